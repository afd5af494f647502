"""Drop-in for ``eval_harness.kernels.einsum_topk_func``.

Reference interface: ``einsum_topk_func(q, k, topk) -> int32 [B, Hq, Sq, topk]``
(eval_harness/kernels/einsum_topk.py:164-225), bound by the ReAttention callers
as the module attribute ``reattention._einsum_topk_func``
(eval_harness/attention_methods/reattention.py:131-137, called at :483).

Differences from the reference launcher, all keyword-only extensions whose
defaults keep the reference call working unchanged:

* ``mode="exact"`` (default) returns the exact top-k of the fp32 scores, i.e.
  what the reference's dense path ``ReAttentionMethod._dense_topk``
  (reattention.py:486-498) selects, sorted by descending score (torch.topk
  order). The reference Triton kernel's per-128-key block-maximum top-{1,4}
  (``mode="blockmax"``) is a separate mode. ``mode="stream"`` gives the exact
  result without a score matrix (raw keys, >= 128 query rows per KV head,
  ``topk <= 4096``); exact mode switches to it by itself for prefill chunks whose
  score matrix would reach 2 GiB.
* Any ``seqlen_q >= 1``, any ``seqlen_k``, any ``1 <= topk <= min(seqlen_k, 16384)``
  in exact mode (the reference needs ``seqlen_q % 128 == 0``, ``seqlen_k % 128 == 0``
  and ``topk in {1, 4}``).
* ``inv_freq`` fuses ``ReAttentionMethod._unrotate_keys`` (reattention.py:743-793):
  ``k`` then holds RoPE-rotated keys at absolute positions ``pos_offset + j``.
* ``causal_offset``: key ``j`` is visible to query row ``s`` iff
  ``j <= causal_offset + s`` (masked keys score ``-inf``).
* ``index_base`` is added to every returned index (sequence shards).
* ``recall_type`` ("qk" default, "qkv", "qkv2") with ``values`` fuses
  ``ReAttentionMethod._apply_recall_weight`` (reattention.py:822-842): each key's
  score is scaled by the L1 / L2 norm of its value row (the norm rounded to the
  values' dtype, as ``values.norm`` returns it). Other recall types raise
  ``ValueError`` with the reference's messages.
* ``return_scores=True`` also returns the fp32 scores of the selected keys.

Argument errors raise ``AssertionError`` like the reference's ``assert``
statements; CUDA failures raise ``PrismLibraryError`` (a ``RuntimeError``).
Both are ``Exception``s, so the caller's ``use_triton_kernel='auto'`` fallback
(reattention.py:408-418) keeps working. There is no CPU or PyTorch fallback.
"""
from __future__ import annotations

import os
from typing import Optional, Tuple, Union

import torch

from . import _lib

_SYNC_CHECK = os.environ.get("PRISM_SYNC_CHECK", "0") not in ("", "0")


def _dtype_code(dt: torch.dtype) -> int:
    return _lib.DTYPE_BF16 if dt == torch.bfloat16 else _lib.DTYPE_FP16


def _rows_contiguous_aligned(k: torch.Tensor) -> bool:
    if k.stride(-2) != k.shape[-1]:
        return False
    esz = k.element_size()
    if k.data_ptr() % 16:
        return False
    return (k.stride(0) * esz) % 16 == 0 and (k.stride(1) * esz) % 16 == 0


def _value_rows_aligned(v: torch.Tensor) -> bool:
    if v.stride(-1) != 1 or v.data_ptr() % 16:
        return False
    esz = v.element_size()
    return all((st * esz) % 16 == 0 for st in v.stride()[:3])


def _recall_weight_code(recall_type: str) -> int:
    """recall_type -> PRISM_RECALL_*, raising like ReAttentionMethod._apply_recall_weight
    (reattention.py:822-842) for the types it rejects."""
    codes = {"qk": _lib.RECALL_QK, "qkv": _lib.RECALL_QKV, "qkv2": _lib.RECALL_QKV2}
    if recall_type in codes:
        return codes[recall_type]
    if recall_type in ("qk_pe", "qkv_pe", "qkv2_pe"):
        raise ValueError(
            f"Unsupported recall_type '{recall_type}' for the hook port: the "
            "'_pe' variants score against position-encoded (rotated) "
            "keys, but this port un-rotates the cache unconditionally "
            "('_pe' variants are not implemented).",
        )
    raise ValueError(f"Unsupported recall_type '{recall_type}'. Use one of: qk, qkv, qkv2.")


def einsum_topk_func(
    q: torch.Tensor,
    k: torch.Tensor,
    topk: int,
    *,
    inv_freq: Optional[torch.Tensor] = None,
    pos_offset: int = 0,
    causal_offset: Optional[int] = None,
    index_base: int = 0,
    return_scores: bool = False,
    mode: str = "exact",
    out: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
    values: Optional[torch.Tensor] = None,
    recall_type: str = "qk",
) -> Union[torch.Tensor, Tuple[torch.Tensor, torch.Tensor]]:
    """Fused (un-rotate +) q·K^T + top-k on the GPU.

    Parameters
    ----------
    q : Tensor [batch, num_heads, seqlen_q, 128], fp16/bf16, CUDA
    k : Tensor [batch, num_kv_heads, seqlen_k, 128], same dtype and device
    topk : int

    Returns
    -------
    indices : int32 Tensor [batch, num_heads, seqlen_q, topk], sorted by
        descending score (and ``scores`` fp32 of the same shape when
        ``return_scores``).

    ``out=(indices, scores)`` writes into caller tensors instead (contiguous,
    int32 and fp32, ``batch * num_heads * seqlen_q * topk`` elements each) and
    returns them.

    ``values`` : Tensor [batch, num_kv_heads, seqlen_k, head_dim_v], the value
    rows of the same keys, needed by ``recall_type`` "qkv" / "qkv2".
    """
    weight_code = _recall_weight_code(recall_type)
    batch, num_heads, seqlen_q, d = q.shape
    batch_k, num_heads_k, seqlen_k, dk = k.shape
    assert q.stride(-1) == 1 and k.stride(-1) == 1
    assert num_heads % num_heads_k == 0, "num_heads must be divisible by num_heads_k"
    assert d == dk and batch_k == batch, (
        f"batch & head dimensions must match, but find q.shape={q.shape} and k.shape={k.shape}"
    )
    assert q.dtype == k.dtype and q.dtype in [torch.float16, torch.bfloat16], (
        "All tensors must have the same type. Only support fp16 and bf16"
    )
    assert q.is_cuda and k.is_cuda, "All tensors must be sent to gpu"
    assert q.device == k.device, "q and k must be on the same device"
    assert d == 128, f"Only support d == 128, but find d={d}"
    if mode in ("exact", "stream"):
        mode_code = _lib.MODE_EXACT if mode == "exact" else _lib.MODE_EXACT_STREAM
        assert 1 <= topk <= seqlen_k, f"need 1 <= topk <= seqlen_k, got topk={topk}, seqlen_k={seqlen_k}"
    elif mode == "blockmax":
        mode_code = _lib.MODE_BLOCKMAX
        assert seqlen_q % 128 == 0 and seqlen_k % 128 == 0, (
            f"blockmax mode needs seqlen_q % 128 == 0 && seqlen_k % 128 == 0, "
            f"but find seqlen_q={seqlen_q}, seqlen_k={seqlen_k}"
        )
        assert topk == 1 or topk == 4, "Only support k == 1 or 4"
    else:
        raise AssertionError(f"unknown mode {mode!r}; use 'exact', 'stream' or 'blockmax'")

    if weight_code != _lib.RECALL_QK:
        assert values is not None, f"recall_type {recall_type!r} needs values"
        assert values.dim() == 4 and tuple(values.shape[:3]) == (batch, num_heads_k, seqlen_k), (
            f"values must be [batch, num_kv_heads, seqlen_k, head_dim_v], got {tuple(values.shape)}"
        )
        assert values.dtype == q.dtype, "values must have the dtype of q and k"
        assert values.device == q.device, "values must be on the device of q"

    lib = _lib.load()
    with torch.cuda.device(q.device):
        if not _rows_contiguous_aligned(k):
            k = k.contiguous()
        if weight_code != _lib.RECALL_QK and not _value_rows_aligned(values):
            values = values.contiguous()
        invf_ptr = None
        if inv_freq is not None:
            assert inv_freq.numel() == d // 2, "inv_freq must have head_dim // 2 entries"
            inv_freq = inv_freq.to(device=q.device, dtype=torch.float32).contiguous()
            invf_ptr = inv_freq.data_ptr()
        causal = -1 if causal_offset is None else int(causal_offset)
        assert causal_offset is None or causal >= 0, "causal_offset must be >= 0"

        if out is not None:
            out_idx, out_scores = out
            n_out = batch * num_heads * seqlen_q * topk
            assert out_idx.dtype == torch.int32 and out_idx.is_contiguous() and out_idx.numel() == n_out
            assert out_scores.dtype == torch.float32 and out_scores.is_contiguous() and out_scores.numel() == n_out
            assert out_idx.device == q.device and out_scores.device == q.device
            return_scores = True
        else:
            out_idx = torch.empty((batch, num_heads, seqlen_q, topk), dtype=torch.int32, device=q.device)
            out_scores = (
                torch.empty((batch, num_heads, seqlen_q, topk), dtype=torch.float32, device=q.device)
                if return_scores else None
            )
        size_fn = (lib.prism_einsum_topk_rope_workspace_size if invf_ptr is not None
                   else lib.prism_einsum_topk_weighted_workspace_size)
        ws_bytes = size_fn(batch, num_heads, num_heads_k, seqlen_q, seqlen_k, topk, mode_code, weight_code)
        ws = torch.empty(max(int(ws_bytes), 256), dtype=torch.uint8, device=q.device)
        stream = torch.cuda.current_stream(q.device).cuda_stream
        if weight_code == _lib.RECALL_QK:
            rc = lib.prism_einsum_topk(
                q.data_ptr(), k.data_ptr(), invf_ptr, _dtype_code(q.dtype),
                batch, num_heads, num_heads_k, seqlen_q, seqlen_k, d,
                _lib.i64_array(q.stride()), _lib.i64_array(k.stride()), int(pos_offset),
                causal, int(topk), mode_code, int(index_base),
                out_idx.data_ptr(), out_scores.data_ptr() if out_scores is not None else None,
                ws.data_ptr(), ws.numel(), stream,
            )
            _lib.check(rc, "prism_einsum_topk")
        else:
            rc = lib.prism_einsum_topk_weighted(
                q.data_ptr(), k.data_ptr(), values.data_ptr(), invf_ptr, _dtype_code(q.dtype),
                batch, num_heads, num_heads_k, seqlen_q, seqlen_k, d, values.shape[-1],
                _lib.i64_array(q.stride()), _lib.i64_array(k.stride()),
                _lib.i64_array(values.stride()), int(pos_offset), causal, weight_code,
                int(topk), mode_code, int(index_base),
                out_idx.data_ptr(), out_scores.data_ptr() if out_scores is not None else None,
                ws.data_ptr(), ws.numel(), stream,
            )
            _lib.check(rc, "prism_einsum_topk_weighted")
        if _SYNC_CHECK:
            read_status(ws)
    if return_scores:
        return out_idx, out_scores
    return out_idx


def read_status(workspace: torch.Tensor) -> None:
    """Synchronise and raise if a kernel reported a device-side error."""
    lib = _lib.load()
    st = _lib.ctypes.c_int(0)
    rc = lib.prism_read_status(workspace.data_ptr(), _lib.ctypes.byref(st),
                               torch.cuda.current_stream(workspace.device).cuda_stream)
    _lib.check(rc, "prism_read_status")
    if st.value != 0:
        raise _lib.PrismLibraryError(f"device status {st.value} reported by a prism kernel")


def topk_merge(cand_scores: torch.Tensor, cand_idx: torch.Tensor, topk: int,
               return_scores: bool = True):
    """Exact top-k of each row of (score, global index) candidate lists.

    ``cand_scores`` fp32 and ``cand_idx`` int32, both ``[rows, n]`` on the
    same CUDA device. Used to merge the per-shard top-k lists of the
    sequence-sharded path after the NCCL all-gather.
    """
    assert cand_scores.dtype == torch.float32 and cand_idx.dtype == torch.int32
    assert cand_scores.shape == cand_idx.shape and cand_scores.dim() == 2
    assert cand_scores.is_cuda and cand_idx.is_cuda
    rows, n = cand_scores.shape
    assert 1 <= topk <= n
    lib = _lib.load()
    with torch.cuda.device(cand_scores.device):
        ld = (n + 3) // 4 * 4
        if cand_scores.stride() != (ld, 1) or cand_scores.data_ptr() % 16:
            s = torch.full((rows, ld), float("-inf"), dtype=torch.float32, device=cand_scores.device)
            s[:, :n] = cand_scores
            cand_scores = s
        if cand_idx.stride() != (ld, 1) or cand_idx.data_ptr() % 16:
            i = torch.zeros((rows, ld), dtype=torch.int32, device=cand_idx.device)
            i[:, :n] = cand_idx
            cand_idx = i
        out_idx = torch.empty((rows, topk), dtype=torch.int32, device=cand_scores.device)
        out_scores = torch.empty((rows, topk), dtype=torch.float32, device=cand_scores.device)
        ws_bytes = int(lib.prism_topk_merge_workspace_size(rows, n))
        ws = torch.empty(max(ws_bytes, 16), dtype=torch.uint8, device=cand_scores.device)
        rc = lib.prism_topk_merge(
            cand_scores.data_ptr(), cand_idx.data_ptr(), rows, n, ld, int(topk),
            out_idx.data_ptr(), out_scores.data_ptr(), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream(cand_scores.device).cuda_stream,
        )
        _lib.check(rc, "prism_topk_merge")
    return (out_idx, out_scores) if return_scores else out_idx


def topk_merge_runs(runs: torch.Tensor, topk: int, return_scores: bool = True):
    """Top-k of the union of sorted runs.

    ``runs`` int32 ``[nruns, 2, rows, run_len]``: plane 0 the fp32 score bits, plane
    1 the global indices, each run's rows sorted like ``einsum_topk_func`` output
    (descending score, then ascending index) — the layout of an all-gather of the
    ranks' results written with ``out=``. Returns int32 indices ``[rows, topk]``
    (and fp32 scores).
    """
    assert runs.dtype == torch.int32 and runs.dim() == 4 and runs.shape[1] == 2
    assert runs.is_cuda
    nruns, _, rows, run_len = runs.shape
    assert 1 <= topk <= run_len
    runs = runs.contiguous()
    lib = _lib.load()
    with torch.cuda.device(runs.device):
        out_idx = torch.empty((rows, topk), dtype=torch.int32, device=runs.device)
        out_scores = torch.empty((rows, topk), dtype=torch.float32, device=runs.device)
        rc = lib.prism_topk_merge_runs(
            runs.data_ptr(), nruns, rows, run_len, int(topk), out_idx.data_ptr(),
            out_scores.data_ptr(), torch.cuda.current_stream(runs.device).cuda_stream,
        )
        _lib.check(rc, "prism_topk_merge_runs")
    return (out_idx, out_scores) if return_scores else out_idx


def post_select(topk_idx: torch.Tensor, n_middle: int, recall_clip: int = -1, span_size: int = 0,
                span_mode: str = "centered") -> torch.Tensor:
    """Sorted, deduplicated middle positions to keep, computed on the device.

    ``topk_idx``: middle-relative indices of any shape (e.g. the ``[B, Hq, Sq, k]``
    output of ``einsum_topk_func``). Equals
    ``ReAttentionMethod._expand_spans(ReAttentionMethod._global_unique(topk_idx,
    recall_clip), n_middle)`` (eval_harness/attention_methods/reattention.py:844-874)
    for ``span_mode="centered"``, and the span arithmetic of
    eval_harness/attention_methods/reattention_exact.py:578-581 for
    ``span_mode="floor"``. Returns an int64 tensor on the same device; reading its
    length synchronises the stream, as ``torch.unique`` does.
    """
    assert topk_idx.is_cuda, "topk_idx must be on the GPU"
    assert n_middle > 0 and span_size >= 0
    modes = {"centered": _lib.SPAN_CENTERED, "floor": _lib.SPAN_FLOOR}
    assert span_mode in modes, f"span_mode must be one of {sorted(modes)}"
    idx = topk_idx.reshape(-1).to(torch.int32).contiguous()
    lib = _lib.load()
    with torch.cuda.device(idx.device):
        out_pos = torch.empty(n_middle, dtype=torch.int32, device=idx.device)
        out_count = torch.zeros(1, dtype=torch.int32, device=idx.device)
        clip = -1 if recall_clip is None else int(recall_clip)
        ws_bytes = int(lib.prism_post_select_workspace_size(n_middle, clip))
        ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=idx.device)
        rc = lib.prism_post_select(
            idx.data_ptr(), idx.numel(), int(n_middle), clip, int(span_size), modes[span_mode],
            out_pos.data_ptr(), out_count.data_ptr(), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream(idx.device).cuda_stream,
        )
        _lib.check(rc, "prism_post_select")
        n = int(out_count.item())
    return out_pos[:n].to(torch.int64)


def sparse_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, key_pos: torch.Tensor, *,
                     q_pos: Optional[torch.Tensor] = None, inv_freq: Optional[torch.Tensor] = None,
                     pe_original: bool = True, scale: Optional[float] = None) -> torch.Tensor:
    """Attention over the selected view, on the GPU (C ABI ``prism_sparse_attention``).

    The step after the recall selection in ReAttentionExactMethod._chunk_attention
    (eval_harness/attention_methods/reattention_exact.py:453-508 and the eager path of
    ``_attend``, :650-661): the view's keys and values are gathered from the raw cache
    ``k``, ``v`` [B, Hkv, S, 128] at the absolute positions ``key_pos`` [nsel], keys and
    queries ``q`` [B, Hq, Sq, 128] are rotated at their RoPE positions (absolute with
    ``pe_original``, else contiguous with the queries last), and
    ``softmax(q k^T * scale) v`` is taken in fp32 with keys past a query's absolute
    position ``q_pos`` masked (default: the last Sq positions of the cache). Returns
    [B, Hq, Sq, 128] in q's dtype; a query that sees no key gives zeros.
    """
    B, Hq, Sq, D = q.shape
    Bk, Hkv, S, Dk = k.shape
    assert v.shape == k.shape and Bk == B and Dk == D, "q, k, v shapes disagree"
    assert q.dtype == k.dtype == v.dtype and q.dtype in (torch.float16, torch.bfloat16), (
        "q, k and v must share one dtype, fp16 or bf16")
    assert q.is_cuda and k.device == q.device and v.device == q.device, "all tensors on one GPU"
    assert Hq % Hkv == 0, "num_heads must be divisible by num_heads_k"
    assert D == 128, f"Only support d == 128, but find d={D}"
    dev = q.device
    key_pos = key_pos.to(device=dev, dtype=torch.int64).contiguous()
    if q_pos is None:
        q_pos = torch.arange(S - Sq, S, device=dev, dtype=torch.int64)
    q_pos = q_pos.to(device=dev, dtype=torch.int64).contiguous()
    assert q_pos.numel() == Sq, "q_pos needs one position per query row"
    if scale is None:
        scale = D ** -0.5
    lib = _lib.load()
    with torch.cuda.device(dev):
        if k.stride(-2) != D or k.stride(-1) != 1:
            k = k.contiguous()
        if v.stride(-2) != D or v.stride(-1) != 1:
            v = v.contiguous()
        if any(s % 4 for s in q.stride()[:3]) or q.stride(-1) != 1:
            q = q.contiguous()
        invf = None
        if inv_freq is not None:
            inv_freq = inv_freq.to(device=dev, dtype=torch.float32).contiguous()
            assert inv_freq.numel() == D // 2, "inv_freq must have head_dim // 2 entries"
            invf = inv_freq.data_ptr()
        out = torch.empty((B, Hq, Sq, D), dtype=q.dtype, device=dev)
        ws_bytes = lib.prism_sparse_attention_workspace_size(B, Hq, Sq, key_pos.numel())
        ws = torch.empty(max(int(ws_bytes), 256), dtype=torch.uint8, device=dev)
        rc = lib.prism_sparse_attention(
            q.data_ptr(), k.data_ptr(), v.data_ptr(), key_pos.data_ptr(), key_pos.numel(),
            q_pos.data_ptr(), invf, 1 if pe_original else 0, float(scale), _dtype_code(q.dtype),
            B, Hq, Hkv, Sq, S, D, _lib.i64_array(q.stride()), _lib.i64_array(k.stride()),
            _lib.i64_array(v.stride()), out.data_ptr(), ws.data_ptr(), ws.numel(),
            torch.cuda.current_stream(dev).cuda_stream,
        )
        _lib.check(rc, "prism_sparse_attention")
        if _SYNC_CHECK:
            read_status(ws)
    return out
