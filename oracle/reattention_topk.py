"""CPU oracle of the ReAttention recall scorer — TEST INFRASTRUCTURE ONLY.

Only the tests, ``__graft_entry__.smoke()`` (as a checker) and ``bench.py``'s
CPU-baseline leg, reference arm and post-timing result check may import this
module. The product path never does.

A plain-PyTorch fp32 restatement, on the CPU, of the reference's dense recall
path (RUSH-Intelligence/Prism-Test, eval_harness/attention_methods/):

* ``build_cos_sin``        _method_base.py:353-381  fp32 angles pos*inv_freq,
                           duplicated halves, cos/sin
* ``rotate_half``          _method_base.py:384-388
* ``apply_rotary_pos_emb`` _method_base.py:324-333
* ``undo_rotary_pos_emb``  _method_base.py:336-350  x*cos + rotate_half(x)*(-sin)
* ``unrotate_keys``        ReAttentionMethod._unrotate_keys, reattention.py:743-793
                           (inv_freq branch :780-784, positions 0..S-1, offset
                           here by ``pos_offset``), evaluated in fp32 on the
                           keys upcast to fp32
* ``repeat_kv``            reattention.py:158-164
* ``dense_topk``           ReAttentionMethod._dense_topk, reattention.py:486-498:
                           einsum("bhqd,bhmd->bhqm") in fp32, then topk (sorted,
                           largest first); a causal mask (-inf) is applied before
                           topk when ``causal_offset`` is given
* ``recall_weights``       ReAttentionMethod._apply_recall_weight, reattention.py:822-842:
                           qkv -> ||v||_1, qkv2 -> ||v||_2 per key, as the
                           values' dtype (``values.norm`` of a bf16/fp16 tensor);
                           the weighted raw key is raw_k (fp32) * that weight
* ``sparse_attention``     ReAttentionExactMethod._chunk_attention's gather + RoPE
                           (reattention_exact.py:453-508) and the eager path of
                           _attend (:650-661), in fp32
* ``blockmax_topk``        the fused Triton kernels einsum_topk.py:21-161 with the
                           4-wide merge of bitonic_merge_wrapper.py:5-52: per
                           128-key block the row maximum (first index on ties),
                           a running top-1 (later block wins ties, ``>=``) or
                           top-4 (strict ``>``, inserted at slot 3, then the
                           2-stage descending merge).

The restatement is pinned by ``tests/golden/`` vectors produced by calling the
reference's own functions (``tests/golden/make_golden.py``).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch


def build_cos_sin(position_ids: torch.Tensor, inv_freq: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """cos, sin of shape [S, D] in fp32 (reference :353-381, batch/head dims dropped)."""
    pos = position_ids.to(torch.float32)
    freqs = torch.einsum("s,d->sd", pos, inv_freq.to(torch.float32))
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def rotate_half(x: torch.Tensor) -> torch.Tensor:
    h = x.shape[-1] // 2
    return torch.cat((-x[..., h:], x[..., :h]), dim=-1)


def apply_rotary_pos_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return (x * cos) + (rotate_half(x) * sin)


def undo_rotary_pos_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    return (x * cos) + (rotate_half(x) * (-sin))


def unrotate_keys(k: torch.Tensor, inv_freq: Optional[torch.Tensor], pos_offset: int = 0) -> torch.Tensor:
    """Raw fp32 keys from RoPE-rotated cached keys [B, Hkv, S, D]."""
    kf = k.to(torch.float32)
    if inv_freq is None:
        return kf
    S = k.shape[2]
    cos, sin = build_cos_sin(torch.arange(pos_offset, pos_offset + S), inv_freq.cpu())
    return undo_rotary_pos_emb(kf, cos, sin)


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1:
        return x
    B, H, S, D = x.shape
    return x[:, :, None].expand(B, H, n_rep, S, D).reshape(B, H * n_rep, S, D)


def dense_scores(q: torch.Tensor, k_raw: torch.Tensor, causal_offset: Optional[int] = None) -> torch.Tensor:
    """fp32 scores [B, Hq, Sq, Sk]."""
    n_rep = max(1, q.shape[1] // k_raw.shape[1])
    scores = torch.einsum("bhqd,bhmd->bhqm", q.to(torch.float32), repeat_kv(k_raw, n_rep).to(torch.float32))
    if causal_offset is not None:
        Sq, Sk = q.shape[2], k_raw.shape[2]
        j = torch.arange(Sk)[None, :]
        i = torch.arange(Sq)[:, None]
        scores = scores.masked_fill(j > causal_offset + i, float("-inf"))
    return scores


def dense_topk(q: torch.Tensor, k: torch.Tensor, topk: int, inv_freq: Optional[torch.Tensor] = None,
               pos_offset: int = 0, causal_offset: Optional[int] = None,
               index_base: int = 0, weights: Optional[torch.Tensor] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """(scores fp32, indices int64) of shape [B, Hq, Sq, topk], largest first.
    ``weights`` [B, Hkv, Sk] (``recall_weights``) scale the raw keys."""
    q = q.cpu()
    k_raw = unrotate_keys(k.cpu(), inv_freq, pos_offset)
    if weights is not None:
        k_raw = k_raw * weights.cpu()[..., None]
    scores = dense_scores(q, k_raw, causal_offset)
    vals, idx = scores.topk(min(topk, scores.shape[-1]), dim=-1)
    return vals, idx + index_base


def dense_topk_by_head(q: torch.Tensor, k: torch.Tensor, topk: int, inv_freq=None, pos_offset: int = 0,
                       causal_offset: Optional[int] = None, index_base: int = 0):
    """``dense_topk`` evaluated one KV head at a time (bounded memory at 1M keys)."""
    B, Hq, Sq, _ = q.shape
    Hkv = k.shape[1]
    G = Hq // Hkv
    vals = []
    idxs = []
    for h in range(Hkv):
        v, i = dense_topk(q[:, h * G:(h + 1) * G], k[:, h:h + 1], topk, inv_freq, pos_offset,
                          causal_offset, index_base)
        vals.append(v)
        idxs.append(i)
    return torch.cat(vals, dim=1), torch.cat(idxs, dim=1)


def blockmax_topk(q: torch.Tensor, k_raw: torch.Tensor, topk: int, block: int = 128) -> torch.Tensor:
    """Indices int32 [B, Hq, Sq, topk] with the Triton kernels' block-maximum semantics.

    ``k_raw`` is used as given (the reference kernel receives raw keys). Scores
    are fp32 dot products of the (bf16/fp16) inputs.
    """
    assert topk in (1, 4)
    s = dense_scores(q.cpu(), k_raw.cpu().to(torch.float32))  # [B,Hq,Sq,Sk]
    B, H, Sq, Sk = s.shape
    nb = Sk // block
    sb = s.reshape(B, H, Sq, nb, block)
    bmax, barg = sb.max(dim=-1)  # torch.max returns the first index of the maximum
    barg = barg + torch.arange(nb)[None, None, None, :] * block
    if topk == 1:
        best = torch.full((B, H, Sq), float("-inf"))
        arg = torch.zeros((B, H, Sq), dtype=torch.int64)
        for t in range(nb):
            m = bmax[..., t] >= best
            best = torch.where(m, bmax[..., t], best)
            arg = torch.where(m, barg[..., t], arg)
        return arg[..., None].to(torch.int32)
    fmin = torch.finfo(torch.float32).min
    vals = torch.full((B, H, Sq, 4), fmin)
    idx = torch.zeros((B, H, Sq, 4), dtype=torch.int64)
    for t in range(nb):
        m = bmax[..., t] > vals[..., 3]
        vals[..., 3] = torch.where(m, bmax[..., t], vals[..., 3])
        idx[..., 3] = torch.where(m, barg[..., t], idx[..., 3])
        # two-stage descending merge: compare (0,2),(1,3) then (0,1),(2,3);
        # swap only when left < right (ties keep their slots)
        for a_, b_ in ((0, 2), (1, 3), (0, 1), (2, 3)):
            sw = vals[..., a_] < vals[..., b_]
            va, vb = vals[..., a_].clone(), vals[..., b_].clone()
            ia, ib = idx[..., a_].clone(), idx[..., b_].clone()
            vals[..., a_] = torch.where(sw, vb, va)
            vals[..., b_] = torch.where(sw, va, vb)
            idx[..., a_] = torch.where(sw, ib, ia)
            idx[..., b_] = torch.where(sw, ia, ib)
    return idx.to(torch.int32)


def score_tolerance(q: torch.Tensor, k_raw: torch.Tensor, rel: float = 1e-3) -> torch.Tensor:
    """Per-(row, key) absolute tolerance: rel * ||q|| * ||k|| ([B, Hq, Sq, Sk]).

    The parity rule: |s - s_ref| <= max(rel * |s_ref|, rel * ||q|| ||k||)."""
    n_rep = max(1, q.shape[1] // k_raw.shape[1])
    qn = q.to(torch.float32).norm(dim=-1)  # [B,Hq,Sq]
    kn = repeat_kv(k_raw, n_rep).norm(dim=-1)  # [B,Hq,Sk]
    return rel * qn[..., :, None] * kn[..., None, :]


def global_unique(topk_idx: torch.Tensor, recall_clip: int) -> torch.Tensor:
    """ReAttentionMethod._global_unique (eval_harness/attention_methods/reattention.py:844-859):
    the sorted unique selected indices, or — when recall_clip >= 0 and more than
    recall_clip survive — the recall_clip most frequently selected (torch.topk over
    the counts; its order among equal counts is unspecified)."""
    flat = topk_idx.reshape(-1).to(torch.int64)
    if recall_clip is None or recall_clip < 0:
        return torch.unique(flat)
    uniq, counts = torch.unique(flat, return_counts=True)
    if uniq.numel() > recall_clip:
        _, keep = torch.topk(counts, k=recall_clip)
        uniq = uniq[keep]
    return uniq


def expand_spans(sel: torch.Tensor, n_middle: int, span_size: int, mode: str = "centered") -> torch.Tensor:
    """Span expansion, clamp to [0, n_middle), unique (sorted).

    centered: ReAttentionMethod._expand_spans (reattention.py:861-874), offsets
    [-(span // 2), (span + 1) // 2), span 0 keeps the positions.
    floor: reattention_exact.py:578-581, offsets [floor(-span / 2), (span + 1) // 2),
    span 0 keeps nothing."""
    if mode == "centered":
        if span_size > 0:
            offsets = torch.arange(-(span_size // 2), (span_size + 1) // 2)
            ids = (sel[:, None] + offsets[None, :]).reshape(-1)
        else:
            ids = sel
    else:
        offsets = torch.arange(-span_size // 2, (span_size + 1) // 2)
        ids = (sel[:, None] + offsets[None, :]).reshape(-1)
    return torch.unique(ids.clamp(0, n_middle - 1))


def recall_weights(values: Optional[torch.Tensor], recall_type: str) -> Optional[torch.Tensor]:
    """Per-key weights [B, Hkv, Sk] (fp32 holding values of the values' dtype) of
    ReAttentionMethod._apply_recall_weight (reattention.py:822-842), or None for "qk".
    The weighted raw key is ``raw_k * weights[..., None]``."""
    if recall_type == "qk":
        return None
    if recall_type == "qkv":
        return values.cpu().norm(p=1, dim=-1).to(torch.float32)
    if recall_type == "qkv2":
        return values.cpu().norm(p=2, dim=-1).to(torch.float32)
    raise ValueError(f"Unsupported recall_type '{recall_type}'. Use one of: qk, qkv, qkv2.")


def sparse_attention(q: torch.Tensor, k_full: torch.Tensor, v_full: torch.Tensor, key_pos: torch.Tensor,
                     q_pos: torch.Tensor, inv_freq: Optional[torch.Tensor], pe_original: bool,
                     scale: float) -> torch.Tensor:
    """Attention over the selected view, fp32 [B, Hq, Sq, D].

    reattention_exact.py:453-508: sel_k / sel_v gathered at the absolute positions
    ``key_pos``; RoPE positions ``key_pos`` / ``q_pos`` (pe_original) or
    ``arange(view_len)`` / its last Sq (contiguous); then _attend's eager path
    (:650-661): repeat_kv, (q k^T) * scale, keys with key_pos > q_pos masked to -inf,
    fp32 softmax, nan_to_num (a row that sees nothing gives zeros), times v."""
    key_pos = key_pos.cpu().long()
    q_pos = q_pos.cpu().long()
    sel_k = k_full.cpu().float()[:, :, key_pos]
    sel_v = v_full.cpu().float()[:, :, key_pos]
    qf = q.cpu().float()
    view_len, q_len = key_pos.numel(), qf.shape[2]
    if inv_freq is not None:
        pe_k = key_pos if pe_original else torch.arange(view_len)
        pe_q = q_pos if pe_original else torch.arange(view_len - q_len, view_len)
        cos_k, sin_k = build_cos_sin(pe_k, inv_freq.cpu())
        sel_k = apply_rotary_pos_emb(sel_k, cos_k, sin_k)
        cos_q, sin_q = build_cos_sin(pe_q, inv_freq.cpu())
        qf = apply_rotary_pos_emb(qf, cos_q, sin_q)
    n_rep = max(1, qf.shape[1] // sel_k.shape[1])
    kk = repeat_kv(sel_k, n_rep)
    vv = repeat_kv(sel_v, n_rep)
    attn = torch.matmul(qf, kk.transpose(2, 3)) * scale
    attn = attn.masked_fill(key_pos[None, :] > q_pos[:, None], float("-inf"))
    attn = torch.softmax(attn, dim=-1, dtype=torch.float32)
    attn = torch.nan_to_num(attn, nan=0.0)
    return torch.matmul(attn, vv)
