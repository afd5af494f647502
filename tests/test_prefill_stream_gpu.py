"""The streaming prefill top-k (sampled per-row thresholds, candidates from the
tcgen05 scorer, per-row selection, exact recompute of missed rows) against the
CPU oracle, through the C ABI. No score matrix is written on this path. RoPE'd
keys reach the same scorer through un-rotated hi / lo key planes."""
import pytest
import torch

from prism_test_b200 import einsum_topk_func, read_status
from prism_test_b200 import kernels, workloads as W
from prism_test_b200 import _lib
from tests.parity import check_parity, check_rows_parity

pytestmark = pytest.mark.gpu

CASES = [
    # B, Hq, Hkv, Sq, Sk, topk, dtype, causal_offset
    (1, 8, 2, 128, 8192, 256, torch.bfloat16, None),
    (1, 8, 2, 160, 12000, 1000, torch.float16, None),   # partial CTA, ragged key tiles
    (1, 4, 1, 64, 20000, 2048, torch.bfloat16, 19936),  # causal chunk at the end of the keys
    (2, 4, 2, 64, 9000, 64, torch.bfloat16, 5000),      # B = 2, causal with later keys masked
    (1, 8, 2, 128, 8192, 4096, torch.bfloat16, None),   # largest streaming k
]


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Sk,topk,dtype,causal", CASES)
def test_stream_parity(B, Hq, Hkv, Sq, Sk, topk, dtype, causal, cuda_device, monkeypatch):
    monkeypatch.setattr(kernels, "_SYNC_CHECK", True)
    g = torch.Generator(device=cuda_device).manual_seed(Sk + topk)
    q = torch.randn(B, Hq, Sq, 128, generator=g, device=cuda_device).to(dtype)
    k = torch.randn(B, Hkv, Sk, 128, generator=g, device=cuda_device).to(dtype)
    idx, sc = einsum_topk_func(q, k, topk, causal_offset=causal, return_scores=True, mode="stream")
    torch.cuda.synchronize()
    check_parity(idx, sc, q, k, topk, None, 0, causal, by_head=True)


def test_stream_rows_seeing_fewer_than_k_keys(cuda_device):
    # causal offset 0: row s sees s + 1 keys; rows below k - 1 continue with the
    # masked keys in ascending index order
    g = torch.Generator(device=cuda_device).manual_seed(2)
    q = torch.randn(1, 4, 128, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(1, 2, 8192, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    a = einsum_topk_func(q, k, 64, causal_offset=0, return_scores=True, mode="stream")
    b = einsum_topk_func(q, k, 64, causal_offset=0, return_scores=True, mode="exact")
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_stream_missed_rows_take_the_exact_fallback(cuda_device, monkeypatch):
    # rows with a zero query score 0 against every key: their threshold admits
    # every key (more than the candidate capacity), so they are recomputed exactly
    monkeypatch.setattr(kernels, "_SYNC_CHECK", True)
    g = torch.Generator(device=cuda_device).manual_seed(4)
    q = torch.randn(1, 8, 128, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    q[0, 3, 5:25] = 0
    k = torch.randn(1, 2, 10000, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    a = einsum_topk_func(q, k, 300, return_scores=True, mode="stream")
    b = einsum_topk_func(q, k, 300, return_scores=True, mode="exact")
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_stream_matches_score_matrix_path(cuda_device):
    # same inputs through both exact paths: identical indices and scores
    g = torch.Generator(device=cuda_device).manual_seed(9)
    q = torch.randn(1, 32, 128, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(1, 8, 16384, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    a = einsum_topk_func(q, k, 1024, causal_offset=16256, return_scores=True, mode="stream")
    b = einsum_topk_func(q, k, 1024, causal_offset=16256, return_scores=True, mode="exact")
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


def test_stream_full_prefill_chunk_sampled_rows(cuda_device, monkeypatch):
    # the full 4096-row x 131072-key causal chunk (exact mode takes the streaming
    # path by itself here); the oracle checks a spread of rows
    monkeypatch.setattr(kernels, "_SYNC_CHECK", True)
    wl = W.WORKLOADS["prefill-chunk-128k"]
    x = W.make_inputs(wl, cuda_device)
    assert x["inv_freq"] is None
    idx, sc = einsum_topk_func(x["q"], x["k"], wl.topk, causal_offset=wl.causal_offset,
                               return_scores=True)
    torch.cuda.synchronize()
    n = wl.B * wl.Hq * wl.Sq
    rows = sorted(set(list(range(0, n, n // 96)) + [1, 4095, 4096, n - 1]))
    check_rows_parity(idx, sc, x["q"], x["k"], wl.topk, rows, wl.causal_offset)


def test_stream_duplicate_keys_tie_by_index(cuda_device):
    # every key appears three times: equal scores must come out lowest index first
    g = torch.Generator(device=cuda_device).manual_seed(21)
    q = torch.randn(1, 8, 128, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    base = torch.randn(1, 2, 3000, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k = base.repeat_interleave(3, dim=2)[:, :, :8192].contiguous()
    a = einsum_topk_func(q, k, 600, return_scores=True, mode="stream")
    b = einsum_topk_func(q, k, 600, return_scores=True, mode="exact")
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


ROPE_CASES = [
    # B, Hq, Hkv, Sq, Sk, topk, dtype, causal_offset, pos_offset
    (1, 8, 2, 128, 8192, 256, torch.bfloat16, None, 0),
    (1, 8, 2, 160, 12000, 1000, torch.float16, None, 70000),  # partial CTA, later positions
    (1, 4, 1, 64, 20000, 2048, torch.bfloat16, 19936, 3),     # causal chunk at the end
    (2, 4, 2, 64, 9000, 64, torch.bfloat16, 5000, 1000),      # B = 2
]


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Sk,topk,dtype,causal,pos", ROPE_CASES)
def test_stream_rope_parity(B, Hq, Hkv, Sq, Sk, topk, dtype, causal, pos, cuda_device, monkeypatch):
    # RoPE'd keys on the streaming path: un-rotated once into hi / lo planes, then
    # the same tcgen05 threshold and candidate passes
    monkeypatch.setattr(kernels, "_SYNC_CHECK", True)
    g = torch.Generator(device=cuda_device).manual_seed(Sk + topk + 1)
    q = torch.randn(B, Hq, Sq, 128, generator=g, device=cuda_device).to(dtype)
    k = torch.randn(B, Hkv, Sk, 128, generator=g, device=cuda_device).to(dtype)
    inv = W.rope_inv_freq(128, 5e5).to(cuda_device)
    idx, sc = einsum_topk_func(q, k, topk, inv_freq=inv, pos_offset=pos, causal_offset=causal,
                               return_scores=True, mode="stream")
    torch.cuda.synchronize()
    check_parity(idx, sc, q, k, topk, inv, pos, causal, by_head=True)


@pytest.mark.parametrize("mode", ["exact", "stream"])
def test_rope_tensor_core_score_matrix_and_stream_agree(mode, cuda_device, monkeypatch):
    # >= 128 query rows per KV head with RoPE'd keys: the score-matrix path also
    # scores on the tensor cores from the planes; both paths meet the oracle
    monkeypatch.setattr(kernels, "_SYNC_CHECK", True)
    g = torch.Generator(device=cuda_device).manual_seed(31)
    q = torch.randn(1, 8, 64, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(1, 2, 5000, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    inv = W.rope_inv_freq(128, 1e4).to(cuda_device)
    idx, sc = einsum_topk_func(q, k, 300, inv_freq=inv, pos_offset=777, return_scores=True, mode=mode)
    torch.cuda.synchronize()
    check_parity(idx, sc, q, k, 300, inv, 777, None, by_head=True)


def test_rope_planes_fall_back_to_cuda_cores_without_room(cuda_device):
    # the plain workspace (no room for the planes): the score-matrix path takes
    # the CUDA-core scorer and still meets the oracle
    lib = _lib.load()
    g = torch.Generator(device=cuda_device).manual_seed(32)
    B, Hq, Hkv, Sq, Sk, topk = 1, 8, 2, 32, 3000, 100
    q = torch.randn(B, Hq, Sq, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(B, Hkv, Sk, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    inv = W.rope_inv_freq(128, 5e5).to(cuda_device)
    plain = lib.prism_einsum_topk_workspace_size(B, Hq, Sq, Sk, topk, _lib.MODE_EXACT)
    rope = lib.prism_einsum_topk_rope_workspace_size(B, Hq, Hkv, Sq, Sk, topk, _lib.MODE_EXACT, _lib.RECALL_QK)
    assert rope > plain
    for nbytes in (plain, rope):
        ws = torch.empty(int(nbytes), dtype=torch.uint8, device=cuda_device)
        oi = torch.empty(B, Hq, Sq, topk, dtype=torch.int32, device=cuda_device)
        os_ = torch.empty(B, Hq, Sq, topk, dtype=torch.float32, device=cuda_device)
        rc = lib.prism_einsum_topk(q.data_ptr(), k.data_ptr(), inv.data_ptr(), _lib.DTYPE_BF16, B, Hq, Hkv, Sq, Sk,
                                   128, _lib.i64_array(q.stride()), _lib.i64_array(k.stride()), 5, -1, topk,
                                   _lib.MODE_EXACT, 0, oi.data_ptr(), os_.data_ptr(), ws.data_ptr(), ws.numel(),
                                   torch.cuda.current_stream().cuda_stream)
        _lib.check(rc, "prism_einsum_topk")
        torch.cuda.synchronize()
        check_parity(oi, os_, q, k, topk, inv, 5, None, by_head=True)


@pytest.mark.parametrize("rope", [False, True])
def test_keys_shared_across_the_batch(rope, cuda_device):
    # keys expanded over the batch (batch stride 0): every batch row reads the one
    # key set, on the tensor-core path with and without RoPE
    g = torch.Generator(device=cuda_device).manual_seed(33)
    q = torch.randn(3, 8, 64, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k1 = torch.randn(1, 2, 4096, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k = k1.expand(3, -1, -1, -1)
    assert k.stride(0) == 0
    inv = W.rope_inv_freq(128, 5e5).to(cuda_device) if rope else None
    for mode in ("exact", "stream"):
        idx, sc = einsum_topk_func(q, k, 200, inv_freq=inv, return_scores=True, mode=mode)
        torch.cuda.synchronize()
        check_parity(idx, sc, q, k.contiguous(), 200, inv, 0, None, by_head=True)


def test_stream_full_rope_prefill_chunk_sampled_rows(cuda_device, monkeypatch):
    # the full 4096-row x 131072-key causal chunk over a RoPE'd cache: un-rotated
    # planes, then the tcgen05 streaming path; the oracle checks a spread of rows
    monkeypatch.setattr(kernels, "_SYNC_CHECK", True)
    wl = W.WORKLOADS["prefill-chunk-128k-rope"]
    x = W.make_inputs(wl, cuda_device)
    assert x["inv_freq"] is not None
    idx, sc = einsum_topk_func(x["q"], x["k"], wl.topk, inv_freq=x["inv_freq"], causal_offset=wl.causal_offset,
                               return_scores=True)
    torch.cuda.synchronize()
    n = wl.B * wl.Hq * wl.Sq
    rows = sorted(set(list(range(0, n, n // 48)) + [1, 4095, 4096, n - 1]))
    check_rows_parity(idx, sc, x["q"], x["k"], wl.topk, rows, wl.causal_offset, inv_freq=x["inv_freq"])
