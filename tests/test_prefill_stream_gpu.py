"""The streaming prefill top-k (sampled per-row thresholds, candidates from the
tcgen05 scorer, per-row selection, exact recompute of missed rows) against the
CPU oracle, through the C ABI. No score matrix is written on this path."""
import pytest
import torch

from prism_test_b200 import einsum_topk_func, read_status
from prism_test_b200 import kernels, workloads as W
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
