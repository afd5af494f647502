"""The tcgen05 tensor-core scorer (many query rows per KV head, raw keys: the
prefill chunk of reattention_exact.py:545-569) against the CPU oracle, through
the C ABI."""
import pytest
import torch

from prism_test_b200 import einsum_topk_func
from tests.parity import check_parity

pytestmark = pytest.mark.gpu

CASES = [
    # B, Hq, Hkv, Sq, Sk, topk, dtype, causal_offset
    (1, 8, 2, 64, 1000, 50, torch.bfloat16, None),     # 256 rows per KV head: one CTA
    (1, 8, 2, 100, 777, 33, torch.float16, None),      # 400 rows: a partial second pair
    (2, 4, 1, 40, 3001, 100, torch.bfloat16, None),    # B = 2, ragged key tiles
    (1, 8, 2, 128, 5000, 200, torch.bfloat16, 4872),   # causal chunk at the end of the keys
    (1, 4, 2, 300, 1200, 20, torch.bfloat16, 900),     # causal, rows that see few keys
    (1, 4, 1, 32, 130, 130, torch.bfloat16, None),     # k = Sk
]


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Sk,topk,dtype,causal", CASES)
def test_prefill_tc_parity(B, Hq, Hkv, Sq, Sk, topk, dtype, causal, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(7 * Sk + Sq)
    q = torch.randn(B, Hq, Sq, 128, generator=g, device=cuda_device).to(dtype)
    k = torch.randn(B, Hkv, Sk, 128, generator=g, device=cuda_device).to(dtype)
    idx, sc = einsum_topk_func(q, k, topk, causal_offset=causal, return_scores=True)
    torch.cuda.synchronize()
    check_parity(idx, sc, q, k, topk, None, 0, causal, by_head=True)


def test_prefill_tc_strided_queries(cuda_device):
    # queries as a slice of a longer chunk (row stride kept, head stride larger)
    g = torch.Generator(device=cuda_device).manual_seed(5)
    qfull = torch.randn(1, 8, 200, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    q = qfull[:, :, 20:170]
    k = torch.randn(1, 2, 1500, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    idx, sc = einsum_topk_func(q, k, 64, return_scores=True)
    torch.cuda.synchronize()
    check_parity(idx, sc, q.contiguous(), k, 64)


def test_prefill_tc_causal_tail_masked(cuda_device):
    # causal offset 0: the first CTA's rows see only the first keys, so most key
    # tiles are never scored for them and must read as masked
    g = torch.Generator(device=cuda_device).manual_seed(12)
    q = torch.randn(1, 4, 128, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(1, 2, 3000, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    idx, sc = einsum_topk_func(q, k, 40, causal_offset=0, return_scores=True)
    torch.cuda.synchronize()
    check_parity(idx, sc, q, k, 40, None, 0, 0, by_head=True)
    # masked keys follow the visible ones in ascending index order
    assert idx[0, 0, 0, :5].tolist() == [0, 1, 2, 3, 4]
