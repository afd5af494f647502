"""Value-weighted recall (recall_type "qkv" / "qkv2") on the GPU through the C ABI
(prism_einsum_topk_weighted), against ReAttentionMethod._apply_recall_weight
(eval_harness/attention_methods/reattention.py:822-842) as restated by the
oracle and pinned by the golden vectors tests/golden/recall_*.npz."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reattention_topk as orc
from prism_test_b200 import einsum_topk_func
from prism_test_b200 import workloads as W
from tests.parity import REL_WEIGHTED, check_parity

pytestmark = pytest.mark.gpu

RECALL = sorted((Path(__file__).resolve().parent / "golden").glob("recall_*.npz"))


def _bf16(z, key):
    return torch.from_numpy(z[key].view(np.int16)).view(torch.bfloat16)


@pytest.mark.parametrize("path", RECALL, ids=[p.stem for p in RECALL])
def test_recall_golden(path, cuda_device):
    z = np.load(path)
    q, k, v = _bf16(z, "q_bf16"), _bf16(z, "k_bf16"), _bf16(z, "v_bf16")
    inv = torch.from_numpy(z["inv_freq"])
    rt, topk, pos = str(z["recall_type"]), int(z["topk"]), int(z["pos_offset"])
    idx, sc = einsum_topk_func(q.to(cuda_device), k.to(cuda_device), topk, inv_freq=inv.to(cuda_device),
                               pos_offset=pos, values=v.to(cuda_device), recall_type=rt, return_scores=True)
    torch.cuda.synchronize()
    w = orc.recall_weights(v, rt)
    check_parity(idx, sc, q, k, topk, inv, pos, rel=REL_WEIGHTED, weights=w)
    # the reference's own sorted scores, rank by rank (near-tie swaps move a
    # value by less than its neighbour's gap)
    ref = torch.from_numpy(z["scores"])
    k_w = orc.unrotate_keys(k, inv, pos) * w[..., None]
    lim = 3 * REL_WEIGHTED * torch.maximum(ref.abs(), q.float().norm(dim=-1)[..., None] * k_w.norm(dim=-1).max())
    assert bool(((sc.cpu() - ref).abs() <= lim).all())
    if "zero_values" in path.stem:
        assert bool(torch.isfinite(sc).all())


CASES = [
    # B, Hq, Hkv, Sq, Sk, topk, dtype, Dv, recall_type — scorer paths: decode
    # (hp / mma), wide rows, general chunked; fp16; value widths other than 128
    (1, 32, 8, 1, 16384, 1024, torch.bfloat16, 128, "qkv2"),
    (1, 32, 8, 1, 5000, 300, torch.bfloat16, 128, "qkv"),
    (2, 8, 2, 2, 2048, 100, torch.float16, 128, "qkv"),
    (2, 8, 2, 2, 2048, 100, torch.float16, 128, "qkv2"),
    (1, 32, 8, 16, 4096, 64, torch.bfloat16, 128, "qkv2"),
    (1, 32, 8, 9, 700, 64, torch.bfloat16, 128, "qkv"),
    (1, 8, 2, 1, 3001, 50, torch.bfloat16, 64, "qkv2"),
    (1, 8, 2, 1, 3001, 50, torch.bfloat16, 256, "qkv"),
    (1, 4, 1, 1, 31, 7, torch.bfloat16, 8, "qkv2"),
]


def _weighted_inputs(B, Hq, Hkv, Sq, Sk, dtype, Dv, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(B, Hq, Sq, 128, generator=g).to(dtype)
    raw = torch.randn(B, Hkv, Sk, 128, generator=g)
    v = (torch.randn(B, Hkv, Sk, Dv, generator=g)
         * torch.exp(0.7 * torch.randn(B, Hkv, Sk, 1, generator=g))).to(dtype)
    inv = W.rope_inv_freq(128, 5e5)
    cos, sin = orc.build_cos_sin(torch.arange(Sk), inv)
    k = orc.apply_rotary_pos_emb(raw, cos, sin).to(dtype)
    return q, k, v, inv


@pytest.mark.parametrize("case", CASES, ids=[f"{c[8]}-{c[1]}x{c[3]}x{c[4]}-Dv{c[7]}-{str(c[6])[6:]}" for c in CASES])
def test_recall_random(case, cuda_device):
    B, Hq, Hkv, Sq, Sk, topk, dtype, Dv, rt = case
    q, k, v, inv = _weighted_inputs(B, Hq, Hkv, Sq, Sk, dtype, Dv, seed=Sk + Dv)
    idx, sc = einsum_topk_func(q.to(cuda_device), k.to(cuda_device), topk, inv_freq=inv.to(cuda_device),
                               values=v.to(cuda_device), recall_type=rt, return_scores=True)
    torch.cuda.synchronize()
    check_parity(idx, sc, q, k, topk, inv, rel=REL_WEIGHTED, weights=orc.recall_weights(v, rt))


def test_recall_strided_values_and_causal(cuda_device):
    # values as the middle slice of a longer cache (row offset 32), and a causal
    # chunk: masked keys stay -inf whatever their weight
    B, Hq, Hkv, Sq, Sk, topk = 1, 4, 2, 5, 300, 20
    q, k, v_full, inv = _weighted_inputs(B, Hq, Hkv, Sq, Sk + 64, torch.bfloat16, 128, seed=11)
    k = k[:, :, :Sk].contiguous()
    v = v_full[:, :, 32:32 + Sk]
    dev_v = v_full.to(cuda_device)[:, :, 32:32 + Sk]
    assert not dev_v.is_contiguous()
    idx, sc = einsum_topk_func(q.to(cuda_device), k.to(cuda_device), topk, inv_freq=inv.to(cuda_device),
                               causal_offset=Sk - Sq, values=dev_v, recall_type="qkv", return_scores=True)
    torch.cuda.synchronize()
    check_parity(idx, sc, q, k, topk, inv, causal_offset=Sk - Sq, rel=REL_WEIGHTED,
                 weights=orc.recall_weights(v, "qkv"))


def test_recall_qk_ignores_values(cuda_device):
    q, k, v, inv = _weighted_inputs(1, 8, 2, 1, 2048, torch.bfloat16, 128, seed=3)
    q, k, v, inv = q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), inv.to(cuda_device)
    a = einsum_topk_func(q, k, 64, inv_freq=inv, return_scores=True)
    b = einsum_topk_func(q, k, 64, inv_freq=inv, return_scores=True, values=v, recall_type="qk")
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])


@pytest.mark.parametrize("topk", [1, 4])
def test_recall_blockmax_exact(topk, cuda_device):
    # small integers and the L1 weight: every weighted score is exact in fp32, so
    # the block-maximum selection matches the oracle exactly, ties included
    B, Hq, Hkv, Sq, Sk = 1, 8, 2, 128, 128 * 12
    g = torch.Generator().manual_seed(17 + topk)
    q = torch.randint(-2, 3, (B, Hq, Sq, 128), generator=g).to(torch.bfloat16)
    k = torch.randint(-2, 3, (B, Hkv, Sk, 128), generator=g).to(torch.bfloat16)
    v = torch.randint(-2, 3, (B, Hkv, Sk, 128), generator=g).to(torch.bfloat16)
    w = orc.recall_weights(v, "qkv")
    want = orc.blockmax_topk(q.float(), k.float() * w[..., None], topk)
    got = einsum_topk_func(q.to(cuda_device), k.to(cuda_device), topk, mode="blockmax",
                           values=v.to(cuda_device), recall_type="qkv").cpu()
    assert torch.equal(got, want)


def test_recall_type_errors(cuda_device):
    q = torch.zeros(1, 4, 1, 128, dtype=torch.bfloat16, device=cuda_device)
    k = torch.zeros(1, 2, 256, 128, dtype=torch.bfloat16, device=cuda_device)
    with pytest.raises(ValueError):
        einsum_topk_func(q, k, 8, values=k, recall_type="qkv_pe")
    with pytest.raises(AssertionError):
        einsum_topk_func(q, k, 8, recall_type="qkv2")  # values missing
    with pytest.raises(AssertionError):
        einsum_topk_func(q, k, 8, values=k[:, :, :100], recall_type="qkv2")  # wrong length


def test_recall_value_rows_with_gaps(cuda_device):
    # value rows of 128 elements every 256 (a view of a wider cache): the
    # general register kernel instead of the bulk-copy ring
    q, k, v_wide, inv = _weighted_inputs(1, 8, 2, 1, 1500, torch.bfloat16, 256, seed=23)
    v = v_wide[..., :128]
    dev_v = v_wide.to(cuda_device)[..., :128]
    assert dev_v.stride(2) == 256
    idx, sc = einsum_topk_func(q.to(cuda_device), k.to(cuda_device), 40, inv_freq=inv.to(cuda_device),
                               values=dev_v, recall_type="qkv2", return_scores=True)
    torch.cuda.synchronize()
    check_parity(idx, sc, q, k, 40, inv, rel=REL_WEIGHTED, weights=orc.recall_weights(v, "qkv2"))
