"""mode="blockmax": the reference Triton kernels' block-maximum top-1 / top-4
(eval_harness/kernels/einsum_topk.py:97-161), checked against the oracle's
restatement (oracle.blockmax_topk)."""
import pytest
import torch

from oracle import reattention_topk as orc
from prism_test_b200 import einsum_topk_func
from prism_test_b200 import workloads as W


def _int_inputs(B, Hq, Hkv, Sq, Sk, seed):
    # small integers: every dot product is exact in fp32 and in the tensor-core
    # path, so the selections must match the oracle exactly, ties included
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-2, 3, (B, Hq, Sq, 128), generator=g).to(torch.bfloat16)
    k = torch.randint(-2, 3, (B, Hkv, Sk, 128), generator=g).to(torch.bfloat16)
    return q, k


@pytest.mark.gpu
@pytest.mark.parametrize("topk", [1, 4])
@pytest.mark.parametrize("shape", [(1, 8, 2, 128, 128 * 40), (2, 4, 4, 128, 256), (1, 32, 8, 128, 128 * 9)])
def test_blockmax_exact_ties(cuda_device, topk, shape):
    B, Hq, Hkv, Sq, Sk = shape
    q, k = _int_inputs(B, Hq, Hkv, Sq, Sk, seed=Sk + topk)
    want = orc.blockmax_topk(q.float(), k.float(), topk)
    got = einsum_topk_func(q.to(cuda_device), k.to(cuda_device), topk, mode="blockmax").cpu()
    assert got.dtype == torch.int32 and got.shape == want.shape
    assert torch.equal(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("topk", [1, 4])
def test_blockmax_rope_keys(cuda_device, topk):
    # RoPE'd keys are un-rotated in the scorer; near-equal block maxima may swap,
    # so each slot's oracle score must match the oracle's slot within tolerance
    B, Hq, Hkv, Sq, Sk = 1, 8, 2, 128, 128 * 24
    g = torch.Generator().manual_seed(5)
    q = torch.randn(B, Hq, Sq, 128, generator=g).to(torch.bfloat16)
    raw = torch.randn(B, Hkv, Sk, 128, generator=g)
    inv = W.rope_inv_freq(128, 5e5)
    cos, sin = orc.build_cos_sin(torch.arange(Sk), inv)
    k = orc.apply_rotary_pos_emb(raw, cos, sin).to(torch.bfloat16)
    k_raw = orc.unrotate_keys(k, inv, 0)
    want = orc.blockmax_topk(q.float(), k_raw, topk)
    got = einsum_topk_func(q.to(cuda_device), k.to(cuda_device), topk, mode="blockmax",
                           inv_freq=inv.to(cuda_device)).cpu()
    scores = orc.dense_scores(q.float(), k_raw)                # [B,Hq,Sq,Sk]
    tol = 1e-3 * q.float().norm(dim=-1, keepdim=True) * k_raw.norm(dim=-1).max()
    s_got = torch.gather(scores, -1, got.long())
    s_want = torch.gather(scores, -1, want.long())
    assert bool(((s_got - s_want).abs() <= tol).all())
    assert float((got == want).float().mean()) > 0.99


# ---- pinned to the reference kernels ------------------------------------------------
# tests/golden/blockmax_*.npz hold the outputs of the reference's own Triton kernels
# (_einsum_topk_1_kernel / _einsum_topk_4_kernel, run by Triton's interpreter on
# integer inputs, tests/golden/make_blockmax_golden.py): exact arithmetic, so the
# oracle and the CUDA path must reproduce them exactly, ties included.
from pathlib import Path  # noqa: E402

import numpy as np  # noqa: E402

BLOCKMAX_GOLDEN = sorted((Path(__file__).parent / "golden").glob("blockmax_*.npz"))


def _golden(path, dtype):
    z = np.load(path)
    q = torch.from_numpy(z["q"]).to(dtype)
    k = torch.from_numpy(z["k"]).to(dtype)
    return q, k, int(z["topk"]), torch.from_numpy(z["out"])


def test_blockmax_golden_present():
    assert len(BLOCKMAX_GOLDEN) >= 6


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("path", BLOCKMAX_GOLDEN, ids=[p.stem for p in BLOCKMAX_GOLDEN])
def test_oracle_matches_reference_kernel(path, dtype):
    q, k, topk, want = _golden(path, dtype)
    got = orc.blockmax_topk(q.float(), k.float(), topk)
    assert torch.equal(got, want)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16], ids=["fp16", "bf16"])
@pytest.mark.parametrize("path", BLOCKMAX_GOLDEN, ids=[p.stem for p in BLOCKMAX_GOLDEN])
def test_blockmax_matches_reference_kernel(cuda_device, path, dtype):
    q, k, topk, want = _golden(path, dtype)
    got = einsum_topk_func(q.to(cuda_device), k.to(cuda_device), topk, mode="blockmax").cpu()
    assert got.dtype == torch.int32 and got.shape == want.shape
    assert torch.equal(got, want)
