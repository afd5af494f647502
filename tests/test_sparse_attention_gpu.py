"""Attention over the selected view (prism_sparse_attention) against the
reference's gather + RoPE + _attend (reattention_exact.py:453-508, 650-661) as
pinned by tests/golden/attn_*.npz, and against the oracle on random views."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reattention_topk as orc
from prism_test_b200 import sparse_attention
from prism_test_b200 import kernels, workloads as W

pytestmark = pytest.mark.gpu

ATTN = sorted((Path(__file__).resolve().parent / "golden").glob("attn_*.npz"))
# the output is rounded to bf16/fp16 (2^-8 / 2^-11 relative); fp32 softmax inside
RTOL, ATOL = 8e-3, 2e-3


def _close(got, want):
    torch.testing.assert_close(got.float().cpu(), want.float(), rtol=RTOL, atol=ATOL)


@pytest.mark.parametrize("path", ATTN, ids=[p.stem for p in ATTN])
def test_sparse_attention_golden(path, cuda_device, monkeypatch):
    monkeypatch.setattr(kernels, "_SYNC_CHECK", True)
    z = np.load(path)
    t = lambda key: torch.from_numpy(z[key].view(np.int16)).view(torch.bfloat16).to(cuda_device)  # noqa: E731
    out = sparse_attention(t("q_bf16"), t("k_bf16"), t("v_bf16"), torch.from_numpy(z["key_pos"]),
                           q_pos=torch.from_numpy(z["q_pos"]), inv_freq=torch.from_numpy(z["inv_freq"]),
                           pe_original=bool(z["pe_original"]), scale=float(z["scale"]))
    torch.cuda.synchronize()
    _close(out, torch.from_numpy(z["out"]))


CASES = [
    # B, Hq, Hkv, Sq, S, nsel, dtype, pe_original, rope
    (1, 32, 8, 1, 131072, 4640, torch.bfloat16, True, True),    # decode: 32 + 128*4 + 4096 view
    (1, 32, 8, 1, 131072, 4640, torch.bfloat16, False, True),   # contiguous re-rotation
    (2, 8, 2, 7, 5000, 900, torch.float16, True, True),         # a small chunk, fp16, B = 2
    (1, 28, 4, 3, 20000, 3000, torch.bfloat16, False, False),   # no RoPE, G = 7
    (1, 4, 4, 1, 100, 1, torch.bfloat16, True, True),           # a one-key view
]


@pytest.mark.parametrize("B,Hq,Hkv,Sq,S,nsel,dtype,pe_original,rope", CASES)
def test_sparse_attention_random(B, Hq, Hkv, Sq, S, nsel, dtype, pe_original, rope, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(S + nsel)
    q = torch.randn(B, Hq, Sq, 128, generator=g, device=cuda_device).to(dtype)
    k = torch.randn(B, Hkv, S, 128, generator=g, device=cuda_device).to(dtype)
    v = torch.randn(B, Hkv, S, 128, generator=g, device=cuda_device).to(dtype)
    # a view: the first keys, a sorted random middle, the tail holding the queries
    tail = min(S, max(Sq, nsel // 4))
    mid = torch.randperm(S - tail, generator=g, device=cuda_device)[: nsel - tail].sort().values
    key_pos = torch.cat([mid, torch.arange(S - tail, S, device=cuda_device)])[:nsel]
    inv = W.rope_inv_freq(128, 5e5) if rope else None
    out = sparse_attention(q, k, v, key_pos, inv_freq=inv, pe_original=pe_original)
    torch.cuda.synchronize()
    q_pos = torch.arange(S - Sq, S)
    want = orc.sparse_attention(q, k, v, key_pos, q_pos, inv, pe_original, 128 ** -0.5)
    _close(out, want)


def test_sparse_attention_out_of_range_position_is_reported(cuda_device):
    q = torch.randn(1, 4, 1, 128, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(1, 2, 64, 128, device=cuda_device).to(torch.bfloat16)
    key_pos = torch.tensor([0, 5, 64], device=cuda_device)  # 64 is past the cache
    with pytest.raises(kernels._lib.PrismLibraryError):
        kernels._SYNC_CHECK, old = True, kernels._SYNC_CHECK
        try:
            sparse_attention(q, k, k, key_pos)
        finally:
            kernels._SYNC_CHECK = old
