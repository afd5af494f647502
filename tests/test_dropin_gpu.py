"""The library as a drop-in for the reference's recall kernel, replayed from the
reference's own caller.

tests/golden/dropin_*.npz record how ``ReAttentionMethod._select_topk`` /
``_kernel_topk`` (eval_harness/attention_methods/reattention.py:398-418, 460-484)
call the module attribute ``_einsum_topk_func(q, k, topk)``: bf16 queries
zero-padded to a multiple of 128 rows and made contiguous, the middle key slice,
``topk = mid_size`` (1, 4 and 64 here, query lengths 1, 50 and 130), and what
``_select_topk`` returned when that call answered with the dense top-k
(tests/golden/make_dropin_golden.py). The reference cannot be imported where the
GPU tests run, so the GPU test replays the recorded call through
``prism_test_b200.einsum_topk_func`` with the same positional arguments, applies
the caller's slice-back (``[:, :, :q_len].long()``), and checks the kernel
contract and the selection.
"""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reattention_topk as orc
from prism_test_b200 import einsum_topk_func
from tests.parity import check_parity

CASES = sorted((Path(__file__).parent / "golden").glob("dropin_*.npz"))


def _load(path):
    z = np.load(path)
    B, Hq, Hkv, q_len, n_middle, mid_size, seed = (int(v) for v in z["shape"])
    g = torch.Generator().manual_seed(seed)
    raw_q = torch.randn(B, Hq, q_len, 128, generator=g)
    k_mid = torch.randn(B, Hkv, n_middle, 128, generator=g).to(torch.bfloat16)
    return z, raw_q, k_mid, q_len, mid_size


def _recorded_call(z, raw_q, k_mid, q_len):
    """The (q, k, topk) the reference's _kernel_topk passed to the kernel."""
    q = torch.zeros(tuple(int(v) for v in z["call_q_shape"]), dtype=torch.bfloat16)
    q[:, :, :q_len] = raw_q.to(torch.bfloat16)
    k = k_mid.contiguous()
    assert tuple(q.stride()) == tuple(int(v) for v in z["call_q_strides"])
    assert tuple(k.shape) == tuple(int(v) for v in z["call_k_shape"])
    assert tuple(k.stride()) == tuple(int(v) for v in z["call_k_strides"])
    return q, k, int(z["call_topk"])


def test_dropin_cases_present():
    assert len(CASES) >= 3


@pytest.mark.parametrize("path", CASES, ids=[p.stem for p in CASES])
def test_recorded_call_matches_the_caller_contract(path):
    z, raw_q, k_mid, q_len, mid_size = _load(path)
    q, k, topk = _recorded_call(z, raw_q, k_mid, q_len)
    # the recorder saw bf16, contiguous q and k, zero padding, the caller's own rows
    assert list(z["call_dtypes"]) == ["torch.bfloat16", "torch.bfloat16"]
    assert all(bool(f) for f in z["call_flags"])
    assert q.shape[2] % 128 == 0 and q.shape[2] >= q_len and topk == mid_size
    assert str(z["selected_dtype"]) == "torch.int64"
    # with a dense kernel the caller returns _dense_topk's selection, and the
    # oracle's dense top-k agrees with both (same fp32 einsum + topk)
    sel = torch.from_numpy(z["selected"]).long()
    dense = torch.from_numpy(z["dense"]).long()
    assert torch.equal(sel, dense)
    _, oi = orc.dense_topk(raw_q.to(torch.bfloat16), k_mid, topk)
    assert torch.equal(oi, dense)


@pytest.mark.gpu
@pytest.mark.parametrize("path", CASES, ids=[p.stem for p in CASES])
def test_dropin_replays_the_reference_caller(cuda_device, path):
    z, raw_q, k_mid, q_len, mid_size = _load(path)
    q, k, topk = _recorded_call(z, raw_q, k_mid, q_len)
    out = einsum_topk_func(q.to(cuda_device), k.to(cuda_device), topk)  # the reference's call
    torch.cuda.synchronize()
    # the kernel contract the caller relies on
    assert out.dtype == torch.int32 and out.device == q.to(cuda_device).device
    assert tuple(out.shape) == (q.shape[0], q.shape[1], q.shape[2], topk)
    # the caller's slice-back
    got = out[:, :, :q_len].long().cpu()
    want = torch.from_numpy(z["selected"]).long()
    assert got.shape == want.shape
    # the selection: the parity rules against the oracle (exact up to near-ties)
    # and, with these inputs, the reference caller's own answer
    st = check_parity(got.to(torch.int32), None, raw_q.to(torch.bfloat16), k_mid, topk)
    if st["swapped"] == 0:  # no near-tie at the k-th score moved a key
        assert torch.equal(got.sort(-1).values, want.sort(-1).values)
    # the zero-padded rows still hold distinct in-range indices
    pad = out[:, :, q_len:].long().cpu()
    if pad.numel():
        assert int(pad.min()) >= 0 and int(pad.max()) < k.shape[2]
        s = pad.sort(-1).values
        assert bool((s[..., 1:] != s[..., :-1]).all())
