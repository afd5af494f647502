"""Host-side behaviour of the drop-in ``einsum_topk_func`` that needs no GPU:
the reference launcher's argument assertions (eval_harness/kernels/
einsum_topk.py:182-195) and the extension arguments' checks."""
import pytest
import torch

from prism_test_b200 import einsum_topk_func


def _qk(**kw):
    q = torch.randn(kw.get("B", 1), kw.get("Hq", 4), kw.get("Sq", 128), kw.get("D", 128), dtype=kw.get("dq", torch.bfloat16))
    k = torch.randn(kw.get("Bk", 1), kw.get("Hkv", 2), kw.get("Sk", 256), kw.get("Dk", 128), dtype=kw.get("dk", torch.bfloat16))
    return q, k


def test_cpu_tensors_rejected_like_reference():
    q, k = _qk()
    with pytest.raises(AssertionError, match="gpu"):
        einsum_topk_func(q, k, 4)


def test_head_divisibility():
    q, k = _qk(Hq=6, Hkv=4)
    with pytest.raises(AssertionError, match="divisible"):
        einsum_topk_func(q, k, 4)


def test_batch_and_dim_mismatch():
    q, k = _qk(Bk=2)
    with pytest.raises(AssertionError, match="must match"):
        einsum_topk_func(q, k, 4)
    q, k = _qk(Dk=64)
    with pytest.raises(AssertionError):
        einsum_topk_func(q, k, 4)


def test_dtype_rules():
    q, k = _qk(dq=torch.float32, dk=torch.float32)
    with pytest.raises(AssertionError, match="fp16 and bf16"):
        einsum_topk_func(q, k, 4)
    q, k = _qk(dq=torch.float16)
    with pytest.raises(AssertionError, match="same type"):
        einsum_topk_func(q, k, 4)


def test_inner_stride():
    q, k = _qk()
    with pytest.raises(AssertionError):
        einsum_topk_func(q.transpose(2, 3), k, 4)


def test_unknown_mode():
    q, k = _qk()
    with pytest.raises(AssertionError):
        einsum_topk_func(q, k, 4, mode="approx")
