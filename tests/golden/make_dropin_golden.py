"""Generates ``dropin_*.npz``: how the reference's ReAttention method calls its
recall kernel, recorded by running the REFERENCE's own caller
(RUSH-Intelligence/Prism-Test, eval_harness/attention_methods/reattention.py):

* ``ReAttentionMethod._select_topk`` (:398-418), with the kernel gate
  ``_should_use_kernel`` (:420-458) forced open (the gate wants CUDA tensors; the
  reference's own tests open it the same way), which calls
* ``ReAttentionMethod._kernel_topk`` (:460-484): cast to bf16, zero-pad the query
  rows to a multiple of 128, ``.contiguous()``, call the module attribute
  ``_einsum_topk_func(q, k, topk)``, slice the rows back and ``.long()``.

The module attribute is bound to a recorder that keeps every argument it receives
and answers with the dense top-k of those very arguments (fp32 einsum +
``torch.topk``, the reference's own ``_dense_topk`` semantics, int32) — the kernel
contract the reference's tests use. Saved per case: the seed and shapes that
regenerate the inputs (torch CPU generator), what the kernel was called with
(shape, dtype, strides, contiguity, the padded rows being zero) and what
``_select_topk`` returned with that kernel, next to ``_dense_topk``'s answer.

The GPU test (tests/test_dropin_gpu.py) replays the recorded call through
``prism_test_b200.einsum_topk_func`` and applies the same slice-back.

Run (needs a checkout of the reference; no GPU):
    python tests/golden/make_dropin_golden.py --reference PATH
"""
from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# name, B, Hq, Hkv, q_len, n_middle, mid_size, seed
CASES = [
    ("dropin_decode_mid4", 1, 8, 2, 1, 1024, 4, 101),
    ("dropin_chunk50_mid64", 1, 4, 2, 50, 512, 64, 102),
    ("dropin_chunk130_mid1", 2, 4, 4, 130, 384, 1, 103),
]


def make_inputs(B, Hq, Hkv, q_len, n_middle, seed):
    """The caller's raw queries (fp32, as the method holds them) and the middle
    slice of the un-rotated key cache, regenerated from the seed."""
    g = torch.Generator().manual_seed(seed)
    raw_q = torch.randn(B, Hq, q_len, 128, generator=g)
    recall_k_mid = torch.randn(B, Hkv, n_middle, 128, generator=g).to(torch.bfloat16)
    return raw_q, recall_k_mid


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PRISM_REFERENCE"),
                    help="root of a RUSH-Intelligence/Prism-Test checkout (or set PRISM_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference PATH or PRISM_REFERENCE")
    sys.path.insert(0, args.reference)
    from unittest.mock import patch

    from eval_harness.attention_methods import reattention as reatt_mod  # noqa: E402
    from eval_harness.attention_methods.reattention import ReAttentionMethod  # noqa: E402

    for (name, B, Hq, Hkv, q_len, n_middle, mid_size, seed) in CASES:
        raw_q, recall_k_mid = make_inputs(B, Hq, Hkv, q_len, n_middle, seed)
        calls = []

        def recorder(q, k, topk):
            calls.append(dict(q_shape=tuple(q.shape), q_dtype=str(q.dtype), q_strides=q.stride(),
                              q_contig=q.is_contiguous(), k_shape=tuple(k.shape), k_dtype=str(k.dtype),
                              k_strides=k.stride(), k_contig=k.is_contiguous(), topk=topk,
                              pad_zero=bool((q[:, :, q_len:] == 0).all()),
                              q_rows_equal=bool(torch.equal(q[:, :, :q_len], raw_q.to(q.dtype))),
                              k_equal=bool(torch.equal(k, recall_k_mid.to(k.dtype)))))
            n_rep = q.shape[1] // k.shape[1]
            kk = k.repeat_interleave(n_rep, dim=1)
            scores = torch.einsum("bhqd,bhmd->bhqm", q.float(), kk.float())
            return scores.topk(topk, dim=-1).indices.to(torch.int32)

        m = ReAttentionMethod(mid_size=mid_size, use_triton_kernel="force")
        with patch.object(reatt_mod, "_einsum_topk_func", recorder), \
                patch.object(ReAttentionMethod, "_should_use_kernel", lambda self, q, k, n: True):
            selected = m._select_topk(raw_q, recall_k_mid, n_middle)
        dense = m._dense_topk(raw_q.to(torch.bfloat16), recall_k_mid, n_middle)
        assert len(calls) == 1, calls
        c = calls[0]
        np.savez_compressed(
            HERE / f"{name}.npz", shape=np.array([B, Hq, Hkv, q_len, n_middle, mid_size, seed]),
            call_q_shape=np.array(c["q_shape"]), call_q_strides=np.array(c["q_strides"]),
            call_k_shape=np.array(c["k_shape"]), call_k_strides=np.array(c["k_strides"]),
            call_dtypes=np.array([c["q_dtype"], c["k_dtype"]]), call_topk=np.array(c["topk"]),
            call_flags=np.array([c["q_contig"], c["k_contig"], c["pad_zero"], c["q_rows_equal"], c["k_equal"]]),
            selected=selected.to(torch.int32).numpy(), selected_dtype=np.array(str(selected.dtype)),
            dense=dense.to(torch.int32).numpy())
        print(f"{name}: kernel called with q {c['q_shape']} {c['q_dtype']}, k {c['k_shape']}, "
              f"topk {c['topk']}; _select_topk -> {tuple(selected.shape)} {selected.dtype}")


if __name__ == "__main__":
    main()
