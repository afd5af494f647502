"""Generates the block-max golden vectors (``blockmax_*.npz``) by running the
REFERENCE's own Triton kernels — ``_einsum_topk_1_kernel`` and
``_einsum_topk_4_kernel`` of eval_harness/kernels/einsum_topk.py (with the 4-wide
merge of eval_harness/kernels/bitonic_merge_wrapper.py) in
RUSH-Intelligence/Prism-Test — under Triton's interpreter (``TRITON_INTERPRET=1``),
which executes the kernel source program by program on the CPU.

The launcher ``einsum_topk_func`` (einsum_topk.py:164-225) asserts CUDA tensors,
so the kernels are launched here the way it launches them: the same grid
``(num_heads, seqlen_q / 128, batch)``, the same strides and the same head ratio.

Queries and keys hold small integers, so every dot product is an exact integer
in fp32 whatever the summation order or TF32 mode: the outputs are the ones the
compiled kernel produces on a GPU, ties included (many block maxima are equal,
which exercises the ``>=`` rule of the top-1 kernel and the strict ``>`` plus the
2-stage merge of the top-4 kernel, and the first-index rule of the row maximum
inside a block). The kernels run on fp16 inputs: the interpreter has no exact
bf16 arithmetic (numpy has no bf16 type; its bf16 dot products here disagree with
exact arithmetic), while the small integers are exact in fp16 and bf16 alike, so
the stored outputs hold for both dtypes (the tests run both).

Run (needs a checkout of the reference and triton; no GPU):
    python tests/golden/make_blockmax_golden.py --reference PATH
"""
from __future__ import annotations

import argparse
import os
import sys
import zlib
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"  # before triton is imported

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent

# name, B, Hq, Hkv, Sq, Sk, topk, value range (integers in [-r, r]), special
CASES = [
    ("blockmax_top1_gqa", 1, 4, 2, 128, 1024, 1, 2, None),
    ("blockmax_top4_gqa", 1, 4, 2, 256, 1024, 4, 2, None),
    ("blockmax_top4_batch", 2, 2, 1, 128, 640, 4, 3, None),
    ("blockmax_top1_mha", 1, 2, 2, 384, 512, 1, 1, None),
    ("blockmax_top4_tied_blocks", 1, 2, 1, 128, 768, 4, 1, "tied"),
    ("blockmax_top1_tied_blocks", 1, 2, 1, 128, 768, 1, 1, "tied"),
]


def make_inputs(B, Hq, Hkv, Sq, Sk, vrange, special, seed):
    g = torch.Generator().manual_seed(seed)
    q = torch.randint(-vrange, vrange + 1, (B, Hq, Sq, 128), generator=g, dtype=torch.int8)
    k = torch.randint(-vrange, vrange + 1, (B, Hkv, Sk, 128), generator=g, dtype=torch.int8)
    if special == "tied":
        # every 128-key block is a copy of the first one: all block maxima tie
        k = k[:, :, :128].repeat(1, 1, Sk // 128, 1).contiguous()
    return q, k


def run_reference(et, triton, q8, k8, topk):
    q = q8.to(torch.float16)
    k = k8.to(torch.float16)
    B, Hq, Sq, _ = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    o = torch.empty((B, Hq, Sq, topk), dtype=torch.int32)
    grid = lambda META: (Hq, triton.cdiv(Sq, META["BLOCK_M"]), B)  # noqa: E731
    args = (q, k, o, q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
            o.stride(0), o.stride(1), o.stride(2), Hq // Hkv, Sk)
    if topk == 1:
        et._einsum_topk_1_kernel[grid](*args, BLOCK_HEADDIM=128)
    else:
        et._einsum_topk_4_kernel[grid](*args)
    return o


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PRISM_REFERENCE"),
                    help="root of a RUSH-Intelligence/Prism-Test checkout (or set PRISM_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference PATH or PRISM_REFERENCE")
    sys.path.insert(0, args.reference)
    import triton  # noqa: E402
    from eval_harness.kernels import einsum_topk as et  # noqa: E402

    for (name, B, Hq, Hkv, Sq, Sk, topk, vrange, special) in CASES:
        q8, k8 = make_inputs(B, Hq, Hkv, Sq, Sk, vrange, special, zlib.crc32(name.encode()))
        out = run_reference(et, triton, q8, k8, topk)
        np.savez_compressed(HERE / f"{name}.npz", q=q8.numpy(), k=k8.numpy(), out=out.numpy(),
                            topk=np.array(topk))
        print(f"{name}: q {tuple(q8.shape)}, k {tuple(k8.shape)}, topk {topk}")


if __name__ == "__main__":
    main()
