"""prism_test_b200 — B200-native (sm_100a) ReAttention recall scorer.

The hot path of Prism-Test's ReAttention method (un-rotate the RoPE'd key
cache, score q·K^T per GQA head, exact per-query top-k) as hand-written CUDA
behind a C ABI (include/prism_b200.h). ``einsum_topk_func`` has the call
signature of ``eval_harness.kernels.einsum_topk_func`` so it can be bound in
its place (``reattention._einsum_topk_func``).
"""
from .kernels import (einsum_topk_func, post_select, read_status, sparse_attention,  # noqa: F401
                      topk_merge, topk_merge_runs)
from ._lib import PrismLibraryError, lib_path, load as load_library  # noqa: F401

__all__ = [
    "einsum_topk_func",
    "topk_merge",
    "topk_merge_runs",
    "post_select",
    "sparse_attention",
    "read_status",
    "PrismLibraryError",
    "load_library",
    "lib_path",
]
