"""prism_topk_merge_noalloc: the merge entry point whose candidate buffers live in a
static device array instead of a caller workspace.

Collected last on purpose: its GPU test must also pass after every other test has
run in the same process (and, run alone, in a fresh one).
"""
import ctypes

import pytest
import torch

from prism_test_b200 import _lib, topk_merge

SCRATCH_BYTES = 8 << 20


@pytest.fixture(scope="module")
def lib():
    from prism_test_b200 import build
    build.build()
    return _lib.load()


def _noalloc(lib, s, i, topk, stream=None):
    rows, n = s.shape
    out_idx = torch.empty((rows, topk), dtype=torch.int32, device=s.device)
    out_scores = torch.empty((rows, topk), dtype=torch.float32, device=s.device)
    if stream is None:
        stream = torch.cuda.current_stream(s.device).cuda_stream
    rc = lib.prism_topk_merge_noalloc(s.data_ptr(), i.data_ptr(), rows, n, s.stride(0), int(topk),
                                      out_idx.data_ptr(), out_scores.data_ptr(), stream)
    _lib.check(rc, "prism_topk_merge_noalloc")
    return out_idx, out_scores


def _shard_candidates(rows, shards, per_shard, seed, device):
    """Per-shard sorted top lists with global indices, as after the all-gather."""
    g = torch.Generator().manual_seed(seed)
    s = torch.randn(rows, shards, per_shard, generator=g).sort(dim=-1, descending=True).values
    base = torch.arange(shards).view(1, shards, 1) * (per_shard * 16)
    i = (base + torch.randperm(per_shard * 16, generator=g)[:per_shard].view(1, 1, per_shard)).expand(rows, -1, -1)
    return (s.reshape(rows, -1).contiguous().to(device), i.reshape(rows, -1).to(torch.int32).contiguous().to(device))


def test_noalloc_rejects_requests_beyond_the_scratch(lib):
    # rejected before any CUDA call, so no device is needed; the pointers are
    # never dereferenced
    rows, n = 65, 65536  # 65 * 16384 * 8 > 8 MiB
    rc = lib.prism_topk_merge_noalloc(16, 16, rows, n, n, 10, 16, None, None)
    assert rc == _lib.PRISM_E_WORKSPACE
    msg = _lib.last_error()
    assert "static merge scratch" in msg and str(SCRATCH_BYTES) in msg, msg
    assert lib.prism_topk_merge_noalloc(None, 16, 4, 64, 64, 10, 16, None, None) == _lib.PRISM_E_INVALID
    assert lib.prism_topk_merge_noalloc(16, 16, 4, 64, 64, 0, 16, None, None) == _lib.PRISM_E_INVALID
    assert lib.prism_topk_merge_noalloc(16, 16, 4, 64, 62, 10, 16, None, None) == _lib.PRISM_E_INVALID


@pytest.mark.gpu
def test_noalloc_matches_workspace_merge_twice_in_a_row(cuda_device, lib):
    # 8 shards x 8192 sorted candidates for 64 rows (the 1M-key sharded decode
    # merge has 32), exactly the 8 MiB scratch limit; then a small case
    big = _shard_candidates(64, 8, 8192, seed=11, device=cuda_device)
    small_s = torch.randn(5, 1000, generator=torch.Generator().manual_seed(12)).to(cuda_device)
    small_i = torch.arange(small_s.shape[1], dtype=torch.int32, device=cuda_device).expand(5, -1).contiguous()
    cases = [(big[0], big[1], 8192), (small_s, small_i, 37)]

    # two calls in a row on one stream, no synchronisation in between
    got = [_noalloc(lib, s, i, k) for s, i, k in cases]
    got_again = [_noalloc(lib, s, i, k) for s, i, k in cases]
    torch.cuda.synchronize()
    for (s, i, k), (gi, gs), (gi2, gs2) in zip(cases, got, got_again):
        ri, rs = topk_merge(s, i, k)
        torch.cuda.synchronize()
        assert torch.equal(gi, ri) and torch.equal(gi2, ri)
        assert torch.equal(gs, rs) and torch.equal(gs2, rs)
        # and against torch.topk (scores exact; index sets equal up to ties)
        ts = s.float().topk(k, dim=-1).values
        assert torch.equal(gs, ts)
