"""prism_topk_merge_noalloc: the merge entry point whose candidate buffers live in a
static device array instead of a caller workspace.

Callers that cannot allocate device memory (a fixed device-memory budget owned by
another allocator, or a path where cudaMalloc's implicit synchronisation is not
acceptable) use this entry point; these tests check that it returns what the
workspace merge returns.

Collected last on purpose: its GPU test must also pass after every other test has
run in the same process (and, run alone, in a fresh one).
"""
import pytest
import torch

from prism_test_b200 import _lib, topk_merge

SCRATCH_BYTES = 8 << 20
KPASS = 131072  # columns the select cluster holds in registers; longer rows are streamed


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


def _distinct_rows(rows, n, seed):
    """Scores that are distinct within each row (so torch.topk has one answer) and
    candidate indices that are a per-row permutation of 3 * column."""
    g = torch.Generator().manual_seed(seed)
    s = torch.stack([torch.randperm(n, generator=g) for _ in range(rows)]).to(torch.float32)
    s = s * (1.0 / n) - 0.5
    i = (torch.stack([torch.randperm(n, generator=g) for _ in range(rows)]) * 3).to(torch.int32)
    return s.contiguous(), i.contiguous()


def _cluster_sampled_mask(n):
    """Columns the cluster select's threshold sample reads for rows held in
    registers (white-box): 8 consecutive columns of every 128, at an offset hashed
    from the chunk number."""
    m = torch.zeros(n, dtype=torch.bool)
    for g in range((n + 127) // 128):
        s = 128 * g + 8 * (((g * 0x9E3779B1) & 0xFFFFFFFF) >> 28)
        if s + 8 <= n:
            m[s:s + 8] = True
    return m


def _sample_defeating_rows(rows, n, seed):
    """Distinct scores whose sampled columns all lie below the rest: the sampled
    threshold admits every unsampled column, far more than the 16384 candidates
    the fast path holds, so the kernel takes its exact path."""
    s, i = _distinct_rows(rows, n, seed)
    m = _cluster_sampled_mask(n)
    assert int((~m).sum()) > 16384
    s = torch.where(m[None, :], s, s + 2.0)
    return s.contiguous(), i


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


def test_noalloc_scratch_bound_of_the_test_cases():
    # the exact-path cases below fill most of the scratch without passing its limit
    assert 63 * 16384 * 8 <= SCRATCH_BYTES < 64 * 16384 * 8 + 1
    assert 8 * 16384 * 8 <= SCRATCH_BYTES


@pytest.mark.gpu
def test_noalloc_matches_workspace_merge_twice_in_a_row(cuda_device, lib):
    # Cases that write the static scratch (fewer than 64 rows, so one 4-CTA cluster
    # per row, whose CTAs exchange the row's candidates through its scratch slice):
    #   rows longer than the 131072 columns a cluster holds in registers (streamed
    #   once), 63 rows x k = 16384 (the exact path fills 63 * 16384 * 8 B, next to
    #   the 8 MiB limit), rows whose threshold sample is defeated (the fast path
    #   falls back to the exact path), and a short row set.
    # Then a case that leaves it alone: 64 rows (one CTA per row, candidates in
    # shared memory).
    torch.manual_seed(0)
    cases = []
    s, i = _distinct_rows(8, 2 * KPASS, seed=21)
    cases.append((s, i, 4096))
    s, i = _distinct_rows(63, KPASS + KPASS // 2, seed=22)
    cases.append((s, i, 16384))
    s, i = _sample_defeating_rows(8, 100000, seed=23)
    cases.append((s, i, 3000))
    s, i = _distinct_rows(5, 1000, seed=25)
    cases.append((s, i, 37))
    s, i = _distinct_rows(64, 65536, seed=24)
    cases.append((s, i, 8192))
    cases = [(s.to(cuda_device), i.to(cuda_device), k) for s, i, k in cases]

    # every case twice, one after the other on one stream and without
    # synchronising: each call after the first finds the scratch full of the
    # previous call's candidates
    got = [_noalloc(lib, s, i, k) for s, i, k in cases]
    got_again = [_noalloc(lib, s, i, k) for s, i, k in cases]
    torch.cuda.synchronize()
    for (s, i, k), (gi, gs), (gi2, gs2) in zip(cases, got, got_again):
        ri, rs = topk_merge(s, i, k)
        torch.cuda.synchronize()
        assert torch.equal(gi, ri) and torch.equal(gi2, ri)
        assert torch.equal(gs, rs) and torch.equal(gs2, rs)
        # and against torch.topk: the scores are distinct, so values and indices
        # are unique and must agree exactly
        tv, tp = s.topk(k, dim=-1)
        assert torch.equal(gs, tv)
        assert torch.equal(gi, torch.gather(i, 1, tp))
