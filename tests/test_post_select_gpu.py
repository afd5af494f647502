"""Device post-selection (prism_post_select) against the reference's
_global_unique + _expand_spans (golden vectors made by the reference itself) and
against the oracle on random inputs."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reattention_topk as orc
from prism_test_b200 import einsum_topk_func, post_select
from prism_test_b200 import workloads as W

pytestmark = pytest.mark.gpu
POST = sorted((Path(__file__).resolve().parent / "golden").glob("post_*.npz"))


@pytest.mark.parametrize("path", POST, ids=[p.stem for p in POST])
def test_post_select_golden(path, cuda_device):
    z = np.load(path)
    idx = torch.from_numpy(z["idx"]).to(cuda_device)
    got = post_select(idx, int(z["n_mid"]), int(z["recall_clip"]), int(z["span"]), str(z["mode"]))
    assert torch.equal(got.cpu(), torch.from_numpy(z["out"]))


@pytest.mark.parametrize("n_mid,span,mode", [(1, 0, "centered"), (1, 3, "floor"), (777, 1, "centered"),
                                             (100000, 16, "centered"), (3000, 0, "floor"), (50, 101, "floor")])
def test_post_select_random(n_mid, span, mode, cuda_device):
    g = torch.Generator().manual_seed(n_mid + span)
    idx = torch.randint(0, n_mid, (4, 8, 1, 32), generator=g)
    got = post_select(idx.to(cuda_device), n_mid, -1, span, mode)
    want = orc.expand_spans(orc.global_unique(idx, -1), n_mid, span, mode)
    assert torch.equal(got.cpu(), want)


def test_post_select_clip_bounds(cuda_device):
    # recall_clip at or above the number of unique picks keeps them all; 0 keeps none
    idx = torch.tensor([5, 5, 9, 100, 9, 5], dtype=torch.int64)
    for clip, want in [(3, [5, 9, 100]), (50, [5, 9, 100]), (0, [])]:
        got = post_select(idx.to(cuda_device), 200, clip, 0, "centered")
        assert got.cpu().tolist() == want
    # clip 2 keeps the two most frequent (5 x3, 9 x2) — no tie at the cut
    assert post_select(idx.to(cuda_device), 200, 2, 0, "centered").cpu().tolist() == [5, 9]


def test_post_select_after_scorer(cuda_device):
    # the op's own top-k feeds the post-selection, as in ReAttentionMethod
    wl = W.small(W.WORKLOADS["decode-128k"], Sk=20000, topk=256)
    x = W.make_inputs(wl, cuda_device)
    idx = einsum_topk_func(x["q"], x["k"], wl.topk, inv_freq=x["inv_freq"])
    got = post_select(idx, wl.Sk, -1, 32, "centered")
    want = orc.expand_spans(orc.global_unique(idx.long().cpu(), -1), wl.Sk, 32, "centered")
    assert torch.equal(got.cpu(), want)
