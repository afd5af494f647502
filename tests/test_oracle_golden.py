"""The CPU oracle against golden vectors produced by the reference's own code
(tests/golden/make_golden.py)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reattention_topk as orc

GOLDEN = sorted(p for p in (Path(__file__).parent / "golden").glob("*.npz")
                if not p.stem.startswith(("post_", "recall_", "attn_", "blockmax_", "dropin_")))


def load_case(path):
    z = np.load(path)
    q = torch.from_numpy(z["q_bf16"].view(np.int16)).view(torch.bfloat16)
    k = torch.from_numpy(z["k_bf16"].view(np.int16)).view(torch.bfloat16)
    inv = torch.from_numpy(z["inv_freq"]) if bool(z["rope"]) else None
    causal = int(z["causal_offset"])
    return dict(q=q, k=k, inv_freq=inv, pos_offset=int(z["pos_offset"]),
                causal_offset=None if causal < 0 else causal, topk=int(z["topk"]),
                idx=torch.from_numpy(z["idx"]), scores=torch.from_numpy(z["scores"]),
                raw=torch.from_numpy(z["raw_keys_ref"]))


def test_golden_present():
    assert len(GOLDEN) >= 8


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_oracle_matches_reference_golden(path):
    c = load_case(path)
    vals, idx = orc.dense_topk(c["q"], c["k"], c["topk"], c["inv_freq"], c["pos_offset"], c["causal_offset"])
    # same torch ops on the same inputs: bit-identical scores
    assert torch.equal(vals, c["scores"])
    if path.stem == "ties_equal_keys":
        # all scores equal: topk order is unspecified, the values are what matter
        assert torch.equal(vals, c["scores"])
    else:
        assert torch.equal(idx, c["idx"])


def test_oracle_unrotation_matches_reference():
    c = load_case(Path(__file__).parent / "golden" / "causal_chunk.npz")
    raw = orc.unrotate_keys(c["k"], c["inv_freq"], c["pos_offset"])
    assert torch.equal(raw, c["raw"])


def test_rope_apply_then_undo_is_identity():
    # mirrors the reference's test_apply_then_undo_is_identity (test_prefill_methods.py:131)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(1, 2, 16, 32, generator=g)
    inv = torch.randn(16, generator=g).abs() * 0.01
    cos, sin = orc.build_cos_sin(torch.arange(16), inv)
    back = orc.undo_rotary_pos_emb(orc.apply_rotary_pos_emb(x, cos, sin), cos, sin)
    torch.testing.assert_close(back, x, atol=1e-5, rtol=1e-5)


def test_rotate_half_values():
    y = orc.rotate_half(torch.tensor([1.0, 2.0, 3.0, 4.0]))
    assert torch.equal(y, torch.tensor([-3.0, -4.0, 1.0, 2.0]))


def test_selection_is_position_agnostic():
    # un-rotating keys rotated at any offset recovers the same selection
    g = torch.Generator().manual_seed(1)
    q = torch.randn(1, 4, 1, 128, generator=g)
    raw = torch.randn(1, 2, 300, 128, generator=g)
    inv = 1.0 / (5e5 ** (torch.arange(0, 128, 2).float() / 128))
    base = orc.dense_topk(q, raw, 10)[1]
    for off in (0, 777, 100000):
        cos, sin = orc.build_cos_sin(torch.arange(off, off + 300), inv)
        rot = orc.apply_rotary_pos_emb(raw, cos, sin)
        assert torch.equal(orc.dense_topk(q, rot, 10, inv, off)[1], base)


def test_blockmax_top1_and_top4_semantics():
    # hand-built scores: block maxima and tie rules of the Triton kernel
    q = torch.zeros(1, 1, 1, 128)
    q[..., 0] = 1.0
    k = torch.zeros(1, 1, 512, 128)
    vals = {5: 3.0, 130: 7.0, 131: 7.0, 300: 5.0, 450: 7.0, 451: 1.0}
    for p, v in vals.items():
        k[0, 0, p, 0] = v
    top1 = orc.blockmax_topk(q, k, 1)
    assert top1.flatten().tolist() == [450]  # later block wins the tie (>=)
    top4 = orc.blockmax_topk(q, k, 4)
    # block maxima: blk0 3.0@5, blk1 7.0@130 (first index), blk2 5.0@300, blk3 7.0@450
    # strict > insertion keeps the earlier 7.0 ahead; the merge keeps tie order
    assert top4.flatten().tolist() == [130, 450, 300, 5]


POST = sorted((Path(__file__).resolve().parent / "golden").glob("post_*.npz"))


@pytest.mark.parametrize("path", POST, ids=[p.stem for p in POST])
def test_post_select_oracle_matches_reference(path):
    z = np.load(path)
    idx = torch.from_numpy(z["idx"])
    sel = orc.global_unique(idx, int(z["recall_clip"]))
    out = orc.expand_spans(sel, int(z["n_mid"]), int(z["span"]), str(z["mode"]))
    assert torch.equal(out, torch.from_numpy(z["out"]))


RECALL = sorted((Path(__file__).resolve().parent / "golden").glob("recall_*.npz"))


def test_recall_golden_present():
    assert len(RECALL) >= 3


@pytest.mark.parametrize("path", RECALL, ids=[p.stem for p in RECALL])
def test_recall_weight_oracle_matches_reference(path):
    """orc.recall_weights + dense_topk against ReAttentionMethod._apply_recall_weight
    + _dense_topk (reattention.py:822-842, 486-498): bit-identical."""
    z = np.load(path)
    c = load_case(path)
    v = torch.from_numpy(z["v_bf16"].view(np.int16)).view(torch.bfloat16)
    w = orc.recall_weights(v, str(z["recall_type"]))
    vals, idx = orc.dense_topk(c["q"], c["k"], c["topk"], c["inv_freq"], c["pos_offset"], weights=w)
    assert torch.equal(vals, c["scores"])
    assert torch.equal(idx, c["idx"])


def test_recall_weights_types():
    v = torch.tensor([[[[3.0, -4.0], [0.0, 0.0]]]]).to(torch.bfloat16)
    assert orc.recall_weights(v, "qk") is None
    assert orc.recall_weights(v, "qkv").tolist() == [[[7.0, 0.0]]]
    assert orc.recall_weights(v, "qkv2").tolist() == [[[5.0, 0.0]]]
    with pytest.raises(ValueError):
        orc.recall_weights(v, "qkv_pe")


ATTN = sorted((Path(__file__).resolve().parent / "golden").glob("attn_*.npz"))


def _attn_case(path):
    z = np.load(path)
    t = lambda key: torch.from_numpy(z[key].view(np.int16)).view(torch.bfloat16)  # noqa: E731
    return (t("q_bf16"), t("k_bf16"), t("v_bf16"), torch.from_numpy(z["key_pos"]),
            torch.from_numpy(z["q_pos"]), torch.from_numpy(z["inv_freq"]), bool(z["pe_original"]),
            float(z["scale"]), torch.from_numpy(z["out"]))


def test_attn_golden_present():
    assert len(ATTN) >= 3


@pytest.mark.parametrize("path", ATTN, ids=[p.stem for p in ATTN])
def test_sparse_attention_oracle_matches_reference(path):
    """orc.sparse_attention against the reference's gather + RoPE + _attend eager path
    (reattention_exact.py:453-508, 650-661)."""
    q, k, v, kp, qp, inv, pe_orig, scale, want = _attn_case(path)
    got = orc.sparse_attention(q, k, v, kp, qp, inv, pe_orig, scale)
    torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-6)
    if "rows_without_keys" in path.stem:
        assert bool((got[:, :, 0] == 0).all())  # the first query row sees no key
