"""Generates the golden vectors in this directory by running the REFERENCE's own
code (RUSH-Intelligence/Prism-Test, imported read-only from a checkout whose root
is given by --reference or the PRISM_REFERENCE environment variable):

    eval_harness/attention_methods/_method_base.py  build_cos_sin,
        apply_rotary_pos_emb, undo_rotary_pos_emb
    eval_harness/attention_methods/reattention.py   ReAttentionMethod._dense_topk,
        ReAttentionMethod._global_unique, ReAttentionMethod._expand_spans,
        ReAttentionMethod._apply_recall_weight
    eval_harness/attention_methods/reattention_exact.py  ReAttentionExactMethod._attend

For each case it draws seeded raw keys and queries, rotates the keys with the
reference's RoPE (fp32), stores them as bf16 (the dtype the GPU path reads),
un-rotates the bf16 keys in fp32 with ``undo_rotary_pos_emb`` and selects with
``_dense_topk``. Output: one .npz per case with the inputs (bf16 as uint16
bits), inv_freq, and the reference's top-k indices and scores.

The checkout is not needed to *use* the vectors; only to regenerate them:
    python tests/golden/make_golden.py --reference PATH
"""
from __future__ import annotations

import argparse
import os
import sys
import zlib
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent

# name, B, Hq, Hkv, Sq, Sk, topk, theta, pos_offset, rope, causal_offset, special
CASES = [
    ("gqa_decode", 1, 8, 2, 1, 1000, 37, 5e5, 0, True, None, None),
    ("mha_multirow_offset", 2, 4, 4, 3, 700, 64, 1e4, 5000, True, None, None),
    ("raw_keys_k_equals_n", 1, 6, 3, 2, 513, 513, 5e5, 0, False, None, None),
    ("causal_chunk", 1, 4, 2, 5, 300, 20, 5e5, 0, True, 295, None),
    ("top1", 1, 4, 1, 2, 384, 1, 5e5, 100, True, None, None),
    ("ties_equal_keys", 1, 4, 2, 1, 256, 10, 5e5, 0, False, None, "ties"),
    ("large_positions", 1, 4, 2, 1, 512, 16, 5e5, 1048000, True, None, None),
    ("outliers_planted", 1, 8, 2, 1, 1536, 128, 1e6, 0, True, None, "planted"),
]


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("PRISM_REFERENCE"),
                    help="root of a RUSH-Intelligence/Prism-Test checkout (or set PRISM_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give the reference checkout with --reference PATH or PRISM_REFERENCE")
    sys.path.insert(0, args.reference)
    from eval_harness.attention_methods._method_base import (  # noqa: E402
        apply_rotary_pos_emb, build_cos_sin, undo_rotary_pos_emb)
    from eval_harness.attention_methods.reattention import ReAttentionMethod  # noqa: E402

    for (name, B, Hq, Hkv, Sq, Sk, topk, theta, pos_offset, rope, causal, special) in CASES:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        D = 128
        q = torch.randn(B, Hq, Sq, D, generator=g).to(torch.bfloat16)
        k_raw = torch.randn(B, Hkv, Sk, D, generator=g)
        if special == "ties":
            k_raw[:, :, :] = k_raw[:, :, :1]  # every key equal -> all scores tie
        if special == "planted":
            k_raw[..., 3] *= 8.0
            k_raw[..., 77] *= 8.0
            for h in range(Hq):
                pos = torch.randperm(Sk, generator=g)[:4]
                qv = q[0, h, 0].float()
                qn = qv / qv.norm()
                for p in pos.tolist():
                    kv = h // (Hq // Hkv)
                    n = k_raw[0, kv, p]
                    k_raw[0, kv, p] = 6.0 * qn * 11.3 + (n - (n @ qn) * qn)
        inv_freq = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).to(torch.float32) / D))
        if rope:
            pos = torch.arange(pos_offset, pos_offset + Sk)
            cos, sin = build_cos_sin(pos, inv_freq, torch.device("cpu"), torch.float32)
            k_cached = apply_rotary_pos_emb(k_raw, cos, sin).to(torch.bfloat16)
            raw_ref = undo_rotary_pos_emb(k_cached.float(), cos, sin)
        else:
            k_cached = k_raw.to(torch.bfloat16)
            raw_ref = k_cached.float()

        method = ReAttentionMethod(mid_size=topk, use_triton_kernel="off")
        if causal is None:
            idx = method._dense_topk(q.float(), raw_ref, Sk)
            n_rep = Hq // Hkv
            rk = raw_ref[:, :, None].expand(B, Hkv, n_rep, Sk, D).reshape(B, Hq, Sk, D)
            full = torch.einsum("bhqd,bhmd->bhqm", q.float(), rk.float())
        else:
            # the dense einsum of _dense_topk with the causal mask applied before topk
            n_rep = Hq // Hkv
            rk = raw_ref[:, :, None].expand(B, Hkv, n_rep, Sk, D).reshape(B, Hq, Sk, D)
            full = torch.einsum("bhqd,bhmd->bhqm", q.float(), rk.float())
            j = torch.arange(Sk)[None, :]
            i = torch.arange(Sq)[:, None]
            full = full.masked_fill(j > causal + i, float("-inf"))
            _, idx = full.topk(topk, dim=-1)
        vals = torch.gather(full, -1, idx)
        np.savez_compressed(
            HERE / f"{name}.npz",
            q_bf16=bf16_bits(q), k_bf16=bf16_bits(k_cached), inv_freq=inv_freq.numpy(),
            rope=np.array(rope), pos_offset=np.array(pos_offset),
            causal_offset=np.array(-1 if causal is None else causal),
            topk=np.array(topk), idx=idx.numpy().astype(np.int64), scores=vals.numpy(),
            raw_keys_ref=raw_ref.numpy() if name == "causal_chunk" else np.zeros(0, np.float32),
        )
        print(name, tuple(q.shape), tuple(k_cached.shape), "topk", topk)
    post_select_cases(ReAttentionMethod)
    recall_weight_cases(ReAttentionMethod, apply_rotary_pos_emb, build_cos_sin, undo_rotary_pos_emb)
    from eval_harness.attention_methods.reattention_exact import ReAttentionExactMethod  # noqa: E402
    sparse_attention_cases(ReAttentionExactMethod, apply_rotary_pos_emb, build_cos_sin)


# value-weighted recall cases: name, recall_type, B, Hq, Hkv, Sq, Sk, topk, theta, pos_offset, zero_rows
RECALL_CASES = [
    ("recall_qkv_gqa_decode", "qkv", 1, 8, 2, 1, 1000, 37, 5e5, 0, 0.0),
    ("recall_qkv2_multirow", "qkv2", 2, 4, 4, 3, 700, 64, 1e4, 5000, 0.0),
    ("recall_qkv2_zero_values", "qkv2", 1, 4, 2, 2, 640, 20, 5e5, 100, 0.05),
]


def recall_weight_cases(ReAttentionMethod, apply_rotary_pos_emb, build_cos_sin, undo_rotary_pos_emb) -> None:
    """Golden vectors of the value-weighted recall: ReAttentionMethod.
    _apply_recall_weight (reattention.py:822-842) on the fp32 un-rotated keys and
    bf16 values, then _dense_topk (reattention.py:486-498). Value rows carry a
    per-row scale (exp of a normal draw) so the weighting changes the selection;
    ``zero_rows`` of them are zero (weight 0)."""
    for (name, rt, B, Hq, Hkv, Sq, Sk, topk, theta, pos_offset, zero_rows) in RECALL_CASES:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        D = 128
        q = torch.randn(B, Hq, Sq, D, generator=g).to(torch.bfloat16)
        k_raw = torch.randn(B, Hkv, Sk, D, generator=g)
        v = torch.randn(B, Hkv, Sk, D, generator=g) * torch.exp(0.7 * torch.randn(B, Hkv, Sk, 1, generator=g))
        if zero_rows > 0:
            v[torch.rand(B, Hkv, Sk, generator=g) < zero_rows] = 0.0
        v = v.to(torch.bfloat16)
        inv_freq = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).to(torch.float32) / D))
        pos = torch.arange(pos_offset, pos_offset + Sk)
        cos, sin = build_cos_sin(pos, inv_freq, torch.device("cpu"), torch.float32)
        k_cached = apply_rotary_pos_emb(k_raw, cos, sin).to(torch.bfloat16)
        raw_ref = undo_rotary_pos_emb(k_cached.float(), cos, sin)
        method = ReAttentionMethod(mid_size=topk, recall_type=rt, use_triton_kernel="off")
        recall_k = method._apply_recall_weight(raw_ref, v)
        idx = method._dense_topk(q.float(), recall_k, Sk)
        n_rep = Hq // Hkv
        rk = recall_k[:, :, None].expand(B, Hkv, n_rep, Sk, D).reshape(B, Hq, Sk, D)
        full = torch.einsum("bhqd,bhmd->bhqm", q.float(), rk.float())
        vals = torch.gather(full, -1, idx)
        np.savez_compressed(
            HERE / f"{name}.npz",
            q_bf16=bf16_bits(q), k_bf16=bf16_bits(k_cached), v_bf16=bf16_bits(v),
            inv_freq=inv_freq.numpy(), rope=np.array(True), pos_offset=np.array(pos_offset),
            causal_offset=np.array(-1), topk=np.array(topk), recall_type=np.array(rt),
            idx=idx.numpy().astype(np.int64), scores=vals.numpy(),
            raw_keys_ref=np.zeros(0, np.float32),
        )
        print(name, rt, tuple(q.shape), tuple(k_cached.shape), "topk", topk)


# post-selection cases: name, n_mid, recall_clip, span_size, span_mode, pattern
POST_CASES = [
    ("post_unique_span32", 60000, -1, 32, "centered", "random"),
    ("post_clip40_span5", 3000, 40, 5, "centered", "frequency"),
    ("post_span0_identity", 2000, -1, 0, "centered", "random"),
    ("post_edges_span7", 600, -1, 7, "centered", "edges"),
    ("post_floor_span5", 3000, -1, 5, "floor", "random"),
    ("post_floor_clip25_span4", 4000, 25, 4, "floor", "frequency"),
]


def post_select_cases(ReAttentionMethod) -> None:
    """Golden vectors of the post-selection: ReAttentionMethod._global_unique and
    _expand_spans (reattention.py:844-874) for the centered spans; for the floor
    spans, _global_unique followed by the span arithmetic of
    reattention_exact.py:578-581 (offsets arange(-span // 2, (span + 1) // 2),
    clamp to the middle, unique), which lives inline in a larger method there."""
    for (name, n_mid, clip, span, mode, pattern) in POST_CASES:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        if pattern == "random":
            idx = torch.randint(0, n_mid, (1, 8, 4, 64), generator=g)
        elif pattern == "edges":
            idx = torch.cat([torch.randint(0, 4, (40,), generator=g),
                             torch.randint(n_mid - 4, n_mid, (40,), generator=g),
                             torch.randint(0, n_mid, (40,), generator=g)])
        else:  # distinct selection counts, so the recall_clip cut has no ties
            pos = torch.randperm(n_mid, generator=g)[:100]
            idx = torch.cat([pos[i:i + 1].repeat(i + 1) for i in range(100)])
            idx = idx[torch.randperm(idx.numel(), generator=g)]
        sel = ReAttentionMethod._global_unique(idx, clip)
        if mode == "centered":
            method = ReAttentionMethod(span_size=span, use_triton_kernel="off")
            out = method._expand_spans(sel, n_mid)
        else:
            offsets = torch.arange(-span // 2, (span + 1) // 2)
            ids = (sel[:, None] + offsets[None, :]).reshape(-1).clamp(0, n_mid - 1)
            out = torch.unique(ids)
        np.savez_compressed(HERE / f"{name}.npz", idx=idx.numpy().astype(np.int64),
                            n_mid=np.array(n_mid), recall_clip=np.array(clip),
                            span=np.array(span), mode=np.array(mode), out=out.numpy().astype(np.int64))
        print(name, idx.numel(), "->", out.numel())


# attention over a selected view: name, B, Hq, Hkv, Sq, S, n_mid_selected, local, pe_original, pattern
ATTN_CASES = [
    ("attn_decode_pe_original", 1, 8, 2, 1, 3000, 300, 256, True, "view"),
    ("attn_chunk_contiguous", 2, 4, 2, 16, 2000, 200, 128, False, "view"),
    ("attn_rows_without_keys", 1, 4, 1, 3, 40, 0, 0, True, "late_keys"),
]


def sparse_attention_cases(ReAttentionExactMethod, apply_rotary_pos_emb, build_cos_sin) -> None:
    """Golden vectors of the attention over the selected view: the gather and RoPE of
    ReAttentionExactMethod._chunk_attention (reattention_exact.py:453-508), run here on
    fp32 copies of bf16 tensors with the reference's build_cos_sin /
    apply_rotary_pos_emb, then its own _attend with the eager path
    (use_flash_attn='off', :650-661)."""
    method = ReAttentionExactMethod(use_flash_attn="off")
    for (name, B, Hq, Hkv, Sq, S, n_sel_mid, local, pe_original, pattern) in ATTN_CASES:
        g = torch.Generator().manual_seed(zlib.crc32(name.encode()))
        D = 128
        q = torch.randn(B, Hq, Sq, D, generator=g).to(torch.bfloat16)
        k = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
        v = torch.randn(B, Hkv, S, D, generator=g).to(torch.bfloat16)
        pos_c = torch.arange(S - Sq, S)
        if pattern == "view":  # [global 32 | recalled middle | local tail]
            gsz = 32
            mid = torch.randperm(S - gsz - local, generator=g)[:n_sel_mid] + gsz
            key_pos = torch.cat([torch.arange(gsz), mid.sort().values, torch.arange(S - local, S)])
        else:  # keys only after the first query rows: those rows see nothing
            pos_c = torch.tensor([5, 15, 25])
            key_pos = torch.arange(10, 21)
        inv_freq = 1.0 / (5e5 ** (torch.arange(0, D, 2, dtype=torch.int64).to(torch.float32) / D))
        gather = key_pos.view(1, 1, -1, 1).expand(B, Hkv, -1, D)
        sel_k = torch.gather(k.float(), 2, gather)
        sel_v = torch.gather(v.float(), 2, gather)
        view_len = key_pos.numel()
        if pe_original:
            pe_key_pos, pe_q_pos = key_pos, pos_c
        else:
            pe_key_pos = torch.arange(view_len)
            pe_q_pos = torch.arange(view_len - Sq, view_len)
        cos_k, sin_k = build_cos_sin(pe_key_pos, inv_freq, torch.device("cpu"), torch.float32)
        sel_k = apply_rotary_pos_emb(sel_k, cos_k, sin_k)
        cos_q, sin_q = build_cos_sin(pe_q_pos, inv_freq, torch.device("cpu"), torch.float32)
        q_rot = apply_rotary_pos_emb(q.float(), cos_q, sin_q)
        scale = D ** -0.5
        out = method._attend(q_rot, sel_k, sel_v, pos_c, key_pos, scale)
        np.savez_compressed(
            HERE / f"{name}.npz",
            q_bf16=bf16_bits(q), k_bf16=bf16_bits(k), v_bf16=bf16_bits(v),
            key_pos=key_pos.numpy().astype(np.int64), q_pos=pos_c.numpy().astype(np.int64),
            inv_freq=inv_freq.numpy(), pe_original=np.array(pe_original), scale=np.array(scale),
            out=out.numpy(),
        )
        print(name, tuple(q.shape), "view", view_len, "pe_original", pe_original)


if __name__ == "__main__":
    main()
