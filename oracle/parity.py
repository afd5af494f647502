"""Parity rules for the recall scorer, checked against the CPU oracle — TEST
INFRASTRUCTURE ONLY (the tests, ``smoke()`` and ``bench.py``'s result check after
its timed region use it as the checker).

* Returned scores agree with the oracle's fp32 score of the same key within
  ``|s - s_ref| <= max(rel * |s_ref|, rel * ||q|| * ||k||)``, rel = 1e-3.
* Returned rows are sorted by descending score.
* Returned indices are distinct and in range.
* The selected index set equals the oracle's except for keys whose oracle score
  lies within that tolerance of the oracle's k-th score (near-ties may swap).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import reattention_topk as orc

REL = 1e-3
# Weighted recall (qkv / qkv2): the key weight is a value-row norm rounded to
# bf16/fp16 like values.norm; a different fp32 summation order can move that
# rounding by one step (2^-8 relative for bf16), so weighted scores get 4e-3.
REL_WEIGHTED = 4e-3


def check_parity(idx: torch.Tensor, scores: Optional[torch.Tensor], q: torch.Tensor, k: torch.Tensor,
                 topk: int, inv_freq: Optional[torch.Tensor] = None, pos_offset: int = 0,
                 causal_offset: Optional[int] = None, index_base: int = 0, rel: float = REL,
                 by_head: bool = False, weights: Optional[torch.Tensor] = None) -> dict:
    """Assert the parity rules; returns a few statistics for reporting."""
    idx = idx.cpu().long() - index_base
    q = q.cpu()
    k = k.cpu()
    B, Hq, Sq, _ = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    G = Hq // Hkv
    assert idx.shape == (B, Hq, Sq, topk), idx.shape
    assert int(idx.min()) >= 0 and int(idx.max()) < Sk, "index out of range"
    stats = dict(max_rel_err=0.0, swapped=0, rows=0)
    inv = inv_freq.cpu() if inv_freq is not None else None
    for hk in range(Hkv):
        k_raw = orc.unrotate_keys(k[:, hk:hk + 1], inv, pos_offset)  # [B,1,Sk,D]
        if weights is not None:  # recall_type qkv / qkv2: raw_k * ||v||
            k_raw = k_raw * weights.cpu()[:, hk:hk + 1, :, None]
        qh = q[:, hk * G:(hk + 1) * G]
        full = orc.dense_scores(qh, k_raw, causal_offset)  # [B,G,Sq,Sk]
        tol = orc.score_tolerance(qh, k_raw, rel)  # [B,G,Sq,Sk]
        ref_vals, ref_idx = full.topk(topk, dim=-1)
        mine = idx[:, hk * G:(hk + 1) * G]
        # distinct
        srt = mine.sort(dim=-1).values
        assert bool((srt[..., 1:] != srt[..., :-1]).all()), "duplicate indices in a row"
        ref_at_mine = torch.gather(full, -1, mine)
        tol_at_mine = torch.gather(tol, -1, mine)
        finite = torch.isfinite(ref_at_mine)
        if scores is not None:
            sc = scores.cpu()[:, hk * G:(hk + 1) * G].float()
            err = (sc - ref_at_mine).abs()
            lim = torch.maximum(rel * ref_at_mine.abs(), tol_at_mine)
            ok = torch.where(finite, err <= lim, sc == ref_at_mine)
            if not bool(ok.all()):
                bad = torch.nonzero(~ok)[:12].tolist()
                detail = [(b_, hk * G + g_, s_, c_, int(mine[b_, g_, s_, c_]),
                           float(sc[b_, g_, s_, c_]), float(ref_at_mine[b_, g_, s_, c_])) for b_, g_, s_, c_ in bad]
                raise AssertionError(
                    f"score mismatch kv head {hk}: {int((~ok).sum())} bad; worst err "
                    f"{float(err[finite].max()):.4g}; (b, head, row, rank, idx, got, ref): {detail}")
            if bool(finite.any()):
                stats["max_rel_err"] = max(stats["max_rel_err"],
                                           float((err[finite] / lim[finite].clamp_min(1e-30)).max()) * rel)
            d = sc[..., 1:] - sc[..., :-1]
            assert bool((d <= 0).all() | torch.isnan(d).any()), "scores not sorted descending"
        # set equality modulo near-ties at the k-th score
        kth = ref_vals[..., -1:]  # [B,G,Sq,1]
        tol_k = torch.maximum(rel * kth.abs(), torch.gather(tol, -1, ref_idx[..., -1:]))
        in_ref = torch.zeros_like(full, dtype=torch.bool).scatter_(-1, ref_idx, True)
        in_mine = torch.zeros_like(full, dtype=torch.bool).scatter_(-1, mine, True)
        diff = in_ref ^ in_mine
        near = (full - kth).abs() <= tol_k
        both_inf = torch.isinf(full) & torch.isinf(kth) & (full == kth)
        bad = diff & ~(near | both_inf)
        assert not bool(bad.any()), f"index sets differ beyond near-ties (kv head {hk}): {int(bad.sum())}"
        stats["swapped"] += int(diff.sum()) // 2
        stats["rows"] += B * G * Sq
    return stats


def check_rows_parity(idx: torch.Tensor, scores: torch.Tensor, q: torch.Tensor, k: torch.Tensor,
                      topk: int, rows, causal_offset: Optional[int] = None, rel: float = REL,
                      inv_freq: Optional[torch.Tensor] = None, pos_offset: int = 0) -> int:
    """The parity rules on selected flattened rows (b, hq, s) only, for shapes whose
    full oracle does not fit in memory; RoPE'd keys (inv_freq given) are un-rotated
    once per (batch, KV head) by the oracle. Returns near-tie swaps."""
    B, Hq, Sq, _ = q.shape
    Hkv, Sk = k.shape[1], k.shape[2]
    G = Hq // Hkv
    idx = idx.reshape(B * Hq * Sq, topk)
    scores = scores.reshape(B * Hq * Sq, topk)
    inv = inv_freq.cpu() if inv_freq is not None else None
    raw = {}  # (b, kv head) -> fp32 raw keys [Sk, D]
    swaps = 0
    for row in rows:
        s = row % Sq
        b, hq = divmod(row // Sq, Hq)
        qv = q[b, hq, s].float().cpu()
        if (b, hq // G) not in raw:
            kh = k[b:b + 1, hq // G:hq // G + 1].cpu()
            raw[(b, hq // G)] = orc.unrotate_keys(kh, inv, pos_offset)[0, 0].float()
        kk = raw[(b, hq // G)]
        full = kk @ qv                                            # [Sk]
        tol = rel * qv.norm() * kk.norm(dim=-1)                   # [Sk]
        if causal_offset is not None:
            full[causal_offset + s + 1:] = float("-inf")
        mine = idx[row].long().cpu()
        sc = scores[row].float().cpu()
        assert int(mine.min()) >= 0 and int(mine.max()) < Sk, f"row {row}: index out of range"
        assert mine.unique().numel() == topk, f"row {row}: duplicate indices"
        ref_at = full[mine]
        finite = torch.isfinite(ref_at)
        lim = torch.maximum(rel * ref_at.abs(), tol[mine])
        ok = torch.where(finite, (sc - ref_at).abs() <= lim, sc == ref_at)
        assert bool(ok.all()), f"row {row}: {int((~ok).sum())} scores off"
        d = sc[1:] - sc[:-1]
        assert bool((d <= 0).all()), f"row {row}: scores not sorted"
        ref_vals, ref_idx = full.topk(topk)
        kth = ref_vals[-1]
        tol_k = max(float(rel * kth.abs()), float(tol[ref_idx[-1]]))
        in_ref = torch.zeros(Sk, dtype=torch.bool)
        in_ref[ref_idx] = True
        in_mine = torch.zeros(Sk, dtype=torch.bool)
        in_mine[mine] = True
        diff = in_ref ^ in_mine
        near = (full - kth).abs() <= tol_k
        both_inf = torch.isinf(full) & torch.isinf(kth) & (full == kth)
        bad = diff & ~(near | both_inf)
        assert not bool(bad.any()), f"row {row}: index sets differ beyond near-ties"
        swaps += int(diff.sum()) // 2
    return swaps
