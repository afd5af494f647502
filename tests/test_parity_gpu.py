"""GPU parity of the CUDA scorer against the CPU oracle (all calls go through
the C ABI of libprism_b200.so via einsum_topk_func)."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import reattention_topk as orc
from prism_test_b200 import einsum_topk_func, topk_merge
from prism_test_b200 import workloads as W
from tests.parity import check_parity

pytestmark = pytest.mark.gpu

GOLDEN = sorted(p for p in (Path(__file__).parent / "golden").glob("*.npz")
                if not p.stem.startswith(("post_", "recall_", "attn_", "blockmax_", "dropin_")))


def _golden(path, dev):
    z = np.load(path)
    q = torch.from_numpy(z["q_bf16"].view(np.int16)).view(torch.bfloat16)
    k = torch.from_numpy(z["k_bf16"].view(np.int16)).view(torch.bfloat16)
    inv = torch.from_numpy(z["inv_freq"]) if bool(z["rope"]) else None
    causal = int(z["causal_offset"])
    return dict(q=q.to(dev), k=k.to(dev), inv_freq=None if inv is None else inv.to(dev),
                pos_offset=int(z["pos_offset"]), causal_offset=None if causal < 0 else causal,
                topk=int(z["topk"]), idx=torch.from_numpy(z["idx"]), scores=torch.from_numpy(z["scores"]))


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_golden_vectors(path, cuda_device):
    c = _golden(path, cuda_device)
    idx, sc = einsum_topk_func(c["q"], c["k"], c["topk"], inv_freq=c["inv_freq"], pos_offset=c["pos_offset"],
                               causal_offset=c["causal_offset"], return_scores=True)
    torch.cuda.synchronize()
    check_parity(idx, sc, c["q"], c["k"], c["topk"], c["inv_freq"], c["pos_offset"], c["causal_offset"])
    # against the reference's own sorted top-k scores, rank by rank: a near-tie
    # swap moves a value by less than its neighbour's gap, so each rank agrees
    # within three times the parity tolerance
    ref_scores = c["scores"]
    finite = torch.isfinite(ref_scores)
    assert torch.equal(torch.isfinite(sc.cpu()), finite)
    qn = c["q"].float().norm(dim=-1).cpu()[..., None]  # [B,Hq,Sq,1]
    kmax = orc.unrotate_keys(c["k"].cpu(), None if c["inv_freq"] is None else c["inv_freq"].cpu(),
                             c["pos_offset"]).norm(dim=-1).max()
    lim = 3e-3 * torch.maximum(ref_scores.abs(), qn * kmax)
    assert bool(((sc.cpu() - ref_scores).abs() <= lim)[finite].all())


CASES = [
    # B, Hq, Hkv, Sq, Sk, topk, rope, dtype
    (1, 32, 8, 1, 16384, 1024, True, torch.bfloat16),
    (1, 32, 8, 1, 5000, 777, True, torch.bfloat16),
    (1, 8, 8, 1, 129, 129, True, torch.bfloat16),
    (1, 4, 1, 1, 3, 2, True, torch.bfloat16),
    (1, 4, 2, 3, 1000, 1, False, torch.bfloat16),
    (2, 8, 2, 2, 2048, 100, True, torch.float16),
    (1, 28, 4, 8, 3000, 500, True, torch.bfloat16),   # 224 rows -> several row chunks per KV head
    (1, 32, 8, 9, 700, 64, True, torch.bfloat16),     # Hq*Sq > 128 -> query chunking
    (3, 12, 3, 1, 4099, 16384 // 8, True, torch.bfloat16),
    (1, 16, 4, 1, 20000, 16384, True, torch.bfloat16),  # largest supported k
    # many query rows per KV head: the queries-as-M tensor-core scorer
    (1, 16, 2, 8, 3001, 300, True, torch.bfloat16),    # 64 rows per KV head, Hkv 2
    (1, 32, 8, 5, 2500, 200, True, torch.float16),     # 20 rows per KV head, fp16
    (1, 32, 8, 8, 2500, 200, False, torch.bfloat16),   # 32 rows per KV head, Hkv 8, raw keys
    (2, 28, 4, 6, 1777, 50, True, torch.float16),      # 42 rows, ragged n-tiles, B = 2
    # the head-pair decode scorer counts the select's threshold sample
    (3, 32, 8, 1, 9000, 700, True, torch.bfloat16),    # 96 rows: one CTA per row
    (1, 8, 4, 1, 200000, 2000, True, torch.bfloat16),  # rows longer than one select pass
    (2, 16, 4, 1, 40001, 4096, True, torch.bfloat16),  # batch 2, ragged length
    (1, 4, 2, 1, 17, 17, True, torch.bfloat16),        # k = Sk: every key a candidate
]


@pytest.mark.parametrize("B,Hq,Hkv,Sq,Sk,topk,rope,dtype", CASES)
def test_random_shapes(B, Hq, Hkv, Sq, Sk, topk, rope, dtype, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(B * 1000 + Sk)
    q = torch.randn(B, Hq, Sq, 128, generator=g, device=cuda_device).to(dtype)
    k = torch.randn(B, Hkv, Sk, 128, generator=g, device=cuda_device).to(dtype)
    inv = W.rope_inv_freq(128, 5e5).to(cuda_device) if rope else None
    idx, sc = einsum_topk_func(q, k, topk, inv_freq=inv, pos_offset=11 if rope else 0, return_scores=True)
    check_parity(idx, sc, q, k, topk, inv, 11 if rope else 0)


def test_causal_prefill_small(cuda_device):
    wl = W.small(W.WORKLOADS["prefill-chunk-128k"], Sk=6000, Sq=64, topk=300)
    x = W.make_inputs(wl, cuda_device)
    idx, sc = einsum_topk_func(x["q"], x["k"], wl.topk, inv_freq=x["inv_freq"],
                               causal_offset=wl.causal_offset, return_scores=True)
    check_parity(idx, sc, x["q"], x["k"], wl.topk, x["inv_freq"], 0, wl.causal_offset)


def test_strided_key_slice_and_index_base(cuda_device):
    # the middle slice of a larger cache, as reattention passes recall_k[:, :, g:S-l]
    g = torch.Generator(device=cuda_device).manual_seed(3)
    cache = torch.randn(1, 4, 3000, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    q = torch.randn(1, 16, 1, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    mid = cache[:, :, 32:2500]
    assert not mid.is_contiguous()
    inv = W.rope_inv_freq(128, 5e5).to(cuda_device)
    idx, sc = einsum_topk_func(q, mid, 50, inv_freq=inv, pos_offset=32, index_base=1000, return_scores=True)
    check_parity(idx, sc, q, mid.contiguous(), 50, inv, 32, index_base=1000)


def test_batch_broadcast_keys(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(4)
    k1 = torch.randn(1, 2, 1024, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k = k1.expand(3, -1, -1, -1)
    assert k.stride(0) == 0
    q = torch.randn(3, 8, 1, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    idx, sc = einsum_topk_func(q, k, 40, return_scores=True)
    check_parity(idx, sc, q, k.contiguous(), 40)


def test_massive_ties_take_lowest_indices(cuda_device):
    # 40000 identical keys: the k-th key has more exact ties than the candidate buffer
    row = torch.randn(128, device=cuda_device).to(torch.bfloat16)
    k = row.expand(1, 1, 40000, 128).contiguous()
    q = torch.randn(1, 2, 1, 128, device=cuda_device).to(torch.bfloat16)
    idx, sc = einsum_topk_func(q, k, 100, return_scores=True)
    assert torch.equal(idx.cpu()[0, 0, 0], torch.arange(100, dtype=torch.int32))
    assert torch.equal(idx.cpu()[0, 1, 0], torch.arange(100, dtype=torch.int32))
    assert bool((sc == sc[..., :1]).all())


def test_planted_keys_are_found(cuda_device):
    wl = W.small(W.WORKLOADS["decode-128k"], Sk=8192, topk=64)
    x = W.make_inputs(wl, cuda_device)
    idx = einsum_topk_func(x["q"], x["k"], wl.topk, inv_freq=x["inv_freq"])
    planted = W.planted_positions(wl)
    G = wl.Hq // wl.Hkv
    for h in range(wl.Hq):
        mine = planted[h // G][(h % G) * wl.planted_per_qhead:(h % G + 1) * wl.planted_per_qhead]
        got = set(idx[0, h, 0].cpu().tolist())
        assert set(mine.tolist()) <= got


def test_deterministic(cuda_device):
    wl = W.small(W.WORKLOADS["shared-context-256k"], Sk=20000, topk=700)
    x = W.make_inputs(wl, cuda_device)
    a = einsum_topk_func(x["q"], x["k"], wl.topk, inv_freq=x["inv_freq"], return_scores=True)
    b = einsum_topk_func(x["q"], x["k"], wl.topk, inv_freq=x["inv_freq"], return_scores=True)
    assert torch.equal(a[0], b[0]) and torch.equal(a[1], b[1])
    check_parity(a[0], a[1], x["q"], x["k"], wl.topk, x["inv_freq"])


def test_topk_merge_matches_torch(cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(9)
    s = torch.randn(6, 3 * 512, generator=g, device=cuda_device)
    i = torch.randperm(100000, generator=g, device=cuda_device)[: 6 * 1536].view(6, 1536).to(torch.int32)
    oi, os_ = topk_merge(s, i, 300)
    rv, rp = s.topk(300, dim=-1)
    assert torch.equal(os_, rv)
    assert torch.equal(oi, torch.gather(i, 1, rp))


def _order_keys(s: torch.Tensor) -> torch.Tensor:
    """The selection's total order as int64 keys: NaN first, +0 above -0, then the
    float order (the order key of the library's selection)."""
    u = s.contiguous().view(torch.int32).long() & 0xFFFFFFFF
    neg = (u & 0x80000000) != 0
    key = torch.where(neg, (~u) & 0xFFFFFFFF, u | 0x80000000)
    return torch.where(torch.isnan(s), torch.full_like(key, 0xFFFFFFFF), key)


def test_streamed_select_signed_zero_nan_inf(cuda_device):
    # rows longer than one pass (streamed): thresholds that land on +0 or -0, NaN
    # and infinities; expected order: order key descending, then the lower index
    g = torch.Generator().manual_seed(41)
    n, k = 300000, 5000
    s = torch.zeros(5, n)
    sign = torch.randint(0, 2, (n,), generator=g).bool()
    s[0] = torch.where(sign, torch.tensor(-0.0), torch.tensor(0.0))
    s[0, torch.randperm(n, generator=g)[:2000]] = torch.randn(2000, generator=g).abs() + 0.1
    s[0, torch.randperm(n, generator=g)[:10]] = float("nan")
    s[1] = -0.0
    s[1, torch.randperm(n, generator=g)[:100]] = torch.rand(100, generator=g) + 1.0
    s[2] = torch.randn(n, generator=g)
    s[2, torch.randperm(n, generator=g)[:7]] = float("inf")
    s[2, torch.randperm(n, generator=g)[:7]] = float("-inf")
    s[3] = -1.0 - torch.rand(n, generator=g)  # few zeros: the threshold can land on +0 itself
    pos = torch.randperm(n, generator=g)
    s[3, pos[:4000]] = torch.rand(4000, generator=g) + 0.5
    s[3, pos[4000:7000]] = 0.0
    s[3, pos[7000:10000]] = -0.0
    s[4] = torch.randn(n, generator=g)  # mostly NaN: NaN keys tie beyond the candidate buffer
    s[4, torch.randperm(n, generator=g)[: n * 2 // 5]] = float("nan")
    i = torch.arange(n, dtype=torch.int32).expand(5, n).contiguous()
    oi, os_ = topk_merge(s.to(cuda_device), i.to(cuda_device), k)
    key = _order_keys(s)
    # descending key, ascending index: sort by index first (stable), then by key
    o = torch.sort(key, dim=-1, descending=True, stable=True).indices[:, :k]
    assert torch.equal(oi.cpu(), o.to(torch.int32))
    got, want = os_.cpu(), torch.gather(s, 1, o)
    assert torch.equal(torch.isnan(got), torch.isnan(want))
    fin = ~torch.isnan(want)
    assert torch.equal(got[fin].view(torch.int32), want[fin].view(torch.int32))


def test_status_word_clean(cuda_device, monkeypatch):
    # with the synchronous check on, every call reads its own device status word
    from prism_test_b200 import kernels
    monkeypatch.setattr(kernels, "_SYNC_CHECK", True)
    q = torch.randn(1, 8, 1, 128, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(1, 2, 50000, 128, device=cuda_device).to(torch.bfloat16)
    einsum_topk_func(q, k, 10, inv_freq=W.rope_inv_freq(128, 5e5).to(cuda_device))
    einsum_topk_func(q, k, 3000)


@pytest.mark.parametrize("name", ["decode-128k", "shared-context-256k"])
def test_full_size_configs(name, cuda_device):
    wl = W.WORKLOADS[name]
    x = W.make_inputs(wl, cuda_device)
    idx, sc = einsum_topk_func(x["q"], x["k"], wl.topk, inv_freq=x["inv_freq"], return_scores=True)
    st = check_parity(idx, sc, x["q"], x["k"], wl.topk, x["inv_freq"])
    assert st["rows"] == wl.B * wl.Hq * wl.Sq


def test_full_size_1m_shard(cuda_device):
    # one of eight sequence shards of the 1M-key config, with its global offset
    wl = W.WORKLOADS["decode-1m-sharded"]
    x = W.make_inputs(wl, cuda_device, shard=(5, 8))
    idx, sc = einsum_topk_func(x["q"], x["k"], wl.topk, inv_freq=x["inv_freq"], pos_offset=x["pos_offset"],
                               index_base=x["index_base"], return_scores=True)
    check_parity(idx, sc, x["q"], x["k"], wl.topk, x["inv_freq"], x["pos_offset"], index_base=x["index_base"])


def _sampled_mask(n, chunk=128):
    """Columns the select kernels' threshold sample reads (white-box): 8 consecutive
    columns of every ``chunk`` at an offset hashed from the chunk number — chunk 128
    for the one-CTA-per-row kernel and for cluster rows held in registers, 256 for
    longer cluster rows."""
    import numpy as np
    shift = 32 - (chunk // 8).bit_length() + 1
    g = np.arange((n + chunk - 1) // chunk, dtype=np.uint64)
    off = ((g * np.uint64(0x9E3779B1)) & np.uint64(0xFFFFFFFF)) >> np.uint64(shift)
    m = np.zeros(n, dtype=bool)
    for gi, o in zip(g.tolist(), off.tolist()):
        s = chunk * gi + 8 * o
        if s + 8 <= n:
            m[s:s + 8] = True
    return torch.from_numpy(m)


def _misleading_keys(n, Hkv, mask, sampled_high, seed):
    """Keys along q's first axis whose magnitudes make the sampled columns all high
    (too few candidates above the sampled threshold) or all low (too many)."""
    g = torch.Generator().manual_seed(seed)
    mag = torch.rand(Hkv, n, generator=g)
    mag = torch.where(mask[None, :], mag + (2.0 if sampled_high else -2.0), mag)
    k = torch.zeros(1, Hkv, n, 128)
    k[0, :, :, 0] = mag
    k[0, :, :, 1:] = 0.01 * torch.randn(Hkv, n, 127, generator=g)
    return k


@pytest.mark.parametrize("sampled_high", [True, False])
@pytest.mark.parametrize("case", ["row-kernel", "cluster", "cluster-long"])
def test_select_threshold_miss_falls_back_exactly(case, sampled_high, cuda_device):
    # every threshold sample the select uses, defeated on purpose: the result must
    # still be the exact top-k (the kernels fall back to the exact radix path)
    if case == "row-kernel":      # 64 rows: one CTA per row
        n, topk, Hq, Hkv, mask = 40000, 3000, 64, 1, _sampled_mask(40000)
    elif case == "cluster":       # 4 rows: one 4-CTA cluster per row, keys in registers
        n, topk, Hq, Hkv, mask = 100000, 3000, 4, 2, _sampled_mask(100000)
    else:                         # the same, rows longer than one pass of the cluster
        n, topk, Hq, Hkv, mask = 300000, 3000, 4, 2, _sampled_mask(300000, 256)
    q = torch.zeros(1, Hq, 1, 128)
    q[..., 0] = 1.0
    k = _misleading_keys(n, Hkv, mask, sampled_high, seed=5)
    q = q.to(torch.bfloat16).to(cuda_device)
    k = k.to(torch.bfloat16).to(cuda_device)
    idx, sc = einsum_topk_func(q, k, topk, return_scores=True)
    check_parity(idx, sc, q, k, topk)


def test_full_size_1m_one_gpu(cuda_device):
    # the whole 1M-key cache on one GPU: rows longer than one select pass, with the
    # scorer's threshold sample
    wl = W.WORKLOADS["decode-1m-sharded"]
    x = W.make_inputs(wl, cuda_device)
    idx, sc = einsum_topk_func(x["q"], x["k"], wl.topk, inv_freq=x["inv_freq"], return_scores=True)
    st = check_parity(idx, sc, x["q"], x["k"], wl.topk, x["inv_freq"])
    assert st["rows"] == 32


def test_topk_merge_large_rows(cuda_device):
    # 8 sorted runs of 8192 (the 8-shard merge of the 1M config) -> sampled path
    g = torch.Generator(device=cuda_device).manual_seed(11)
    runs = [torch.randn(32, 8192, generator=g, device=cuda_device).sort(dim=-1, descending=True).values
            for _ in range(8)]
    s = torch.cat(runs, dim=1)
    i = (torch.arange(8 * 8192, device=cuda_device, dtype=torch.int32)[None, :] * 3).expand(32, -1).contiguous()
    oi, os_ = topk_merge(s, i, 8192)
    rv, rp = s.topk(8192, dim=-1)
    assert torch.equal(os_, rv)
    assert torch.equal(oi, torch.gather(i, 1, rp))


@pytest.mark.gpu
@pytest.mark.parametrize("nruns,run_len,topk", [(2, 8192, 8192), (8, 8192, 8192), (4, 1000, 300), (3, 5000, 5000)])
def test_topk_merge_runs_matches_torch(cuda_device, nruns, run_len, topk):
    # sorted runs with distinct global indices, as the sharded path gathers them;
    # one run holds a block of much larger scores (a skewed shard)
    from prism_test_b200 import topk_merge_runs
    rows = 6
    g = torch.Generator().manual_seed(nruns * 131 + run_len)
    s = torch.randn(nruns, rows, run_len, generator=g)
    s[0, :, : run_len // 3] += 4.0
    perm = torch.randperm(nruns * run_len * 4, generator=g)[: nruns * run_len].view(nruns, 1, run_len)
    idx = perm.expand(nruns, rows, run_len).to(torch.int32)
    # sort each run by (score desc, index asc)
    order = torch.argsort(idx.long(), dim=-1, stable=True)
    s = torch.gather(s, -1, order)
    idx = torch.gather(idx, -1, order)
    v, p = torch.sort(s, dim=-1, descending=True, stable=True)
    idx = torch.gather(idx, -1, p)
    runs = torch.stack([v.view(torch.int32), idx], dim=1).to(cuda_device)  # [nruns, 2, rows, len]
    oi, os_ = topk_merge_runs(runs, topk)
    flat_s = v.permute(1, 0, 2).reshape(rows, -1)
    flat_i = idx.permute(1, 0, 2).reshape(rows, -1)
    o2 = torch.argsort(flat_i.long(), dim=-1, stable=True)
    fs, fi = torch.gather(flat_s, -1, o2), torch.gather(flat_i, -1, o2)
    ws, wp = torch.sort(fs, dim=-1, descending=True, stable=True)
    wi = torch.gather(fi, -1, wp)
    assert torch.equal(os_.cpu(), ws[:, :topk])
    assert torch.equal(oi.cpu(), wi[:, :topk])


@pytest.mark.gpu
def test_wide_rows_causal(cuda_device):
    # 56 rows per KV head (8 queries x 7 heads) with a causal mask
    g = torch.Generator(device=cuda_device).manual_seed(77)
    q = torch.randn(1, 28, 8, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(1, 4, 4000, 128, generator=g, device=cuda_device).to(torch.bfloat16)
    inv = W.rope_inv_freq(128, 1e6).to(cuda_device)
    idx, sc = einsum_topk_func(q, k, 400, inv_freq=inv, causal_offset=3990, return_scores=True)
    check_parity(idx, sc, q, k, 400, inv, 0, 3990)


# ---- streaming top-k on the queries-as-M scorer (many rows per KV head, long context) --
# A threshold sample (every 16th stage of 128 / Hkv positions), per-row thresholds,
# a candidate pass and the streaming selection with its exact fallback: no score
# matrix. Taken for exact calls with Sq >= 2, >= 64 rows, Sk >= 32768, topk * 16 <= Sk.
@pytest.mark.parametrize("B,Hq,Hkv,Sq,Sk,topk,rope,dtype,causal", [
    (1, 28, 4, 8, 40000, 1000, True, torch.bfloat16, None),      # ragged Sk, RoPE
    (1, 28, 4, 8, 40000, 1000, True, torch.bfloat16, 39990),     # causal chunk tail
    (1, 16, 2, 8, 65536, 4096, False, torch.float16, None),      # raw fp16 keys, Hkv 2
    (2, 32, 8, 4, 36000, 500, True, torch.bfloat16, None),       # batch 2, Hkv 8
])
def test_wide_stream_shapes(B, Hq, Hkv, Sq, Sk, topk, rope, dtype, causal, cuda_device):
    g = torch.Generator(device=cuda_device).manual_seed(Sk + Hq)
    q = torch.randn(B, Hq, Sq, 128, generator=g, device=cuda_device).to(dtype)
    k = torch.randn(B, Hkv, Sk, 128, generator=g, device=cuda_device).to(dtype)
    inv = W.rope_inv_freq(128, 1e6).to(cuda_device) if rope else None
    idx, sc = einsum_topk_func(q, k, topk, inv_freq=inv, pos_offset=5 if rope else 0,
                               causal_offset=causal, return_scores=True)
    check_parity(idx, sc, q, k, topk, inv, 5 if rope else 0, causal)


@pytest.mark.parametrize("Hkv,dtype", [(4, torch.bfloat16), (2, torch.float16)])
def test_wide_stream_concentrated_hits_overflow_segments(Hkv, dtype, cuda_device):
    # 600 keys in one stretch of the cache aligned with every query row of their head:
    # the CTAs covering that stretch find far more than a candidate segment holds
    # (64 per row and CTA half), and the rest goes to the rows' lists through their
    # counters
    g = torch.Generator(device=cuda_device).manual_seed(41)
    B, Sq, Sk, topk = 1, 8, 40000, 2000
    Hq = Hkv * 7
    G = Hq // Hkv
    dirs = torch.randn(Hkv, 128, generator=g, device=cuda_device)
    dirs = dirs / dirs.norm(dim=-1, keepdim=True)
    # every query row of head h: a common direction dirs[h] plus noise
    q = torch.randn(B, Hq, Sq, 128, generator=g, device=cuda_device) + \
        3.0 * dirs.repeat_interleave(G, dim=0)[None, :, None, :]
    k = torch.randn(B, Hkv, Sk, 128, generator=g, device=cuda_device)
    for h in range(Hkv):
        k[0, h, 10000:10600] = 4.0 * 11.3 * dirs[h] + 0.5 * k[0, h, 10000:10600]
    q, k = q.to(dtype), k.to(dtype)
    idx, sc = einsum_topk_func(q, k, topk, return_scores=True)
    check_parity(idx, sc, q, k, topk)
    # most of the planted keys are in every row's top-k
    planted = ((idx >= 10000) & (idx < 10600)).sum(-1).float()
    assert float(planted.min()) > 300


@pytest.mark.parametrize("sampled_high", [True, False])
def test_wide_stream_threshold_miss_falls_back_exactly(sampled_high, cuda_device):
    # keys along q whose magnitudes make the sampled stages (positions p with
    # (p // 32) % 16 == 0 for Hkv = 4) all high (too few candidates) or all low
    # (too many): the rows are recomputed exactly, RoPE included
    B, Hq, Hkv, Sq, Sk, topk = 1, 28, 4, 8, 36000, 800
    q = torch.zeros(B, Hq, Sq, 128)
    q[..., 0] = 1.0
    q[..., 64] = 0.5
    pos = torch.arange(Sk)
    mask = (pos // 32) % 16 == 0
    gen = torch.Generator().manual_seed(9)
    mag = torch.rand(Hkv, Sk, generator=gen)
    mag = torch.where(mask[None, :], mag + (2.0 if sampled_high else -2.0), mag)
    raw = torch.zeros(B, Hkv, Sk, 128)
    raw[0, :, :, 0] = mag
    raw[0, :, :, 1:] = 0.01 * torch.randn(Hkv, Sk, 127, generator=gen)
    inv = W.rope_inv_freq(128, 1e6)
    cos, sin = W.rope_cos_sin(pos, inv)
    k = W.apply_rope(raw, cos, sin).to(torch.bfloat16).to(cuda_device)
    q = q.to(torch.bfloat16).to(cuda_device)
    idx, sc = einsum_topk_func(q, k, topk, inv_freq=inv.to(cuda_device), return_scores=True)
    check_parity(idx, sc, q, k, topk, inv.to(cuda_device))
