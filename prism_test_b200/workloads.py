"""Seeded synthetic inputs for the recall scorer's benchmark configurations.

No public dataset is involved: each configuration is the shape / distribution of
a ReAttention recall call (one layer, one decode step or one prefill chunk),
generated on the target device:

* queries ``q ~ N(0, 1)``, raw keys ``N(0, 1)`` or Student-t(3);
* optional outlier channels (4 per KV head, scaled x8);
* optional planted keys per query head whose raw score is ``+z`` standard
  deviations of that head's score distribution;
* cached keys = RoPE(raw keys) at absolute positions ``0 .. Sk-1`` with the HF
  ``rotate_half`` layout and fp32 angles ``fp32(pos) * inv_freq`` — the keys the
  reference un-rotates in ``ReAttentionMethod._unrotate_keys``
  (eval_harness/attention_methods/reattention.py:743-793) — stored in bf16;
  the prefill chunk keeps raw keys (no RoPE), as the exact method's cache does.

Key generation is chunked along the sequence with a per-chunk seed, so a
sequence shard ``[start, stop)`` can be generated on its own rank and equals
the same slice of the full sequence.
"""
from __future__ import annotations

import dataclasses
from typing import Dict, Optional

import torch

CHUNK = 1 << 16


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    B: int
    Hq: int
    Hkv: int
    Sq: int
    Sk: int
    theta: float
    topk: int
    dtype: torch.dtype = torch.bfloat16
    causal_offset: Optional[int] = None
    key_dist: str = "normal"          # "normal" | "student_t3"
    outlier_channels: int = 0         # per KV head, scaled by 8
    planted_per_qhead: int = 0
    planted_sigma: float = 6.0
    D: int = 128
    rope: bool = True                 # cached keys RoPE-rotated (else raw, pre-RoPE)

    @property
    def kv_bytes(self) -> int:
        """Bytes of cached K the scorer must read (2 bytes per element)."""
        return self.B * self.Hkv * self.Sk * self.D * 2

    def with_(self, **kw) -> "Workload":
        return dataclasses.replace(self, **kw)


WORKLOADS: Dict[str, Workload] = {
    # the reference's CPU-runnable case: decode, 16K keys
    "cpu-ref-16k": Workload("cpu-ref-16k", 1, 32, 8, 1, 16384, 5e5, 1024,
                            planted_per_qhead=16, planted_sigma=6.0),
    # decode top-k at 128K keys (single GPU headline)
    "decode-128k": Workload("decode-128k", 1, 32, 8, 1, 131072, 5e5, 4096,
                            outlier_channels=4, planted_per_qhead=16, planted_sigma=6.0),
    # prefill chunk: 4096 query rows against 128K keys, causal; raw (pre-RoPE) keys,
    # as the exact method's cache holds them (reattention_exact.py:545-547)
    "prefill-chunk-128k": Workload("prefill-chunk-128k", 1, 32, 8, 4096, 131072, 5e5, 2048,
                                   causal_offset=126976, rope=False),
    # the same chunk cut to its last 512 query rows (profiling-sized)
    "prefill-chunk-128k-512rows": Workload("prefill-chunk-128k-512rows", 1, 32, 8, 512, 131072,
                                           5e5, 2048, causal_offset=130560, rope=False),
    # the same chunk over a RoPE'd cache (keys un-rotated on the device first)
    "prefill-chunk-128k-rope": Workload("prefill-chunk-128k-rope", 1, 32, 8, 4096, 131072, 5e5, 2048,
                                        causal_offset=126976, rope=True),
    # 1M-key decode, sequence-sharded over N GPUs
    "decode-1m-sharded": Workload("decode-1m-sharded", 1, 32, 8, 1, 1 << 20, 5e5, 8192,
                                  planted_per_qhead=64, planted_sigma=5.0),
    # 8 questions sharing one 256K-key context, heavy-tailed keys (near-ties)
    "shared-context-256k": Workload("shared-context-256k", 1, 28, 4, 8, 262144, 1e6, 4096,
                                    key_dist="student_t3"),
}


def rope_inv_freq(D: int, theta: float) -> torch.Tensor:
    """HF default RoPE inverse frequencies, fp32 on the CPU:
    1 / theta ** (arange(0, D, 2) / D)."""
    return 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.int64).to(torch.float32) / D))


def rope_cos_sin(pos: torch.Tensor, inv_freq: torch.Tensor):
    """cos/sin [S, D] for positions ``pos`` (fp32 angles, HF duplicated halves)."""
    freqs = pos.to(torch.float32)[:, None] * inv_freq.to(pos.device, torch.float32)[None, :]
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos(), emb.sin()


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    half = x.shape[-1] // 2
    rot = torch.cat([-x[..., half:], x[..., :half]], dim=-1)
    return x * cos + rot * sin


def _gen(device, seed: int) -> torch.Generator:
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    return g


def _raw_key_chunk(wl: Workload, start: int, stop: int, device, seed: int) -> torch.Tensor:
    """Raw (pre-RoPE) fp32 keys for positions [start, stop), chunk-seeded."""
    parts = []
    c0 = start // CHUNK
    c1 = (stop - 1) // CHUNK
    for c in range(c0, c1 + 1):
        g = _gen(device, seed * 1_000_003 + 17 + c)
        n = min(CHUNK, wl.Sk - c * CHUNK)
        shape = (wl.B, wl.Hkv, n, wl.D)
        if wl.key_dist == "normal":
            x = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
        elif wl.key_dist == "student_t3":
            z = torch.randn(shape, generator=g, device=device, dtype=torch.float32)
            chi2 = torch.zeros(shape, device=device, dtype=torch.float32)
            for _ in range(3):
                chi2 += torch.randn(shape, generator=g, device=device, dtype=torch.float32) ** 2
            x = z / torch.sqrt(chi2 / 3.0)
        else:
            raise ValueError(wl.key_dist)
        lo = max(start, c * CHUNK) - c * CHUNK
        hi = min(stop, c * CHUNK + n) - c * CHUNK
        parts.append(x[:, :, lo:hi])
    return torch.cat(parts, dim=2) if len(parts) > 1 else parts[0]


def make_queries(wl: Workload, device, seed: int = 0) -> torch.Tensor:
    g = _gen(device, seed * 1_000_003 + 1)
    q = torch.randn((wl.B, wl.Hq, wl.Sq, wl.D), generator=g, device=device, dtype=torch.float32)
    return q.to(wl.dtype)


def _outlier_scale(wl: Workload, device, seed: int) -> torch.Tensor:
    """Per-(KV head, channel) multiplier [Hkv, D]."""
    scale = torch.ones((wl.Hkv, wl.D), dtype=torch.float32)
    if wl.outlier_channels:
        g = _gen("cpu", seed * 1_000_003 + 5)
        for h in range(wl.Hkv):
            ch = torch.randperm(wl.D, generator=g)[: wl.outlier_channels]
            scale[h, ch] = 8.0
    return scale.to(device)


def planted_positions(wl: Workload, seed: int = 0) -> torch.Tensor:
    """[Hkv, G * planted_per_qhead] distinct positions (CPU, int64)."""
    G = wl.Hq // wl.Hkv
    n = G * wl.planted_per_qhead
    g = _gen("cpu", seed * 1_000_003 + 7)
    out = torch.empty((wl.Hkv, n), dtype=torch.int64)
    for h in range(wl.Hkv):
        out[h] = torch.randperm(wl.Sk, generator=g)[:n]
    return out


def make_keys(wl: Workload, device, q: torch.Tensor, inv_freq: torch.Tensor,
              start: int = 0, stop: Optional[int] = None, seed: int = 0) -> torch.Tensor:
    """RoPE-rotated cached keys for positions [start, stop) in ``wl.dtype``."""
    stop = wl.Sk if stop is None else stop
    G = wl.Hq // wl.Hkv
    scale = _outlier_scale(wl, device, seed)
    var = scale.square()  # per-channel variance of the raw keys (normal case)
    planted = planted_positions(wl, seed) if wl.planted_per_qhead else None
    out = torch.empty((wl.B, wl.Hkv, stop - start, wl.D), dtype=wl.dtype, device=device)
    for c0 in range(start, stop, CHUNK):
        c1 = min(stop, c0 + CHUNK)
        raw = _raw_key_chunk(wl, c0, c1, device, seed) * scale[None, :, None, :]
        if planted is not None:
            qf = q.float()
            for hk in range(wl.Hkv):
                pos = planted[hk]
                sel = (pos >= c0) & (pos < c1)
                if not bool(sel.any()):
                    continue
                for slot in torch.nonzero(sel).flatten().tolist():
                    p = int(pos[slot])
                    hq = hk * G + slot // wl.planted_per_qhead
                    for b in range(wl.B):
                        qv = qf[b, hq, 0]
                        qn = qv / qv.norm()
                        sigma = torch.sqrt((qv.square() * var[hk]).sum())
                        z = wl.planted_sigma * sigma / qv.norm()
                        n = raw[b, hk, p - c0]
                        raw[b, hk, p - c0] = z * qn + (n - (n @ qn) * qn)
        if wl.rope:
            cos, sin = rope_cos_sin(torch.arange(c0, c1, device=device), inv_freq)
            raw = apply_rope(raw, cos, sin)
        out[:, :, c0 - start:c1 - start] = raw.to(wl.dtype)
    return out


def make_values(wl: Workload, device, start: int = 0, stop: Optional[int] = None,
                seed: int = 0) -> torch.Tensor:
    """Cached value rows [B, Hkv, stop - start, D] in ``wl.dtype`` for the
    value-weighted recall (qkv / qkv2): normal rows, each scaled by exp(0.7 z),
    z normal, so that the value norms vary by about 2x either way and change the
    selection. Chunk-seeded like the keys, so a shard is a slice of the whole."""
    stop = wl.Sk if stop is None else stop
    out = torch.empty((wl.B, wl.Hkv, stop - start, wl.D), dtype=wl.dtype, device=device)
    for c in range(start // CHUNK, (stop - 1) // CHUNK + 1):
        g = _gen(device, seed * 1_000_003 + 7_000_001 + c)
        n = min(CHUNK, wl.Sk - c * CHUNK)
        x = torch.randn((wl.B, wl.Hkv, n, wl.D), generator=g, device=device, dtype=torch.float32)
        x *= torch.exp(0.7 * torch.randn((wl.B, wl.Hkv, n, 1), generator=g, device=device))
        a, b = max(start, c * CHUNK), min(stop, c * CHUNK + n)
        out[:, :, a - start:b - start] = x[:, :, a - c * CHUNK:b - c * CHUNK].to(wl.dtype)
    return out


def make_inputs(wl: Workload, device, seed: int = 0, shard: Optional[tuple] = None) -> dict:
    """All inputs of one scorer call. ``shard=(rank, world)`` keeps only that
    rank's contiguous slice of the keys; ``pos_offset``/``index_base`` then give
    the slice's first absolute position / global index."""
    q = make_queries(wl, device, seed)
    inv_freq = rope_inv_freq(wl.D, wl.theta)
    start, stop = 0, wl.Sk
    if shard is not None:
        rank, world = shard
        per = wl.Sk // world
        assert per * world == wl.Sk, "Sk must divide evenly over the shards"
        start, stop = rank * per, (rank + 1) * per
    k = make_keys(wl, device, q, inv_freq.to(device), start, stop, seed)
    return dict(q=q, k=k, inv_freq=inv_freq.to(device) if wl.rope else None, pos_offset=start,
                index_base=start,
                topk=wl.topk, causal_offset=wl.causal_offset, start=start, stop=stop)


def small(wl: Workload, Sk: int, Sq: Optional[int] = None, topk: Optional[int] = None) -> Workload:
    """A reduced copy of a workload for quick parity checks."""
    Sq = wl.Sq if Sq is None else Sq
    topk = min(wl.topk if topk is None else topk, Sk)
    causal = None
    if wl.causal_offset is not None:
        causal = max(0, Sk - Sq)
    planted = min(wl.planted_per_qhead, max(0, Sk // (4 * (wl.Hq // wl.Hkv))))
    return wl.with_(name=wl.name + f"@{Sk}", Sk=Sk, Sq=Sq, topk=topk, causal_offset=causal,
                    planted_per_qhead=planted)


def algorithmic_bytes(wl: Workload) -> int:
    """HBM bytes the scorer must move per call: the cached keys once."""
    return wl.kv_bytes


def causal_flops(wl: Workload) -> float:
    """2*D*Hq*sum_i(visible keys of row i) (the dense bound when not causal)."""
    if wl.causal_offset is None:
        vis = wl.Sq * wl.Sk
    else:
        vis = sum(min(wl.Sk, wl.causal_offset + i + 1) for i in range(wl.Sq))
    return 2.0 * wl.D * wl.Hq * wl.B * vis

