#!/usr/bin/env python
"""Benchmark of the ReAttention recall scorer (un-rotate + q·K^T + exact top-k).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl prism|reference]
                    [--workload NAME]

Metric: KV tokens scored and top-k'd per second (keys of the cached sequence
processed per second, all heads), whole job.

The headline workload is ``decode-1m-sharded`` at every N (strong scaling on one
configuration): one decode step, 32 query / 8 KV heads, head_dim 128, 1,048,576
RoPE'd bf16 keys, k = 8192 per query head. At N = 1 one GPU holds the whole 2 GB
cache; at N > 1 (one process per GPU, launched by torchrun) the keys are split
evenly over the ranks and every rank's merge kernel reads the other ranks' sorted
runs from their GPUs over NVLink (peer-mapped buffers; ``--exchange nccl``: NCCL
all-gather, then merge).

The same line carries sub-records measured in the same run: ``decode_128k``
(N = 1 only: 131072 keys, k = 4096) and ``shared_context_256k`` (every N: 8
queries over 262144 Student-t keys, 28 / 4 heads, k = 4096, sequence-sharded at
N > 1). ``--workload NAME`` measures one workload alone.

A step is one full call of the op on resident inputs; W untimed steps, then K
steps timed with CUDA events between barriers, max over ranks. The key caches
(268 MB per rank at the least) are larger than the 126 MB L2, so no flush is
needed between steps. ``e2e`` repeats the K steps through the same public call
with pinned host inputs copied in and the result (indices + scores) copied out
inside the timed region. After the timed region every workload's result is
checked (``parity``): the ranks agree, a sharded result equals a one-GPU call
over the whole cache bit for bit, and whole rows match the CPU oracle under the
parity rules. ``--impl reference`` times the reference's dense PyTorch path
restated in the CPU oracle on the host cores (rank 0 only).
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "KV tokens scored+top-k'd/sec"
UNIT = "KV tokens/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="prism", choices=["prism", "reference"])
    ap.add_argument("--workload", default=None)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-sub", action="store_true",
                    help="measure the headline workload only (no decode_128k / shared_context_256k records)")
    ap.add_argument("--recall-type", default="qk", choices=["qk", "qkv", "qkv2"],
                    help="value-norm weighting of the keys (qkv: L1, qkv2: L2)")
    ap.add_argument("--chunks", type=int, default=0,
                    help="sharded path: groups of KV heads whose exchange is pipelined "
                         "(0: 2 when the KV heads split evenly, else 1)")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="sharded path: peer: runs read over NVLink from peer-mapped buffers; "
                         "nccl: all-gather of the runs, then a local merge")
    ap.add_argument("--stage", default="recall", choices=["recall", "attention", "merge"],
                    help="attention: time the attention over a selected view instead of the recall; "
                         "merge: time the sharded path's run merge for N ranks on one GPU (--runs)")
    ap.add_argument("--runs", type=int, default=8,
                    help="merge stage: number of sorted runs (the ranks of the sharded decode)")
    return ap.parse_args()


def run_merge(args):
    """The sharded path's run merge on one GPU: the top-k of --runs sorted runs per row,
    each the local top-k of one rank of decode-1m-sharded (32 rows, k = 8192, distinct
    global indices, scores of a normal score tail), in the gathered layout
    [runs, 2, rows, k]. The work of each rank's merge kernel in the N-GPU step, without
    the interconnect."""
    from prism_test_b200 import _lib, topk_merge_runs
    from prism_test_b200 import workloads as W
    dev = torch.device("cuda", 0)
    wl = W.WORKLOADS[args.workload or "decode-1m-sharded"]
    nruns, rows, k = args.runs, wl.B * wl.Hq * wl.Sq, wl.topk
    g = torch.Generator(device=dev).manual_seed(3)
    s = torch.randn(nruns, rows, k, generator=g, device=dev).sort(dim=-1, descending=True).values
    idx = (torch.arange(nruns * k, device=dev, dtype=torch.int32).view(nruns, 1, k)
           .expand(nruns, rows, k).contiguous())
    runs = torch.stack([s.view(torch.int32), idx], dim=1).contiguous()
    lib = _lib.load()
    step = lambda: topk_merge_runs(runs, k)  # noqa: E731
    for _ in range(max(3, args.warmup)):
        oi, os_ = step()
    torch.cuda.synchronize()
    ref = s.permute(1, 0, 2).reshape(rows, -1).topk(k, dim=-1).values
    if not torch.equal(os_, ref):
        raise SystemExit("run merge result differs from torch.topk over the union")
    lib.prism_profile_start(args.steps + 16)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    lib.prism_profile_stop()
    n_m = _lib.ctypes.c_int64(0)
    t_m = _lib.ctypes.c_double(0.0)
    lib.prism_profile_read(_lib.KERNEL_MERGE, _lib.ctypes.byref(n_m), _lib.ctypes.byref(t_m))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    line = {
        "metric": "run-merge candidates/sec", "value": nruns * rows * k * args.steps / (ms * 1e-3),
        "unit": "candidates/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "u64 keys (fp32 score, int32 index)", "data": "synthetic",
        "config": {"workload": wl.name, "stage": "run merge", "runs": nruns, "rows": rows, "topk": k},
        "launch_ms": t_m.value / max(1, n_m.value),
        "gpu_launches": args.steps, "timing": "CUDA graph of one call, replayed",
    }
    print(json.dumps(line), flush=True)
    return 0


def run_attention(args):
    """Attention over a selected view on one GPU: the step after the recall in the
    exact method. The view of a decode step on the workload's cache: 32 global
    positions, 4096 recalled middle positions, the 4096-position local window."""
    from prism_test_b200 import _lib, sparse_attention
    from prism_test_b200 import workloads as W
    dev = torch.device("cuda", 0)
    wl = W.WORKLOADS[args.workload or "decode-128k"]
    lib = _lib.load()
    g = torch.Generator(device=dev).manual_seed(1)
    q = torch.randn(wl.B, wl.Hq, 1, wl.D, generator=g, device=dev).to(wl.dtype)
    k = torch.randn(wl.B, wl.Hkv, wl.Sk, wl.D, generator=g, device=dev).to(wl.dtype)
    v = torch.randn(wl.B, wl.Hkv, wl.Sk, wl.D, generator=g, device=dev).to(wl.dtype)
    loc, glob, mid = 4096, 32, 4096
    middle = torch.randperm(wl.Sk - glob - loc, generator=g, device=dev)[:mid].sort().values + glob
    key_pos = torch.cat([torch.arange(glob, device=dev), middle,
                         torch.arange(wl.Sk - loc, wl.Sk, device=dev)])
    inv = W.rope_inv_freq(wl.D, wl.theta).to(dev)
    step = lambda: sparse_attention(q, k, v, key_pos, inv_freq=inv, pe_original=True)  # noqa: E731
    for _ in range(max(3, args.warmup)):
        step()
    torch.cuda.synchronize()
    lib.prism_profile_start(2 * args.steps + 16)
    for _ in range(args.steps):
        step()
    torch.cuda.synchronize()
    lib.prism_profile_stop()
    n_a = _lib.ctypes.c_int64(0)
    t_a = _lib.ctypes.c_double(0.0)
    lib.prism_profile_read(_lib.KERNEL_ATTN, _lib.ctypes.byref(n_a), _lib.ctypes.byref(t_a))
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1)
    nsel = key_pos.numel()
    bytes_per_call = nsel * wl.B * wl.Hkv * wl.D * 2 * 2  # gathered key and value rows
    launch_ms = t_a.value / max(1, n_a.value)
    peak, peak_kind = measured_peaks()
    achieved = bytes_per_call / (launch_ms * 1e-3) / 1e9
    line = {
        "metric": "view KV tokens attended/sec", "value": nsel * args.steps / (ms * 1e-3),
        "unit": "KV tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup),
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32 (bf16 in)", "data": "synthetic",
        "config": {"workload": wl.name, "stage": "attention over the selected view",
                   "view": {"global": glob, "recalled": mid, "local": loc}, "q_len": 1},
        "roofline": {"bound": "hbm", "unit": "GB/s", "bytes_per_launch": bytes_per_call,
                     "achieved": achieved, "peak": peak, "frac": achieved / peak,
                     "peak_source": peak_kind, "launch_ms": launch_ms},
        # per call: the RoPE angle table, the split partials, the split merge
        "gpu_launches": 3 * args.steps, "timing": "CUDA graph of one call, replayed",
    }
    print(json.dumps(line), flush=True)
    return 0


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def pick_workload(args, world):
    from prism_test_b200 import workloads as W
    name = args.workload or "decode-1m-sharded"
    return W.WORKLOADS[name]


def config_of(wl, world, recall_type="qk", exchange="peer"):
    return {
        "workload": wl.name, "B": wl.B, "Hq": wl.Hq, "Hkv": wl.Hkv, "Sq": wl.Sq, "Sk": wl.Sk,
        "topk": wl.topk, "head_dim": wl.D, "rope_theta": wl.theta, "key_dtype": "bf16",
        "causal_offset": wl.causal_offset, "shards": world,
        "parallelism": "single GPU" if world == 1 else
                       f"sequence-sharded x{world} (" + (
                           "peer-mapped exchange over NVLink: each rank's merge kernel reads the other ranks' "
                           "runs from their GPUs" if exchange == "peer" else
                           "NCCL all-gather pipelined over KV-head groups + device merge") + ")",
        "l2": "inputs larger than L2 (cached keys %d MB per rank > 126 MB), no flush" % (wl.kv_bytes // world >> 20),
        "recall_type": recall_type,
    }


# ---------------------------------------------------------------- clocks (NVML)
class ClockSampler:
    """Samples SM clock and throttle reasons on a background thread."""

    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
        0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
        0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
    }

    def __init__(self, index: int, period_s: float = 0.002):
        self.ok = False
        self.samples = []
        self.reasons = 0
        self.period = period_s
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:  # noqa: BLE001
            self.max_mhz = None

    def _sample(self):
        self.samples.append(self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM))
        try:
            self.reasons |= int(self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
        except Exception:  # noqa: BLE001
            self.reasons |= int(self.nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h))

    def _loop(self):
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def start(self):
        if not self.ok:
            return
        self._stop = threading.Event()
        self._sample()
        self.t = threading.Thread(target=self._loop, daemon=True)
        self.t.start()

    def stop(self):
        if not self.ok:
            return
        self._stop.set()
        self.t.join()
        self._sample()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        names = [n for b, n in self.REASONS.items() if self.reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


def measured_peaks(kind: str = "hbm_gbs"):
    """A measured peak (hbm_gbs, bf16_tflops or bf16_tflops_sustained) and its source."""
    fallback = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            d = json.loads(p.read_text())
            return float(d[kind]), "measured"
        except Exception:  # noqa: BLE001
            pass
    return fallback[kind], "fallback"


def prefill_flops(wl) -> float:
    """Algorithmic FLOPs of one prefill-chunk call: 2 * D per (query row, visible key)."""
    vis = 0
    for s in range(wl.Sq):
        n = wl.Sk if wl.causal_offset is None else min(wl.Sk, wl.causal_offset + s + 1)
        vis += max(0, n)
    return 2.0 * wl.D * wl.B * wl.Hq * vis


def ncu_traffic(kernel: str, workload: str):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, if any."""
    p = ROOT / "profiles" / "traffic.json"
    if not p.exists():
        return None
    try:
        d = json.loads(p.read_text())
        return d.get(workload, {}).get(kernel)
    except Exception:  # noqa: BLE001
        return None


# ---------------------------------------------------------------- CPU baseline
def cpu_sample_plan(wl, whole_heads: int):
    """(sub-workload, fraction of the whole call it is, description) of a bounded CPU
    sample. Prefill chunks (Sq >= 128): the 128 query rows of the last 32 positions of
    one KV head's group (the rows that see the most keys), extrapolated linearly over
    the rows — the full score matrix would not fit in host memory. Otherwise
    `whole_heads` KV heads with their query groups."""
    if wl.Sq >= 128:
        G = wl.Hq // wl.Hkv
        rows = 32
        causal = None if wl.causal_offset is None else wl.causal_offset + wl.Sq - rows
        sub = wl.with_(Hkv=1, Hq=G, Sq=rows, causal_offset=causal, planted_per_qhead=0)
        frac = G * rows / (wl.B * wl.Hq * wl.Sq)
        return sub, frac, (f"{G * rows} of {wl.B * wl.Hq * wl.Sq} query rows (the last {rows} "
                           f"positions of one KV head group), extrapolated")
    sub = wl.with_(Hkv=whole_heads, Hq=whole_heads * (wl.Hq // wl.Hkv))
    frac = whole_heads / wl.Hkv
    return sub, frac, ("full call" if whole_heads == wl.Hkv else f"{whole_heads} of {wl.Hkv} KV heads")


def cpu_baseline(wl, max_seconds=20.0, recall_type="qk"):
    """The reference's dense CPU path (oracle restatement) on the host cores.

    Runs whole calls (or, when one call would exceed the budget, one KV head of
    it and scales by the number of KV heads) and returns KV tokens/s."""
    from oracle import reattention_topk as orc
    from prism_test_b200 import workloads as W
    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    heads = wl.Hkv if wl.Sk * wl.Sq <= (1 << 17) * 8 else 1
    sub, frac, what = cpu_sample_plan(wl, heads)
    x = W.make_inputs(sub, "cpu")
    v = W.make_values(sub, "cpu") if recall_type != "qk" else None

    def call():
        w = orc.recall_weights(v, recall_type)
        orc.dense_topk(x["q"], x["k"], sub.topk, x["inv_freq"], 0, sub.causal_offset, weights=w)

    call()  # warm-up
    times = []
    t_budget = time.perf_counter()
    while len(times) < 5 and time.perf_counter() - t_budget < max_seconds:
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
    best = min(times)
    value = wl.Sk * frac / best
    sample = (f"{what} of {wl.name} "
              f"({'un-rotate fp32, ' if wl.rope else ''}{'value norms, ' if recall_type != 'qk' else ''}"
              f"einsum, topk), best of {len(times)} after 1 warm-up")
    return {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample,
            "seconds_per_call": best / frac}


def run_reference(args):
    world, rank, _ = dist_env()
    if rank != 0:
        return 0
    wl = pick_workload(args, world)
    from oracle import reattention_topk as orc
    from prism_test_b200 import workloads as W
    torch.set_num_threads(os.cpu_count() or 1)
    cores = torch.get_num_threads()
    # bounded sample per step: one KV head (and its query group) of the workload
    sub, frac, what = cpu_sample_plan(wl, 1)
    x = W.make_inputs(sub, "cpu")
    rt = args.recall_type
    v = W.make_values(sub, "cpu") if rt != "qk" else None

    def call():
        w = orc.recall_weights(v, rt)
        orc.dense_topk(x["q"], x["k"], sub.topk, x["inv_freq"], 0, sub.causal_offset, weights=w)

    steps, warm = max(1, args.steps), max(0, args.warmup)
    est = None
    for _ in range(max(1, warm)):
        t0 = time.perf_counter()
        call()
        est = time.perf_counter() - t0
    # keep the whole run within a few minutes
    steps = min(steps, max(3, int(120.0 / max(est, 1e-3))))
    t0 = time.perf_counter()
    for _ in range(steps):
        call()
    dt = (time.perf_counter() - t0) / steps
    value = wl.Sk * frac / dt  # KV tokens (the whole call) per second
    sample = (f"{what} of {wl.name} per step ({'un-rotate fp32, ' if wl.rope else ''}einsum, topk); "
              f"{steps} steps")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": warm, "ms_per_step": dt * 1e3, "higher_is_better": True,
        "scaling": "strong" if wl.name == "decode-1m-sharded" or world > 1 else "weak", "vs_baseline": None,
        "dtype": "f32 (host cores)",
        "data": "synthetic", "config": config_of(wl, world, rt, args.exchange),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------- GPU arm
# (name in kernels_ms_per_step, kernel id of the library's profiling aid)
KERNEL_IDS = (("score", "KERNEL_SCORE"), ("select", "KERNEL_SELECT"), ("merge", "KERNEL_MERGE"),
              ("value_norms", "KERNEL_WEIGHT"), ("score_weighting", "KERNEL_SCALE"),
              ("threshold", "KERNEL_THRESHOLD"), ("unrotate", "KERNEL_UNROTATE"))


class Ranks:
    """This process's place in the job (one process per GPU) and the helpers that
    every rank calls in the same order."""

    def __init__(self, world, rank, local, dev):
        self.world, self.rank, self.local, self.dev = world, rank, local, dev

    def barrier(self):
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        import torch.distributed as dist
        t = torch.tensor([v], device=self.dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def all_equal(self, t: torch.Tensor) -> bool:
        """Whether every rank holds the same small int64 tensor."""
        if self.world == 1:
            return True
        import torch.distributed as dist
        hi, lo = t.clone(), t.clone()
        dist.all_reduce(hi, op=dist.ReduceOp.MAX)
        dist.all_reduce(lo, op=dist.ReduceOp.MIN)
        return bool(torch.equal(hi, lo))


def kernel_times(lib):
    """{name: (launches, total ms)} of the library's event pairs since profiling started."""
    import ctypes
    from prism_test_b200 import _lib
    out = {}
    for name, attr in KERNEL_IDS:
        n, t = ctypes.c_int64(0), ctypes.c_double(0.0)
        lib.prism_profile_read(getattr(_lib, attr), ctypes.byref(n), ctypes.byref(t))
        out[name] = (n.value, t.value)
    return out


def result_check(wl, ranks: Ranks, x: dict, v, idx, sc, recall_type: str, budget_s: float = 60.0) -> dict:
    """The result of one step, checked after the timed region:

    * every rank holds the same result (checksums compared over the process group);
    * at N > 1, rank 0 regenerates the whole key cache from the same seeds and the
      sharded result must equal a one-GPU call over it bit for bit (same scores for
      the same keys, ties toward lower indices);
    * rank 0 checks whole query-head groups of rows, one KV head at a time, spread
      over the heads, against the CPU oracle with the parity rules (scores within
      1e-3, index sets equal up to near-ties at the k-th score), until the budget
      is spent (at least one KV head)."""
    from prism_test_b200 import einsum_topk_func
    from prism_test_b200 import workloads as W
    rows = idx.numel() // wl.topk
    ck = torch.stack([idx.long().sum(), sc.view(torch.int32).long().sum(),
                      (idx.reshape(rows, -1)[:, ::97].long() * 131).sum()])
    out = {"rows": rows, "ranks_agree": ranks.all_equal(ck)}
    if ranks.rank != 0:
        return out
    t0 = time.perf_counter()
    q, k, vv, inv = x["q"], x["k"], v, x["inv_freq"]
    if ranks.world > 1:
        full = W.make_inputs(wl, ranks.dev)
        q, k, inv = full["q"], full["k"], full["inv_freq"]
        vv = W.make_values(wl, ranks.dev) if recall_type != "qk" else None
        ri, rs = einsum_topk_func(q, k, wl.topk, inv_freq=inv, return_scores=True,
                                  causal_offset=wl.causal_offset, values=vv, recall_type=recall_type)
        torch.cuda.synchronize()
        out["bitwise_equal_single_gpu"] = bool(torch.equal(ri, idx) and torch.equal(rs, sc))
        del ri, rs
    from oracle import reattention_topk as orc
    from oracle.parity import REL, REL_WEIGHTED, check_parity
    G = wl.Hq // wl.Hkv
    order = []
    for h in [0, wl.Hkv - 1] + list(range(wl.Hkv // 2, wl.Hkv - 1)) + list(range(1, wl.Hkv // 2)):
        if 0 <= h < wl.Hkv and h not in order:
            order.append(h)
    checked, swaps, worst, err = 0, 0, 0.0, None
    inv_c = inv.cpu() if inv is not None else None
    for h in order:
        if checked and time.perf_counter() - t0 > budget_s:
            break
        sl = slice(h * G, (h + 1) * G)
        w = orc.recall_weights(vv[:, h:h + 1].cpu(), recall_type) if recall_type != "qk" else None
        try:
            st = check_parity(idx[:, sl], sc[:, sl], q[:, sl].cpu(), k[:, h:h + 1].cpu(), wl.topk,
                              inv_c, 0, wl.causal_offset, 0,
                              rel=REL if recall_type == "qk" else REL_WEIGHTED, weights=w)
        except AssertionError as e:  # noqa: PERF203
            err = f"KV head {h}: {str(e)[:300]}"
            checked += wl.B * G * wl.Sq
            break
        checked += st["rows"]
        swaps += st["swapped"]
        worst = max(worst, st["max_rel_err"])
    ok = err is None and out["ranks_agree"] and out.get("bitwise_equal_single_gpu", True)
    out.update({"rows_checked": checked, "near_tie_swaps": swaps, "max_rel_err": worst, "ok": bool(ok),
                "rule": "scores within 1e-3 of the fp32 oracle (x max(|s|, ||q|| ||k||)); index sets "
                        "equal up to near-ties at the k-th score",
                "seconds": round(time.perf_counter() - t0, 1)})
    if err:
        out["error"] = err
    return out


def measure(wl, args, ranks: Ranks, *, e2e: bool, cpu_base: bool, clocks_on: bool) -> dict:
    """One workload on every rank: W warm-up steps, a profiling pass (every library
    launch between its own pair of events), then K steps as replays of a CUDA graph of
    one call (host Python/ctypes overhead would otherwise starve the device), timed
    between CUDA events with all ranks entering together, max over ranks; then, if
    asked, the end-to-end pass and the CPU baseline; then the result check."""
    from prism_test_b200 import _lib, einsum_topk_func
    from prism_test_b200 import workloads as W
    from prism_test_b200.sharded import shard_bounds, sharded_einsum_topk
    lib = _lib.load()
    world, rank, dev = ranks.world, ranks.rank, ranks.dev
    start, stop = shard_bounds(wl.Sk, rank, world)
    x = W.make_inputs(wl, dev, shard=(rank, world) if world > 1 else None)
    q, k, inv = x["q"], x["k"], x["inv_freq"]
    rt = args.recall_type
    v = W.make_values(wl, dev, start, stop) if rt != "qk" else None
    exchange = None
    if world > 1 and args.exchange == "peer":
        from prism_test_b200.peer_exchange import PeerExchange
        exchange = PeerExchange(wl.B * wl.Hq * wl.Sq, wl.topk, dev)
    chunks = 1 if exchange is not None else (args.chunks or (2 if wl.Hkv % 2 == 0 else 1))

    def step(qq, kk, vv=v):
        if world == 1:
            return einsum_topk_func(qq, kk, wl.topk, inv_freq=inv, return_scores=True,
                                    causal_offset=wl.causal_offset, values=vv, recall_type=rt)
        return sharded_einsum_topk(qq, kk, wl.topk, shard_start=start, inv_freq=inv, return_scores=True,
                                   v_shard=vv, recall_type=rt, chunks=chunks, exchange=exchange)

    warm = max(3, args.warmup)
    for _ in range(warm):
        step(q, k)
    torch.cuda.synchronize()
    ranks.barrier()
    torch.cuda.synchronize()

    # per-kernel device times: every launch bracketed by events (profiling mode)
    lib.prism_profile_start(8 * args.steps + 16)
    n0 = lib.prism_launch_count()
    for _ in range(args.steps):
        step(q, k)
    torch.cuda.synchronize()
    lib.prism_profile_stop()
    launches_per_step = (lib.prism_launch_count() - n0) / args.steps
    ktimes = kernel_times(lib)
    ranks.barrier()
    torch.cuda.synchronize()

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(2):
            step(q, k)
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step(q, k)
    for _ in range(3):
        graph.replay()
    torch.cuda.synchronize()
    if exchange is not None:
        exchange.timings(reset=True)
    clocks = ClockSampler(ranks.local) if clocks_on else None
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    if clocks:
        clocks.start()
    torch.cuda.synchronize()
    ranks.barrier()  # every rank enters the timed region together
    torch.cuda.synchronize()
    ev0.record()
    for _ in range(args.steps):
        graph.replay()
    ev1.record()
    torch.cuda.synchronize()
    if clocks:
        clocks.stop()
    ranks.barrier()
    torch.cuda.synchronize()
    ms = ranks.max(ev0.elapsed_time(ev1))
    del graph  # a graph holding NCCL work must go before the process group
    torch.cuda.synchronize()
    xtime = None
    if exchange is not None:
        # device time per merge in the timed steps, the slowest rank's
        tm = exchange.timings(reset=True)
        xtime = {key: ranks.max(tm[key]) for key in ("wait_us", "merge_us", "ack_us")}
        xtime["what"] = ("per peer merge, slowest rank: waiting for every rank's run from the merge's "
                         "start, merging, waiting for the acknowledgements (%globaltimer)")

    n_sc, t_sc = ktimes["score"]
    score_ms = ranks.max(t_sc / max(1, n_sc))  # the slowest rank's scorer launch
    res = {"wl": wl, "start": start, "stop": stop, "ms": ms, "ms_per_step": ms / args.steps,
           "score_ms": score_ms,
           "value": wl.Sk * args.steps / (ms * 1e-3), "launches": int(round(launches_per_step * args.steps)),
           "launches_per_step": launches_per_step, "ktimes": ktimes,
           "clocks": clocks.summary() if clocks else None, "chunks": chunks,
           "exchange": "peer" if exchange is not None else ("nccl" if world > 1 else None),
           "exchange_timing": xtime}

    # ---- end to end through the public call, host buffers ----
    if e2e:
        q_h = q.cpu().pin_memory()
        k_h = k.cpu().pin_memory()
        rows = wl.B * wl.Hq * wl.Sq
        idx_h = torch.empty((rows * wl.topk,), dtype=torch.int32).pin_memory()
        sc_h = torch.empty((rows * wl.topk,), dtype=torch.float32).pin_memory()
        q_d = torch.empty_like(q)
        k_d = torch.empty_like(k)
        v_h = v.cpu().pin_memory() if v is not None else None
        v_d = torch.empty_like(v) if v is not None else None

        def e2e_step():
            q_d.copy_(q_h, non_blocking=True)
            k_d.copy_(k_h, non_blocking=True)
            if v_d is not None:
                v_d.copy_(v_h, non_blocking=True)
            oi, os_ = step(q_d, k_d, v_d)
            idx_h.copy_(oi.reshape(-1), non_blocking=True)
            sc_h.copy_(os_.reshape(-1), non_blocking=True)

        for _ in range(2):
            e2e_step()
        torch.cuda.synchronize()
        ranks.barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize()
        ranks.barrier()
        torch.cuda.synchronize()
        ems = ranks.max(e0.elapsed_time(e1))
        res["e2e"] = {"value": wl.Sk * args.steps / (ems * 1e-3), "unit": UNIT,
                      "h2d_bytes_per_step": int(q_h.numel() * q_h.element_size() + k_h.numel() * k_h.element_size()
                                                + (v_h.numel() * v_h.element_size() if v_h is not None else 0)) * world,
                      "d2h_bytes_per_step": int(idx_h.numel() * 4 + sc_h.numel() * 4) * world,
                      "ms_per_step": ems / args.steps}
        del q_h, k_h, v_h, q_d, k_d, v_d

    if cpu_base and rank == 0 and world == 1:
        res["cpu_baseline"] = cpu_baseline(wl, recall_type=rt)

    # ---- the result of one more step, checked (not timed) ----
    idx, sc = step(q, k)
    torch.cuda.synchronize()
    res["parity"] = result_check(wl, ranks, x, v, idx, sc, rt)
    if exchange is not None:
        res["exchange_status"] = int(ranks.max(float(exchange.status())))
        exchange.close()
    del x, q, k, v, idx, sc
    torch.cuda.empty_cache()
    return res


def path_of(wl, rt="qk", sk=None) -> str:
    """The library path a workload takes (the dispatch of prism_einsum_topk in exact
    mode): "prefill" (Sq >= 128: tcgen05 candidate pass, tensor-bound), "wide" (many
    query rows share one long context: tcgen05 queries-as-M candidate pass, HBM-bound)
    or "decode" (the streaming decode scorer). ``sk``: the keys of this rank's shard."""
    sk = wl.Sk if sk is None else sk
    if wl.Sq >= 128:
        return "prefill"
    rows = wl.B * wl.Hq * wl.Sq
    if (rt == "qk" and wl.Sq >= 2 and rows >= 64 and sk >= 32768 and wl.topk <= 4096
            and wl.topk * 16 <= sk and wl.Hkv in (2, 4) and wl.Hq // wl.Hkv * wl.Sq <= 64):
        return "wide"
    return "decode"


def dtype_of(wl, rt="qk", sk=None) -> str:
    return {"prefill": "bf16 in, fp32 accumulate (tcgen05)",
            "wide": "fp32 keys as bf16 hi + lo, fp32 accumulate (tcgen05)",
            "decode": "f32 (tf32 MMA)"}[path_of(wl, rt, sk)]


def roofline_of(res, rt="qk") -> tuple:
    """(roofline of the dominant kernel, roofline of the whole step) of one measurement."""
    wl = res["wl"]
    score_ms = res["score_ms"]
    prefill = wl.Sq >= 128  # the tcgen05 path: tensor-bound
    if prefill:
        work = prefill_flops(wl)
        peak, src = measured_peaks("bf16_tflops_sustained")
        achieved = work / (score_ms * 1e-3) / 1e12
        roof = {"bound": "tensor", "unit": "TFLOP/s", "flops_per_launch": work,
                "kernel": "prefill candidate pass (tcgen05 kind::f16 M128 N128, TMEM accumulators, "
                          "threshold epilogue" + (", hi + lo un-rotated key planes: twice the MMAs of the "
                                                  "FLOPs counted)" if wl.rope else ")"),
                "peak_note": "sustained bf16 GEMM peak: the kernel runs inside a long step loop"}
        step_work = work
        step_achieved = work / (res["ms_per_step"] * 1e-3) / 1e12
    else:
        work = (res["stop"] - res["start"]) * wl.B * wl.Hkv * wl.D * 2  # keys of this rank, read once
        peak, src = measured_peaks()
        achieved = work / (score_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "unit": "GB/s", "bytes_per_launch": work,
                "kernel": ("queries-as-M candidate pass (tcgen05 kind::f16 M128 N64, query rows in "
                           "TMEM, keys un-rotated once into bf16 hi + lo tiles, threshold epilogue)"
                           if path_of(wl, rt, res["stop"] - res["start"]) == "wide" else
                           "decode scorer (TMA ring, fused inverse RoPE, fp32 q·K^T)")}
        step_work = work
        step_achieved = work / (res["ms_per_step"] * 1e-3) / 1e9
    roof.update(achieved=achieved, peak=peak, frac=achieved / peak, peak_source=src,
                traffic=ncu_traffic("score", wl.name) if res["stop"] - res["start"] == wl.Sk else None,
                launch_ms=score_ms)
    step_roof = {"what": "the whole step (score + select (+ exchange and merge)) against the same "
                         "algorithmic work and peak", "achieved": step_achieved, "peak": peak,
                 "unit": roof["unit"], "frac": step_achieved / peak, "work_per_step": step_work}
    return roof, step_roof


def kernels_ms(res, steps):
    return {name: t / max(1, steps) for name, (n, t) in res["ktimes"].items()}


def sub_record(res, args) -> dict:
    """A compact record of a secondary workload measured in the same run."""
    wl = res["wl"]
    roof, step_roof = roofline_of(res, args.recall_type)
    return {"workload": wl.name, "value": res["value"], "unit": UNIT, "ms_per_step": res["ms_per_step"],
            "dtype": dtype_of(wl, args.recall_type, res["stop"] - res["start"]),
            "config": config_of(wl, res_world(res), args.recall_type, res["exchange"] or "peer"),
            "roofline": roof, "step_roofline": step_roof, "kernels_ms_per_step": kernels_ms(res, args.steps),
            "gpu_launches_per_step": res["launches_per_step"], "parity": res["parity"],
            **({"exchange_timing": res["exchange_timing"]} if res.get("exchange_timing") else {}),
            **({"exchange_status": res["exchange_status"]} if "exchange_status" in res else {})}


def res_world(res):
    wl = res["wl"]
    return max(1, wl.Sk // max(1, res["stop"] - res["start"]))


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.stage == "attention":
        return run_attention(args)
    if args.stage == "merge":
        return run_merge(args)
    world, rank, local = dist_env()
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torchrun")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        # generous: rank 0 checks the result against the CPU oracle while the others wait
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=600))
    from prism_test_b200 import workloads as W
    ranks = Ranks(world, rank, local, dev)
    rt = args.recall_type
    wl = pick_workload(args, world)
    main_res = measure(wl, args, ranks, e2e=not args.no_e2e, cpu_base=not args.no_cpu_baseline, clocks_on=True)
    subs = {}
    if args.workload is None and not args.no_sub:
        # the 128K decode step at N = 1, and the shared-context workload at every N
        names = (["decode-128k"] if world == 1 else []) + ["shared-context-256k"]
        for name in names:
            subs[name.replace("-", "_")] = sub_record(
                measure(W.WORKLOADS[name], args, ranks, e2e=False, cpu_base=False, clocks_on=False), args)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    roof, step_roof = roofline_of(main_res, rt)
    line = {
        "metric": METRIC, "value": main_res["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": max(3, args.warmup), "ms_per_step": main_res["ms_per_step"], "higher_is_better": True,
        "scaling": "strong" if wl.name == "decode-1m-sharded" or world > 1 else "weak", "vs_baseline": None,
        "dtype": dtype_of(wl, rt, main_res["stop"] - main_res["start"]),
        "data": "synthetic (seeded; see prism_test_b200/workloads.py)",
        "config": config_of(wl, world, rt, main_res["exchange"] or "peer"),
        "roofline": roof,
        "step_roofline": step_roof,
        "kernels_ms_per_step": kernels_ms(main_res, args.steps),
        "gpu_launches": main_res["launches"],
        "timing": "CUDA graph of one call, replayed",
        "clocks": main_res["clocks"],
        "e2e": main_res.get("e2e"),
        "cpu_baseline": main_res.get("cpu_baseline"),
        "parity": main_res["parity"],
    }
    if "exchange_status" in main_res:
        line["exchange_status"] = main_res["exchange_status"]  # 0: every bounded peer wait succeeded
    if main_res.get("exchange_timing"):
        line["exchange_timing"] = main_res["exchange_timing"]
    line.update(subs)
    print(json.dumps(line), flush=True)
    ok = main_res["parity"]["ok"] and all(s["parity"].get("ok", False) for s in subs.values())
    return 0 if ok else 1


if __name__ == "__main__":
    sys.exit(main())
