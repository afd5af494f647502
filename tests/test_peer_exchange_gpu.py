"""The run merge of the sequence-sharded path and its peer exchange on the GPU.

* prism_topk_merge_runs on edge cases: equal scores across runs, duplicate
  (-inf, INT32_MAX) padding entries, k below the summary width, 16 runs, runs
  longer than k, and ties at the threshold that overflow the shared-memory staging.
  The expected result is torch.topk over the union (reattention.py:497) with ties
  toward the lower index, as the single-GPU path returns it.
* prism_peer_publish / prism_peer_merge with the ranks emulated on one GPU (their
  buffers side by side; every wait is already satisfied when it starts: every
  rank publishes before any merge, and only the last merge waits for the acks,
  which the earlier merges have sent), over several steps.
* A ready flag that nothing sets: the bounded wait expires and the status word
  reports it (the kernel returns; the context stays usable).
* Two real ranks on two GPUs (CUDA IPC mappings, NCCL for the handles), when the
  machine has them: the sharded call with the peer exchange against both shards'
  local top-k merged on one GPU, eagerly and replayed from a CUDA graph.
"""
import ctypes
import datetime
import os
import socket
import traceback

import pytest
import torch

from prism_test_b200 import _lib, einsum_topk_func, topk_merge_runs
from prism_test_b200 import workloads as W
from prism_test_b200.peer_exchange import _DeviceArray

pytestmark = pytest.mark.gpu

INT32_MAX = torch.iinfo(torch.int32).max


def _sorted_runs(s: torch.Tensor, idx: torch.Tensor):
    """Sort every run's rows by (score desc, index asc); [nruns, rows, len] each."""
    order = torch.argsort(idx.long(), dim=-1, stable=True)
    s, idx = torch.gather(s, -1, order), torch.gather(idx, -1, order)
    v, p = torch.sort(s, dim=-1, descending=True, stable=True)
    return v, torch.gather(idx, -1, p)


def _expected(v: torch.Tensor, idx: torch.Tensor, topk: int):
    nruns, rows, n = v.shape
    fs = v.permute(1, 0, 2).reshape(rows, -1)
    fi = idx.permute(1, 0, 2).reshape(rows, -1)
    o = torch.argsort(fi.long(), dim=-1, stable=True)
    fs, fi = torch.gather(fs, -1, o), torch.gather(fi, -1, o)
    ws, wp = torch.sort(fs, dim=-1, descending=True, stable=True)
    return ws[:, :topk], torch.gather(fi, -1, wp)[:, :topk]


def _runs(nruns, rows, run_len, seed, kind="normal", pad=0):
    g = torch.Generator().manual_seed(seed)
    if kind == "normal":
        s = torch.randn(nruns, rows, run_len, generator=g)
    elif kind == "ties":  # few distinct values: many equal scores across runs
        s = torch.randint(-3, 4, (nruns, rows, run_len), generator=g).float()
    elif kind == "flat":  # every score equal: the threshold ties everything
        s = torch.zeros(nruns, rows, run_len)
    else:
        raise ValueError(kind)
    perm = torch.randperm(nruns * run_len * 2, generator=g)[: nruns * run_len].view(nruns, 1, run_len)
    idx = perm.expand(nruns, rows, run_len).to(torch.int32).clone()
    v, idx = _sorted_runs(s, idx)
    if pad:  # the last `pad` entries of every run: a shard shorter than k
        v[:, :, run_len - pad:] = float("-inf")
        idx[:, :, run_len - pad:] = INT32_MAX
    return v, idx


@pytest.mark.parametrize("nruns,rows,run_len,topk,kind,pad", [
    (8, 32, 8192, 8192, "normal", 0),     # the 8-way decode-1m merge
    (2, 4, 2048, 2048, "ties", 0),
    (5, 3, 700, 100, "ties", 0),          # k below 128: one summary entry per candidate
    (16, 2, 300, 1, "normal", 0),         # 16 runs, k = 1
    (3, 5, 4000, 2500, "normal", 0),      # runs longer than k
    (4, 3, 1000, 1000, "normal", 600),    # duplicate (-inf, INT32_MAX) padding in every run
    (2, 2, 16384, 16384, "flat", 0),      # ties beyond the staging capacity
    (2, 3, 12800, 12800, "normal", 0),    # a long staging (one tree level)
    (4, 3, 14000, 14000, "normal", 0),    # two tree buffers do not fit: ranking by binary searches
    (7, 4, 3000, 2900, "ties", 40),       # an odd number of runs: a list without a partner
    # more rows than a wave of 4-CTA clusters: one CTA per row, several per SM
    (2, 224, 4096, 4096, "normal", 0),    # the 2-rank shared-context merge
    (8, 224, 4096, 4096, "ties", 0),
    (5, 50, 3000, 2900, "normal", 30),
    (4, 40, 14000, 14000, "normal", 0),   # ranking by binary searches
    (2, 40, 16384, 16384, "flat", 0),     # ties beyond the staging capacity
    (16, 40, 2000, 1500, "normal", 0),    # more runs than the CTA's warps
    (1, 100, 3000, 2000, "ties", 0),      # one run: the tree has no level
])
def test_merge_runs_edge_cases(cuda_device, nruns, rows, run_len, topk, kind, pad):
    v, idx = _runs(nruns, rows, run_len, seed=nruns * 1000 + topk, kind=kind, pad=pad)
    runs = torch.stack([v.view(torch.int32), idx], dim=1).to(cuda_device)
    oi, os_ = topk_merge_runs(runs, topk)
    ws, wi = _expected(v, idx, topk)
    assert torch.equal(os_.cpu(), ws)
    assert torch.equal(oi.cpu(), wi)


class _Buffers:
    """Exchange buffers of `world` emulated ranks, all on this GPU."""

    def __init__(self, world, rows, topk):
        self.lib = _lib.load()
        self.world, self.rows, self.topk = world, rows, topk
        nbytes = self.lib.prism_peer_buffer_bytes(rows, topk)
        assert nbytes == _lib.PEER_HEADER_BYTES + rows * topk * 8
        self.ptrs = []
        for _ in range(world):
            p = ctypes.c_void_p()
            h = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
            _lib.check(self.lib.prism_peer_alloc(nbytes, ctypes.byref(p), h), "prism_peer_alloc")
            self.ptrs.append(p.value)
        self.arr = (ctypes.c_void_p * world)(*self.ptrs)

    def run(self, r, device):
        return torch.as_tensor(_DeviceArray(self.ptrs[r] + _lib.PEER_HEADER_BYTES,
                                            (2, self.rows, self.topk), "<i4"), device=device)

    def status(self, r):
        st = ctypes.c_int(0)
        _lib.check(self.lib.prism_read_status(ctypes.c_void_p(self.ptrs[r]), ctypes.byref(st),
                                              torch.cuda.current_stream().cuda_stream), "prism_read_status")
        return st.value

    def free(self):
        torch.cuda.synchronize()
        for p in self.ptrs:
            _lib.check(self.lib.prism_peer_free(ctypes.c_void_p(p)), "prism_peer_free")


def test_peer_merge_emulated_ranks(cuda_device):
    world, rows, topk = 4, 6, 1000
    bufs = _Buffers(world, rows, topk)
    lib, stream = bufs.lib, torch.cuda.current_stream().cuda_stream
    try:
        for step in range(3):
            kind = "ties" if step == 1 else "normal"
            v, idx = _runs(world, rows, topk, seed=50 + step, kind=kind)
            for r in range(world):
                bufs.run(r, cuda_device).copy_(torch.stack([v[r].view(torch.int32), idx[r]]).to(cuda_device))
            for r in range(world):
                _lib.check(lib.prism_peer_publish(bufs.arr, world, r, stream), "prism_peer_publish")
            outs = []
            for r in range(world):
                oi = torch.empty(rows, topk, dtype=torch.int32, device=cuda_device)
                os_ = torch.empty(rows, topk, dtype=torch.float32, device=cuda_device)
                _lib.check(lib.prism_peer_merge(bufs.arr, world, r, rows, topk, int(r == world - 1), 0,
                                                oi.data_ptr(), os_.data_ptr(), stream), "prism_peer_merge")
                outs.append((oi, os_))
            torch.cuda.synchronize()
            ws, wi = _expected(v, idx, topk)
            for r in range(world):
                assert bufs.status(r) == 0
                assert torch.equal(outs[r][1].cpu(), ws)
                assert torch.equal(outs[r][0].cpu(), wi)
    finally:
        bufs.free()


def test_peer_merge_wait_expires(cuda_device):
    # rank 1 never publishes: rank 0's merge gives up after 20 ms per wait and says so
    world, rows, topk = 2, 2, 64
    bufs = _Buffers(world, rows, topk)
    lib, stream = bufs.lib, torch.cuda.current_stream().cuda_stream
    try:
        _lib.check(lib.prism_peer_publish(bufs.arr, world, 0, stream), "prism_peer_publish")
        oi = torch.empty(rows, topk, dtype=torch.int32, device=cuda_device)
        os_ = torch.empty(rows, topk, dtype=torch.float32, device=cuda_device)
        _lib.check(lib.prism_peer_merge(bufs.arr, world, 0, rows, topk, 1, 20_000_000,
                                        oi.data_ptr(), os_.data_ptr(), stream), "prism_peer_merge")
        torch.cuda.synchronize()
        assert bufs.status(0) == 1
        assert bufs.status(0) == 0  # read and reset
        x = torch.ones(4, device=cuda_device)  # the context is still usable
        assert float((x * 2).sum()) == 8.0
    finally:
        bufs.free()


def test_peer_exchange_argument_errors(cuda_device):
    bufs = _Buffers(2, 2, 64)
    lib, stream = bufs.lib, torch.cuda.current_stream().cuda_stream
    try:
        assert lib.prism_peer_publish(bufs.arr, 0, 0, stream) == _lib.PRISM_E_UNSUPPORTED
        assert lib.prism_peer_publish(bufs.arr, 2, 2, stream) == _lib.PRISM_E_INVALID
        mis = (ctypes.c_void_p * 2)(bufs.ptrs[0], bufs.ptrs[1] + 16)
        assert lib.prism_peer_publish(mis, 2, 0, stream) == _lib.PRISM_E_INVALID
        assert lib.prism_peer_merge(bufs.arr, 2, 0, 2, 64, 1, 0, None, None, stream) == _lib.PRISM_E_INVALID
    finally:
        bufs.free()


# ---- the single C-ABI sharded call ------------------------------------------------------
def _sharded_c(lib, q, k_shard, inv, start, topk, bufs, world, rank, wait_acks=1):
    """prism_sharded_topk through the C ABI: this rank's local top-k into its exchange
    run, the publish and the merge; int32 / fp32 [B, Hq, Sq, topk]."""
    B, Hq, Sq, D = q.shape
    Hkv, Sk = k_shard.shape[1], k_shard.shape[2]
    out_i = torch.empty((B, Hq, Sq, topk), dtype=torch.int32, device=q.device)
    out_s = torch.empty((B, Hq, Sq, topk), dtype=torch.float32, device=q.device)
    ws_bytes = lib.prism_einsum_topk_workspace_size(B, Hq, Sq, Sk, topk, _lib.MODE_EXACT)
    ws = torch.empty(int(ws_bytes), dtype=torch.uint8, device=q.device)
    stream = torch.cuda.current_stream(q.device).cuda_stream
    rc = lib.prism_sharded_topk(q.data_ptr(), k_shard.data_ptr(), inv.data_ptr() if inv is not None else None,
                                0, B, Hq, Hkv, Sq, Sk, D, _lib.i64_array(q.stride()), _lib.i64_array(k_shard.stride()),
                                int(start), int(topk), bufs, world, rank, wait_acks, 0,
                                out_i.data_ptr(), out_s.data_ptr(), ws.data_ptr(), ws.numel(), stream)
    _lib.check(rc, "prism_sharded_topk")
    return out_i, out_s


def test_sharded_c_abi_one_rank(cuda_device):
    # world = 1: the call's merge of one run returns the local top-k of the shard
    # at its global offset, exactly as prism_einsum_topk does
    lib = _lib.load()
    g = torch.Generator().manual_seed(3)
    B, Hq, Hkv, Sk, topk, start = 1, 8, 2, 20000, 700, 123456
    q = torch.randn(B, Hq, 1, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    k = torch.randn(B, Hkv, Sk, 128, generator=g).to(torch.bfloat16).to(cuda_device)
    inv = W.rope_inv_freq(128, 5e5).to(cuda_device)
    rows = B * Hq
    nbytes = lib.prism_peer_buffer_bytes(rows, topk)
    own = ctypes.c_void_p()
    handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
    _lib.check(lib.prism_peer_alloc(nbytes, ctypes.byref(own), handle), "prism_peer_alloc")
    try:
        bufs = (ctypes.c_void_p * 1)(own.value)
        want_i, want_s = einsum_topk_func(q, k, topk, inv_freq=inv, pos_offset=start, index_base=start,
                                          return_scores=True)
        for _ in range(3):  # several steps on one buffer
            gi, gs = _sharded_c(lib, q, k, inv, start, topk, bufs, 1, 0)
            torch.cuda.synchronize()
            assert torch.equal(gi, want_i) and torch.equal(gs, want_s)
        # argument checks: a shard shorter than k, a rank outside the world
        short = k[:, :, :topk - 1]
        with pytest.raises(AssertionError, match="at least topk"):
            _sharded_c(lib, q, short.contiguous(), inv, start, topk, bufs, 1, 0)
        with pytest.raises(AssertionError, match="outside"):
            _sharded_c(lib, q, k, inv, start, topk, bufs, 1, 1)
    finally:
        torch.cuda.synchronize()
        lib.prism_peer_free(own)


# ---- two ranks on two GPUs ------------------------------------------------------------
def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _two_gpu_worker(rank, world, port, errq):
    try:
        import torch.distributed as dist

        from prism_test_b200.peer_exchange import PeerExchange
        from prism_test_b200.sharded import shard_bounds, sharded_einsum_topk
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=60))
        B, Hq, Hkv, Sk, topk = 1, 8, 2, 2 * 16384, 1000
        g = torch.Generator().manual_seed(7)
        q = torch.randn(B, Hq, 1, 128, generator=g).to(torch.bfloat16)
        k = torch.randn(B, Hkv, Sk, 128, generator=g).to(torch.bfloat16)
        inv = W.rope_inv_freq(128, 5e5)
        start, stop = shard_bounds(Sk, rank, world)
        qd, kd, invd = q.to(dev), k[:, :, start:stop].contiguous().to(dev), inv.to(dev)
        rows = B * Hq
        # expected: both shards' local top-k computed here, merged here
        runs = []
        for r in range(world):
            s0, s1 = shard_bounds(Sk, r, world)
            li, ls = einsum_topk_func(qd, k[:, :, s0:s1].contiguous().to(dev), topk, inv_freq=invd,
                                      pos_offset=s0, index_base=s0, return_scores=True)
            runs.append(torch.stack([ls.reshape(rows, topk).view(torch.int32), li.reshape(rows, topk)]))
        want_i, want_s = topk_merge_runs(torch.stack(runs), topk)
        want_i, want_s = want_i.reshape(B, Hq, 1, topk), want_s.reshape(B, Hq, 1, topk)
        ex = PeerExchange(rows, topk, dev)
        try:
            def step():
                return sharded_einsum_topk(qd, kd, topk, shard_start=start, inv_freq=invd,
                                           return_scores=True, exchange=ex)
            for _ in range(3):
                gi, gs = step()
                assert torch.equal(gi, want_i) and torch.equal(gs, want_s)
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(side):
                step()
            torch.cuda.current_stream().wait_stream(side)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                gi, gs = step()
            for _ in range(3):
                graph.replay()
                torch.cuda.synchronize()
                assert torch.equal(gi, want_i) and torch.equal(gs, want_s)
            del graph
            # the same step through the single C-ABI call, on the same exchange
            lib = _lib.load()
            for _ in range(2):
                ci, cs = _sharded_c(lib, qd, kd, invd, start, topk, ex._bufs, world, rank)
                torch.cuda.synchronize()
                assert torch.equal(ci, want_i) and torch.equal(cs, want_s)
            # steps whose local top-k the caller writes into the run (publish + merge
            # path) between single-call steps, whose merges leave the read
            # acknowledgements to the next step
            def wrapped(*a, **kw):
                return einsum_topk_func(*a, **kw)
            for fn in (wrapped, None, wrapped, None):
                gi, gs = sharded_einsum_topk(qd, kd, topk, shard_start=start, inv_freq=invd,
                                             return_scores=True, exchange=ex, local_topk=fn)
                torch.cuda.synchronize()
                assert torch.equal(gi, want_i) and torch.equal(gs, want_s)
            assert ex.status() == 0
        finally:
            ex.close()
        dist.destroy_process_group()
        errq.put((rank, "ok"))
    except Exception:  # noqa: BLE001
        errq.put((rank, traceback.format_exc()))


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2,
                    reason="needs two GPUs")
def test_peer_exchange_two_gpus():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_two_gpu_worker, args=(r, 2, port, errq)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(errq.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert results == {0: "ok", 1: "ok"}, results
