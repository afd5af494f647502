"""Exchange of the sequence-sharded path's local top-k runs over NVLink.

The reference is single-GPU; this is the B200 exchange for a key sequence split
over the GPUs of one node (one process per GPU). Instead of all-gathering every
rank's run and merging the gathered copy, every rank keeps its run in a
peer-mapped buffer (CUDA IPC) and each rank's merge kernel reads the runs it
needs straight from the other GPUs' memory: only the prefixes of the runs at or
above the merge threshold (about k + (N + 1) * k / 128 entries per row) cross
NVLink, instead of N * k per row.

Per step, on the current stream of every rank (``prism_peer_*`` in
include/prism_b200.h):

1. the local top-k is written into :attr:`PeerExchange.run` (after
   :meth:`PeerExchange.wait_acks` when the previous step was a
   :meth:`PeerExchange.sharded_topk`);
2. ``prism_peer_publish`` marks this rank's run of the step ready on every rank;
3. ``prism_peer_merge`` waits for every rank's run, merges, acknowledges the reads
   and waits until this rank's run has been read everywhere.

:meth:`PeerExchange.sharded_topk` runs the three steps as one C call and moves
the last wait to the start of the next step, where it overlaps the scorer.

Steps are counted on the device, so the whole step can be captured in a CUDA
graph and replayed. Every wait is bounded (``timeout_s``); an expired wait sets
the status word :meth:`status` reads, and the exchange must then be rebuilt.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch
import torch.distributed as dist

from . import _lib


class _DeviceArray:
    """A raw device pointer as a ``__cuda_array_interface__`` object."""

    def __init__(self, ptr: int, shape, typestr: str):
        self.__cuda_array_interface__ = {
            "shape": tuple(shape), "typestr": typestr, "data": (int(ptr), False), "version": 3,
            "strides": None,
        }


class PeerExchange:
    """Peer-mapped exchange buffers of one process group (one rank per GPU).

    ``rows`` x ``topk`` is the shape of every rank's local top-k (rows = B * Hq * Sq).
    Construction is collective: every rank of ``group`` must create its exchange
    with the same arguments, in the same order relative to other collectives.
    """

    def __init__(self, rows: int, topk: int, device: torch.device, group=None,
                 timeout_s: float = 2.0):
        lib = _lib.load()
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > _lib.PEER_MAX_RANKS:
            raise ValueError(f"at most {_lib.PEER_MAX_RANKS} ranks, got {self.world}")
        self.rows, self.topk = int(rows), int(topk)
        self.device = torch.device(device)
        self.group = group
        self.timeout_ns = int(timeout_s * 1e9)
        self._opened = []
        with torch.cuda.device(self.device):
            nbytes = lib.prism_peer_buffer_bytes(self.rows, self.topk)
            if nbytes == 0:
                raise ValueError("rows and topk must be positive")
            own = ctypes.c_void_p()
            handle = ctypes.create_string_buffer(_lib.IPC_HANDLE_BYTES)
            _lib.check(lib.prism_peer_alloc(nbytes, ctypes.byref(own), handle), "prism_peer_alloc")
            self._own = own.value
            try:
                handles = [None] * self.world
                dist.all_gather_object(handles, handle.raw, group=group)
                ptrs = []
                for r, h in enumerate(handles):
                    if r == self.rank:
                        ptrs.append(self._own)
                        continue
                    p = ctypes.c_void_p()
                    hb = ctypes.create_string_buffer(h, _lib.IPC_HANDLE_BYTES)
                    _lib.check(lib.prism_peer_open(hb, ctypes.byref(p)), "prism_peer_open")
                    self._opened.append(p.value)
                    ptrs.append(p.value)
            except BaseException:
                # undo this rank's mappings and buffer; the other ranks see the
                # failure as an error of their next collective
                for p in self._opened:
                    lib.prism_peer_close(ctypes.c_void_p(p))
                self._opened = []
                lib.prism_peer_free(ctypes.c_void_p(self._own))
                self._own = None
                raise
        self._bufs = (ctypes.c_void_p * self.world)(*ptrs)
        self._ws = None  # scratch of sharded_topk, grown on demand
        # this rank's run, int32 [2, rows, topk]: fp32 score bits, global indices
        self.run = torch.as_tensor(
            _DeviceArray(self._own + _lib.PEER_HEADER_BYTES, (2, self.rows, self.topk), "<i4"),
            device=self.device)
        dist.barrier(group)

    def merge(self, out_idx: torch.Tensor, out_scores: torch.Tensor) -> None:
        """Publish this rank's run and merge every rank's run into out_idx / out_scores
        ([rows, topk] int32 / fp32), on the current stream."""
        assert out_idx.shape == (self.rows, self.topk) and out_idx.dtype == torch.int32
        assert out_scores.shape == (self.rows, self.topk) and out_scores.dtype == torch.float32
        assert out_idx.is_contiguous() and out_scores.is_contiguous()
        lib = _lib.load()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(lib.prism_peer_publish(self._bufs, self.world, self.rank, stream), "prism_peer_publish")
        _lib.check(lib.prism_peer_merge(self._bufs, self.world, self.rank, self.rows, self.topk, 1,
                                        self.timeout_ns, out_idx.data_ptr(), out_scores.data_ptr(), stream),
                   "prism_peer_merge")

    def wait_acks(self) -> None:
        """On the current stream: wait until every rank has read this rank's run of
        the current step. Needed before writing :attr:`run` when the previous step
        ran :meth:`sharded_topk` (whose merge does not wait for the reads)."""
        lib = _lib.load()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(lib.prism_peer_wait_acks(self._bufs, self.world, self.rank, self.timeout_ns, stream),
                   "prism_peer_wait_acks")

    def sharded_topk(self, q: torch.Tensor, k_shard: torch.Tensor, shard_start: int,
                     inv_freq: Optional[torch.Tensor], out_idx: torch.Tensor,
                     out_scores: torch.Tensor) -> None:
        """One sequence-sharded step in one C call (``prism_sharded_topk``): the exact
        local top-k of ``k_shard`` (keys at global positions / indices from
        ``shard_start``) written into this rank's run, the publish and the merge into
        out_idx / out_scores ([rows, topk]). The wait for the other ranks to have read
        the previous step's run runs on the device while this step's scorer runs."""
        assert out_idx.shape == (self.rows, self.topk) and out_idx.dtype == torch.int32
        assert out_scores.shape == (self.rows, self.topk) and out_scores.dtype == torch.float32
        assert out_idx.is_contiguous() and out_scores.is_contiguous()
        lib = _lib.load()
        B, Hq, Sq, D = q.shape
        Hkv, Sk = k_shard.shape[1], k_shard.shape[2]
        if B * Hq * Sq != self.rows:
            raise ValueError(f"exchange built for {self.rows} rows, call has {B * Hq * Sq}")
        dtype = _lib.DTYPE_BF16 if q.dtype == torch.bfloat16 else _lib.DTYPE_FP16
        if inv_freq is not None:
            ws_bytes = int(lib.prism_einsum_topk_rope_workspace_size(B, Hq, Hkv, Sq, Sk, self.topk,
                                                                     _lib.MODE_EXACT, _lib.RECALL_QK))
        else:
            ws_bytes = int(lib.prism_einsum_topk_workspace_size(B, Hq, Sq, Sk, self.topk, _lib.MODE_EXACT))
        if self._ws is None or self._ws.numel() < ws_bytes:
            self._ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self.device)
        inv = None
        if inv_freq is not None:
            inv = inv_freq.to(device=self.device, dtype=torch.float32).contiguous()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        rc = lib.prism_sharded_topk(
            q.data_ptr(), k_shard.data_ptr(), inv.data_ptr() if inv is not None else None, dtype,
            B, Hq, Hkv, Sq, Sk, D, _lib.i64_array(q.stride()), _lib.i64_array(k_shard.stride()),
            int(shard_start), self.topk, self._bufs, self.world, self.rank, 1, self.timeout_ns,
            out_idx.data_ptr(), out_scores.data_ptr(), self._ws.data_ptr(), self._ws.numel(), stream)
        _lib.check(rc, "prism_sharded_topk")

    def status(self) -> int:
        """The exchange's device status word (0, or 1 after an expired wait); resets it."""
        lib = _lib.load()
        st = ctypes.c_int(0)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(lib.prism_read_status(ctypes.c_void_p(self._own), ctypes.byref(st), stream),
                   "prism_read_status")
        return st.value

    def timings(self, reset: bool = True) -> dict:
        """This rank's merges since the last reset, in device time: how many, and the
        microseconds per merge spent waiting for the ranks' runs (from the merge's
        start), merging, and waiting for the other ranks' acknowledgements."""
        lib = _lib.load()
        out = (ctypes.c_uint64 * 4)()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        _lib.check(lib.prism_peer_read_timings(ctypes.c_void_p(self._own), out, 1 if reset else 0, stream),
                   "prism_peer_read_timings")
        n = int(out[0])
        per = (lambda v: v / n / 1e3) if n else (lambda v: 0.0)
        return {"merges": n, "wait_us": per(out[1]), "merge_us": per(out[2]), "ack_us": per(out[3])}

    def close(self) -> None:
        """Collective: unmaps the peers' buffers and frees this rank's."""
        if self._own is None:
            return
        lib = _lib.load()
        torch.cuda.synchronize(self.device)
        dist.barrier(self.group)  # nobody reads another rank's buffer any more
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.check(lib.prism_peer_close(ctypes.c_void_p(p)), "prism_peer_close")
            self._opened = []
            self.run = None
            dist.barrier(self.group)  # every mapping of this rank's buffer is gone
            _lib.check(lib.prism_peer_free(ctypes.c_void_p(self._own)), "prism_peer_free")
        self._own = None
