"""Sequence-sharded recall scoring across the GPUs of one node.

The reference is single-GPU (it has no distributed code); this is the B200
extension for key caches beyond one GPU's budget. Rank ``r`` of ``N`` holds the
contiguous key slice ``[r*Sk/N, (r+1)*Sk/N)`` of every KV head and:

1. runs the exact local top-k (``einsum_topk_func`` with ``pos_offset`` and
   ``index_base`` = the slice start, so RoPE positions and returned indices are
   global), with fp32 scores;
2. writes its result straight into an int32 ``[2, rows, topk]`` buffer (score
   bits, global indices) and all-gathers it (one NCCL collective over NVLink);
3. merges the N sorted runs per row on the device (``topk_merge_runs``, reading
   the gathered buffer in place): the global top-k is always contained in the
   union of the local top-k lists.

With ``chunks`` > 1 the KV heads are taken in that many groups: a group's local
top-k is all-gathered asynchronously (NCCL on its own stream) while the next
group is scored, so only the last group's exchange is exposed; the merges run at
the end, one per group.

With ``exchange`` (a :class:`~prism_test_b200.peer_exchange.PeerExchange`) steps 2
and 3 go over peer-mapped memory instead: the local top-k is written into the
rank's exchange buffer and each rank's merge kernel reads the other ranks' runs
straight from their GPUs over NVLink, after a device-side ready flag per rank (no
NCCL call, no gathered copy).

Every rank ends with the global result, equal to ``torch.topk`` over the whole
sequence (``ReAttentionMethod._dense_topk``, reattention.py:486-498), ties
broken toward lower global indices.
"""
from __future__ import annotations

from typing import Callable, Optional

import torch
import torch.distributed as dist

from .kernels import einsum_topk_func, topk_merge_runs


def shard_bounds(Sk_total: int, rank: int, world: int):
    """[start, stop) of rank's contiguous slice; Sk_total must divide evenly."""
    per = Sk_total // world
    if per * world != Sk_total:
        raise ValueError(f"sequence length {Sk_total} does not split evenly over {world} ranks")
    return rank * per, (rank + 1) * per


def _all_gather(packed: torch.Tensor, world: int, group, async_op: bool = False):
    """[world, *packed.shape] gathered buffer (and the async work handle, or None)."""
    out = torch.empty((world, *packed.shape), dtype=packed.dtype, device=packed.device)
    if dist.get_backend(group) == "nccl":
        work = dist.all_gather_into_tensor(out, packed, group=group, async_op=async_op)
    else:
        work = dist.all_gather(list(out.unbind(0)), packed, group=group, async_op=async_op)
    return (out, work) if async_op else out


def merge_candidates_torch(cand_s: torch.Tensor, cand_i: torch.Tensor, topk: int):
    """Host/CPU merge with the same result as the device merge (lowest index wins ties)."""
    order = torch.argsort(cand_i, dim=-1, stable=True)
    s = torch.gather(cand_s, -1, order)
    i = torch.gather(cand_i, -1, order)
    v, p = torch.sort(s, dim=-1, descending=True, stable=True)
    return torch.gather(i, -1, p[:, :topk]), v[:, :topk]


def sharded_einsum_topk(
    q: torch.Tensor,
    k_shard: torch.Tensor,
    topk: int,
    *,
    shard_start: int,
    inv_freq: Optional[torch.Tensor] = None,
    group=None,
    return_scores: bool = False,
    local_topk: Optional[Callable] = None,
    merge: Optional[Callable] = None,
    v_shard: Optional[torch.Tensor] = None,
    recall_type: str = "qk",
    chunks: int = 1,
    exchange=None,
):
    """Global exact top-k over a key sequence split across the ranks of ``group``.

    ``k_shard`` is this rank's slice ``[B, Hkv, Sk/N, 128]`` whose first key sits
    at absolute position / global index ``shard_start``. Returns int32 indices
    ``[B, Hq, Sq, topk]`` (and fp32 scores) on every rank.
    ``local_topk`` / ``merge`` default to the CUDA kernels; tests substitute
    CPU implementations to run the exchange over gloo. ``recall_type`` "qkv" /
    "qkv2" weights each key by the norm of its value row in ``v_shard`` (the
    same slice of the value cache), as ``einsum_topk_func`` does. ``chunks``
    (dividing Hkv) pipelines the exchange over groups of KV heads. ``exchange``
    (a ``PeerExchange`` built for ``B * Hq * Sq`` rows and ``topk``) exchanges the
    runs over peer-mapped memory instead of NCCL; ``chunks`` must then be 1.
    """
    local_topk = local_topk or einsum_topk_func
    world = dist.get_world_size(group)
    B, Hq, Sq, _ = q.shape
    Hkv = k_shard.shape[1]
    if chunks < 1 or Hkv % chunks:
        raise ValueError(f"chunks={chunks} must divide the {Hkv} KV heads")
    hk, hq = Hkv // chunks, Hq // chunks
    if exchange is not None:
        if chunks != 1:
            raise ValueError("the peer exchange takes the KV heads in one group (chunks=1)")
        rows = B * Hq * Sq
        if (exchange.rows, exchange.topk) != (rows, topk):
            raise ValueError(f"exchange built for {exchange.rows} x {exchange.topk}, call needs {rows} x {topk}")
        out_i = torch.empty((rows, topk), dtype=torch.int32, device=q.device)
        out_s = torch.empty((rows, topk), dtype=torch.float32, device=q.device)
        if recall_type == "qk" and local_topk is einsum_topk_func and k_shard.shape[2] >= topk:
            # one C call: local top-k into the run, publish, merge
            exchange.sharded_topk(q, k_shard, shard_start, inv_freq, out_i, out_s)
        else:
            extra = {} if recall_type == "qk" else dict(values=v_shard, recall_type=recall_type)
            exchange.wait_acks()  # the run may still be read by a sharded_topk step's merges
            _local_packed(local_topk, q, k_shard, topk, inv_freq, shard_start, extra, dest=exchange.run)
            exchange.merge(out_i, out_s)
        out_i, out_s = out_i.reshape(B, Hq, Sq, topk), out_s.reshape(B, Hq, Sq, topk)
        return (out_i, out_s) if return_scores else out_i
    pending = []
    for c in range(chunks):
        qc = q[:, c * hq:(c + 1) * hq]
        kc = k_shard[:, c * hk:(c + 1) * hk]
        extra = {} if recall_type == "qk" else dict(values=v_shard[:, c * hk:(c + 1) * hk],
                                                     recall_type=recall_type)
        packed = _local_packed(local_topk, qc, kc, topk, inv_freq, shard_start, extra)
        pending.append(_all_gather(packed, world, group, async_op=True))
    outs_i, outs_s = [], []
    for gathered, work in pending:
        if work is not None:
            work.wait()
        rows = gathered.shape[2]
        if merge is None:
            out_i, out_s = topk_merge_runs(gathered, topk)  # [world, 2, rows, topk]: sorted runs
        else:
            cand_s = gathered[:, 0].permute(1, 0, 2).reshape(rows, world * topk).contiguous().view(torch.float32)
            cand_i = gathered[:, 1].permute(1, 0, 2).reshape(rows, world * topk).contiguous()
            out_i, out_s = merge(cand_s, cand_i, topk)
        outs_i.append(out_i.reshape(B, hq, Sq, topk))
        outs_s.append(out_s.reshape(B, hq, Sq, topk))
    out_i = outs_i[0] if chunks == 1 else torch.cat(outs_i, dim=1)
    if return_scores:
        return out_i, (outs_s[0] if chunks == 1 else torch.cat(outs_s, dim=1))
    return out_i


def _local_packed(local_topk, q, k_shard, topk, inv_freq, shard_start, extra, dest=None) -> torch.Tensor:
    """This rank's exact local top-k as an int32 [2, rows, topk] buffer (score bits,
    global indices), sorted; a shard shorter than topk is padded with -inf.
    Written into ``dest`` when given."""
    B, Hq, Sq, _ = q.shape
    rows = B * Hq * Sq
    kl = min(topk, k_shard.shape[2])
    packed = dest if dest is not None else torch.empty((2, rows, topk), dtype=torch.int32, device=q.device)
    if kl == topk and local_topk is einsum_topk_func:
        local_topk(q, k_shard, kl, inv_freq=inv_freq, pos_offset=shard_start, index_base=shard_start,
                   out=(packed[1], packed[0].view(torch.float32)), **extra)
    else:
        idx, sc = local_topk(q, k_shard, kl, inv_freq=inv_freq, pos_offset=shard_start,
                             index_base=shard_start, return_scores=True, **extra)
        packed[0, :, :kl] = sc.reshape(rows, kl).contiguous().view(torch.int32)
        packed[1, :, :kl] = idx.reshape(rows, kl)
        if kl < topk:  # a shard shorter than k contributes -inf padding
            packed[0, :, kl:] = torch.tensor(float("-inf"), dtype=torch.float32).view(torch.int32).item()
            packed[1, :, kl:] = torch.iinfo(torch.int32).max
    return packed
