"""Host logic of the sequence-sharded path over gloo on the CPU (world size 2
and 4): shard bounds, global positions / indices, the packed all-gather and the
merge, against the single-process oracle. Also a rank that dies before the
exchange: the survivor's collective ends with an error instead of hanging."""
import os
import socket
import traceback

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cpu_local(q, k, kl, inv_freq=None, pos_offset=0, index_base=0, return_scores=True, values=None,
               recall_type="qk"):
    from oracle import reattention_topk as orc
    vals, idx = orc.dense_topk(q, k, kl, inv_freq, pos_offset, None, index_base,
                               weights=orc.recall_weights(values, recall_type))
    return idx.to(torch.int32), vals


class _HostExchange:
    """Stand-in for PeerExchange on the CPU (the same interface: the local top-k is
    written into ``run``, then ``merge`` fills the outputs), exchanging the runs
    with a gloo all-gather and merging with the host merge; the peer-mapped GPU
    buffers themselves are tested in tests/test_peer_exchange_gpu.py."""

    def __init__(self, rows, topk):
        self.rows, self.topk = rows, topk
        self.run = torch.zeros((2, rows, topk), dtype=torch.int32)
        self.merges = 0
        self.ack_waits = 0

    def wait_acks(self):
        # the all-gather of merge() already completed every read of the run
        self.ack_waits += 1

    def merge(self, out_idx, out_scores):
        from prism_test_b200.sharded import merge_candidates_torch
        world = dist.get_world_size()
        runs = [torch.empty_like(self.run) for _ in range(world)]
        dist.all_gather(runs, self.run)
        g = torch.stack(runs)  # [world, 2, rows, topk]
        cand_s = g[:, 0].permute(1, 0, 2).reshape(self.rows, -1).contiguous().view(torch.float32)
        cand_i = g[:, 1].permute(1, 0, 2).reshape(self.rows, -1).contiguous()
        i, s = merge_candidates_torch(cand_s, cand_i, self.topk)
        out_idx.copy_(i)
        out_scores.copy_(s)
        self.merges += 1


def _put_and_exit(q, item):
    q.put(item)
    q.close()
    q.join_thread()  # flush before the hard exit
    os._exit(0)


def _worker(rank, world, port, case, q, k_full, inv, topk, errq, v_full=None):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        import datetime
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=10))
        from prism_test_b200.sharded import merge_candidates_torch, shard_bounds, sharded_einsum_topk
        start, stop = shard_bounds(k_full.shape[2], rank, world)
        if case == "die" and rank == 1:
            os._exit(0)  # leaves between steps, before the exchange
        rt = "qkv2" if case == "qkv2" else "qk"
        chunks = 2 if case == "chunks2" else 1
        v_shard = v_full[:, :, start:stop] if v_full is not None else None
        exchange = None
        if case == "exchange":
            rows = q.shape[0] * q.shape[1] * q.shape[2]
            exchange = _HostExchange(rows, topk)
            for bad in (dict(chunks=2), dict(topk=topk - 1)):  # rejected before any exchange
                try:
                    sharded_einsum_topk(q, k_full[:, :, start:stop], bad.get("topk", topk), shard_start=start,
                                        inv_freq=inv, local_topk=_cpu_local, exchange=exchange,
                                        chunks=bad.get("chunks", 1))
                except ValueError:
                    pass
                else:
                    raise AssertionError(f"{bad} was not rejected")
        try:
            idx, sc = sharded_einsum_topk(q, k_full[:, :, start:stop], topk, shard_start=start,
                                          inv_freq=inv, return_scores=True, local_topk=_cpu_local,
                                          merge=merge_candidates_torch, v_shard=v_shard, recall_type=rt,
                                          chunks=chunks, exchange=exchange)
        except Exception as e:  # noqa: BLE001
            if case == "die":
                _put_and_exit(errq, ("ok-error", rank, type(e).__name__))
            raise
        if case == "die":
            _put_and_exit(errq, ("no-error", rank, ""))
        from oracle import reattention_topk as orc
        from tests.parity import check_parity
        w = orc.recall_weights(v_full, rt)
        check_parity(idx, sc, q, k_full, topk, inv, 0, weights=w)
        errq.put(("ok", rank, ""))
        dist.destroy_process_group()
    except Exception:  # noqa: BLE001
        errq.put(("fail", rank, traceback.format_exc()))


def _run(world, case, Sk, topk, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, 8, 2, 128, generator=g).to(torch.bfloat16)
    raw = torch.randn(1, 2, Sk, 128, generator=g)
    inv = 1.0 / (5e5 ** (torch.arange(0, 128, 2, dtype=torch.int64).float() / 128))
    from prism_test_b200.workloads import apply_rope, rope_cos_sin
    cos, sin = rope_cos_sin(torch.arange(Sk), inv)
    k = apply_rope(raw, cos, sin).to(torch.bfloat16)
    v = (torch.randn(1, 2, Sk, 128, generator=g) * torch.exp(0.7 * torch.randn(1, 2, Sk, 1, generator=g))
         ).to(torch.bfloat16) if case == "qkv2" else None
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, case, q, k, inv, topk, errq, v)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
    out = []
    while not errq.empty():
        out.append(errq.get())
    return out


@pytest.mark.parametrize("world,Sk,topk", [(2, 1000, 50), (4, 1024, 300), (2, 64, 40)])
def test_sharded_matches_oracle(world, Sk, topk):
    res = _run(world, "ok", Sk, topk)
    assert sorted(r[1] for r in res) == list(range(world)), res
    for status, rank, msg in res:
        assert status == "ok", msg


def test_sharded_value_weighted_matches_oracle():
    res = _run(2, "qkv2", 1000, 60, seed=4)
    assert sorted(r[1] for r in res) == [0, 1], res
    for status, rank, msg in res:
        assert status == "ok", msg


def test_sharded_chunked_exchange_matches_oracle():
    # two groups of KV heads, each exchanged on its own (asynchronous) all-gather
    res = _run(2, "chunks2", 1000, 50, seed=6)
    assert sorted(r[1] for r in res) == [0, 1], res
    for status, rank, msg in res:
        assert status == "ok", msg


def test_sharded_exchange_path_matches_oracle():
    # the exchange= path of sharded_einsum_topk (local top-k written into the
    # exchange's run, one merge call), with a host stand-in for the peer buffers
    res = _run(2, "exchange", 1000, 50, seed=8)
    assert sorted(r[1] for r in res) == [0, 1], res
    for status, rank, msg in res:
        assert status == "ok", msg


def test_dead_rank_surfaces_as_error():
    res = _run(2, "die", 512, 20)
    assert res and all(s == "ok-error" for s, _, _ in res), res
