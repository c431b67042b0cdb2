"""Host logic of the vocab-parallel head on CPU ranks (gloo, world size 2): shard-geometry
validation of TPHead (sampling/tp_head.py:25-60), TorchGroup.all_gather along any dim, and
global_topk (two all-gathers + merge_topk, sampling/tp_head.py:9-14,76-82) against the oracle's
merge.  The fused per-rank head and the merge kernel are GPU tests (test_gpu_lmhead.py)."""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle as O


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from dspine_b200.lmhead import TPHead, TorchGroup
        grp = TorchGroup()
        V, H, k = 1000, 16, 7
        start, end = V * rank // world, V * (rank + 1) // world
        w = torch.zeros(end - start + 3, H, dtype=torch.bfloat16)  # padded shard
        head = TPHead(w, start, end, V, grp)
        assert head.geometry == tuple((V * r // world, V * (r + 1) // world, end - start + 3)
                                      for r in range(world))
        # all_gather along the last dim
        x = torch.full((2, 3), float(rank))
        y = grp.all_gather(x, dim=-1)
        assert y.shape == (2, 3 * world) and float(y[0, 3]) == 1.0
        # global_topk == oracle merge of the concatenated candidates
        g = torch.Generator().manual_seed(rank)
        vals = torch.randint(0, 5, (4, k), generator=g).float()  # many ties across ranks
        ids = torch.randint(start, end, (4, k), generator=g)
        gv, gi = head.global_topk(vals, ids, k)
        all_v = grp.all_gather(vals, dim=-1).numpy()
        all_i = grp.all_gather(ids, dim=-1).numpy()
        ev, ei = O.merge_topk(all_v, all_i, k)
        assert np.array_equal(gi.numpy(), ei) and np.array_equal(gv.numpy(), ev)
        # shards that do not partition the vocabulary are refused on every rank
        bad = False
        try:
            TPHead(w, start, end - 1 if rank == 0 else end, V, grp)
        except ValueError:
            bad = True
        assert bad
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


def test_tp_head_host_logic_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res


def _sync_worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from dspine_b200.runtime.tp_sync import TpCoordinator
        tp = TpCoordinator()
        acc = torch.full((4,), rank, dtype=torch.int32)
        bonus = torch.full((4,), 100 + rank, dtype=torch.int64)
        out = torch.full((4, 16), 7 * rank, dtype=torch.int64)
        ptrs = (acc.data_ptr(), bonus.data_ptr(), out.data_ptr())
        tp.sync_accept(acc, None, bonus, out)
        ok = (acc == 0).all() and (bonus == 100).all() and (out == 0).all()
        ok = ok and ptrs == (acc.data_ptr(), bonus.data_ptr(), out.data_ptr())
        ok = ok and acc.dtype == torch.int32
        dist.destroy_process_group()
        q.put((rank, "ok" if ok else "mismatch"))
    except Exception as e:
        q.put((rank, repr(e)))


def test_sync_accept_broadcasts_in_place_two_ranks():
    """runtime/tp_sync.py:67-106: rank 0's accept buffers reach every rank, in place."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_sync_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res


def _rescore_worker(rank, world, port, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from dspine_b200.layers.fp8 import gather
        from dspine_b200.lmhead import TPHead, TorchGroup

        # the per-rank dot is a GPU kernel; on CPU ranks it is the reference's CPU formula
        # (sampling/tp_head.py:100-101), which leaves the exchange logic under test
        def cpu_rescore(torch_mod, weight, ids, hidden, *, fp32_output=False):
            return (weight[ids].float() * hidden[:, None].float()).sum(-1).to(hidden.dtype)
        gather.rescore = cpu_rescore
        V, H = 1000, 16
        g = torch.Generator().manual_seed(0)
        full = torch.randn(V, H, generator=g).to(torch.bfloat16)
        hidden = torch.randn(3, H, generator=g).to(torch.bfloat16)
        ids = torch.randint(0, V, (3, 128), generator=g)
        ids[0, :4] = V                                # padding ids score 0 on every rank
        start, end = V * rank // world, V * (rank + 1) // world
        shard = torch.cat([full[start:end], torch.zeros(5, H, dtype=torch.bfloat16)])
        head = TPHead(shard, start, end, V, TorchGroup())
        got = head.rescore(ids, hidden)
        safe = ids.clamp(0, V - 1)
        expected = (full[safe].float() * hidden[:, None].float()).sum(-1).to(hidden.dtype)
        expected[0, :4] = 0
        assert torch.equal(got, expected)
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # report to the parent instead of hanging it
        q.put((rank, repr(e)))


def test_tp_rescore_exchange_two_ranks():
    """TPHead.rescore (sampling/tp_head.py:91-103): the owner rank's dot, zeros elsewhere, one
    all-reduce: every rank ends with the full-vocabulary scores."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rescore_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "ok", 1: "ok"}, res
