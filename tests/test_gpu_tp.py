"""Vocab-parallel TP head on 2/4/8 GPUs (NCCL) at config 3's shapes (hidden 5120, 32 requests x
16 rows, k = 20, V = 151936): every rank's fused shard head + one all-gather + the merge kernel
must give, on every rank, exactly the unsharded head's top-k ids and values (and its logsumexp
within 1e-5), the greedy accept decision made from them must be identical on every rank and to
TP = 1 (sampling/tp_head.py:17-103; runtime/tp_sync.py:67-106 broadcasts the accept result
instead of recomputing it), and the ids must be a top-k of the fp32 product computed by torch
(ties and bf16 rounding midpoints within the product's error admit either neighbour), with
values equal to the fp32 logits rounded to bf16 and the logsumexp within 1e-4 of torch's.
Skipped with fewer than 2 GPUs."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

V, H, ROWS, K, B = 151936, 5120, 512, 20, 32


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _inputs(dev):
    g = torch.Generator(device=dev).manual_seed(1234)
    x = torch.randn(ROWS, H, generator=g, device=dev).to(torch.bfloat16)
    w = (torch.randn(V, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    cand = torch.randint(0, V, (B, 16), generator=g, device=dev)
    caps = torch.randint(1, 17, (B,), generator=g, device=dev, dtype=torch.int32)
    return x, w, cand, caps


def _matches_fp32_reference(x, w, ids, vals, lse):
    """ids / values / logsumexp against torch's fp32 product of the same bf16 operands."""
    ref = torch.cat([x.float() @ w[i:i + 16384].float().T for i in range(0, V, 16384)], dim=1)
    kth = ref.topk(K, dim=1).values[:, -1:]
    # error scale of an fp32 dot of length H: |x| . |w| * H * 2^-24, and one bf16 ulp
    mag = torch.cat([x.float().abs() @ w[i:i + 16384].float().abs().T for i in range(0, V, 16384)], dim=1)
    tol = (mag * H * 2.0 ** -24).gather(1, ids) + kth.abs() * 2.0 ** -8
    picked = ref.gather(1, ids)
    if not bool((picked >= kth - tol).all()):
        return False
    above = (ref > kth + tol.max(dim=1, keepdim=True).values)
    if not bool((above.sum(1) <= K).all()):
        return False
    hit = torch.zeros_like(above).scatter_(1, ids, True)
    if bool((above & ~hit).any()):
        return False
    if not bool(((vals - picked).abs() <= picked.abs() * 2.0 ** -8 + tol).all()):
        return False
    return bool((lse - torch.logsumexp(ref, dim=1)).abs().max() <= 1e-4)


def _worker(rank, world, port, q):
    import datetime
    import torch.distributed as dist
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        from dspine_b200 import accept, lmhead
        x, w, cand, caps = _inputs(dev)
        start, end = V * rank // world, V * (rank + 1) // world
        shard = w[start:end].contiguous()
        head = lmhead.TPHead(shard, start, end, V, lmhead.TorchGroup())
        ids, vals, lse = head.topk_lse(x, K)
        # make the top-1 of each row disagree with about a third of the drafts
        cand[:, 1:] = ids[:B * 16, 0].view(B, 16)[:, :-1]
        cand[::3, 5] += 1
        acc = accept.accept_greedy(cand, ids[:B * 16, 0].view(B, 16), caps)
        f_ids, f_vals, f_lse = lmhead.lmhead_topk(x, w, K)
        f_acc = accept.accept_greedy(cand, f_ids[:B * 16, 0].view(B, 16), caps)
        torch.cuda.synchronize()
        ok = torch.equal(ids, f_ids) and torch.equal(vals, f_vals)
        ok = ok and bool((lse - f_lse).abs().max() <= 1e-5)
        ok = ok and _matches_fp32_reference(x, w, ids, vals, lse)
        ok = ok and all(torch.equal(a, b) for a, b in zip(acc, f_acc))
        # identical on every rank
        flat = torch.cat([ids.view(-1).float(), vals.view(-1), lse, acc[0].float(), acc[2].float()])
        allf = [torch.empty_like(flat) for _ in range(world)]
        dist.all_gather(allf, flat)
        same = all(torch.equal(allf[0], a) for a in allf)
        dist.barrier(device_ids=[rank])
        dist.destroy_process_group()
        q.put((rank, "ok" if ok and same else f"mismatch ok={ok} same={same}"))
    except Exception as e:
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_tp_head_equals_unsharded_on_every_rank(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
    assert all(v == "ok" for v in res.values()), res
