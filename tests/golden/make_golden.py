"""Generate the golden fixtures that pin the CPU oracle to the reference implementation.

Run in a container that has the reference checkout (read-only) and Triton:

    PYTHONDONTWRITEBYTECODE=1 TRITON_INTERPRET=1 python tests/golden/make_golden.py /path/to/reference

It imports the reference package ``sglang_dspine`` and its test helpers, executes the
reference's own kernels on CPU tensors under the Triton interpreter (the same mechanism the
reference's tests/test_random.py:245-251 uses), and writes inputs plus outputs as small
``.npz`` files next to this script.  The GPU box and the test suite never import the
reference: they only read these files.

Fixture groups (reference function -> file):
  chain     sampling/rejection.py:101-153 sample_capped_chain_from_probs   chain.npz
  sparse    sampling/sparse/accept.py:422-543 compress_probs/accept_sparse  sparse.npz
  target    tests/ref_utils.py:79-108 ref_target_row (float64)             target.npz
  topk      kernels/dspine.py:165-207 topk_ids                             topk.npz
  uniforms  sampling/random.py:22-43 _cpu_uniforms                         uniforms.npz
  sps       verification/sps.py:35-58 allocate_verify_lens                 sps.npz
  merge     sampling/tp_head.py:9-14 merge_topk                            merge.npz
  greedy    verification/caps.py:32-59 _accept_capped, ragged.py:51-76     greedy.npz
"""

import os
import sys
import tempfile
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def _install_stubs():
    """sampling/random.py imports SGLang's murmur helpers at module level; its CPU path
    (_cpu_uniforms) does not use them, so an import-only stub suffices."""
    names = ["sglang", "sglang.kernels", "sglang.kernels.ops", "sglang.kernels.ops.sampling",
             "sglang.kernels.ops.sampling.murmur_hash"]
    for n in names:
        if n not in sys.modules:
            sys.modules[n] = types.ModuleType(n)
    sys.modules["sglang.kernels.ops.sampling.murmur_hash"].murmur3_mix = None
    sys.modules["sglang.kernels.ops.sampling.murmur_hash"].fmix32 = None


def _buffers(torch, bs):
    return (torch.empty(bs, dtype=torch.int32), torch.empty(bs, dtype=torch.int32),
            torch.empty(bs, dtype=torch.int64), torch.empty((bs, 16), dtype=torch.int64),
            torch.empty(bs, dtype=torch.int32))


def _np(t):
    return t.detach().cpu().numpy()


def gen_chain(torch):
    from sglang_dspine.sampling.rejection import sample_capped_chain_from_probs

    out = {}
    specs = [(9, 257, 0), (5, 1031, 1), (16, 97, 2), (3, 1543, 3)]
    for ci, (bs, V, seed) in enumerate(specs):
        g = torch.Generator().manual_seed(4100 + seed)
        p = torch.softmax(torch.randn(bs, 16, V, generator=g) * 2, -1)
        q = torch.softmax(torch.randn(bs, 15, V, generator=g) * 2, -1)
        if seed % 2 == 0:  # filtered rows: zero out part of the support
            p = p * (torch.rand(bs, 16, V, generator=g) > 0.5)
            p = p / p.sum(-1, keepdim=True)
        cand = torch.zeros(bs, 16, dtype=torch.int64)
        # drafts mostly from the high-p region of the target so that chains get long
        for b in range(bs):
            for s in range(15):
                cand[b, s + 1] = torch.multinomial(p[b, s], 1, generator=g)[0]
        caps = 1 + torch.arange(bs, dtype=torch.int32) % 16
        caps[0] = 16
        u = torch.rand(bs, 15, generator=g) * 0.6
        uf = torch.rand(bs, generator=g)
        prefix = torch.arange(bs, dtype=torch.int32) + 100
        u[0] = 0  # all accepted
        if bs > 1:  # zero residual: p == q on the rejected row
            q[1] = p[1, :15]
            u[1] = 1
        if bs > 2:  # invalid q values are clamped
            q[2, :, :3] = -1.0
        outs = _buffers(torch, bs)
        sample_capped_chain_from_probs(candidates=cand, target_probs=p.float().contiguous(),
                                       draft_probs=q.float().contiguous(), verify_lens=caps,
                                       uniforms=u, uniform_final=uf, prefix_lens=prefix,
                                       outputs=outs)
        for name, val in (("cand", cand), ("p", p.float()), ("q", q.float()), ("caps", caps),
                          ("u", u), ("uf", uf), ("prefix", prefix)):
            out[f"c{ci}_{name}"] = _np(val)
        for name, val in zip(("accept", "commit", "bonus", "output", "new_seq"), outs):
            out[f"c{ci}_{name}"] = _np(val)
    out["n"] = np.array(len(specs))
    return out


def gen_sparse(torch):
    from sglang_dspine.sampling.sparse.accept import accept_sparse, compress_probs

    out = {}
    ci = 0
    for bs in (1, 9, 32):
        for kind in ("compact", "overflow", "pure_packed", "dense"):
            g = torch.Generator().manual_seed(713 + bs)
            vocab = 257
            caps = torch.arange(bs, dtype=torch.int32) % 16 + 1
            caps[0] = 16
            offsets = torch.cat((torch.zeros(1, dtype=torch.int64), caps.long().cumsum(0)))[:-1]
            rows = int(caps.sum())
            p = torch.zeros((rows, vocab))
            support = torch.tensor([0, 2, 3, 7, 11, 13, 15])
            p[:, support] = torch.softmax(torch.randn(rows, len(support), generator=g), -1)
            qids = torch.arange(16, dtype=torch.int64).expand(bs, 15, 16).contiguous()
            qvals = torch.softmax(torch.randn((bs, 15, 16), generator=g), -1)
            cand = torch.zeros((bs, 16), dtype=torch.int64)
            cand[:, 1:] = torch.multinomial(qvals.reshape(-1, 16), 1, generator=g).reshape(bs, 15)
            u = torch.full((bs, 15), 0.371)
            uf = torch.linspace(0.071, 0.917, bs)
            prefix = torch.arange(bs, dtype=torch.int32) + 8191
            cand[0, 1:] = 0
            u[0] = 0
            if bs > 1:
                lo = int(offsets[1])
                hi = lo + int(caps[1])
                same = torch.softmax(torch.arange(16, dtype=torch.float32), 0)
                p[lo:hi] = 0
                p[lo:hi, :16] = same
                qvals[1] = same
                u[1] = 1
            if kind in ("overflow", "dense"):
                p[::11] = torch.softmax(torch.randn((len(p[::11]), vocab), generator=g), -1)
            packed = None
            if kind != "dense":
                packed = compress_probs(torch, p, capacity=32)
                ids, values, lengths, overflow = packed
                lane = torch.arange(32)[None, :]
                perm = (lengths[:, None] - 1 - lane).clamp_min(0).long()
                packed = (ids.gather(1, perm).where(lane < lengths[:, None], -1),
                          values.gather(1, perm).where(lane < lengths[:, None], 0), lengths,
                          overflow)
                for name, val in zip(("ids", "vals", "lens", "ovf"), packed):
                    out[f"c{ci}_{name}"] = _np(val)
                for name, val in zip(("cids", "cvals", "clens", "covf"),
                                     compress_probs(torch, p, capacity=32)):
                    out[f"c{ci}_{name}"] = _np(val)
            outs = _buffers(torch, bs)
            accept_sparse(torch, candidates=cand, dense_p=None if kind == "pure_packed" else p,
                          packed=packed, q_ids=qids, q_values=qvals, verify_lens=caps,
                          uniforms=u, uniform_final=uf, prefix_lens=prefix, outputs=outs,
                          row_offsets=offsets, vocab_size=vocab)
            for name, val in (("cand", cand), ("p", p), ("qids", qids), ("qvals", qvals),
                              ("caps", caps), ("u", u), ("uf", uf), ("prefix", prefix),
                              ("offsets", offsets)):
                out[f"c{ci}_{name}"] = _np(val)
            out[f"c{ci}_kind"] = np.array(kind)
            for name, val in zip(("accept", "commit", "bonus", "output", "new_seq"), outs):
                out[f"c{ci}_{name}"] = _np(val)
            ci += 1
    out["n"] = np.array(ci)
    return out


def gen_target(torch, ref_dir):
    sys.path.insert(0, str(Path(ref_dir) / "tests"))
    from ref_utils import ref_target_row

    out = {}
    ci = 0
    g = torch.Generator().manual_seed(0)
    params = [(0.6, 20, 0.95), (1.0, 7, 1.0), (1.2, 1 << 30, 0.6), (0.9, 30, 0.9),
              (0.3, 50, 0.8), (1.5, 1 << 30, 1.0), (0.05, 20, 0.85), (2.0, 3, 0.99)]
    for (T, k, tp) in params:
        for rep in range(3):
            V = [200, 97, 1000][rep]
            l = torch.randn(V, generator=g) * 3
            ref = ref_target_row(l, T, k, tp, 0.0, "flashinfer")
            out[f"c{ci}_logits"] = _np(l.float())
            out[f"c{ci}_params"] = np.array([T, k, tp], dtype=np.float64)
            out[f"c{ci}_p"] = _np(ref)
            ci += 1
    out["n"] = np.array(ci)
    return out


def gen_topk(torch):
    from sglang_dspine.kernels.dspine import topk_ids

    out = {}
    ci = 0
    g = torch.Generator().manual_seed(11)
    for (rows, V, k, dtype) in ((3, 4096, 16, torch.float32), (2, 3000, 8, torch.bfloat16),
                                (4, 1531, 4, torch.float32), (2, 4096, 32, torch.bfloat16)):
        x = (torch.randn(rows, V, generator=g) * 4).round() / 4  # many ties
        x = x.to(dtype)
        ids = topk_ids(x, k)
        out[f"c{ci}_x"] = _np(x.float())
        out[f"c{ci}_k"] = np.array(k)
        out[f"c{ci}_bf16"] = np.array(dtype == torch.bfloat16)
        out[f"c{ci}_ids"] = _np(ids)
        ci += 1
    out["n"] = np.array(ci)
    return out


def gen_uniforms(torch):
    from sglang_dspine.sampling.random import _cpu_uniforms

    seeds = torch.tensor([0, -1, -(2**63), 2**63 - 1, 2**40 + 7, 7, 123])
    positions = torch.tensor([0, 19, 214, 8192, 131071, 29, 811])
    out = {"seeds": _np(seeds), "positions": _np(positions)}
    for stream in range(4):
        out[f"s{stream}"] = _np(_cpu_uniforms(seeds, positions, 15, stream))
    return out


def gen_sps(torch):
    from sglang_dspine.verification.sps import allocate_verify_lens

    out = {}
    ci = 0
    for bs in (1, 3, 9, 17, 65):
        g = torch.Generator().manual_seed(714)
        raw = torch.rand((bs, 15), generator=g)
        raw[::2] = 1
        table = torch.linspace(0.1, 1.0, 16).expand(15, 16).contiguous()
        for budget in (bs, bs * 7 + (bs > 1), bs * 16):
            lens = allocate_verify_lens(raw, table, torch.arange(15), budget)
            out[f"c{ci}_raw"] = _np(raw)
            out[f"c{ci}_table"] = _np(table)
            out[f"c{ci}_budget"] = np.array(budget)
            out[f"c{ci}_lens"] = _np(lens)
            ci += 1
    # fp32 extremes (tests/test_sps.py:379-416 construction)
    gamma, bs = 15, 4
    conditional = torch.tensor([
        [1.0] * gamma,
        [1.0, 1.0 - 2**-24, 1.0 - 2**-23] * 5,
        [1e-30, 1.0, 1e-30] + [1.0] * 12,
        [1.0, torch.finfo(torch.float32).tiny, 1.0, 1e-10] + [1.0] * 11,
    ], dtype=torch.float32)
    table = conditional.T.contiguous()
    raw = torch.tensor([0.125, 0.375, 0.625, 0.875])[:, None].expand(bs, gamma).contiguous()
    for budget in range(bs, bs * (gamma + 1) + 1, 3):
        lens = allocate_verify_lens(raw, table, torch.arange(gamma), budget)
        out[f"c{ci}_raw"] = _np(raw)
        out[f"c{ci}_table"] = _np(table)
        out[f"c{ci}_budget"] = np.array(budget)
        out[f"c{ci}_lens"] = _np(lens)
        ci += 1
    # bucketize boundaries
    g = torch.Generator().manual_seed(715)
    raw = torch.rand((33, 15), generator=g)
    boundaries = torch.tensor([0.2, 0.5, 0.5, 0.8])
    table = torch.rand((15, 5), generator=g)
    for budget in (33, 200, 33 * 16):
        lens = allocate_verify_lens(raw, table, torch.arange(15), budget, boundaries)
        out[f"c{ci}_raw"] = _np(raw)
        out[f"c{ci}_table"] = _np(table)
        out[f"c{ci}_budget"] = np.array(budget)
        out[f"c{ci}_boundaries"] = _np(boundaries)
        out[f"c{ci}_lens"] = _np(lens)
        ci += 1
    out["n"] = np.array(ci)
    return out


def gen_merge(torch):
    from sglang_dspine.sampling.tp_head import merge_topk

    out = {}
    g = torch.Generator().manual_seed(21)
    ci = 0
    for (n, m, k) in ((4, 40, 20), (3, 16, 8), (2, 160, 20)):
        v = ((torch.randn(n, m, generator=g) * 2).round() / 2).to(torch.bfloat16)
        ids = torch.randint(0, 151936, (n, m), generator=g)
        vals, sel = merge_topk(v, ids, k)
        out[f"c{ci}_v"] = _np(v.float())
        out[f"c{ci}_ids"] = _np(ids)
        out[f"c{ci}_k"] = np.array(k)
        out[f"c{ci}_outv"] = _np(vals.float())
        out[f"c{ci}_outi"] = _np(sel)
        ci += 1
    # the known answer of tests/test_tp_head.py:49-53
    v = torch.tensor([[9, 8, 8, 9, 8, 8]], dtype=torch.bfloat16)
    ids = torch.tensor([[0, 1, 2, 4, 5, 6]])
    vals, sel = merge_topk(v, ids, 4)
    out[f"c{ci}_v"] = _np(v.float())
    out[f"c{ci}_ids"] = _np(ids)
    out[f"c{ci}_k"] = np.array(4)
    out[f"c{ci}_outv"] = _np(vals.float())
    out[f"c{ci}_outi"] = _np(sel)
    ci += 1
    out["n"] = np.array(ci)
    return out


def gen_greedy(torch):
    from sglang_dspine.verification.caps import _accept_capped
    from sglang_dspine.verification.ragged import _accept

    out = {}
    g = torch.Generator().manual_seed(5)
    ci = 0
    for bs, cap in ((7, 16), (9, 5), (4, 1)):
        top1 = torch.randint(0, 5, (bs, 16), generator=g)
        cand = torch.zeros(bs, 16, dtype=torch.int64)
        cand[:, 1:] = torch.where(torch.rand(bs, 15, generator=g) < 0.8, top1[:, :15],
                                  torch.randint(0, 5, (bs, 15), generator=g))
        prefix = torch.arange(bs, dtype=torch.int32) + 3
        outs = _buffers(torch, bs)
        a, c, bo, o, ns = outs
        _accept_capped[(bs,)](cand, top1, a, c, bo, o, prefix, ns, T=16, CAP=cap, WIDTH=16)
        for name, val in (("cand", cand), ("top1", top1), ("prefix", prefix)):
            out[f"c{ci}_{name}"] = _np(val)
        out[f"c{ci}_caps"] = np.full(bs, cap, np.int32)
        for name, val in zip(("accept", "commit", "bonus", "output", "new_seq"), outs):
            out[f"c{ci}_{name}"] = _np(val)
        ci += 1
    for bs in (6, 17):
        top1 = torch.randint(0, 4, (bs, 16), generator=g)
        cand = torch.zeros(bs, 16, dtype=torch.int64)
        cand[:, 1:] = torch.where(torch.rand(bs, 15, generator=g) < 0.85, top1[:, :15],
                                  torch.randint(0, 4, (bs, 15), generator=g))
        lens = 1 + torch.arange(bs, dtype=torch.int32) % 16
        prefix = torch.arange(bs, dtype=torch.int32)
        outs = _buffers(torch, bs)
        a, c, bo, o, ns = outs
        _accept[(bs,)](cand, top1, lens, a, c, bo, o, prefix, ns, T=16)
        for name, val in (("cand", cand), ("top1", top1), ("prefix", prefix), ("caps", lens)):
            out[f"c{ci}_{name}"] = _np(val)
        for name, val in zip(("accept", "commit", "bonus", "output", "new_seq"), outs):
            out[f"c{ci}_{name}"] = _np(val)
        ci += 1
    out["n"] = np.array(ci)
    return out


def main(ref_dir):
    os.environ.setdefault("TRITON_INTERPRET", "1")
    os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(ref_dir))
    _install_stubs()
    import torch

    torch.manual_seed(0)
    groups = {
        "chain": lambda: gen_chain(torch),
        "sparse": lambda: gen_sparse(torch),
        "target": lambda: gen_target(torch, ref_dir),
        "topk": lambda: gen_topk(torch),
        "uniforms": lambda: gen_uniforms(torch),
        "sps": lambda: gen_sps(torch),
        "merge": lambda: gen_merge(torch),
        "greedy": lambda: gen_greedy(torch),
    }
    only = set(sys.argv[2:])
    for name, fn in groups.items():
        if only and name not in only:
            continue
        data = fn()
        np.savez_compressed(HERE / f"{name}.npz", **data)
        print(name, "->", HERE / f"{name}.npz")


if __name__ == "__main__":
    main(Path(sys.argv[1]) if len(sys.argv) > 1 else Path(tempfile.gettempdir()))
