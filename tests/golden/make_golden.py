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
  serial    kernels/dspine.py:210-351,616-772 serial_table / serial_chain /
            build_serial_tables / serial_sample_chain, and tests/ref_utils.py:12-76
            ref_sample_chain / ref_refine_table                             serial.npz
  fp8       layers/fp8/coarse.py FullVFP8Coarse (weight quantization), _scale/_quantize,
            stable_local_topk; layers/fp8/gather.py rescore / select16      fp8.npz
  target_minp  tests/ref_utils.py:79-108 ref_target_row with min-p, both backends  target_minp.npz
  sparse_target  sampling/sparse/target.py:95-178 build_sparse_target (CPU branch)  sparse_target.npz
  adjust    sampling/compact.py:14-79 adjust_logits (pure torch, CPU tensors)       adjust.npz
  fullv     configs 0, 1 and 4 at V = 151936: ref_target_row rows +
            sampling/rejection.py:101-153 sample_capped_chain_from_probs     fullv.npz
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


def _serial_refine_inputs(torch, g, bs, T, H, R, C, V, k):
    import math
    bf = torch.bfloat16
    m, n = bs * T, bs * (T - 1)
    d = dict(
        raw=torch.randn(m, H, generator=g).to(bf),
        rms=(torch.rand(m, generator=g) + 0.5).float(),
        packed=torch.randn(m, 3 * R, generator=g).to(bf),
        codebook=(torch.randn(V, C, generator=g) / math.sqrt(C)).to(bf),
        pg=(torch.randn(R, C, generator=g) / math.sqrt(C)).to(bf),
        pv=(torch.randn(R, C, generator=g) / math.sqrt(C)).to(bf),
        gb=(torch.randn(R, generator=g) * 0.1).to(bf),
        w_last=(torch.randn(H, R, generator=g) / math.sqrt(R)).to(bf),
        norm_w=(1.0 + 0.1 * torch.randn(H, generator=g)).to(bf),
        lm=(torch.randn(V, H, generator=g) / math.sqrt(H)).to(bf),
    )
    d["cand"] = torch.stack([torch.randperm(V, generator=g)[:k].sort().values
                             for _ in range(n)]).contiguous()
    d["input_ids"] = torch.randint(0, V, (m,), generator=g)
    d["anchors"] = d["input_ids"].view(bs, T)[:, 0].contiguous()
    return d


def gen_serial(torch, ref_dir):
    """Sampled chain: the reference kernel (under the interpreter) and ref_sample_chain on the
    same inputs.  Greedy table: build_serial_tables -> serial_table -> serial_chain (with
    confidences), plus the fp64 refinement table ref_refine_table the chain approximates."""
    sys.path.insert(0, str(Path(ref_dir) / "tests"))
    from ref_utils import ref_refine_table, ref_sample_chain
    from sglang_dspine.kernels import dspine as K

    out = {}
    g = torch.Generator().manual_seed(31)
    ci = 0
    chain_cases = [
        # (T, k, per-request (temperature, top_k, top_p, min_p, greedy), table scale)
        (5, 8, [(1.0, 8, 1.0, 0.0, 0), (0.7, 3, 0.8, 0.1, 0), (1.5, 8, 0.5, 0.0, 0),
                (1.0, 8, 1.0, 0.3, 0), (0.3, 1, 1.0, 0.0, 0), (1.0, 1, 1.0, 0.0, 1)], 3.0),
        (16, 16, [(1.0, 16, 1.0, 0.0, 0), (0.6, 4, 0.9, 0.05, 0), (1.3, 16, 0.7, 0.0, 0),
                  (1.0, 2, 1.0, 0.0, 0), (0.8, 16, 0.95, 0.1, 0), (1.0, 1, 1.0, 0.0, 0),
                  (2.0, 8, 0.5, 0.2, 0), (1.0, 1, 1.0, 0.0, 1)], 3.0),
        (4, 32, [(1.0, 32, 1.0, 0.0, 0), (0.9, 10, 0.85, 0.02, 0), (1.0, 32, 0.6, 0.0, 1)], 2.0),
        (3, 64, [(1.0, 64, 1.0, 0.0, 0), (0.7, 40, 0.9, 0.0, 0), (1.0, 5, 1.0, 0.0, 1)], 2.0),
        (3, 4, [(1.0, 4, 1.0, 0.0, 0), (0.5, 2, 0.7, 0.05, 0), (1.0, 5, 0.65, 0.2, 0)], 2.0),
    ]
    for (T, k, params, scale) in chain_cases:
        bs = len(params)
        n = bs * (T - 1)
        table = (torch.randn(n, k, k, generator=g) * scale).contiguous()
        cand = torch.stack([torch.randperm(151936, generator=g)[:k].sort().values
                            for _ in range(n)]).contiguous()
        gtok = cand[torch.arange(n), torch.randint(0, k, (n,), generator=g)].contiguous()
        u = torch.rand(n, generator=g)
        staged = (torch.tensor([1.0 / p[0] for p in params], dtype=torch.float32),
                  torch.tensor([p[1] for p in params], dtype=torch.int32),
                  torch.tensor([p[2] for p in params], dtype=torch.float32),
                  torch.tensor([p[3] for p in params], dtype=torch.float32),
                  torch.tensor([p[4] for p in params], dtype=torch.int32))
        tok = torch.full((n,), -1, dtype=torch.int64)
        q = torch.full((n, k), -1.0)
        conf = torch.full((n,), -0.25)
        K.serial_sample_chain(table, *staged, u, cand, gtok, tok, q, T, confidence_out=conf)
        rtok, rq = ref_sample_chain(table, *staged, u, cand, gtok, T)
        for name, val in (("table", table), ("inv_t", staged[0]), ("top_k", staged[1]),
                          ("top_p", staged[2]), ("min_p", staged[3]), ("greedy", staged[4]),
                          ("u", u), ("cand", cand), ("gtok", gtok), ("tok", tok), ("q", q),
                          ("conf", conf), ("ref_tok", rtok), ("ref_q", rq)):
            out[f"c{ci}_{name}"] = _np(val)
        out[f"c{ci}_T"] = np.array(T)
        ci += 1
    # exact tie between lanes 2 and 6 with top_k = 1: the lower lane wins
    T, k = 3, 8
    n = T - 1
    table = torch.zeros(n, k, k)
    table[:, :, 2] = 5.0
    table[:, :, 6] = 5.0
    cand = torch.arange(k, dtype=torch.int64).repeat(n, 1) + 100
    gtok = cand[:, 0].clone()
    staged = (torch.ones(1), torch.tensor([1], dtype=torch.int32), torch.ones(1), torch.zeros(1),
              torch.zeros(1, dtype=torch.int32))
    tok = torch.full((n,), -1, dtype=torch.int64)
    q = torch.full((n, k), -1.0)
    conf = torch.full((n,), -0.25)
    u = torch.zeros(n)
    K.serial_sample_chain(table, *staged, u, cand, gtok, tok, q, T, confidence_out=conf)
    rtok, rq = ref_sample_chain(table, *staged, u, cand, gtok, T)
    for name, val in (("table", table), ("inv_t", staged[0]), ("top_k", staged[1]),
                      ("top_p", staged[2]), ("min_p", staged[3]), ("greedy", staged[4]),
                      ("u", u), ("cand", cand), ("gtok", gtok), ("tok", tok), ("q", q),
                      ("conf", conf), ("ref_tok", rtok), ("ref_q", rq)):
        out[f"c{ci}_{name}"] = _np(val)
    out[f"c{ci}_T"] = np.array(T)
    ci += 1
    out["n_chain"] = np.array(ci)

    ti = 0
    for (bs, T, H, R, C, V, k, head) in ((2, 4, 512, 128, 64, 1024, 8, False),
                                         (2, 5, 1024, 256, 128, 2048, 16, False),
                                         (3, 3, 512, 128, 64, 512, 2, False),
                                         (1, 3, 512, 128, 64, 1024, 64, False),
                                         (2, 4, 512, 128, 64, 1024, 8, True)):
        d = _serial_refine_inputs(torch, g, bs, T, H, R, C, V, k)
        n = bs * (T - 1)
        tg, tsv = K.build_serial_tables(d["lm"], d["norm_w"], d["w_last"],
                                        torch.cat((d["pg"], d["pv"]), 0), d["codebook"])
        chead = d["lm"][d["cand"]].contiguous() if head else None
        conf = torch.empty(n, k)
        idx = K.serial_table(d["raw"], d["norm_w"], d["cand"], d["input_ids"], d["lm"], tg, tsv,
                             d["packed"], d["rms"], d["gb"], T, confidence=conf,
                             candidate_head=chead)
        chain = torch.full((n,), -1, dtype=torch.int64)
        cconf = torch.full((n,), -1.0)
        K.serial_chain(idx, d["cand"], chain, T, confidence=conf, confidence_out=cconf)
        ref = ref_refine_table(d["raw"], d["rms"], d["packed"][:, :R], d["anchors"], d["cand"],
                               d["codebook"], d["pg"], d["pv"], d["gb"], d["w_last"], d["norm_w"],
                               d["lm"], 1e-6, T)
        # only the table rows the kernels read (candidate and sender ids) are stored; every
        # other row of lm / tg / tsv may hold anything without changing a result
        used = torch.unique(torch.cat((d["cand"].flatten(), d["anchors"])))

        def bits(t):
            return _np(t.contiguous().view(torch.int16))

        out[f"t{ti}_dims"] = np.array([bs, T, H, R, C, V, k, int(head)])
        out[f"t{ti}_used"] = _np(used)
        for name in ("raw", "norm_w", "gb"):
            out[f"t{ti}_{name}"] = bits(d[name])
        out[f"t{ti}_query"] = bits(d["packed"][:, :R])
        out[f"t{ti}_lm"] = bits(d["lm"][used])
        out[f"t{ti}_tg"] = bits(tg[used])
        out[f"t{ti}_tsv"] = bits(tsv[used])
        for name in ("rms", "cand", "input_ids"):
            out[f"t{ti}_{name}"] = _np(d[name])
        for name, val in (("idx", idx), ("conf", conf), ("chain", chain), ("chain_conf", cconf),
                          ("ref_table", ref)):
            out[f"t{ti}_{name}"] = _np(val)
        ti += 1
    out["n_table"] = np.array(ti)
    return out


def gen_fp8(torch):
    """layers/fp8/coarse.py FullVFP8Coarse.__init__ (weight quantization), _scale/_quantize
    (hidden rows), stable_local_topk (portable argsort path), and layers/fp8/gather.py rescore
    and select16 (Triton kernels under the interpreter).  torch's CPU _scaled_mm refuses
    per-row scales, so the coarse GEMM itself has no CPU fixture."""
    from sglang_dspine.layers.fp8 import coarse, gather

    out = {}
    g = torch.Generator().manual_seed(13)
    # the reference test's exact two-column head (tests/test_topk_compat_cuda.py:103-109)
    w2 = torch.zeros(512, 512, dtype=torch.bfloat16)
    w2[:, 0] = torch.arange(512).remainder(47).bfloat16() / 32
    w2[:, 1] = torch.arange(512).remainder(31).bfloat16() / 64
    # a random head with an all-zero row and a tiny row
    wr = (torch.randn(300, 256, generator=g) * 0.05).bfloat16()
    wr[7] = 0
    wr[8] = 0
    wr[8, 3] = 1e-30
    for name, w in (("two", w2), ("rand", wr)):
        local = coarse.FullVFP8Coarse(torch, w)
        out[f"{name}_w"] = _np(w.float())
        out[f"{name}_wq"] = _np(local.weight8.view(torch.uint8))
        out[f"{name}_ws"] = _np(local.weight_scale[0])
    hidden = (torch.randn(6, 256, generator=g) * torch.tensor([[0.01], [1], [30], [0], [2], [5]])).bfloat16()
    scale = coarse._scale(torch, hidden)
    out["hidden"] = _np(hidden.float())
    out["hidden_q"] = _np(coarse._quantize(torch, hidden, scale).view(torch.uint8))
    out["hidden_s"] = _np(scale[:, 0])
    # stable top-k of tied bf16 scores
    scores = ((torch.randn(5, 3000, generator=g) * 3).round() / 2).bfloat16()
    scores[1] = 1.0
    scores[2, ::5] = float("-inf")
    out["topk_scores"] = _np(scores.float())
    for k in (1, 16, 128):
        out[f"topk_ids_{k}"] = _np(coarse.stable_local_topk(scores, k, None)[1])
    # rescore + select16 on the random head
    ids = torch.stack([torch.randperm(300, generator=g)[:128] for _ in range(6)])
    rescored = gather.rescore(torch, wr, ids, hidden)
    out["rescore_ids"] = _np(ids)
    out["rescore_scores"] = _np(rescored.float())
    out["rescore_top16"] = _np(gather.select16(torch, rescored, ids))
    # select16 on heavily tied scores
    tied = ((torch.randn(4, 128, generator=g)).round() / 2).bfloat16()
    tied_ids = torch.stack([torch.randperm(1000, generator=g)[:128] for _ in range(4)])
    out["tied_scores"] = _np(tied.float())
    out["tied_ids"] = _np(tied_ids)
    out["tied_top16"] = _np(gather.select16(torch, tied, tied_ids))
    return out


def gen_target_minp(torch):
    """ref_target_row (tests/ref_utils.py:79-108, float64) with min-p on, for the flashinfer
    backend (sequential top-k -> top-p -> min-p) and the pytorch backend (joint top-k / top-p
    and min-p), and with min-p off for the pytorch backend."""
    from ref_utils import ref_target_row

    out = {}
    ci = 0
    g = torch.Generator().manual_seed(11)
    params = [(0.7, 20, 0.9, 0.05), (1.0, 1 << 30, 0.95, 0.01), (1.3, 50, 1.0, 0.1),
              (0.5, 30, 0.8, 0.0), (1.0, 8, 0.6, 0.02), (2.0, 1 << 30, 1.0, 0.3),
              (0.9, 100, 0.7, 0.001), (1.1, 5, 0.99, 0.5)]
    for (T, k, tp, mp) in params:
        for backend in ("flashinfer", "pytorch"):
            for rep in range(2):
                V = [317, 2048][rep]
                l = torch.randn(V, generator=g) * 3
                if rep == 1:
                    l = l.bfloat16().float()  # quantised: ties everywhere
                ref = ref_target_row(l, T, k, tp, mp, backend)
                out[f"c{ci}_logits"] = _np(l.float())
                out[f"c{ci}_params"] = np.array([T, k, tp, mp], dtype=np.float64)
                out[f"c{ci}_backend"] = np.array(backend)
                out[f"c{ci}_p"] = _np(ref)
                ci += 1
    out["n"] = np.array(ci)
    return out


def gen_sparse_target(torch):
    """build_sparse_target's CPU branch (sampling/sparse/target.py:156-178) on CPU logits:
    random rows, bf16-quantised rows (ties at the k-th p), all-equal rows (overflow), a
    cutting top-p and every top-k in [1, 32]; compact rows mapped by row_to_request."""
    import types as _t

    from sglang_dspine.sampling.sparse.target import build_sparse_target

    out = {}
    ci = 0
    g = torch.Generator().manual_seed(23)
    for V, rows in ((257, 24), (4099, 16), (1000, 40)):
        for kind in ("random", "quantised", "ties"):
            bs = 8
            temps = 0.3 + 1.2 * torch.rand(bs, generator=g)
            ks = torch.randint(1, 33, (bs,), generator=g, dtype=torch.int32)
            tps = torch.where(torch.rand(bs, generator=g) < 0.5, torch.ones(bs),
                              0.5 + 0.5 * torch.rand(bs, generator=g))
            l = torch.randn(rows, V, generator=g) * 2.5
            if kind == "quantised":
                l = (l * 2).round() / 2  # many equal values, ties at the k-th p
            elif kind == "ties":
                l = (l > 1.5).float() * 3.0  # a plateau of equal tops: overflow rows
                l[::5] = 0.0                   # all-equal rows
            r2r = torch.randint(0, bs, (rows,), generator=g)
            info = _t.SimpleNamespace(temperatures=temps[:, None], top_ks=ks, top_ps=tps,
                                      min_ps=torch.zeros(bs), max_top_k=int(ks.max()),
                                      need_min_p_sampling=False, is_any_greedy=False)
            res = build_sparse_target(l, info, row_to_request=r2r, capacity=32,
                                      sampling_backend="flashinfer")
            ids, vals, lens, ovf = res.packed
            out[f"c{ci}_logits"] = _np(l.float())
            out[f"c{ci}_temp"] = _np(temps[r2r].float())
            out[f"c{ci}_topk"] = _np(ks[r2r])
            out[f"c{ci}_topp"] = _np(tps[r2r].float())
            out[f"c{ci}_ids"] = _np(ids)
            out[f"c{ci}_vals"] = _np(vals)
            out[f"c{ci}_lens"] = _np(lens)
            out[f"c{ci}_ovf"] = _np(ovf)
            ovf_rows = np.flatnonzero(_np(ovf))
            out[f"c{ci}_ovf_rows"] = ovf_rows
            out[f"c{ci}_dense"] = _np(res.dense_p[torch.as_tensor(ovf_rows, dtype=torch.long)])
            ci += 1
    out["n"] = np.array(ci)
    return out


class _Info:
    """SamplingBatchInfo stand-in for adjust_logits: the fields it reads and len()."""

    def __init__(self, bs, **fields):
        self._bs = bs
        self.__dict__.update(fields)

    def __len__(self):
        return self._bs


def _xgrammar_apply(logits, vocab_mask):
    """xgrammar's token-bitmask semantics (SGLang's XGrammarGrammar.apply_vocab_mask): bit i of
    row r's int32 words clear means token i is disallowed (-inf)."""
    import torch

    V = logits.shape[-1]
    shifts = torch.arange(32, dtype=torch.int32)
    bits = ((vocab_mask[:, :, None] >> shifts) & 1).reshape(vocab_mask.shape[0], -1)[:, :V]
    logits.masked_fill_(bits == 0, float("-inf"))


def gen_adjust(torch):
    """sampling/compact.py:14-79 adjust_logits on CPU tensors (pure torch in the reference):
    additive and scaling penalties, two penalizers of an orchestrator (multiplicative, then
    additive), a grammar bitmask applied through the grammar's own apply_vocab_mask (xgrammar
    semantics) and a logit bias; full [B, T, V] blocks and packed rows with row_to_request;
    bf16 and fp32 logits."""
    import types as _t

    from sglang_dspine.sampling.compact import adjust_logits

    out = {}
    ci = 0
    g = torch.Generator().manual_seed(31)
    B, T, V = 4, 16, 517
    words = (V + 31) // 32
    for dtype in (torch.float32, torch.bfloat16):
        for packed in (False, True):
            add = torch.randn(B, V, generator=g)
            scl = 1.0 + torch.rand(B, V, generator=g)
            bias = torch.randn(B, V, generator=g) * 0.5
            mask = torch.randint(-2**31, 2**31 - 1, (B, words), generator=g,
                                 dtype=torch.int64).to(torch.int32)
            pen_scale = 1.0 + 0.5 * torch.rand(B, V, generator=g)
            pen_add = torch.randn(B, V, generator=g) * 0.25
            mult = _t.SimpleNamespace(is_prepared=lambda: True, is_multiplicative=True,
                                      get_scaling_penalties=lambda s=pen_scale: s)
            addp = _t.SimpleNamespace(is_prepared=lambda: True, is_multiplicative=False,
                                      apply=lambda b, a=pen_add: b.add_(a))
            idle = _t.SimpleNamespace(is_prepared=lambda: False, is_multiplicative=False)
            info = _Info(B, acc_additive_penalties=add, acc_scaling_penalties=scl,
                         penalizer_orchestrator=_t.SimpleNamespace(
                             is_required=True, penalizers={"m": mult, "i": idle, "a": addp}),
                         grammar_mask=_t.SimpleNamespace(
                             vocab_mask=mask, grammar=_t.SimpleNamespace(apply_vocab_mask=_xgrammar_apply)),
                         logit_bias=bias)
            if packed:
                rows = 37
                r2r = torch.randint(0, B, (rows,), generator=g)
                x = (torch.randn(rows, V, generator=g) * 3).to(dtype)
            else:
                r2r = None
                x = (torch.randn(B, T, V, generator=g) * 3).to(dtype)
            y = x.clone()
            adjust_logits(y, info, r2r)
            for name, val in (("add", add), ("scl", scl), ("bias", bias), ("mask", mask),
                              ("pen_scale", pen_scale), ("pen_add", pen_add)):
                out[f"c{ci}_{name}"] = _np(val)
            out[f"c{ci}_r2r"] = _np(r2r) if r2r is not None else np.zeros(0, np.int64)
            out[f"c{ci}_x"] = _np(x.float())
            out[f"c{ci}_y"] = _np(y.float())
            out[f"c{ci}_bf16"] = np.array(dtype == torch.bfloat16)
            ci += 1
    out["n"] = np.array(ci)
    return out


def _fullv_case(torch, batch, ref_target_row, chain):
    """Reference outputs of one benchmark batch at the full vocabulary: target rows through
    ref_target_row (float64, then float32) or a one-hot at the lowest-index argmax for greedy
    requests (runtime/worker.py:461-469), q rows the same filter on the draft logits (one-hot
    at the drafted token for greedy requests), then the reference's
    sample_capped_chain_from_probs under the Triton interpreter."""
    B, V = batch.B, batch.V
    lens = batch.verify_lens.tolist()
    P = torch.zeros(B, 16, V)
    Q = torch.zeros(B, 15, V)
    for b in range(B):
        T, k, tp = float(batch.temperature[b]), int(batch.top_k[b]), float(batch.top_p[b])
        greedy = k <= 1 or not T > 0
        for s in range(lens[b]):
            row = batch.target_logits[int(batch.target_rows[b]) + s]
            if greedy:
                P[b, s, int(row.argmax())] = 1.0
            else:
                P[b, s] = ref_target_row(row.float(), T, k, tp, 0.0, "flashinfer").float()
        for s in range(lens[b] - 1):
            if greedy:
                Q[b, s, int(batch.candidates[b, s + 1])] = 1.0
            else:
                row = batch.draft_logits[int(batch.draft_rows[b]) + s]
                Q[b, s] = ref_target_row(row.float(), T, k, tp, 0.0, "flashinfer").float()
    outs = _buffers(torch, B)
    chain(candidates=batch.candidates, target_probs=P.contiguous(), draft_probs=Q.contiguous(),
          verify_lens=batch.verify_lens, uniforms=batch.uniforms,
          uniform_final=batch.uniform_final, prefix_lens=batch.prefix_lens, outputs=outs)
    # distance of each bonus draw from the nearest CDF step, relative to the draw's mass
    # (float64 over the float32 rows the reference kernel consumed)
    margin = np.zeros(B)
    for b in range(B):
        a = int(outs[0][b])
        p = P[b, a].double()
        if a == lens[b] - 1:
            w = p
        else:
            w = (p - Q[b, a].double().clamp(0, 1)).clamp_min(0)
            if float(w.sum()) <= 0:
                w = p
        cdf = torch.cumsum(w, 0)
        thr = float(batch.uniform_final[b]) * float(cdf[-1])
        j = int(outs[2][b])
        lo = float(cdf[j - 1]) if j > 0 else 0.0
        margin[b] = min(abs(thr - lo), abs(float(cdf[j]) - thr)) / float(cdf[-1])
    return outs, margin


def gen_fullv(torch):
    """Benchmark configurations at V = 151936 pinned to the reference itself: configs 0, 1
    and 4 whole (dspine_b200.workloads), outputs of the reference's
    sample_capped_chain_from_probs over ref_target_row probabilities.  Only the outputs, a
    fingerprint of the regenerated inputs and the draw margins are stored; the tests
    regenerate the inputs from the same seeds."""
    from ref_utils import ref_target_row
    from sglang_dspine.sampling.rejection import sample_capped_chain_from_probs

    sys.path.insert(0, str(HERE.parents[1]))
    from dspine_b200 import workloads

    out = {}
    for name, batch in (("config0", workloads.config0()), ("config1", workloads.config1()),
                        ("config4", workloads.config4())):
        outs, margin = _fullv_case(torch, batch, ref_target_row, sample_capped_chain_from_probs)
        out[f"{name}_fingerprint"] = workloads.fingerprint(batch)
        out[f"{name}_margin"] = margin
        for key, val in zip(("accept", "commit", "bonus", "output", "new_seq"), outs):
            out[f"{name}_{key}"] = _np(val)
    return out


def main(ref_dir):
    os.environ.setdefault("TRITON_INTERPRET", "1")
    os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(ref_dir))
    _install_stubs()
    import torch

    torch.manual_seed(0)
    sys.path.insert(0, str(Path(ref_dir) / "tests"))
    groups = {
        "chain": lambda: gen_chain(torch),
        "sparse": lambda: gen_sparse(torch),
        "target": lambda: gen_target(torch, ref_dir),
        "topk": lambda: gen_topk(torch),
        "uniforms": lambda: gen_uniforms(torch),
        "sps": lambda: gen_sps(torch),
        "merge": lambda: gen_merge(torch),
        "greedy": lambda: gen_greedy(torch),
        "serial": lambda: gen_serial(torch, ref_dir),
        "fp8": lambda: gen_fp8(torch),
        "fullv": lambda: gen_fullv(torch),
        "target_minp": lambda: gen_target_minp(torch),
        "sparse_target": lambda: gen_sparse_target(torch),
        "adjust": lambda: gen_adjust(torch),
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
