"""Parity of the draft-side serial chains (dsv_serial_sample_chain, dsv_serial_table,
dsv_serial_chain) with the reference kernels and the CPU oracle.

Reference semantics: kernels/dspine.py:210-324 (_serial_table, _serial_chain) and 616-772
(_serial_sample_chain); the reference's tests pin them the same way (tests/test_cuda.py:141-450,
tests/test_sampled_confidence.py): sampled tokens exact, q within rtol 1e-5 / atol 1e-6,
greedy-table picks an argmax of the fp64 table up to accumulation error.  Fixtures in
tests/golden/serial.npz hold the reference kernels' own outputs.
"""

import math

import numpy as np
import pytest
import torch

import oracle.serial as OS
from dspine_b200.kernels import dspine as K
from tests.helpers import serial_chain_case, serial_scores, serial_table_case

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLDEN = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "serial.npz")


def run_chain(inp, conf_fill=-0.25, with_conf=True):
    n, k = inp["cand"].shape
    t = lambda a, dt: torch.as_tensor(np.asarray(a), dtype=dt, device=DEV).contiguous()  # noqa: E731
    out_tok = torch.full((n,), -1, dtype=torch.int64, device=DEV)
    out_q = torch.full((n, k), -1.0, device=DEV)
    conf = torch.full((n,), conf_fill, device=DEV) if with_conf else None
    K.serial_sample_chain(t(inp["table"], torch.float32), t(inp["inv_t"], torch.float32),
                          t(inp["top_k"], torch.int32), t(inp["top_p"], torch.float32),
                          t(inp["min_p"], torch.float32), t(inp["greedy"], torch.int32),
                          t(inp["u"], torch.float32), t(inp["cand"], torch.int64),
                          t(inp["greedy_tok"], torch.int64), out_tok, out_q, inp["T"],
                          confidence_out=conf)
    torch.cuda.synchronize()
    return out_tok.cpu().numpy(), out_q.cpu().numpy(), None if conf is None else conf.cpu().numpy()


@pytest.mark.parametrize("ci", range(int(GOLDEN["n_chain"])))
def test_sample_chain_matches_reference_kernel(ci):
    inp, ref = serial_chain_case(GOLDEN, ci)
    tok, q, conf = run_chain(inp)
    np.testing.assert_array_equal(tok, ref["tok"])
    np.testing.assert_allclose(q, ref["q"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(q.sum(-1), np.ones(len(q)), rtol=0, atol=1e-5)
    np.testing.assert_allclose(conf, ref["conf"], rtol=1e-5, atol=1e-6)  # greedy rows keep -0.25
    lane = (inp["cand"] == tok[:, None]).argmax(-1)
    assert (q[np.arange(len(q)), lane] > 0).all()


def random_chain_case(seed, bs, T, k, scale=3.0):
    g = np.random.default_rng(seed)
    n = bs * (T - 1)
    inp = dict(
        table=(g.standard_normal((n, k, k)) * scale).astype(np.float32),
        inv_t=(1.0 / g.uniform(0.3, 2.0, bs)).astype(np.float32),
        top_k=np.where(g.random(bs) < 0.3, k, g.integers(1, k + 1, bs)).astype(np.int32),
        top_p=np.where(g.random(bs) < 0.3, 1.0, g.uniform(0.3, 1.0, bs)).astype(np.float32),
        min_p=np.where(g.random(bs) < 0.5, 0.0, g.uniform(0.0, 0.3, bs)).astype(np.float32),
        greedy=(g.random(bs) < 0.15).astype(np.int32),
        u=g.random(n).astype(np.float32),
        T=T,
    )
    inp["cand"] = np.stack([np.sort(g.choice(151936, k, replace=False)) for _ in range(n)]).astype(np.int64)
    inp["greedy_tok"] = inp["cand"][np.arange(n), g.integers(0, k, n)]
    return inp


@pytest.mark.parametrize("k", [1, 2, 3, 8, 16, 31, 32, 33, 48, 64])
def test_sample_chain_matches_oracle_any_width(k):
    inp = random_chain_case(100 + k, bs=24, T=16, k=k)
    tok, q, conf = run_chain(inp, conf_fill=float("nan"))
    otok, oq, oconf = OS.sample_chain(**inp)
    np.testing.assert_array_equal(tok, otok)
    np.testing.assert_allclose(q, oq, rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(conf, oconf, rtol=1e-5, atol=1e-6, equal_nan=True)


def test_sample_chain_without_confidence_is_identical():
    inp = random_chain_case(7, bs=9, T=16, k=16)
    tok_a, q_a, _ = run_chain(inp)
    tok_b, q_b, _ = run_chain(inp, with_conf=False)
    assert np.array_equal(tok_a, tok_b) and np.array_equal(q_a.view(np.int32), q_b.view(np.int32))


def test_sample_chain_ties_break_to_lower_lane():
    T, k = 3, 8
    n = T - 1
    table = np.zeros((n, k, k), np.float32)
    table[:, :, 2] = 5.0
    table[:, :, 6] = 5.0
    cand = np.tile(np.arange(k, dtype=np.int64) + 100, (n, 1))
    inp = dict(table=table, inv_t=np.ones(1, np.float32), top_k=np.ones(1, np.int32),
               top_p=np.ones(1, np.float32), min_p=np.zeros(1, np.float32),
               greedy=np.zeros(1, np.int32), u=np.zeros(n, np.float32), cand=cand,
               greedy_tok=cand[:, 0].copy(), T=T)
    tok, q, _ = run_chain(inp)
    assert tok.tolist() == [102, 102] and q[:, 2].tolist() == [1.0, 1.0]


def test_confidence_follows_the_sampled_prefix():
    """Confidence of row i is max softmax(table[i, sender]) with sender = the lane actually
    drawn on row i-1, taken before filtering (tests/test_sampled_confidence.py semantics)."""
    width, k = 4, 4
    dist = np.array([[0.899, 0.099, 0.001, 0.001], [0.4, 0.3, 0.2, 0.1],
                     [0.6, 0.2, 0.1, 0.1], [0.25, 0.25, 0.25, 0.25]], np.float32)
    table = np.broadcast_to(np.log(dist), (width - 1, k, k)).copy()
    table[0] = np.broadcast_to(np.log(dist[1]), (k, k))
    cand = np.tile(np.arange(10, 10 + k, dtype=np.int64), (width - 1, 1))

    def run(draws):
        inp = dict(table=table, inv_t=np.ones(1, np.float32), top_k=np.full(1, k, np.int32),
                   top_p=np.ones(1, np.float32), min_p=np.zeros(1, np.float32),
                   greedy=np.zeros(1, np.int32), u=np.array(draws, np.float32), cand=cand,
                   greedy_tok=cand[:, 0].copy(), T=width)
        return run_chain(inp, conf_fill=-1.0)

    first = run([0.05, 0.2, 0.4])
    changed_first = run([0.55, 0.2, 0.4])
    changed_second = run([0.05, 0.95, 0.4])
    assert first[0][0] != changed_first[0][0]
    assert first[2][0] == changed_first[2][0] and first[2][1] != changed_first[2][1]
    assert first[0][1] != changed_second[0][1]
    assert first[2][1] == changed_second[2][1] and first[2][2] != changed_second[2][2]


def test_prefilter_confidence_when_q_is_one_hot():
    p = np.array([[0.85, 0.14, 0.009, 0.001], [0.99, 0.008, 0.001, 0.001]], np.float32)
    k, width, temp = 4, 2, 0.7
    table = np.broadcast_to((np.log(p) * temp)[:, None, :], (2, k, k)).astype(np.float32).copy()
    inp = dict(table=table, inv_t=np.full(2, 1 / temp, np.float32), top_k=np.full(2, 5, np.int32),
               top_p=np.full(2, 0.8, np.float32), min_p=np.full(2, 0.05, np.float32),
               greedy=np.zeros(2, np.int32), u=np.array([0.2, 0.8], np.float32),
               cand=np.tile(np.arange(k, dtype=np.int64), (2, 1)), greedy_tok=np.zeros(2, np.int64),
               T=width)
    _, q, conf = run_chain(inp)
    np.testing.assert_allclose(q.max(-1), np.ones(2), rtol=0, atol=1e-6)
    np.testing.assert_allclose(conf, p.max(-1), rtol=1e-5, atol=1e-6)


def table_tensors(case):
    bf = lambda a: torch.as_tensor(a, device=DEV).to(torch.bfloat16).contiguous()  # noqa: E731
    m = case["bs"] * case["T"]
    packed = torch.zeros(m, 3 * case["R"], dtype=torch.bfloat16, device=DEV)
    packed[:, : case["R"]] = bf(case["query"])
    cand = torch.as_tensor(case["cand"], device=DEV)
    lm = bf(case["lm"])
    return dict(raw=bf(case["raw"]), norm_w=bf(case["norm_w"]), cand=cand,
                input_ids=torch.as_tensor(case["input_ids"], device=DEV), lm=lm,
                tg=bf(case["tg"]), tsv=bf(case["tsv"]), packed=packed,
                rms=torch.as_tensor(case["rms"], device=DEV), gb=bf(case["gb"]),
                head=lm[cand].contiguous() if case["head"] else None)


def run_table(case):
    g = table_tensors(case)
    n, k = case["cand"].shape
    conf = torch.empty(n, k, device=DEV)
    idx = K.serial_table(g["raw"], g["norm_w"], g["cand"], g["input_ids"], g["lm"], g["tg"],
                         g["tsv"], g["packed"], g["rms"], g["gb"], case["T"], confidence=conf,
                         candidate_head=g["head"])
    chain = torch.full((n,), -1, dtype=torch.int64, device=DEV)
    cconf = torch.full((n,), -1.0, device=DEV)
    K.serial_chain(idx, g["cand"], chain, case["T"], confidence=conf, confidence_out=cconf)
    torch.cuda.synchronize()
    return idx.cpu().numpy(), conf.cpu().numpy(), chain.cpu().numpy(), cconf.cpu().numpy()


@pytest.mark.parametrize("ti", range(int(GOLDEN["n_table"])))
def test_serial_table_matches_reference_kernel(ti):
    """Picks equal the reference kernel's wherever the fp64 scores separate the best lane from
    the runner-up by more than the fp32 accumulation error; every pick is an admissible argmax;
    confidences within 2e-4; the greedy walk equals the reference walk where picks agree."""
    case, ref = serial_table_case(GOLDEN, ti)
    idx, conf, chain, cconf = run_table(case)
    s, bound = serial_scores(case)
    tol = 2e-5 * bound.max(axis=2)
    picked = np.take_along_axis(s, idx[..., None], axis=2)[..., 0]
    assert (picked >= s.max(axis=2) - tol).all()
    top2 = np.sort(s, axis=2)[..., -2:]
    clear = (top2[..., 1] - top2[..., 0]) > 2 * tol
    assert clear.mean() > 0.9
    np.testing.assert_array_equal(idx[clear], ref["idx"][clear])
    np.testing.assert_allclose(conf, ref["conf"], rtol=2e-4, atol=1e-6)
    ochain, ocout = OS.chain(idx, case["cand"], case["T"], conf)
    np.testing.assert_array_equal(chain, ochain)
    np.testing.assert_array_equal(cconf, ocout)
    if (idx == ref["idx"]).all():
        np.testing.assert_array_equal(chain, ref["chain"])


def _assert_chain_is_refined_argmax(out, cand, ref, bs, T):
    """The pick of every drafted row is an argmax of the redone last write (fp64) up to bf16
    table rounding (tests/test_cuda.py:297-313)."""
    for b in range(bs):
        j = 0
        for i in range(T - 1):
            nn = b * (T - 1) + i
            lane = int(np.nonzero(cand[nn] == out[nn])[0][0])
            row = ref[nn, j]
            assert row[lane] >= row.max() - 2e-2 * np.abs(row).max(), (b, i)
            j = lane


@pytest.mark.parametrize("ti", range(int(GOLDEN["n_table"])))
def test_greedy_chain_follows_refined_argmax(ti):
    case, ref = serial_table_case(GOLDEN, ti)
    _, _, chain, _ = run_table(case)
    _assert_chain_is_refined_argmax(chain, case["cand"], ref["ref_table"], case["bs"], case["T"])


def test_refine_tables_realistic_shapes():
    """H=4096, R=512, C=1024, V=4096, K=16, T=16: tables built on the GPU, greedy chain
    checked against the fp64 redone last write."""
    bs, T, H, R, C, V, k = 2, 16, 4096, 512, 1024, 4096, 16
    m, n = bs * T, bs * (T - 1)
    g = torch.Generator().manual_seed(5)
    bf = torch.bfloat16

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g) * scale).to(bf)

    raw, packed = rnd(m, H), rnd(m, 3 * R)
    rms = torch.rand(m, generator=g) + 0.5
    codebook = rnd(V, C, scale=1 / math.sqrt(C))
    pg, pv = rnd(R, C, scale=1 / math.sqrt(C)), rnd(R, C, scale=1 / math.sqrt(C))
    gb, w_last = rnd(R, scale=0.1), rnd(H, R, scale=1 / math.sqrt(R))
    norm_w = (1 + 0.1 * torch.randn(H, generator=g)).to(bf)
    lm = rnd(V, H, scale=1 / math.sqrt(H))
    cand = torch.stack([torch.randperm(V, generator=g)[:k].sort().values for _ in range(n)])
    input_ids = torch.randint(0, V, (m,), generator=g)
    anchors = input_ids.view(bs, T)[:, 0]
    d = lambda x: x.to(DEV).contiguous()  # noqa: E731
    tg, tsv = K.build_serial_tables(d(lm), d(norm_w), d(w_last), d(torch.cat((pg, pv), 0)),
                                    d(codebook))
    idx = K.serial_table(d(raw), d(norm_w), d(cand), d(input_ids), d(lm), tg, tsv, d(packed),
                         d(rms), d(gb), T)
    out = torch.empty(n, dtype=torch.int64, device=DEV)
    K.serial_chain(idx, d(cand), out, T)
    torch.cuda.synchronize()
    f = lambda x: x.float().numpy()  # noqa: E731
    lmf = f(lm)
    ref = OS.refine_table(f(raw), rms.numpy(), f(packed[:, :R]), anchors.numpy(), cand.numpy(),
                          f(codebook), f(pg), f(pv), f(gb), f(w_last), f(norm_w),
                          lambda ids: lmf[ids], 1e-6, T)
    _assert_chain_is_refined_argmax(out.cpu().numpy(), cand.numpy(), ref, bs, T)


def test_serial_chain_lane_outside_range_selects_zero():
    T, k = 4, 4
    n = T - 1
    idx = torch.tensor([[1, 0, 0, 0], [0, 9, 0, 0], [3, 0, 0, 0]], dtype=torch.int64, device=DEV)
    cand = torch.arange(n * k, dtype=torch.int64, device=DEV).view(n, k) + 50
    conf = torch.rand(n, k, device=DEV)
    out = torch.full((n,), -1, dtype=torch.int64, device=DEV)
    cout = torch.full((n,), -1.0, device=DEV)
    K.serial_chain(idx, cand, out, T, confidence=conf, confidence_out=cout)
    torch.cuda.synchronize()
    o, c = OS.chain(idx.cpu().numpy(), cand.cpu().numpy(), T, conf.cpu().numpy())
    assert out.cpu().tolist() == o.tolist() == [51, 0, 58]
    np.testing.assert_array_equal(cout.cpu().numpy(), c)


def test_serial_table_flags_out_of_range_ids():
    case, _ = serial_table_case(GOLDEN, 0)
    case = dict(case)
    cand = case["cand"].copy()
    cand[1, 3] = case["V"] + 5  # row 1 reads it as a candidate, row 2 as a sender
    case["cand"] = cand
    idx, conf, _, _ = run_table(case)
    assert (idx[1] == -1).all() and np.isnan(conf[1]).all()
    assert (idx[2] == -1).all()
    assert (idx[0] >= 0).all()
