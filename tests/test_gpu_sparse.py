"""Parity of the sparse-q rejection and probability compression with the reference's own
kernel outputs (golden sparse.npz: dense, compact, overflow-mixed and pure-packed targets, raw
denominators) and with the CPU oracle on seeded inputs (sampling/sparse/accept.py:94-543).
Integer outputs and compressed entries: bit-exact."""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle as O
from dspine_b200.sampling.sparse.accept import accept_sparse, compress_probs
from dspine_b200.verify import new_outputs

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"
NAMES = ("accept", "commit", "bonus", "output", "new_seq")


def t(x):
    return torch.as_tensor(np.ascontiguousarray(x)).to(DEV)


def cases(d):
    return sorted({int(k.split("_")[0][1:]) for k in d.files if k.startswith("c") and "_" in k})


def run(cand, dense, packed, qids, qvals, caps, u, uf, prefix, offsets=None, vocab=None,
        denominator=None):
    B = cand.shape[0]
    out = new_outputs(B, DEV)
    accept_sparse(torch, candidates=t(cand), dense_p=None if dense is None else t(dense),
                  packed=None if packed is None else tuple(t(x) for x in packed),
                  q_ids=t(qids), q_values=t(qvals), verify_lens=t(caps), uniforms=t(u),
                  uniform_final=t(uf), prefix_lens=t(prefix), outputs=out,
                  row_offsets=None if offsets is None else t(offsets), vocab_size=vocab,
                  denominator=None if denominator is None else t(denominator),
                  raw_fallback=denominator is not None)
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in out]


def test_accept_sparse_matches_reference_golden():
    d = np.load(GOLDEN / "sparse.npz")
    for c in cases(d):
        kind = str(d[f"c{c}_kind"])
        packed = None if kind == "dense" else tuple(d[f"c{c}_{n}"] for n in ("ids", "vals", "lens", "ovf"))
        dense = None if kind == "pure_packed" else d[f"c{c}_p"]
        got = run(d[f"c{c}_cand"], dense, packed, d[f"c{c}_qids"], d[f"c{c}_qvals"],
                  d[f"c{c}_caps"], d[f"c{c}_u"], d[f"c{c}_uf"], d[f"c{c}_prefix"],
                  d[f"c{c}_offsets"], d[f"c{c}_p"].shape[-1])
        for name, g in zip(NAMES, got):
            assert np.array_equal(g, d[f"c{c}_{name}"]), (c, kind, name)


def test_compress_probs_matches_reference_golden():
    d = np.load(GOLDEN / "sparse.npz")
    seen = 0
    for c in cases(d):
        if f"c{c}_cids" not in d.files:
            continue
        seen += 1
        ids, vals, lens, ovf = compress_probs(torch, t(d[f"c{c}_p"]), capacity=32)
        torch.cuda.synchronize()
        assert np.array_equal(ids.cpu().numpy(), d[f"c{c}_cids"]), c
        assert np.array_equal(vals.cpu().numpy(), d[f"c{c}_cvals"]), c
        assert np.array_equal(lens.cpu().numpy(), d[f"c{c}_clens"]), c
        assert np.array_equal(ovf.cpu().numpy(), d[f"c{c}_covf"]), c
    assert seen > 0


def random_sparse(seed, B, V, width):
    rng = np.random.default_rng(seed)
    rows = B * 16
    logits = rng.normal(0, 2.5, (rows, V)).astype(np.float32)
    p = np.exp(logits - logits.max(-1, keepdims=True))
    keep = rng.random((rows, V)) < 0.3
    p = np.where(keep, p, 0.0)
    p = (p / p.sum(-1, keepdims=True)).astype(np.float32)
    cand = rng.integers(0, V, (B, 16)).astype(np.int64)
    # candidates drawn from p so that some are accepted
    for r in range(B):
        for s in range(15):
            cand[r, s + 1] = rng.choice(V, p=p[r * 16 + s] / p[r * 16 + s].sum())
    qids = rng.integers(0, V, (B, 15, 16)).astype(np.int64)
    qids[:, :, 0] = cand[:, 1:]
    qids[:, :, 1] = cand[:, 1:]                      # duplicate ids sum
    qvals = (rng.random((B, 15, 16)) * 0.3).astype(np.float32)
    qvals[0, :, 2] = 1.5                             # out of [0,1]: clamped to 0 in the residual
    caps = rng.integers(1, 17, B).astype(np.int32)
    u = rng.random((B, 15)).astype(np.float32)
    u[0] = 0.0
    caps[0] = 16
    uf = rng.random(B).astype(np.float32)
    uf[1] = 1.0
    prefix = rng.integers(0, 100, B).astype(np.int32)
    ids, vals, lens, ovf = O.compress_probs(p, capacity=width)
    return cand, p, (ids, vals, lens, ovf), qids, qvals, caps, u, uf, prefix


@pytest.mark.parametrize("B,V,width", [(8, 257, 32), (12, 4099, 64), (6, 151936, 32)])
def test_accept_sparse_matches_oracle(B, V, width):
    cand, p, packed, qids, qvals, caps, u, uf, prefix = random_sparse(B * 31 + V, B, V, width)
    offsets = (np.arange(B) * 16).astype(np.int64)
    # dense
    want = O.accept_sparse(cand, p, None, qids, qvals, caps, u, uf, prefix, row_offsets=offsets)
    got = run(cand, p, None, qids, qvals, caps, u, uf, prefix, offsets)
    for name, g, w in zip(NAMES, got, want):
        assert np.array_equal(g, w), ("dense", name)
    # packed with dense fallback for overflowed rows
    want = O.accept_sparse(cand, p, packed, qids, qvals, caps, u, uf, prefix, row_offsets=offsets)
    got = run(cand, p, packed, qids, qvals, caps, u, uf, prefix, offsets)
    for name, g, w in zip(NAMES, got, want):
        assert np.array_equal(g, w), ("packed", name)
    # raw dense rows with per-row denominators
    den = (1.0 + np.random.default_rng(1).random(B * 16)).astype(np.float32)
    raw = (p * den[:, None]).astype(np.float32)
    want = O.accept_sparse(cand, raw, None, qids, qvals, caps, u, uf, prefix, row_offsets=offsets,
                           denominator=den)
    got = run(cand, raw, None, qids, qvals, caps, u, uf, prefix, offsets, denominator=den)
    for name, g, w in zip(NAMES, got, want):
        assert np.array_equal(g, w), ("raw", name)


@pytest.mark.parametrize("V,cap", [(97, 8), (4099, 64), (151936, 32)])
def test_compress_probs_matches_oracle(V, cap):
    rng = np.random.default_rng(V)
    p = rng.random((40, V)).astype(np.float32)
    p[p < 0.9995] = 0.0                                  # sparse rows
    p[3, :] = 0.0                                         # empty row
    p[5, 7] = -1.0                                        # a bad entry
    p[6, 9] = np.nan
    got = compress_probs(torch, t(p), capacity=cap)
    torch.cuda.synchronize()
    want = O.compress_probs(p, capacity=cap)
    for g, w in zip(got, want):
        assert np.array_equal(g.cpu().numpy(), w)
