"""Parity of the per-request kernels with the CPU oracle and the reference's golden vectors:
greedy capped accept (dsv_accept_greedy vs verification/caps.py:32-59, golden greedy.npz),
seeded uniforms (dsv_uniforms vs sampling/random.py:22-43 _cpu_uniforms, golden uniforms.npz),
SPS lengths/index (dsv_sps_plan vs verification/sps.py:27-58, golden sps.npz) and the
standalone accept-compact (dsv_accept_compact vs the oracle's restated commit contract).
All outputs are integers or exactly-rounded floats: compared bit for bit."""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle as O
from dspine_b200 import accept
from dspine_b200.sampling import random as R
from dspine_b200.verification import sps

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"


def t(x, dtype=None):
    return torch.as_tensor(np.asarray(x), dtype=dtype).to(DEV)


def test_greedy_matches_golden_and_oracle():
    g = np.load(GOLDEN / "greedy.npz")
    for c in range(int(g["n"])):
        cand, top1 = g[f"c{c}_cand"], g[f"c{c}_top1"]
        caps, prefix = g[f"c{c}_caps"], g[f"c{c}_prefix"]
        out = accept.accept_greedy(t(cand), t(top1), t(caps), t(prefix))
        torch.cuda.synchronize()
        for name, got in zip(("accept", "commit", "bonus", "output", "new_seq"), out):
            assert np.array_equal(got.cpu().numpy(), g[f"c{c}_{name}"]), (c, name)


@pytest.mark.parametrize("B", [1, 7, 64, 300])
def test_greedy_random_matches_oracle_strided_top1(B):
    rng = np.random.default_rng(B)
    cand = rng.integers(0, 50, (B, 16)).astype(np.int64)
    top1 = cand.copy()
    top1[:, :-1] = cand[:, 1:]
    flip = rng.random((B, 16)) < 0.15
    top1[flip] = rng.integers(0, 50, flip.sum())
    caps = rng.integers(1, 17, B).astype(np.int32)
    prefix = rng.integers(0, 1000, B).astype(np.int32)
    want = O.accept_greedy(cand, top1, caps, prefix)
    # top1 as column 0 of a [B*16, 5] array (the merged top-k ids of a head)
    wide = np.zeros((B * 16, 5), np.int64)
    wide[:, 0] = top1.reshape(-1)
    wide[:, 1:] = -7
    ids = t(wide)
    out = accept.accept_greedy(t(cand), ids[:, 0].view(B, 16), t(caps), t(prefix))
    torch.cuda.synchronize()
    for got, exp in zip(out, want):
        assert np.array_equal(got.cpu().numpy(), exp)


def test_uniforms_match_golden_bitwise():
    g = np.load(GOLDEN / "uniforms.npz")
    seeds, pos = t(g["seeds"]), t(g["positions"])
    for s in range(4):
        got = R.seeded_uniforms(seeds, pos, 15, s).cpu().numpy()
        assert np.array_equal(got.view(np.uint32), g[f"s{s}"].view(np.uint32))
    got32 = R.seeded_uniforms(seeds, pos.to(torch.int32), 15, 1).cpu().numpy()
    assert np.array_equal(got32, g["s1"])


def test_uniforms_random_match_oracle():
    rng = np.random.default_rng(5)
    seeds = rng.integers(-2**63, 2**63 - 1, 513, dtype=np.int64)
    pos = rng.integers(0, 2**40, 513).astype(np.int64)
    for width in (1, 15, 300):
        got = R.seeded_uniforms(t(seeds), t(pos), width, 2).cpu().numpy()
        assert np.array_equal(got, O.uniforms(seeds, pos, width, 2))


def test_sps_matches_golden():
    g = np.load(GOLDEN / "sps.npz")
    for c in range(int(g["n"])):
        raw, table, budget = g[f"c{c}_raw"], g[f"c{c}_table"], int(g[f"c{c}_budget"])
        bnd = g[f"c{c}_boundaries"] if f"c{c}_boundaries" in g.files else None
        lens, qo, index = sps.sps_plan(t(raw), t(table), torch.arange(15, device=DEV), budget,
                                       None if bnd is None else t(bnd))
        torch.cuda.synchronize()
        assert np.array_equal(lens.cpu().numpy(), g[f"c{c}_lens"]), c
        e_qo, e_index = O.sps_index(g[f"c{c}_lens"])
        assert np.array_equal(qo.cpu().numpy(), e_qo) and np.array_equal(index.cpu().numpy(), e_index)


@pytest.mark.parametrize("B,nb", [(256, 16), (1024, 7), (33, 4)])
def test_sps_random_matches_oracle(B, nb):
    rng = np.random.default_rng(B + nb)
    raw = rng.random((B, 15)).astype(np.float32)
    raw[rng.random((B, 15)) < 0.05] = 1.0  # bin edge
    table = np.clip(rng.random((15, nb)), 0.05, 0.999).astype(np.float32)
    table[3] = table[2]                     # ties in survival
    for budget in (B, B * 4, B * 16, B + 1):
        lens = sps.allocate_verify_lens(t(raw), t(table), torch.arange(15, device=DEV), budget)
        torch.cuda.synchronize()
        assert np.array_equal(lens.cpu().numpy(), O.sps_lens(raw, table, budget))


@pytest.mark.parametrize("B", [1, 64, 1500])
def test_accept_compact_matches_oracle(B):
    rng = np.random.default_rng(B)
    lens = rng.integers(1, 17, B).astype(np.int32)
    commit = np.minimum(rng.integers(1, 17, B), lens).astype(np.int32)
    output = rng.integers(0, 151936, (B, 16)).astype(np.int64)
    slots = rng.permutation(B * 16 + 64)[: B * 16].astype(np.int32)
    rows = (np.arange(B) * 16).astype(np.int64)
    comp = accept.accept_compact(t(commit), t(lens), t(output), t(slots), t(rows))
    torch.cuda.synchronize()
    tok, sl, off, fr, foff = O.accept_compact(commit, lens, output, slots, rows)
    n, m = int(off[-1]), int(foff[-1])
    assert np.array_equal(comp.offsets.cpu().numpy(), off)
    assert np.array_equal(comp.freed_offsets.cpu().numpy(), foff)
    assert np.array_equal(comp.tokens[:n].cpu().numpy(), tok)
    assert np.array_equal(comp.kept_slots[:n].cpu().numpy(), sl)
    assert np.array_equal(comp.freed_slots[:m].cpu().numpy(), fr)
    assert accept.workspace_for(B, DEV).error_word() == 0
