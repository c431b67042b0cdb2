"""Parity of dsv_chain_from_probs (sample_capped_chain_from_probs, sampling/rejection.py:101-153)
with the reference's own kernel outputs (golden chain.npz, produced by the reference) and with
the CPU oracle on seeded inputs: ragged caps, all-accepted blocks, zero residual mass (fallback
to p), out-of-range draft tokens, q outside [0,1], u = 0 and u >= 1, large vocabularies.
Integer outputs: bit-exact."""

from pathlib import Path

import numpy as np
import pytest
import torch

import oracle as O
from dspine_b200.sampling.rejection import sample_capped_chain_from_probs
from dspine_b200.verify import new_outputs

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLDEN = Path(__file__).resolve().parent / "golden"
NAMES = ("accept", "commit", "bonus", "output", "new_seq")


def run(cand, p, q, caps, u, uf, prefix):
    t = lambda x: torch.as_tensor(np.ascontiguousarray(x)).to(DEV)  # noqa: E731
    B = cand.shape[0]
    out = new_outputs(B, DEV)
    sample_capped_chain_from_probs(candidates=t(cand), target_probs=t(p), draft_probs=t(q),
                                   verify_lens=t(caps), uniforms=t(u), uniform_final=t(uf),
                                   prefix_lens=t(prefix), outputs=out)
    torch.cuda.synchronize()
    return [o.cpu().numpy() for o in out]


def test_chain_from_probs_matches_reference_golden():
    d = np.load(GOLDEN / "chain.npz")
    cases = sorted({int(k.split("_")[0][1:]) for k in d.files if k.startswith("c") and "_" in k})
    for c in cases:
        got = run(d[f"c{c}_cand"], d[f"c{c}_p"], d[f"c{c}_q"], d[f"c{c}_caps"], d[f"c{c}_u"],
                  d[f"c{c}_uf"], d[f"c{c}_prefix"])
        for name, g in zip(NAMES, got):
            assert np.array_equal(g, d[f"c{c}_{name}"]), (c, name)


def random_case(seed, B, V):
    rng = np.random.default_rng(seed)
    logits = rng.normal(0, 2.5, (B, 16, V)).astype(np.float32)
    p = np.exp(logits - logits.max(-1, keepdims=True))
    p = (p / p.sum(-1, keepdims=True)).astype(np.float32)
    q = np.exp(logits[:, :15] + rng.normal(0, 1, (B, 15, V)))
    q = (q / q.sum(-1, keepdims=True)).astype(np.float32)
    cand = np.zeros((B, 16), np.int64)
    for b in range(B):
        for s in range(15):
            cand[b, s + 1] = rng.choice(V, p=q[b, s] / q[b, s].sum())
    caps = rng.integers(1, 17, B).astype(np.int32)
    u = rng.random((B, 15)).astype(np.float32)
    uf = rng.random(B).astype(np.float32)
    prefix = rng.integers(0, 5000, B).astype(np.int32)
    # edge cases
    u[0] = 0.0                      # accept everything q agrees with
    caps[0] = 16
    q[1] = p[1, :15]                # identical q: residual zero -> fallback to p
    u[1] = 0.0
    cand[2, 3] = V + 5              # out of range draft token: rejected
    q[3, :, : V // 2] = 1.5         # q > 1 clamps to 0 in the residual
    uf[4] = 1.0                     # u >= 1: no crossing -> V - 1
    uf[5] = 0.0
    return cand, p, q, caps, u, uf, prefix


@pytest.mark.parametrize("B,V", [(8, 97), (16, 4099), (12, 151936)])
def test_chain_from_probs_matches_oracle(B, V):
    case = random_case(B * 1000 + V, B, V)
    got = run(*case)
    want = O.chain_from_probs(*case)
    for name, g, w in zip(NAMES, got, want):
        assert np.array_equal(g, w), name


def test_chain_from_probs_argument_errors():
    B, V = 2, 33
    z = lambda *s, dt=torch.float32: torch.zeros(*s, dtype=dt, device=DEV)  # noqa: E731
    good = dict(candidates=z(B, 16, dt=torch.int64), target_probs=z(B, 16, V),
                draft_probs=z(B, 15, V), verify_lens=z(B, dt=torch.int32), uniforms=z(B, 15),
                uniform_final=z(B), prefix_lens=z(B, dt=torch.int32), outputs=new_outputs(B, DEV))
    with pytest.raises(ValueError, match="target"):
        sample_capped_chain_from_probs(**{**good, "target_probs": z(B, 15, V)})
    with pytest.raises(ValueError, match="draft q"):
        sample_capped_chain_from_probs(**{**good, "draft_probs": z(B, 16, V)})
    with pytest.raises(ValueError, match="contiguous"):
        sample_capped_chain_from_probs(**{**good, "uniforms": z(15, B).T})
