"""The plugin seams at the reference's module paths, called as SGLang calls them.

Each shim keeps the reference's name, signature and result layout; `sampling_info` objects
carry the SamplingBatchInfo fields the reference reads (tests/ref_utils.py:150-162:
temperatures [bs, 1], top_ks, top_ps, min_ps and the need_* / greedy flags).  Results are
compared with the CPU oracle on the same inputs and seeded uniforms:

- runtime/worker.py build_dspine_target_probs (:440-470), every filter mode, bf16 and fp32;
- runtime/worker.py dspine_accept_sampling (:511-581) and seam C accept_dspine_sampled_round
  (:1092-1115) through DSpineVerifier and sampling/target.py TargetDistribution (:34-122),
  on its sparse and its dense path;
- verification/caps.py VerifyCaps.accept (:331-379) and verification/ragged.py
  RaggedVerifyCaps.accept (:282-335), greedy and sampled rounds;
- verification/sps.py device_plan (:61-99).
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle as O
from dspine_b200 import workloads
from dspine_b200.runtime import worker as W
from dspine_b200.sampling import random as R
from dspine_b200.verification import caps, ragged, sps

pytestmark = pytest.mark.gpu
DEV = "cuda"
T = 16


def info(temperature, top_k, top_p, min_p=None, greedy=False, need_k=None, need_p=None):
    bs = len(temperature)
    top_k = torch.as_tensor(top_k, dtype=torch.int32)
    return SimpleNamespace(
        temperatures=torch.as_tensor(temperature, dtype=torch.float32).view(bs, 1).to(DEV),
        top_ks=top_k.to(DEV),
        top_ps=torch.as_tensor(top_p, dtype=torch.float32).to(DEV),
        min_ps=torch.as_tensor(min_p if min_p is not None else [0.0] * bs,
                               dtype=torch.float32).to(DEV),
        need_top_k_sampling=bool((top_k < W.TOPK_ALL).any()) if need_k is None else need_k,
        need_top_p_sampling=bool(any(p < 1 for p in top_p)) if need_p is None else need_p,
        need_min_p_sampling=min_p is not None,
        is_all_greedy=False, is_any_greedy=greedy, max_top_k=int(top_k.max()))


def logits_rows(rows, V, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(rows, V, generator=g) * 2.5
    x[torch.arange(rows), torch.randint(0, V, (rows,), generator=g)] += 8.0
    return x.to(dtype)


@pytest.mark.parametrize("backend,min_p", [("flashinfer", None), ("flashinfer", [0.02, 0.0, 0.1]),
                                           ("pytorch", None), ("pytorch", [0.05, 0.2, 0.0])])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_build_dspine_target_probs(backend, min_p, dtype):
    bs, V = 3, 4099
    x = logits_rows(bs * T, V, dtype, 3 + len(backend))
    si = info([0.8, 1.2, 0.6], [20, W.TOPK_ALL, 50], [0.9, 0.95, 1.0], min_p)
    got = W.build_dspine_target_probs(next_token_logits=x.to(DEV), sampling_info=si,
                                      block_size=T, bs=bs, sampling_backend=backend)
    torch.cuda.synchronize()
    assert got.shape == (bs, T, V) and got.dtype == torch.float32
    mode = O.filter_mode(backend, min_p is not None)
    want = O.target_probs(x.float().numpy(), [0.8, 1.2, 0.6], [20, W.TOPK_ALL, 50],
                          [0.9, 0.95, 1.0], rows_per_request=T, mode=mode,
                          min_p=None if min_p is None else np.asarray(min_p, np.float32))
    assert np.array_equal(got.reshape(bs * T, V).cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_build_dspine_target_probs_unflagged_filters_are_off():
    """A filter whose need_* flag is off is not applied (runtime/worker.py:476-479)."""
    bs, V = 2, 1031
    x = logits_rows(bs * T, V, torch.float32, 9)
    si = info([1.0, 1.0], [5, 7], [0.5, 0.6], need_k=False, need_p=False)
    got = W.build_dspine_target_probs(next_token_logits=x.to(DEV), sampling_info=si,
                                      block_size=T, bs=bs, sampling_backend="flashinfer")
    want = O.target_probs(x.numpy(), [1.0, 1.0], [W.TOPK_ALL] * 2, [1.0, 1.0], rows_per_request=T)
    assert np.array_equal(got.reshape(bs * T, V).cpu().numpy().view(np.uint32), want.view(np.uint32))


class Sampler(SimpleNamespace):
    """The draft sampler state seam C reads (the reference's DSpineDraftSampler)."""


def sampled_round(bs, V, seed, greedy_rows=()):
    """Candidates drawn from a sparse q over 16 ids per row, seeded request uniforms."""
    g = torch.Generator().manual_seed(seed)
    ids = torch.stack([torch.randperm(V, generator=g)[:16] for _ in range(bs * 15)]).view(bs, 15, 16)
    q = torch.softmax(torch.randn(bs, 15, 16, generator=g) * 2, -1)
    cand = torch.zeros(bs, T, dtype=torch.int64)
    cand[:, 0] = torch.randint(0, V, (bs,), generator=g)
    pick = torch.multinomial(q.view(-1, 16), 1, generator=g).view(bs, 15)
    cand[:, 1:] = ids.gather(2, pick[..., None])[..., 0]
    seeds = torch.randint(-2**62, 2**62, (bs,), generator=g, dtype=torch.int64)
    positions = torch.randint(0, 4096, (bs,), generator=g, dtype=torch.int64)
    rng = R.RequestRNG()
    rng.stage(seeds.to(DEV), positions.to(DEV))
    sampler = Sampler(round_sampled=True, round_bs=bs, k=16, candidate_out=ids.to(DEV),
                      q_out=q.to(DEV), random=rng)
    u = O.uniforms(seeds.numpy(), positions.numpy(), 15, R.ACCEPT)
    uf = O.uniforms(seeds.numpy(), positions.numpy(), 1, R.BONUS)[:, 0]
    return sampler, cand, u, uf


def oracle_sparse_accept(cand, p, packed, sampler, u, uf, lens, prefix):
    return O.accept_sparse(cand.numpy(), p, packed, sampler.candidate_out.cpu().numpy(),
                           sampler.q_out.cpu().numpy(), lens, u, uf, prefix)


def test_dspine_accept_sampling_matches_oracle():
    bs, V = 5, 4099
    x = logits_rows(bs * T, V, torch.float32, 21)
    sampler, cand, u, uf = sampled_round(bs, V, 4)
    si = info([0.9] * bs, [W.TOPK_ALL] * bs, [1.0] * bs)
    acc, bonus = W.dspine_accept_sampling(
        candidates=cand.to(DEV), target_logits=x.to(DEV), candidate_ids=sampler.candidate_out,
        q_rows=sampler.q_out, sampling_info=si, sampling_backend="flashinfer",
        dense_q=None, random_state=sampler.random)
    torch.cuda.synchronize()
    p = O.target_probs(x.numpy(), [0.9] * bs, [W.TOPK_ALL] * bs, [1.0] * bs, rows_per_request=T)
    want = oracle_sparse_accept(cand, p, None, sampler, u, uf, np.full(bs, 16, np.int32),
                                np.zeros(bs, np.int32))
    assert np.array_equal(acc.cpu().numpy(), want[0]) and np.array_equal(bonus.cpu().numpy(), want[2])
    assert acc.dtype == torch.int32 and bonus.dtype == torch.int64


@pytest.mark.parametrize("path", ["sparse", "dense_packed", "dense_unfiltered", "no_target_distribution"])
def test_seam_c_through_the_active_worker(path):
    """accept_dspine_sampled_round -> the worker's _accept_sampled_round -> TargetDistribution:
    the sparse joint target (top-k <= 32, no greedy rows), the dense target packed by
    compress_probs (a greedy row present), the dense unfiltered target, and the worker without
    a TargetDistribution (dspine_accept_sampling)."""
    bs, V = 4, 3001
    x = logits_rows(bs * T, V, torch.bfloat16, 31)
    sampler, cand, u, uf = sampled_round(bs, V, 5)
    temps, ks, ps = [0.8, 1.0, 1.3, 0.7], [20, 32, 8, 16], [0.9, 1.0, 0.95, 0.85]
    greedy = path == "dense_packed"
    if greedy:
        ks = [1, 32, 8, 16]
    if path in ("dense_unfiltered", "no_target_distribution"):
        ks, ps = [W.TOPK_ALL] * bs, [1.0] * bs
    si = info(temps, ks, ps, greedy=greedy)
    verifier = W.DSpineVerifier(sampler, use_target_distribution=path != "no_target_distribution")
    W.set_active_worker(verifier)
    try:
        acc, bonus = W.accept_dspine_sampled_round(candidates=cand.to(DEV), next_token_logits=x.to(DEV),
                                                   sampling_info=si, max_top_k=max(ks))
        torch.cuda.synchronize()
    finally:
        W.set_active_worker(None)
    lens, prefix = np.full(bs, 16, np.int32), np.zeros(bs, np.int32)
    if path == "sparse":
        rows_t = np.repeat(np.asarray(temps, np.float32), T)
        ids, vals, ln, ovf, dense = O.sparse_target(x.float().numpy(), rows_t, np.repeat(ks, T),
                                                    np.repeat(np.asarray(ps, np.float32), T), 32)
        want = oracle_sparse_accept(cand, dense, (ids, vals, ln, ovf), sampler, u, uf, lens, prefix)
    else:
        p = O.target_probs(x.float().numpy(), temps, ks, ps, rows_per_request=T)
        packed = O.compress_probs(p, capacity=32) if path == "dense_packed" else None
        want = oracle_sparse_accept(cand, p, packed, sampler, u, uf, lens, prefix)
    assert np.array_equal(acc.cpu().numpy(), want[0]), path
    assert np.array_equal(bonus.cpu().numpy(), want[2]), path


def test_seam_c_refuses_a_round_without_its_sampled_chain():
    sampler, cand, _, _ = sampled_round(2, 257, 1)
    sampler.round_sampled = False
    W.set_active_worker(W.DSpineVerifier(sampler))
    try:
        with pytest.raises(RuntimeError, match="without this round's sampled draft chain"):
            W.accept_dspine_sampled_round(candidates=cand.to(DEV),
                                          next_token_logits=torch.zeros(32, 257, device=DEV),
                                          sampling_info=info([1.0, 1.0], [4, 4], [1.0, 1.0]))
    finally:
        W.set_active_worker(None)
    with pytest.raises(RuntimeError, match="before the DSpine worker exists"):
        W.accept_dspine_sampled_round(candidates=cand, next_token_logits=None, sampling_info=None)


def greedy_batch(bs, V, seed, full_accept_rows=()):
    x = logits_rows(bs * T, V, torch.float32, seed)
    top1 = O.argmax_rows(x.numpy()).reshape(bs, T)
    g = torch.Generator().manual_seed(seed)
    cand = torch.from_numpy(top1.copy())
    cand = torch.roll(cand, 1, dims=1)  # draft s+1 = top1 of row s
    cand[:, 0] = torch.randint(0, V, (bs,), generator=g)
    # break each chain at a random depth
    for b in range(bs):
        if b not in full_accept_rows:
            cand[b, int(torch.randint(1, T, (1,), generator=g))] = (V - 1)
    return x, cand, top1


def test_verify_caps_accept_greedy_and_sampled():
    bs, V, active = 6, 2053, 11
    x, cand, top1 = greedy_batch(bs, V, 41, full_accept_rows=(0,))
    sampler, _, u, uf = sampled_round(bs, V, 6)
    verifier = W.DSpineVerifier(sampler)
    ctl = caps.VerifyCaps(verifier, full=T, active=active)
    prefix = torch.arange(bs, dtype=torch.int32) + 100
    got = ctl.accept(candidates=cand.to(DEV), next_token_logits=x.to(DEV), sampling_info=None,
                     draft_input=None, prefix_lens=prefix.to(DEV), bs=bs)
    torch.cuda.synchronize()
    want = O.accept_greedy(cand.numpy(), top1, np.full(bs, active, np.int32), prefix.numpy())
    for g, w in zip(got, want):
        assert np.array_equal(g.cpu().numpy(), w)
    # the sampled round of the same controller: every request capped at `active`
    ctl.sampled_round = True
    si = info([1.0] * bs, [W.TOPK_ALL] * bs, [1.0] * bs)
    sampled_cand = cand.clone()
    got = ctl.accept(candidates=sampled_cand.to(DEV), next_token_logits=x.to(DEV),
                     sampling_info=si, draft_input=None, prefix_lens=prefix.to(DEV), bs=bs)
    torch.cuda.synchronize()
    p = O.target_probs(x.numpy(), [1.0] * bs, [W.TOPK_ALL] * bs, [1.0] * bs, rows_per_request=T)
    want = oracle_sparse_accept(sampled_cand, p, None, sampler, u, uf,
                                np.full(bs, active, np.int32), prefix.numpy())
    for g, w in zip(got, want):
        assert np.array_equal(g.cpu().numpy(), w)
    assert ctl.sampled_executions == 1
    ctl.executed_width = active - 1
    with pytest.raises(RuntimeError, match="confirmed shortened target forward"):
        ctl.accept(candidates=cand.to(DEV), next_token_logits=x.to(DEV), sampling_info=None,
                   draft_input=None, prefix_lens=prefix.to(DEV), bs=bs)


def test_ragged_verify_caps_accept_greedy():
    bs, V = 7, 1031
    x, cand, top1 = greedy_batch(bs, V, 43, full_accept_rows=(1, 2))
    lens = torch.tensor([16, 3, 1, 9, 16, 5, 12], dtype=torch.int32)
    sampler, _, _, _ = sampled_round(bs, V, 7)
    ctl = ragged.RaggedVerifyCaps(W.DSpineVerifier(sampler), full=T)
    ctl.ragged_round, ctl.batch_size, ctl.tokens, ctl.executed_tokens = True, bs, int(lens.sum()), int(lens.sum())
    ctl.layout = SimpleNamespace(verify_lens=lens.to(DEV))
    prefix = torch.zeros(bs, dtype=torch.int32)
    got = ctl.accept(candidates=cand.to(DEV), next_token_logits=x.to(DEV), sampling_info=None,
                     draft_input=None, prefix_lens=prefix.to(DEV), bs=bs)
    torch.cuda.synchronize()
    want = O.accept_greedy(cand.numpy(), top1, lens.numpy(), prefix.numpy())
    for g, w in zip(got, want):
        assert np.array_equal(g.cpu().numpy(), w)


def test_sps_device_plan():
    rng = np.random.default_rng(3)
    B = 40
    raw = rng.random((B, 15)).astype(np.float32)
    table = np.clip(rng.random((15, 8)), 0.05, 0.999).astype(np.float32)
    cfg = SimpleNamespace(min_verify_len=1, survival_eps=0.0)
    budget = B * 5
    layout, index = sps.device_plan(torch.from_numpy(raw).to(DEV), torch.from_numpy(table).to(DEV),
                                    torch.arange(15, device=DEV), budget, cfg)
    torch.cuda.synchronize()
    lens = O.sps_lens(raw, table, budget)
    qo, idx = O.sps_index(lens)
    assert np.array_equal(layout.verify_lens.cpu().numpy(), lens)
    assert np.array_equal(layout.qo_indptr_device.cpu().numpy(), qo)
    assert np.array_equal(index.cpu().numpy(), idx)
    with pytest.raises(ValueError, match="one root per request"):
        sps.device_plan(torch.from_numpy(raw).to(DEV), torch.from_numpy(table).to(DEV),
                        torch.arange(15, device=DEV), budget,
                        SimpleNamespace(min_verify_len=2, survival_eps=0.0))
