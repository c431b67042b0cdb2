"""Same-coins equivalence of the sparse and dense verification paths, as the reference tests it
(tests/test_p_distribution_reference.py:255-318, tests/test_dynamic_sampling.py:218-303): with
identical candidates, uniforms and bonus uniforms, rejection against the packed / sparse target
(build_sparse_target -> accept_sparse, packed ids in either order; TargetDistribution.sample_prefix
with the sparse q) must give exactly the outputs of the dense chain over the dense target
(sample_capped_chain_from_probs, build_dspine_target_probs), at every cap and for the flashinfer
and pytorch filter modes with min-p."""

from types import SimpleNamespace
from unittest.mock import patch

import pytest
import torch

from dspine_b200.logits import target_probs
from dspine_b200.runtime.worker import build_dspine_target_probs
from dspine_b200.sampling.rejection import sample_capped_chain_from_probs
from dspine_b200.sampling.sparse.accept import accept_sparse
from dspine_b200.sampling.sparse.target import build_sparse_target
from dspine_b200.sampling.target import TargetDistribution

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _buffers(bs, width=16):
    return (torch.empty(bs, device=DEV, dtype=torch.int32),
            torch.empty(bs, device=DEV, dtype=torch.int32),
            torch.empty(bs, device=DEV, dtype=torch.int64),
            torch.empty((bs, width), device=DEV, dtype=torch.int64),
            torch.empty(bs, device=DEV, dtype=torch.int32))


@pytest.mark.parametrize("bs", [3, 9, 32])
@pytest.mark.parametrize("reverse_packed", [False, True])
def test_packed_rejection_matches_dense_chain_with_identical_coins(bs, reverse_packed):
    g = torch.Generator(device=DEV).manual_seed(1907 + bs)
    width, vocab, k = 16, 257, 16
    lens = torch.tensor(([1, 2, 8, 16] * bs)[:bs], dtype=torch.int32, device=DEV)
    offsets = torch.cat((torch.zeros(1, dtype=torch.int32, device=DEV), lens.cumsum(0).int()))[:-1]
    requests = torch.repeat_interleave(torch.arange(bs, device=DEV, dtype=torch.int32), lens)
    info = SimpleNamespace(
        temperatures=torch.linspace(.7, 1.4, bs, device=DEV).view(-1, 1),
        top_ks=torch.full((bs,), 20, dtype=torch.int32, device=DEV),
        top_ps=torch.linspace(.65, .95, bs, device=DEV), min_ps=torch.zeros(bs, device=DEV),
        need_top_k_sampling=True, need_top_p_sampling=True, need_min_p_sampling=False,
        is_any_greedy=False, is_all_greedy=False, max_top_k=20)
    logits = torch.randn((requests.numel(), vocab), device=DEV, generator=g) * 2
    req = requests.long()
    p = target_probs(logits, info.temperatures.view(-1)[req], info.top_ks[req], info.top_ps[req])
    result = build_sparse_target(logits, info, row_to_request=requests, row_offsets=offsets,
                                 verify_lens=lens)
    assert result is not None
    ids, values, lengths, overflow = result.packed
    cols = torch.arange(ids.shape[1], device=DEV)[None]
    valid = cols < lengths[:, None]
    rebuilt = torch.zeros_like(p).scatter_add_(1, ids.long().clamp_min(0), values * valid)
    dense_rows = overflow.bool()
    rebuilt[dense_rows] = result.dense_p[dense_rows]
    assert torch.equal(rebuilt, p)  # the packed target is the dense target, bit for bit
    packed = result.packed
    if reverse_packed:
        order = torch.where(valid, lengths[:, None] - 1 - cols, cols).long()
        packed = ids.gather(1, order), values.gather(1, order), lengths, overflow
    dense_p = torch.zeros((bs, width, vocab), device=DEV)
    dense_p[..., 0] = 1.0
    q_ids = torch.empty((bs, width - 1, k), device=DEV, dtype=torch.int64)
    for b in range(bs):
        start, count = int(offsets[b]), int(lens[b])
        dense_p[b, :count] = p[start:start + count]
        for depth in range(width - 1):
            q_ids[b, depth] = p[start + min(depth, count - 1)].topk(k).indices.sort().values
    q_values = torch.softmax(torch.randn((bs, width - 1, k), device=DEV, generator=g), -1)
    chosen = torch.multinomial(q_values.reshape(-1, k), 1, generator=g).view(bs, width - 1, 1)
    candidates = torch.cat((torch.zeros((bs, 1), device=DEV, dtype=torch.int64),
                            q_ids.gather(-1, chosen).squeeze(-1)), 1)
    dense_q = torch.zeros((bs, width - 1, vocab), device=DEV).scatter_(-1, q_ids, q_values)
    coins = torch.rand((bs, width - 1), device=DEV, generator=g)
    bonus_coins = torch.rand(bs, device=DEV, generator=g)
    for b in range(0, bs, 2):  # every cap reached: the terminal bonus row of each length
        for depth in range(width - 1):
            candidates[b, depth + 1] = p[int(offsets[b]) + min(depth, int(lens[b]) - 1)].argmax()
        coins[b].zero_()
    prefix = torch.arange(bs, device=DEV, dtype=torch.int32) + 8190
    actual, expected = _buffers(bs), _buffers(bs)
    accept_sparse(torch, candidates=candidates, dense_p=result.dense_p, packed=packed,
                  q_ids=q_ids, q_values=q_values, verify_lens=lens, uniforms=coins,
                  uniform_final=bonus_coins, prefix_lens=prefix, outputs=actual,
                  row_offsets=offsets, vocab_size=vocab)
    sample_capped_chain_from_probs(candidates=candidates, target_probs=dense_p, draft_probs=dense_q,
                                   verify_lens=lens, uniforms=coins, uniform_final=bonus_coins,
                                   prefix_lens=prefix, outputs=expected)
    torch.cuda.synchronize()
    assert all(torch.equal(a, e) for a, e in zip(actual, expected))
    assert torch.equal(actual[0][::2], lens[::2] - 1)


@pytest.mark.parametrize("bs", [1, 9, 17, 33])
@pytest.mark.parametrize("backend", ["flashinfer", "pytorch"])
@pytest.mark.parametrize("kind", ["unfiltered", "mixed", "joint"])
def test_sparse_q_rejection_matches_dense_target_with_identical_coins(bs, backend, kind):
    g = torch.Generator(device=DEV).manual_seed(83)
    t, k, vocab = 16, 16, 97
    info = SimpleNamespace(
        temperatures=torch.full((bs, 1), 0.7, device=DEV),
        top_ks=torch.full((bs,), 1 << 30, dtype=torch.int32, device=DEV),
        top_ps=torch.ones(bs, device=DEV), min_ps=torch.zeros(bs, device=DEV),
        need_top_k_sampling=False, need_top_p_sampling=False, need_min_p_sampling=False,
        is_any_greedy=False, is_all_greedy=False, max_top_k=1 << 30)
    if kind != "unfiltered":
        info.need_top_k_sampling = info.need_top_p_sampling = True
        info.temperatures = torch.linspace(0.4, 1.8, bs, device=DEV).view(bs, 1)
        info.top_ks = torch.tensor([1, 7, 20, 1 << 30], device=DEV,
                                   dtype=torch.int32).repeat(bs)[:bs]
        info.top_ps = torch.linspace(0.5, 1, bs, device=DEV)
        info.is_any_greedy = True
        info.max_top_k = int(info.top_ks.max())
        if kind == "mixed":
            info.need_min_p_sampling = True
            info.min_ps = torch.linspace(0, 0.3, bs, device=DEV)
    logits = torch.randn((bs * t, vocab), device=DEV, generator=g) * 2
    ids = torch.arange(k, device=DEV).expand(bs, t - 1, k).contiguous()
    q = torch.softmax(torch.randn((bs, t - 1, k), device=DEV, generator=g), -1)
    draws = torch.multinomial(q.reshape(-1, k), 1, generator=g).view(bs, t - 1)
    candidates = torch.cat((torch.zeros((bs, 1), device=DEV, dtype=torch.int64), draws), 1)
    caps = 1 + torch.arange(bs, device=DEV, dtype=torch.int32) % t
    prefix = torch.arange(bs, device=DEV, dtype=torch.int32) + 8190
    uniforms = torch.rand((bs, t - 1), device=DEV, generator=g)
    final = torch.rand(bs, device=DEV, generator=g)
    actual, expected = _buffers(bs, t), _buffers(bs, t)
    sampler = SimpleNamespace(round_sampled=True, round_bs=bs, k=k, candidate_out=ids, q_out=q,
                              random=None)
    worker = SimpleNamespace(block_size=t, _dspine_sampler=sampler, sampling_backend=backend,
                             _next_accept_bonus_buffers=lambda size: actual)
    with patch("dspine_b200.sampling.random.verification_uniforms",
               return_value=(uniforms, final)):
        got = TargetDistribution(worker).sample_prefix(
            candidates=candidates, next_token_logits=logits, sampling_info=info,
            prefix_lens=prefix, bs=bs, verify_lens=caps)
    assert got is actual
    p = build_dspine_target_probs(next_token_logits=logits, sampling_info=info, block_size=t,
                                  bs=bs, sampling_backend=backend)
    dense_q = torch.zeros((bs, t - 1, vocab), device=DEV).scatter_(-1, ids, q)
    sample_capped_chain_from_probs(candidates=candidates, target_probs=p, draft_probs=dense_q,
                                   verify_lens=caps, uniforms=uniforms, uniform_final=final,
                                   prefix_lens=prefix, outputs=expected)
    torch.cuda.synchronize()
    assert all(torch.equal(a, e) for a, e in zip(actual, expected))
