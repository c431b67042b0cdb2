"""Parity of the standalone target probabilities (dsv_target_probs, runtime/worker.py:440-508)
and of build_sparse_target (sampling/sparse/target.py:95-178) with the CPU oracle: the kept
set is the canonical exact one and p_i = exp2c((l_i - m) c) * (1 / S_kept), so the dense rows
are compared bit for bit, over every selection path (greedy, top-k window, nucleus histogram,
keep-all, ties, -inf masks, tiny vocabularies)."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle as O
from dspine_b200 import logits as L
from dspine_b200 import workloads
from dspine_b200.sampling.sparse.target import build_sparse_target

pytestmark = pytest.mark.gpu

DEV = "cuda"


def params(seed, R):
    g = torch.Generator().manual_seed(seed)
    T = torch.rand(R, generator=g) * 1.8
    T[torch.rand(R, generator=g) < 0.2] = 0.0
    ks = torch.tensor([workloads.TOPK_OFF, 1, 3, 20, 50, 300], dtype=torch.int32)
    k = ks[torch.randint(0, len(ks), (R,), generator=g)]
    p = torch.where(torch.rand(R, generator=g) < 0.3, torch.ones(R), 0.5 + 0.5 * torch.rand(R, generator=g))
    return T, k, p


@pytest.mark.parametrize("rows,rpr,V,mode", [(48, 16, 4099, "normal"), (40, 1, 151936, "normal"),
                                             (32, 4, 257, "ties"), (32, 8, 1031, "neginf"),
                                             (12, 1, 97, "normal")])
def test_target_probs_match_oracle(rows, rpr, V, mode):
    R = rows // rpr
    T, k, p = params(rows * 7 + V, R)
    g = torch.Generator().manual_seed(V)
    x = torch.randn(rows, V, generator=g) * 2.5
    x[:, 3] += 8.0
    if mode == "ties":
        x = (x * 2).round() / 2
    if mode == "neginf":
        x[:, ::5] = -float("inf")
    xb = x.to(torch.bfloat16)
    got = L.target_probs(xb.to(DEV), T, k, p, rows_per_request=rpr)
    torch.cuda.synchronize()
    want = O.target_probs(xb.float().numpy(), T.numpy(), k.numpy(), p.numpy(), rows_per_request=rpr)
    g_ = got.cpu().numpy()
    assert np.array_equal(g_.view(np.uint32), want.view(np.uint32))


def test_target_probs_config1_rows():
    b = workloads.config1(device="cpu")
    rows = int(b.target_logits.shape[0]) // 16 * 16
    rpr = 16
    R = rows // rpr
    got = L.target_probs(b.target_logits[:rows].to(DEV), b.temperature[:R], b.top_k[:R],
                         b.top_p[:R], rows_per_request=rpr)
    torch.cuda.synchronize()
    want = O.target_probs(b.target_logits[:rows].float().numpy(), b.temperature[:R].numpy(),
                          b.top_k[:R].numpy(), b.top_p[:R].numpy(), rows_per_request=rpr)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_build_sparse_target_packs_the_kept_sets():
    rows, V, cap = 48, 4099, 32
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(rows, V, generator=g) * 3.0).to(torch.bfloat16)
    B = rows // 16
    info = SimpleNamespace(temperatures=torch.full((B,), 0.7), top_ks=torch.tensor([20, 32, 5], dtype=torch.int32),
                           top_ps=torch.tensor([0.9, 0.95, 1.0]), max_top_k=32,
                           need_min_p_sampling=False, is_any_greedy=False)
    st = build_sparse_target(x.to(DEV), SimpleNamespace(**{k: (v.to(DEV) if torch.is_tensor(v) else v)
                                                          for k, v in vars(info).items()}),
                             capacity=cap)
    torch.cuda.synchronize()
    T = info.temperatures.repeat_interleave(16).numpy()
    K = info.top_ks.repeat_interleave(16).numpy()
    P = info.top_ps.repeat_interleave(16).numpy()
    p = O.target_probs(x.float().numpy(), T, K, P, rows_per_request=1)
    want = O.compress_probs(p, capacity=cap)
    for got, w in zip(st.packed, want):
        assert np.array_equal(got.cpu().numpy(), w)
    assert np.array_equal(st.dense_p.cpu().numpy().view(np.uint32), p.view(np.uint32))
    # the dense path is required for greedy rows, min-p or an unbounded top-k
    assert build_sparse_target(x.to(DEV), SimpleNamespace(max_top_k=64, is_any_greedy=False),
                               capacity=cap) is None
    assert build_sparse_target(x.to(DEV), SimpleNamespace(max_top_k=8, is_any_greedy=True),
                               capacity=cap) is None
