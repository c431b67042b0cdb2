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


SPARSE_FIX = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "sparse_target.npz")


def _sparse_info(temp, topk, topp, max_k):
    return SimpleNamespace(temperatures=torch.as_tensor(temp).to(DEV), top_ks=torch.as_tensor(topk).to(DEV),
                           top_ps=torch.as_tensor(topp).to(DEV), max_top_k=int(max_k),
                           need_min_p_sampling=False, is_any_greedy=False)


def _check_sparse(st, want_ids, want_vals, want_lens, want_ovf, want_dense_rows, ovf_rows, tag):
    ids, vals, lens, ovf = (t.cpu().numpy() for t in st.packed)
    np.testing.assert_array_equal(ovf, want_ovf, err_msg=f"{tag} overflow")
    np.testing.assert_array_equal(lens, want_lens, err_msg=f"{tag} lengths")
    keep = want_ovf == 0
    np.testing.assert_array_equal(ids[keep], want_ids[keep], err_msg=f"{tag} ids")
    np.testing.assert_allclose(vals[keep], want_vals[keep], rtol=1e-5, atol=1e-7, err_msg=f"{tag} values")
    dense = st.dense_p.cpu().numpy()[ovf_rows]
    np.testing.assert_allclose(dense, want_dense_rows, rtol=1e-5, atol=1e-7, err_msg=f"{tag} dense")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_build_sparse_target_matches_reference_cpu_branch(dtype):
    """GPU build_sparse_target against the reference's own CPU branch (sparse/target.py:156-178,
    tests/golden/sparse_target.npz): random, quantised (ties at the k-th p) and plateau rows,
    top-k 1..32, cutting and open top-p.  bf16 runs the cases whose logits are bf16-exact."""
    d = SPARSE_FIX
    ran = 0
    for ci in range(int(d["n"])):
        x = torch.from_numpy(d[f"c{ci}_logits"])
        if dtype == torch.bfloat16 and not torch.equal(x.to(torch.bfloat16).float(), x):
            continue
        rows = x.shape[0]
        info = _sparse_info(d[f"c{ci}_temp"], d[f"c{ci}_topk"], d[f"c{ci}_topp"],
                            int(d[f"c{ci}_topk"].max()))
        st = build_sparse_target(x.to(dtype).to(DEV), info,
                                 row_to_request=torch.arange(rows, device=DEV), capacity=32)
        torch.cuda.synchronize()
        _check_sparse(st, d[f"c{ci}_ids"], d[f"c{ci}_vals"], d[f"c{ci}_lens"], d[f"c{ci}_ovf"],
                      d[f"c{ci}_dense"], d[f"c{ci}_ovf_rows"], f"case {ci} {dtype}")
        ran += 1
    assert ran >= 3


@pytest.mark.parametrize("dtype,V", [(torch.bfloat16, 151936), (torch.float32, 151936),
                                     (torch.bfloat16, 3001)])
def test_build_sparse_target_matches_oracle(dtype, V):
    """GPU == oracle exactly (ids, lengths, overflow, the fp32 bits of values and of dense
    overflow rows) on config-1-like rows, the offsets row mapping, all-equal and plateau rows."""
    B = 6
    g = torch.Generator().manual_seed(V)
    lens = torch.tensor([3, 1, 5, 2, 4, 1])
    offsets = torch.cat([torch.zeros(1, dtype=torch.int64), lens.cumsum(0)])
    rows = int(lens.sum())
    x = torch.randn(rows, V, generator=g) * 2.5
    x[torch.arange(rows), torch.randint(0, V, (rows,), generator=g)] += 8
    x[3] = 0.0                                   # all equal: overflow
    x[5, :] = -5.0
    x[5, :40] = 2.0                              # a plateau of 40 tied tops: overflow
    x[7] = (x[7] * 2).round() / 2                # ties at the k-th p
    x = x.to(dtype)
    temp = torch.tensor([0.7, 1.0, 1.3, 0.5, 1.0, 0.9])
    topk = torch.tensor([20, 32, 1, 8, 32, 5], dtype=torch.int32)
    topp = torch.tensor([0.9, 1.0, 0.95, 0.8, 0.6, 1.0])
    st = build_sparse_target(x.to(DEV), _sparse_info(temp, topk, topp, 32),
                             row_offsets=offsets.to(DEV), capacity=32)
    torch.cuda.synchronize()
    req = torch.searchsorted(offsets[1:], torch.arange(rows), right=True)
    ids, vals, ln, ovf, dense = O.sparse_target(x.float().numpy(), temp[req].numpy(),
                                                topk[req].numpy(), topp[req].numpy(), 32)
    assert ovf.sum() >= 2
    g_ids, g_vals, g_lens, g_ovf = (t.cpu().numpy() for t in st.packed)
    np.testing.assert_array_equal(g_ovf, ovf)
    np.testing.assert_array_equal(g_lens, ln)
    np.testing.assert_array_equal(g_ids, ids)
    assert np.array_equal(g_vals.view(np.uint32), vals.view(np.uint32))
    o = np.flatnonzero(ovf)
    assert np.array_equal(st.dense_p.cpu().numpy()[o].view(np.uint32), dense[o].view(np.uint32))


def test_build_sparse_target_gating():
    """The dense path is required for greedy rows, min-p, another backend or an unbounded
    top-k (sparse/target.py:106-111); those calls return None without launching."""
    x = torch.zeros(4, 97, device=DEV)
    assert build_sparse_target(x, SimpleNamespace(max_top_k=64, is_any_greedy=False), capacity=32) is None
    assert build_sparse_target(x, SimpleNamespace(max_top_k=8, is_any_greedy=True), capacity=32) is None
    assert build_sparse_target(x, SimpleNamespace(max_top_k=8, need_min_p_sampling=True)) is None
    assert build_sparse_target(x, SimpleNamespace(max_top_k=8), sampling_backend="pytorch") is None


@pytest.mark.parametrize("mode", [0, 1, 2])
@pytest.mark.parametrize("dtype,V,rpr", [(torch.float32, 4099, 4), (torch.float32, 151936, 1),
                                         (torch.bfloat16, 4099, 4), (torch.float32, 97, 3)])
def test_target_probs_modes_and_fp32_match_oracle(mode, dtype, V, rpr):
    """dsv_target_probs_ex: fp32 logits through the cluster kernel, bf16 through the row kernel,
    with min-p and each filter mode; the dense rows equal the oracle's bit for bit."""
    rows = 24 if V < 100000 else 6
    rows -= rows % rpr
    R = rows // rpr
    T, k, p = params(rows * 11 + V + mode, R)
    g = torch.Generator().manual_seed(V + mode)
    mp = torch.rand(R, generator=g) * 0.2
    mp[::3] = 0.0
    x = torch.randn(rows, V, generator=g) * 2.5
    x[:, 7] += 8.0
    x = x.to(dtype)
    got = L.target_probs(x.to(DEV), T, k, p, rows_per_request=rpr, min_p=mp, mode=mode)
    torch.cuda.synchronize()
    want = O.target_probs(x.float().numpy(), T.numpy(), k.numpy(), p.numpy(),
                          rows_per_request=rpr, min_p=mp.numpy(), mode=mode)
    assert np.array_equal(got.cpu().numpy().view(np.uint32), want.view(np.uint32))
