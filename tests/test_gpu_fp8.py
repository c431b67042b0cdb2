"""Parity of the FP8 coarse retrieval + BF16 rescore (dsv_fp8_quantize_rows,
dsv_fp8_coarse_scores, dsv_topk_ranked, dsv_rescore_select16) with the CPU oracle.

Reference semantics: layers/fp8/coarse.py:19-113 and layers/fp8/gather.py:7-79.  The
reference's own end-to-end test (tests/test_topk_compat_cuda.py:82-132) builds a head whose
dot products are exact (two non-zero columns) so that every stage is compared with atol 0; the
first test repeats that construction.  Elsewhere: quantization bit-exact; coarse scores within
one bf16 rounding plus the fp32 accumulation error of the exact float64 product; the ranked
top-k and the 16 selection rounds exact on the GPU's own scores; rescored scores within one
bf16 rounding plus the fp32 accumulation error.
"""

import numpy as np
import pytest
import torch

import oracle.fp8 as OF
from dspine_b200.layers.fp8 import coarse as C
from dspine_b200.layers.fp8 import gather as G

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _bf16_np(t):
    return t.float().cpu().numpy()


def test_exact_two_column_head_end_to_end():
    """tests/test_topk_compat_cuda.py:103-132: results equal the oracle exactly, eager and
    after negating the hidden rows."""
    w = torch.zeros(512, 512, dtype=torch.bfloat16)
    w[:, 0] = torch.arange(512).remainder(47).bfloat16() / 32
    w[:, 1] = torch.arange(512).remainder(31).bfloat16() / 64
    local = C.FullVFP8Coarse(torch, w.to(DEV))
    hidden = torch.zeros(4, 512, device=DEV, dtype=torch.bfloat16)
    hidden[:, :2] = torch.tensor([[1, 2], [2, -1], [-1, 1], [0, 0]], device=DEV)
    wq_ref, sw_ref = OF.quantize_rows(_bf16_np(w))
    np.testing.assert_array_equal(local.weight8.view(torch.uint8).cpu().numpy(), wq_ref)
    np.testing.assert_array_equal(local.weight_scale.cpu().numpy()[0], sw_ref)
    for _ in range(2):
        top16, ids, scores = local.retrieve_and_rescore(hidden)
        torch.cuda.synchronize()
        h = _bf16_np(hidden)
        xq, sx = OF.quantize_rows(h)
        coarse = OF.coarse_fp32_small(xq, sx, wq_ref, sw_ref)
        ref_ids = OF.lexical_topk(coarse, 128)
        np.testing.assert_array_equal(ids.cpu().numpy(), ref_ids)
        exact, _ = OF.rescore_exact(_bf16_np(w), ref_ids, h)
        ref_scores = OF._bf16(exact.astype(np.float32))
        np.testing.assert_array_equal(_bf16_np(scores), ref_scores)
        np.testing.assert_array_equal(top16.cpu().numpy(), OF.select16(ref_scores, ref_ids))
        hidden.neg_()
    assert local.error_word() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_quantize_rows_bit_exact(dtype):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((37, 1000)) * rng.uniform(1e-3, 50, size=(37, 1))).astype(np.float32)
    x[5] = 0.0
    x[6, 3:] = 0.0
    x[7, 11] = np.nan      # torch's amax propagates NaN: scale 1, NaN entries code NaN
    x[8, 2] = -np.inf      # scale inf: the inf entry codes NaN, the rest 0
    t = torch.from_numpy(x).to(dtype).to(DEV)
    q, s = C.quantize_rows(t)
    torch.cuda.synchronize()
    q_ref, s_ref = OF.quantize_rows(t.float().cpu().numpy())
    np.testing.assert_array_equal(s.cpu().numpy(), s_ref)
    q = q.cpu().numpy()
    is_nan = (q_ref & 0x7F) == 0x7F        # either e4m3 NaN code: the sign is arithmetic's choice
    np.testing.assert_array_equal((q & 0x7F) == 0x7F, is_nan)
    np.testing.assert_array_equal(q[~is_nan], q_ref[~is_nan])
    assert is_nan[7].sum() == 1 and is_nan[8].sum() == 1


@pytest.mark.parametrize("m,v,h", [(200, 3000, 1024), (5, 256, 128), (130, 8200, 512)])
def test_coarse_scores_match_oracle(m, v, h):
    rng = np.random.default_rng(m + v + h)
    x = torch.from_numpy(rng.standard_normal((m, h)).astype(np.float32)).bfloat16().to(DEV)
    w = torch.from_numpy((rng.standard_normal((v, h)) * 0.05).astype(np.float32)).bfloat16().to(DEV)
    xq, sx = C.quantize_rows(x)
    wq, sw = C.quantize_rows(w)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    got = C.coarse_scores(xq, sx, wq, sw, err=err)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    exact, bound = OF.coarse_exact(xq.cpu().numpy(), sx.cpu().numpy(), wq.cpu().numpy(), sw.cpu().numpy())
    diff = np.abs(_bf16_np(got) - exact)
    tol = 2.0 ** -8 * np.abs(exact) + 2.0 ** -12 * bound
    assert (diff <= tol).all(), float((diff - tol).max())


@pytest.mark.parametrize("v,k", [(100, 1), (100, 7), (100, 100), (512, 128), (3000, 16),
                                 (3000, 128), (151936, 128), (151936, 100)])
def test_ranked_topk_matches_lexical_order(v, k):
    rng = np.random.default_rng(v * 7 + k)
    x = rng.integers(-20, 20, size=(9, v)).astype(np.float32) / 4   # many ties
    x[1] = 1.0
    x[2, ::3] = -np.inf
    t = torch.from_numpy(x).bfloat16().to(DEV)
    vals, ids = C.stable_local_topk(t, k)
    torch.cuda.synchronize()
    ref = OF.lexical_topk(_bf16_np(t), k)
    np.testing.assert_array_equal(ids.cpu().numpy(), ref)
    np.testing.assert_array_equal(_bf16_np(vals), np.take_along_axis(_bf16_np(t), ref, 1))


@pytest.mark.parametrize("fp32_output", [False, True])
def test_rescore_and_select16_match_oracle(fp32_output):
    rng = np.random.default_rng(5)
    V, H, M = 5000, 1024, 37
    w = torch.from_numpy((rng.standard_normal((V, H)) * 0.05).astype(np.float32)).bfloat16().to(DEV)
    hidden = torch.from_numpy(rng.standard_normal((M, H)).astype(np.float32)).bfloat16().to(DEV)
    ids_np = np.stack([rng.choice(V, 128, replace=False) for _ in range(M)]).astype(np.int64)
    ids_np[3, 7] = -1                       # out of range: scores -inf
    ids_np[4, 9] = V
    ids = torch.from_numpy(ids_np).to(DEV)
    scores, top16 = G.rescore_select16(torch, w, ids, hidden, fp32_output=fp32_output)
    torch.cuda.synchronize()
    got = scores.float().cpu().numpy()
    assert got[3, 7] == -np.inf and got[4, 9] == -np.inf
    safe = np.clip(ids_np, 0, V - 1)
    exact, bound = OF.rescore_exact(_bf16_np(w), safe, _bf16_np(hidden))
    ok = np.ones_like(got, bool)
    ok[3, 7] = ok[4, 9] = False
    tol = (0 if fp32_output else 2.0 ** -8) * np.abs(exact) + 2.0 ** -12 * bound
    assert (np.abs(got - exact)[ok] <= tol[ok]).all()
    np.testing.assert_array_equal(top16.cpu().numpy(), OF.select16(got, ids_np))
    # the selection alone on given (tied) scores
    tied = torch.from_numpy(np.round(got * 2) / 2).to(scores.dtype).to(DEV).contiguous()
    sel = G.select16(torch, tied, ids)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(sel.cpu().numpy(), OF.select16(tied.float().cpu().numpy(), ids_np))


class _OneRank:
    world_size = 1

    def all_gather(self, tensor, dim=0):
        return tensor

    def all_reduce(self, tensor):
        return tensor


def test_retrieve_and_rescore_random_and_single_shard_tp():
    """The full pipeline on a random head: coarse ids are the lexical top-128 of the coarse
    scores, top16 the selection of the rescored candidates; a one-rank TP head (padded
    shard, sampling/tp_head.py:91-103 rescore) gives the same tokens."""
    from dspine_b200.lmhead import TPHead

    rng = np.random.default_rng(9)
    V, H, M = 8192, 512, 64
    w = torch.from_numpy((rng.standard_normal((V, H)) * 0.05).astype(np.float32)).bfloat16().to(DEV)
    hidden = torch.from_numpy(rng.standard_normal((M, H)).astype(np.float32)).bfloat16().to(DEV)
    local = C.FullVFP8Coarse(torch, w)
    top16, ids, scores = local.retrieve_and_rescore(hidden)
    xq, sx = C.quantize_rows(hidden)
    coarse = C.coarse_scores(xq, sx, local.weight8.view(torch.uint8), local.weight_scale.reshape(-1))
    torch.cuda.synchronize()
    ids_np = ids.cpu().numpy()
    np.testing.assert_array_equal(ids_np, OF.lexical_topk(_bf16_np(coarse), 128))
    exact, bound = OF.rescore_exact(_bf16_np(w), ids_np, _bf16_np(hidden))
    got = _bf16_np(scores)
    assert (np.abs(got - exact) <= 2.0 ** -8 * np.abs(exact) + 2.0 ** -12 * bound).all()
    np.testing.assert_array_equal(top16.cpu().numpy(), OF.select16(got, ids_np))
    # one-rank TP head over a shard padded by 64 rows
    padded = torch.cat([w, torch.zeros(64, H, dtype=w.dtype, device=DEV)])
    head = TPHead(padded, 0, V, V, _OneRank())
    tp = C.FullVFP8Coarse(torch, padded, head)
    t16, tids, tscores = tp.retrieve_and_rescore(hidden)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(tids.cpu().numpy(), ids_np)
    np.testing.assert_array_equal(t16.cpu().numpy(), top16.cpu().numpy())
    np.testing.assert_array_equal(_bf16_np(tscores), got)
    assert local.error_word() == 0 and tp.error_word() == 0


GOLDEN = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "fp8.npz")


def test_reference_fixtures():
    """tests/golden/fp8.npz (the reference's own FullVFP8Coarse quantization, _scale/_quantize,
    stable_local_topk, gather.rescore and gather.select16): quantization, the stable top-k and
    the selection exact; rescored scores within one bf16 ulp of the reference's (its fixture
    was stored by the Triton interpreter, which truncates to bf16) and within half an ulp plus
    the fp32 accumulation bound of the exact dot."""
    for name in ("two", "rand"):
        w = torch.from_numpy(GOLDEN[f"{name}_w"]).bfloat16().to(DEV)
        local = C.FullVFP8Coarse(torch, w) if w.shape[1] % 128 == 0 else None
        q, s = C.quantize_rows(w)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(q.cpu().numpy(), GOLDEN[f"{name}_wq"])
        np.testing.assert_array_equal(s.cpu().numpy(), GOLDEN[f"{name}_ws"])
        if local is not None:
            np.testing.assert_array_equal(local.weight8.view(torch.uint8).cpu().numpy(), GOLDEN[f"{name}_wq"])
    hidden = torch.from_numpy(GOLDEN["hidden"]).bfloat16().to(DEV)
    q, s = C.quantize_rows(hidden)
    scores = torch.from_numpy(GOLDEN["topk_scores"]).bfloat16().to(DEV)
    tops = {k: C.stable_local_topk(scores, k)[1] for k in (1, 16, 128)}
    w = torch.from_numpy(GOLDEN["rand_w"]).bfloat16().to(DEV)
    ids = torch.from_numpy(GOLDEN["rescore_ids"]).to(DEV)
    got, top16 = G.rescore_select16(torch, w, ids, hidden)
    ref_scores = torch.from_numpy(GOLDEN["rescore_scores"]).bfloat16().to(DEV)
    sel_ref = G.select16(torch, ref_scores, ids)
    tied = torch.from_numpy(GOLDEN["tied_scores"]).bfloat16().to(DEV)
    sel_tied = G.select16(torch, tied, torch.from_numpy(GOLDEN["tied_ids"]).to(DEV))
    torch.cuda.synchronize()
    np.testing.assert_array_equal(q.cpu().numpy(), GOLDEN["hidden_q"])
    np.testing.assert_array_equal(s.cpu().numpy(), GOLDEN["hidden_s"])
    for k, t in tops.items():
        np.testing.assert_array_equal(t.cpu().numpy(), GOLDEN[f"topk_ids_{k}"])
    exact, bound = OF.rescore_exact(GOLDEN["rand_w"], GOLDEN["rescore_ids"], GOLDEN["hidden"])
    g = _bf16_np(got)
    assert (np.abs(g - exact) <= 2.0 ** -8 * np.abs(exact) + 2.0 ** -12 * bound).all()
    assert (np.abs(g - GOLDEN["rescore_scores"]) <= 2.0 ** -7 * np.abs(exact) + 2.0 ** -11 * bound).all()
    np.testing.assert_array_equal(top16.cpu().numpy(), OF.select16(g, GOLDEN["rescore_ids"]))
    np.testing.assert_array_equal(sel_ref.cpu().numpy(), GOLDEN["rescore_top16"])
    np.testing.assert_array_equal(sel_tied.cpu().numpy(), GOLDEN["tied_top16"])


def test_retrieve_and_rescore_replays_in_a_cuda_graph():
    """tests/test_topk_compat_cuda.py:121-132: the step captured once in a CUDA graph and
    replayed on new hidden rows gives the eager results."""
    w = torch.zeros(512, 512, dtype=torch.bfloat16)
    w[:, 0] = torch.arange(512).remainder(47).bfloat16() / 32
    w[:, 1] = torch.arange(512).remainder(31).bfloat16() / 64
    local = C.FullVFP8Coarse(torch, w.to(DEV))
    hidden = torch.zeros(4, 512, device=DEV, dtype=torch.bfloat16)
    hidden[:, :2] = torch.tensor([[1, 2], [2, -1], [-1, 1], [0, 0]], device=DEV)
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            local.retrieve_and_rescore(hidden)
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    try:
        with torch.cuda.graph(graph):
            replayed = local.retrieve_and_rescore(hidden)
        for _ in range(2):
            hidden.neg_()
            graph.replay()
            eager = local.retrieve_and_rescore(hidden)
            torch.cuda.synchronize()
            for a, b in zip(replayed, eager):
                assert torch.equal(a, b)
    finally:
        graph.reset()
