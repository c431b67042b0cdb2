"""Parity of the standalone top-k ids (dsv_topk_ids) with the reference kernel and the oracle.

Reference semantics: kernels/dspine.py:165-207 topk_ids (two stages over 64-wide chunks): the
k ids of the largest values of each row, ascending by id, ties at the k-th place to the lower
id.  tests/golden/topk.npz holds the reference kernel's own outputs; the oracle (the row's
top-k by value descending, id ascending) is pinned against them.  Ids are compared exactly.
"""

import numpy as np
import pytest
import torch

import oracle as O
from dspine_b200.kernels import dspine as K

pytestmark = pytest.mark.gpu

DEV = "cuda"
GOLDEN = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "topk.npz")
DTYPES = {"bf16": torch.bfloat16, "fp32": torch.float32, "fp16": torch.float16}


def run(x, k, dtype=torch.float32):
    t = torch.as_tensor(np.asarray(x, np.float32)).to(dtype).to(DEV)
    got = K.topk_ids(t, k)
    torch.cuda.synchronize()
    return got.cpu().numpy(), t.float().cpu().numpy()


def check(x, k, dtype=torch.float32):
    got, xr = run(x, k, dtype)
    np.testing.assert_array_equal(got, O.topk_ids(xr, k))


def test_golden_reference_outputs():
    for ci in range(int(GOLDEN["n"])):
        x, k = GOLDEN[f"c{ci}_x"], int(GOLDEN[f"c{ci}_k"])
        dtype = torch.bfloat16 if bool(GOLDEN[f"c{ci}_bf16"]) else torch.float32
        got, _ = run(x, k, dtype)
        np.testing.assert_array_equal(got, GOLDEN[f"c{ci}_ids"], err_msg=f"case {ci}")


@pytest.mark.parametrize("dtype", list(DTYPES))
@pytest.mark.parametrize("k", [1, 2, 4, 8, 16, 32, 64])
def test_random_rows(dtype, k):
    rng = np.random.default_rng({"bf16": 1, "fp32": 2, "fp16": 3}[dtype] * 100 + k)
    for v in (64 * k, 3001, 32000):
        if -(-v // 64) < k:
            continue
        check(rng.standard_normal((5, v)).astype(np.float32) * 4, k, DTYPES[dtype])


@pytest.mark.parametrize("dtype", list(DTYPES))
def test_heavy_ties(dtype):
    """Few distinct values: the k-th place straddles many equal values, chunk maxima tie."""
    rng = np.random.default_rng(7)
    for k in (1, 8, 64):
        x = rng.integers(0, 5, size=(6, 9000)).astype(np.float32)
        x[1] = 3.0                                   # every value equal
        x[2, :4096] = -np.inf                        # -inf prefix
        check(x, k, DTYPES[dtype])


def test_signed_zeros_inf_nan():
    """-0 equals +0 (ties to the lower id); -inf and +inf rank as numbers; NaN below all."""
    x = np.zeros((4, 4096), np.float32)
    x[0, ::2] = -0.0
    x[1, :] = -np.inf
    x[1, 100:110] = -0.0
    x[1, 3000] = np.inf
    x[2, :] = np.nan
    x[2, 1000:1100] = np.arange(100, dtype=np.float32)
    x[3, 7::13] = np.nan
    x[3, 4000] = np.inf
    for k in (1, 16, 64):
        for dt in DTYPES.values():
            check(x, k, dt)


def test_full_vocab_and_max_vocab():
    rng = np.random.default_rng(11)
    for v, k in ((151936, 16), (262144, 64), (262144, 1)):
        x = rng.standard_normal((3, v)).astype(np.float32)
        x[1, -1] = 100.0                             # the last element of the row wins
        check(x, k, torch.bfloat16)


def test_many_rows_and_strided_rows():
    """More rows than the grid (grid-stride loop); rows with a pitch above the vocabulary."""
    rng = np.random.default_rng(12)
    x = rng.standard_normal((1500, 640)).astype(np.float32)
    check(x, 8, torch.bfloat16)
    wide = torch.as_tensor(rng.standard_normal((7, 5000)).astype(np.float32)).to(DEV)
    view = wide[:, 100:4200]
    got = K.topk_ids(view, 32)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy(), O.topk_ids(view.cpu().numpy(), 32))


def test_out_argument_and_empty():
    x = torch.randn(3, 2048, device=DEV)
    out = torch.full((3, 4), -7, dtype=torch.int64, device=DEV)
    assert K.topk_ids(x, 4, out=out) is out
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), O.topk_ids(x.cpu().numpy(), 4))
    empty = K.topk_ids(torch.empty(0, 2048, device=DEV), 4)
    assert tuple(empty.shape) == (0, 4)
