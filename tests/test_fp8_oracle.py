"""The FP8 retrieval oracle pinned on the CPU: its e4m3 encoder against torch's
float8_e4m3fn conversion, its row quantization against the reference's _scale/_quantize
formulas (layers/fp8/coarse.py:41-55) run by torch on the CPU, and its selection rules against
known answers (coarse.py:19-35 lower-index ties; gather.py:37-50 selection rounds)."""

import numpy as np
import torch

import oracle.fp8 as OF


def test_e4m3_encoder_matches_torch():
    rng = np.random.default_rng(0)
    vals = np.concatenate([
        rng.standard_normal(20000) * 50,
        rng.standard_normal(5000) * 0.01,          # subnormal range
        np.ldexp(1.0, np.arange(-12, 9)),           # powers of two
        (np.arange(1, 256) / 8.0),                  # midpoints / exact values
        [0.0, -0.0, 448.0, -448.0, 2.0 ** -9, 2.0 ** -10, 3 * 2.0 ** -10, 2.0 ** -6 - 2.0 ** -10],
    ]).astype(np.float32)
    vals = np.clip(vals, -448, 448).astype(np.float32)
    # every midpoint between neighbouring codes (ties to even)
    finite = OF.e4m3_decode(np.arange(0, 0x7F, dtype=np.uint8))
    mids = ((finite[1:] + finite[:-1]) / 2).astype(np.float32)
    vals = np.concatenate([vals, mids, -mids])
    ref = torch.from_numpy(vals).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    np.testing.assert_array_equal(OF.e4m3_encode(vals), ref)


def test_decode_encode_round_trip():
    codes = np.array([c for c in range(256) if c & 0x7F != 0x7F], np.uint8)
    np.testing.assert_array_equal(OF.e4m3_encode(OF.e4m3_decode(codes).astype(np.float32)), codes)


def test_quantize_rows_matches_reference_formula():
    rng = np.random.default_rng(1)
    x = (rng.standard_normal((6, 700)) * rng.uniform(0.01, 30, size=(6, 1))).astype(np.float32)
    x[2] = 0.0                                     # all-zero row: scale 1
    x[3, 5] = 1e-30                                # tiny row maximum
    x[3, 6:] = 0.0
    x[4, 17] = np.nan                              # NaN row: amax NaN, scale 1, NaN codes
    x[5, 3] = np.inf                               # inf row: scale inf, inf / inf = NaN code
    xt = torch.from_numpy(x).bfloat16().float()    # bf16 inputs, as the hidden rows
    maximum = xt.abs().amax(dim=1, keepdim=True)
    scale = torch.where(maximum > 0, maximum / 448.0, torch.ones_like(maximum)).float()
    q_ref = (xt / scale).clamp(-448.0, 448.0).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    q, s = OF.quantize_rows(xt.numpy())
    np.testing.assert_array_equal(s, scale[:, 0].numpy())
    # e4m3 has two NaN codes (0x7F, 0xFF); which sign a NaN carries depends on the arithmetic
    # that produced it (the host's inf / inf is negative, a GPU's canonical NaN positive)
    is_nan = (q_ref & 0x7F) == 0x7F
    np.testing.assert_array_equal((q & 0x7F) == 0x7F, is_nan)
    np.testing.assert_array_equal(q[~is_nan], q_ref[~is_nan])
    assert is_nan[4].sum() == 1 and is_nan[5].sum() == 1


def test_lexical_topk_and_select16_known_answers():
    scores = np.array([[1.0, 3.0, 3.0, 2.0, 3.0] + [0.0] * 15], np.float32)
    np.testing.assert_array_equal(OF.lexical_topk(scores, 4), [[1, 2, 4, 3]])
    ids = np.arange(100, 120)[None, :]
    got = OF.select16(scores, ids)
    expected = sorted([101, 102, 104, 103, 100] + [105 + i for i in range(11)])
    np.testing.assert_array_equal(got, [expected])


GOLDEN = np.load(__import__("pathlib").Path(__file__).resolve().parent / "golden" / "fp8.npz")


def test_quantization_matches_reference_fixtures():
    """FullVFP8Coarse.__init__ and _scale/_quantize of the reference (tests/golden/fp8.npz)."""
    for name in ("two", "rand"):
        q, s = OF.quantize_rows(GOLDEN[f"{name}_w"])
        np.testing.assert_array_equal(q, GOLDEN[f"{name}_wq"])
        np.testing.assert_array_equal(s, GOLDEN[f"{name}_ws"])
    q, s = OF.quantize_rows(GOLDEN["hidden"])
    np.testing.assert_array_equal(q, GOLDEN["hidden_q"])
    np.testing.assert_array_equal(s, GOLDEN["hidden_s"])


def test_lexical_topk_matches_reference_stable_topk():
    for k in (1, 16, 128):
        np.testing.assert_array_equal(OF.lexical_topk(GOLDEN["topk_scores"], k), GOLDEN[f"topk_ids_{k}"])


def test_rescore_and_select16_match_reference_kernels():
    """gather.rescore (fp32 sums stored bf16) within one bf16 ulp plus the fp32 accumulation
    bound (the fixture ran under the Triton interpreter, whose fp32 -> bf16 store truncates
    where the GPU rounds to nearest); select16 exact on the reference's own stored scores."""
    exact, bound = OF.rescore_exact(GOLDEN["rand_w"], GOLDEN["rescore_ids"], GOLDEN["hidden"])
    ref = GOLDEN["rescore_scores"]
    assert (np.abs(ref - exact) <= 2.0 ** -7 * np.abs(exact) + 2.0 ** -12 * bound).all()
    np.testing.assert_array_equal(OF.select16(ref, GOLDEN["rescore_ids"]), GOLDEN["rescore_top16"])
    np.testing.assert_array_equal(OF.select16(GOLDEN["tied_scores"], GOLDEN["tied_ids"]),
                                  GOLDEN["tied_top16"])
