"""Pin the CPU oracle to the reference: every fixture under tests/golden was produced by the
reference's own code (tests/golden/make_golden.py).  Integer and index outputs must match
exactly; target probabilities within the reference's own tolerance (tests/test_sampling.py:
62-92: exact support, rtol 1e-5, atol 1e-7)."""

from pathlib import Path

import numpy as np
import pytest

import oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name):
    return np.load(GOLDEN / f"{name}.npz")


def cases(data):
    return range(int(data["n"]))


NAMES = ("accept", "commit", "bonus", "output", "new_seq")


def assert_outputs(got, data, ci):
    for name, val in zip(NAMES, got):
        np.testing.assert_array_equal(val, data[f"c{ci}_{name}"], err_msg=f"case {ci} {name}")


def test_chain_matches_reference_kernel():
    d = load("chain")
    for ci in cases(d):
        got = O.chain_from_probs(d[f"c{ci}_cand"], d[f"c{ci}_p"], d[f"c{ci}_q"], d[f"c{ci}_caps"],
                                 d[f"c{ci}_u"], d[f"c{ci}_uf"], d[f"c{ci}_prefix"])
        assert_outputs(got, d, ci)


def test_sparse_accept_matches_reference_kernel():
    d = load("sparse")
    for ci in cases(d):
        kind = str(d[f"c{ci}_kind"])
        packed = None
        if kind != "dense":
            packed = tuple(d[f"c{ci}_{n}"] for n in ("ids", "vals", "lens", "ovf"))
        dense = None if kind == "pure_packed" else d[f"c{ci}_p"]
        got = O.accept_sparse(d[f"c{ci}_cand"], dense, packed, d[f"c{ci}_qids"],
                              d[f"c{ci}_qvals"], d[f"c{ci}_caps"], d[f"c{ci}_u"], d[f"c{ci}_uf"],
                              d[f"c{ci}_prefix"], row_offsets=d[f"c{ci}_offsets"],
                              vocab_size=d[f"c{ci}_p"].shape[-1])
        assert_outputs(got, d, ci)


def test_compress_probs_matches_reference_kernel():
    d = load("sparse")
    seen = 0
    for ci in cases(d):
        if f"c{ci}_cids" not in d:
            continue
        got = O.compress_probs(d[f"c{ci}_p"], capacity=32)
        for g, name in zip(got, ("cids", "cvals", "clens", "covf")):
            np.testing.assert_array_equal(g, d[f"c{ci}_{name}"])
        seen += 1
    assert seen > 0


def test_target_probs_match_float64_reference_rows():
    d = load("target")
    for ci in cases(d):
        T, k, tp = d[f"c{ci}_params"]
        got = O.target_probs(d[f"c{ci}_logits"][None], [T], [int(k)], [tp])[0]
        ref = d[f"c{ci}_p"]
        np.testing.assert_array_equal(got > 0, ref > 0, err_msg=f"support differs case {ci}")
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-7, err_msg=f"case {ci}")


def test_target_probs_hand_computed_rows():
    """tests/test_sampling.py:38-59 and tests/test_p_distribution_reference.py:56-61."""
    logits = np.log(np.array([[4.0, 3.0, 2.0, 1.0]], np.float32))
    got = O.target_probs(logits, [1.0], [2], [0.5])
    np.testing.assert_allclose(got[0], [4 / 7, 3 / 7, 0, 0], rtol=0, atol=1e-6)
    got = O.target_probs(logits, [1.0], [1 << 30], [0.75])
    np.testing.assert_allclose(got[0], [4 / 9, 3 / 9, 2 / 9, 0], rtol=0, atol=1e-6)


def test_greedy_rows_take_first_argmax():
    """tests/test_dynamic_sampling.py:308-338: all-equal greedy rows pick id 0."""
    logits = np.zeros((2, 97), np.float32)
    got = O.target_probs(logits, [0.7, 0.7], [1, 1], [0.8, 0.8])
    assert got[0, 0] == 1 and np.count_nonzero(got[0]) == 1
    assert got[1, 0] == 1 and np.count_nonzero(got[1]) == 1


def test_topk_ids_match_reference_kernel():
    d = load("topk")
    for ci in cases(d):
        got = O.topk_ids(d[f"c{ci}_x"], int(d[f"c{ci}_k"]))
        np.testing.assert_array_equal(got, d[f"c{ci}_ids"], err_msg=f"case {ci}")


def test_topk_lowest_id_ties_known_answer():
    """tests/test_topk_compat.py:70-84."""
    scores = np.tile((np.arange(257) % 7).astype(np.float32), (2, 1))
    scores[1, 254:] = -np.inf
    for k in (16, 128):
        vals, ids = O.topk_sorted(scores, k)
        for r in range(2):
            row = scores[r].tolist()
            expected = sorted(range(257), key=lambda i: (-row[i], i))[:k]
            assert ids[r].tolist() == expected


def test_uniforms_match_reference_bitwise():
    d = load("uniforms")
    for stream in range(4):
        got = O.uniforms(d["seeds"], d["positions"], 15, stream)
        np.testing.assert_array_equal(got, d[f"s{stream}"])


def test_sps_lens_match_reference():
    d = load("sps")
    for ci in cases(d):
        bnd = d[f"c{ci}_boundaries"] if f"c{ci}_boundaries" in d else None
        got = O.sps_lens(d[f"c{ci}_raw"], d[f"c{ci}_table"], int(d[f"c{ci}_budget"]), bnd)
        np.testing.assert_array_equal(got, d[f"c{ci}_lens"], err_msg=f"case {ci}")


def test_sps_index_layout():
    """tests/test_sps.py:237-240: index = [b*16+i for i < len_b]."""
    lens = np.array([1, 3, 16, 2], np.int32)
    qo, index = O.sps_index(lens)
    assert qo.tolist() == [0, 1, 4, 20, 22]
    assert index.tolist() == [b * 16 + i for b, n in enumerate(lens) for i in range(n)]


def test_merge_topk_matches_reference():
    d = load("merge")
    for ci in cases(d):
        v, i = O.merge_topk(d[f"c{ci}_v"], d[f"c{ci}_ids"], int(d[f"c{ci}_k"]))
        np.testing.assert_array_equal(i, d[f"c{ci}_outi"], err_msg=f"case {ci}")
        np.testing.assert_array_equal(v, d[f"c{ci}_outv"], err_msg=f"case {ci}")


def test_greedy_accept_matches_reference_kernels():
    d = load("greedy")
    for ci in cases(d):
        got = O.accept_greedy(d[f"c{ci}_cand"], d[f"c{ci}_top1"], d[f"c{ci}_caps"],
                              d[f"c{ci}_prefix"])
        assert_outputs(got, d, ci)


def test_exp2_within_one_ulp():
    ys = np.linspace(-125, 0, 20001).astype(np.float32)
    got = np.array([O.exp2(float(y)) for y in ys], np.float64)
    ex = np.exp2(ys.astype(np.float64))
    ulp = np.spacing(ex.astype(np.float32)).astype(np.float64)
    assert (np.abs(got - ex) / ulp).max() < 1.0
    assert O.exp2(0.0) == 1.0
    assert O.exp2(-126.0) == 0.0


def test_fix_is_round_half_even():
    assert O.fix(1.0) == 1 << 40
    assert O.fix(0.0) == 0 and O.fix(-1.0) == 0 and O.fix(float("nan")) == 0
    assert O.fix(2.0) == 1 << 40
    assert O.fix(2.0 ** -41) == 0          # exactly one half rounds to even
    assert O.fix(2.0 ** -40) == 1
    assert O.fix(3 * 2.0 ** -41) == 2       # 1.5 -> 2


def test_scale_floor_exact():
    m = (1 << 40) + 12345
    for u in (0.0, 0.5, 0.25, 0.999999940395, 1e-30):
        exp = int(np.floor(np.float64(np.float32(u)) * m)) if u > 1e-20 else 0
        assert O.scale_floor(u, m) == exp
    assert O.scale_floor(-0.5, m) == -1
    assert O.scale_floor(1.0, m) == -2
    assert O.scale_floor(float("nan"), m) == -2


def test_accept_compact_layout():
    commit = np.array([1, 3, 2], np.int32)
    lens = np.array([4, 3, 16], np.int32)
    output = np.arange(48, dtype=np.int64).reshape(3, 16)
    slots = np.arange(1000, 1048, dtype=np.int32)
    rows = np.array([0, 16, 32], np.int64)
    tok, sl, off, fr, foff = O.accept_compact(commit, lens, output, slots, rows)
    assert off.tolist() == [0, 1, 4, 6]
    assert tok.tolist() == [0, 16, 17, 18, 32, 33]
    assert sl.tolist() == [1000, 1016, 1017, 1018, 1032, 1033]
    assert foff.tolist() == [0, 3, 3, 17]
    assert fr.tolist() == [1001, 1002, 1003] + list(range(1034, 1048))


# ---- draft-side serial chains (kernels/dspine.py:210-324, 616-772) -----------------------------

def test_sample_chain_oracle_matches_reference_kernel():
    """Tokens exact, q and confidence within fp32 rounding of the reference kernel (run under
    the Triton interpreter); the reference's own test oracle agrees on the same inputs."""
    import oracle.serial as OS
    from tests.helpers import serial_chain_case

    d = load("serial")
    for ci in range(int(d["n_chain"])):
        inp, ref = serial_chain_case(d, ci)
        tok, q, conf = OS.sample_chain(**inp)
        np.testing.assert_array_equal(tok, ref["tok"], err_msg=f"case {ci}")
        np.testing.assert_array_equal(tok, ref["ref_tok"], err_msg=f"case {ci}")
        np.testing.assert_allclose(q, ref["q"], rtol=1e-5, atol=1e-6, err_msg=f"case {ci}")
        np.testing.assert_allclose(q, ref["ref_q"], rtol=1e-5, atol=1e-6, err_msg=f"case {ci}")
        sampled = ~np.isnan(conf)
        np.testing.assert_allclose(conf[sampled], ref["conf"][sampled], rtol=1e-5, atol=1e-6)
        assert (ref["conf"][~sampled] == np.float32(-0.25)).all()  # greedy rows untouched


def test_serial_table_oracle_pins_reference_kernel():
    """The reference kernel's best lane is an argmax of the fp64 scores within the fp32
    accumulation error, and its confidence matches; the greedy walk of its table is the
    reference walk bit for bit."""
    import oracle.serial as OS
    from tests.helpers import serial_scores, serial_table_case

    d = load("serial")
    for ti in range(int(d["n_table"])):
        case, ref = serial_table_case(d, ti)
        s, bound = serial_scores(case)
        tol = 2e-5 * bound.max(axis=2)
        picked = np.take_along_axis(s, ref["idx"][..., None], axis=2)[..., 0]
        assert (picked >= s.max(axis=2) - tol).all(), f"table case {ti}"
        idx, conf = OS.table_idx_conf(s, case["rms"], case["T"])
        np.testing.assert_allclose(conf, ref["conf"], rtol=2e-4, atol=1e-6, err_msg=f"case {ti}")
        out, cout = OS.chain(ref["idx"], case["cand"], case["T"], ref["conf"])
        np.testing.assert_array_equal(out, ref["chain"])
        np.testing.assert_array_equal(cout, ref["chain_conf"])


def test_target_probs_min_p_and_pytorch_backend_match_reference_rows():
    """ref_target_row with min-p on (flashinfer: sequential top-k -> top-p -> min-p; pytorch:
    joint top-k / top-p and min-p) and the pytorch backend with min-p off: exact support,
    values within rtol 1e-5 (target_minp.npz)."""
    d = load("target_minp")
    for ci in cases(d):
        T, k, tp, mp = d[f"c{ci}_params"]
        backend = str(d[f"c{ci}_backend"])
        mode = O.filter_mode(backend, mp > 0)
        got = O.target_probs(d[f"c{ci}_logits"][None], [T], [int(k)], [tp], min_p=[mp],
                             mode=mode)[0]
        ref = d[f"c{ci}_p"]
        np.testing.assert_array_equal(got > 0, ref > 0,
                                      err_msg=f"support differs case {ci} ({backend}, {mp})")
        np.testing.assert_allclose(got, ref, rtol=1e-5, atol=1e-7, err_msg=f"case {ci}")


def test_sparse_target_matches_reference_cpu_branch():
    """build_sparse_target's CPU branch (sampling/sparse/target.py:156-178): lengths, overflow
    flags and the packed ids of packed rows exact, their values and the dense overflow rows
    within rtol 1e-5, on
    random, bf16-like quantised (ties at the k-th p) and plateau / all-equal rows."""
    d = load("sparse_target")
    n_ovf = 0
    for ci in cases(d):
        ids, vals, lens, ovf, dense = O.sparse_target(
            d[f"c{ci}_logits"], d[f"c{ci}_temp"], d[f"c{ci}_topk"], d[f"c{ci}_topp"], 32)
        np.testing.assert_array_equal(ovf, d[f"c{ci}_ovf"], err_msg=f"overflow case {ci}")
        np.testing.assert_array_equal(lens, d[f"c{ci}_lens"], err_msg=f"lengths case {ci}")
        # packed entries of overflow rows are unused (accept_sparse reads the dense row), and
        # the reference fills them from whichever tied ids torch.topk returned
        keep = d[f"c{ci}_ovf"] == 0
        np.testing.assert_array_equal(ids[keep], d[f"c{ci}_ids"][keep], err_msg=f"ids case {ci}")
        np.testing.assert_allclose(vals[keep], d[f"c{ci}_vals"][keep], rtol=1e-5, atol=1e-7,
                                   err_msg=f"values case {ci}")
        rows = d[f"c{ci}_ovf_rows"]
        n_ovf += len(rows)
        np.testing.assert_allclose(dense[rows], d[f"c{ci}_dense"], rtol=1e-5, atol=1e-7,
                                   err_msg=f"dense overflow rows case {ci}")
    assert n_ovf > 0
