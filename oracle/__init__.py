"""CPU oracle for the DSpine draft-block verification path -- TEST INFRASTRUCTURE ONLY.

This package is the checker that the CUDA product (package ``dspine_b200``) is compared
against.  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU-baseline leg
and its ``--impl reference`` arm) may import it; product code never does.

The arithmetic is defined in ``dsv_oracle.c``: exact 2^-40 fixed-point integer sums for every
sum that feeds a decision, and a fixed fp32 exp2 (Cody-Waite + degree-6 polynomial), so that
decisions are a function of the inputs alone.  Each wrapper names the reference function it
restates (paths inside the reference project, package ``sglang_dspine``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lib = None

F32P = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
I64P = np.ctypeslib.ndpointer(dtype=np.int64, flags="C_CONTIGUOUS")


def build() -> Path:
    """Compile the oracle library (make -C oracle)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


class RowDesc(ctypes.Structure):
    _fields_ = [
        ("greedy", ctypes.c_int32),
        ("argmax", ctypes.c_int32),
        ("m", ctypes.c_float),
        ("c", ctypes.c_float),
        ("kstar", ctypes.c_uint32),
        ("tie_cut", ctypes.c_int32),
        ("n_kept", ctypes.c_int32),
        ("s_total", ctypes.c_uint64),
        ("s_kept", ctypes.c_uint64),
        ("inv_s", ctypes.c_float),
    ]


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        build()
    L = ctypes.CDLL(str(_LIB_PATH))
    c = ctypes
    L.or_exp2.restype = c.c_float
    L.or_exp2.argtypes = [c.c_float]
    L.or_fix.restype = c.c_uint64
    L.or_fix.argtypes = [c.c_float]
    L.or_key_f32.restype = c.c_uint32
    L.or_key_f32.argtypes = [c.c_float]
    L.or_scale_floor.restype = c.c_int64
    L.or_scale_floor.argtypes = [c.c_float, c.c_uint64]
    L.or_process_row.restype = None
    L.or_process_row.argtypes = [F32P, c.c_int32, c.c_float, c.c_int32, c.c_float,
                                 c.POINTER(RowDesc)]
    L.or_process_row_ex.restype = None
    L.or_process_row_ex.argtypes = [F32P, c.c_int32, c.c_float, c.c_int32, c.c_float, c.c_float,
                                    c.c_int32, c.POINTER(RowDesc)]
    L.or_minp_floor.restype = c.c_uint32
    L.or_minp_floor.argtypes = [c.c_float, c.c_float, c.c_float]
    L.or_target_probs_ex.restype = None
    L.or_target_probs_ex.argtypes = [F32P, c.c_int64, c.c_int32, c.c_int32, F32P, I32P, F32P,
                                     c.c_void_p, c.c_int32, F32P, c.c_int32]
    L.or_verify_logits_ex.restype = None
    L.or_verify_logits_ex.argtypes = [c.c_int32, c.c_int32, I64P, F32P, I64P, c.c_void_p, I64P,
                                      c.c_int64, F32P, I32P, F32P, c.c_void_p, c.c_int32, I32P,
                                      F32P, F32P, I32P, I32P, I32P, I64P, I64P, I32P, c.c_int32]
    L.or_sparse_target.restype = None
    L.or_sparse_target.argtypes = [F32P, c.c_int64, c.c_int32, F32P, I32P, F32P, c.c_int32,
                                   I32P, F32P, I32P, I32P, F32P, c.c_int32]
    L.or_target_probs.restype = None
    L.or_target_probs.argtypes = [F32P, c.c_int64, c.c_int32, c.c_int32, F32P, I32P, F32P,
                                  F32P, c.c_int32]
    L.or_chain_from_probs.restype = None
    L.or_chain_from_probs.argtypes = [c.c_int32, c.c_int32, I64P, F32P, F32P, I32P, F32P,
                                      F32P, I32P, I32P, I32P, I64P, I64P, I32P]
    L.or_verify_logits.restype = None
    L.or_verify_logits.argtypes = [c.c_int32, c.c_int32, I64P, F32P, I64P, c.c_void_p, I64P,
                                   c.c_int64, F32P, I32P, F32P, I32P, F32P, F32P, I32P, I32P,
                                   I32P, I64P, I64P, I32P, c.c_int32]
    L.or_accept_sparse.restype = None
    L.or_accept_sparse.argtypes = [c.c_int32, c.c_int32, I64P, c.c_void_p, c.c_void_p,
                                   c.c_void_p, c.c_void_p, c.c_void_p, c.c_int32, I64P, F32P,
                                   I32P, F32P, F32P, I32P, c.c_void_p, c.c_void_p, I32P, I32P,
                                   I64P, I64P, I32P]
    L.or_compress_probs.restype = None
    L.or_compress_probs.argtypes = [F32P, c.c_int64, c.c_int32, c.c_int32, I32P, F32P, I32P,
                                    I32P]
    L.or_accept_greedy.restype = None
    L.or_accept_greedy.argtypes = [c.c_int32, I64P, I64P, I32P, I32P, I32P, I32P, I64P, I64P,
                                   I32P]
    L.or_argmax_rows.restype = None
    L.or_argmax_rows.argtypes = [F32P, c.c_int64, c.c_int32, c.c_int64, I64P]
    L.or_topk_ids.restype = None
    L.or_topk_ids.argtypes = [F32P, c.c_int64, c.c_int32, c.c_int64, c.c_int32, I64P]
    L.or_topk_sorted.restype = None
    L.or_topk_sorted.argtypes = [F32P, c.c_int64, c.c_int32, c.c_int64, c.c_int32, F32P, I64P]
    L.or_uniforms.restype = None
    L.or_uniforms.argtypes = [I64P, I64P, c.c_int32, c.c_int32, c.c_int32, F32P]
    L.or_sps_lens.restype = None
    L.or_sps_lens.argtypes = [c.c_int32, F32P, F32P, c.c_int32, c.c_void_p, c.c_int32,
                              c.c_int32, I32P]
    L.or_sps_index.restype = None
    L.or_sps_index.argtypes = [c.c_int32, I32P, c.c_int32, I64P, I64P]
    L.or_accept_compact.restype = None
    L.or_accept_compact.argtypes = [c.c_int32, I32P, I32P, I64P, I32P, I64P, I64P, I32P, I32P,
                                    I32P, I32P]
    L.or_merge_topk.restype = None
    L.or_merge_topk.argtypes = [c.c_int64, c.c_int32, F32P, I64P, c.c_int32, F32P, I64P]
    _lib = L
    return L


def _f32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.float32))


def _i32(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.int32))


def _i64(x):
    return np.ascontiguousarray(np.asarray(x, dtype=np.int64))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _nthreads(n):
    return int(n if n is not None else (os.cpu_count() or 1))


# ---- scalars --------------------------------------------------------------------------


def exp2(y: float) -> float:
    return lib().or_exp2(float(y))


def fix(x: float) -> int:
    return int(lib().or_fix(float(x)))


def key_f32(v: float) -> int:
    return int(lib().or_key_f32(float(v)))


def scale_floor(u: float, m: int) -> int:
    return int(lib().or_scale_floor(float(u), int(m)))


# ---- target distribution (runtime/worker.py:440-508) -----------------------------------


# filter modes of runtime/worker.py:473-508 (dsv_oracle.h OR_JOINT / OR_SEQ / OR_TORCH)
JOINT, SEQUENTIAL, TORCH = 0, 1, 2


def filter_mode(sampling_backend: str, need_min_p: bool) -> int:
    """The filter mode of a batch: the pytorch backend, or flashinfer with the batch's min-p
    flag deciding between the sequential and the joint filter (runtime/worker.py:473-508)."""
    if sampling_backend == "pytorch":
        return TORCH
    if sampling_backend == "flashinfer":
        return SEQUENTIAL if need_min_p else JOINT
    raise ValueError(f"unsupported sampling backend {sampling_backend!r}")


def process_row(logits, temperature, top_k, top_p, min_p=0.0, mode=JOINT) -> RowDesc:
    l = _f32(logits).reshape(-1)
    d = RowDesc()
    lib().or_process_row_ex(l, l.size, float(temperature), int(top_k), float(top_p),
                            float(min_p), int(mode), ctypes.byref(d))
    return d


def minp_floor(m, c, min_p) -> int:
    return int(lib().or_minp_floor(float(m), float(c), float(min_p)))


def target_probs(logits, temperature, top_k, top_p, rows_per_request=1, nthreads=None,
                 min_p=None, mode=JOINT):
    """Dense p [rows, V] of build_dspine_target_probs; temperature/top_k/top_p (and min_p)
    are per request; request of row r = r // rows_per_request; mode = filter mode."""
    l = _f32(logits)
    rows, V = l.shape
    out = np.empty_like(l)
    mp = None if min_p is None else _f32(min_p).reshape(-1)
    lib().or_target_probs_ex(l, rows, V, int(rows_per_request), _f32(temperature).reshape(-1),
                             _i32(top_k).reshape(-1), _f32(top_p).reshape(-1), _ptr(mp),
                             int(mode), out, _nthreads(nthreads))
    return out


def sparse_target(logits, temperature, top_k, top_p, capacity=32, nthreads=None):
    """build_sparse_target (sampling/sparse/target.py:95-178) per row: returns (ids i32
    [rows, capacity], values f32, lengths i32, overflow i32, dense f32 [rows, V] with the
    overflow rows written and the others zero).  temperature/top_k/top_p are per row."""
    l = _f32(logits)
    rows, V = l.shape
    ids = np.empty((rows, capacity), np.int32)
    vals = np.empty((rows, capacity), np.float32)
    lens = np.empty(rows, np.int32)
    ovf = np.empty(rows, np.int32)
    dense = np.zeros_like(l)
    lib().or_sparse_target(l, rows, V, _f32(temperature).reshape(-1), _i32(top_k).reshape(-1),
                           _f32(top_p).reshape(-1), int(capacity), ids, vals, lens, ovf, dense,
                           _nthreads(nthreads))
    return ids, vals, lens, ovf, dense


# ---- rejection (sampling/rejection.py:12-153) ------------------------------------------


def _outputs(B):
    return (np.empty(B, np.int32), np.empty(B, np.int32), np.empty(B, np.int64),
            np.empty((B, 16), np.int64), np.empty(B, np.int32))


def chain_from_probs(candidates, target_probs, draft_probs, verify_lens, uniforms,
                     uniform_final, prefix_lens):
    """sample_capped_chain_from_probs with the exact residual CDF; returns the 5 outputs."""
    cand = _i64(candidates)
    p = _f32(target_probs)
    q = _f32(draft_probs)
    B = cand.shape[0]
    V = p.shape[-1]
    out = _outputs(B)
    lib().or_chain_from_probs(B, V, cand, p, q, _i32(verify_lens), _f32(uniforms),
                              _f32(uniform_final), _i32(prefix_lens), *out)
    return out


def verify_logits(candidates, target_logits, target_rows, draft_logits, draft_rows,
                  temperature, top_k, top_p, verify_lens, uniforms, uniform_final,
                  prefix_lens, nthreads=None, min_p=None, mode=JOINT):
    """Fused logits -> target p, draft q -> chain + residual bonus.  target_logits/draft_logits
    are [rows, V] (any float dtype, computed in fp32); target_rows[b] / draft_rows[b] give the
    first row of request b.  draft_logits=None: q is one-hot at the drafted token."""
    cand = _i64(candidates)
    tl = _f32(target_logits)
    V = tl.shape[-1]
    B = cand.shape[0]
    dl = None if draft_logits is None else _f32(draft_logits)
    if dl is not None and dl.shape[-1] != V:
        raise ValueError("draft vocab differs")
    out = _outputs(B)
    drows = _i64(draft_rows if draft_rows is not None else np.zeros(B))
    mp = None if min_p is None else _f32(min_p).reshape(-1)
    lib().or_verify_logits_ex(B, V, cand, tl, _i64(target_rows), _ptr(dl), drows, V,
                              _f32(temperature), _i32(top_k), _f32(top_p), _ptr(mp), int(mode),
                              _i32(verify_lens), _f32(uniforms), _f32(uniform_final),
                              _i32(prefix_lens), *out, _nthreads(nthreads))
    return out


def accept_sparse(candidates, dense_p, packed, q_ids, q_values, verify_lens, uniforms,
                  uniform_final, prefix_lens, row_offsets=None, vocab_size=None,
                  denominator=None):
    """accept_sparse (sampling/sparse/accept.py:463-543) with the exact residual CDF."""
    cand = _i64(candidates)
    B = cand.shape[0]
    dp = None if dense_p is None else _f32(dense_p)
    if dp is not None:
        V = dp.shape[-1]
        dp = dp.reshape(-1, V)
    else:
        V = int(vocab_size)
    if packed is not None:
        ids, vals, lens, ovf = packed
        ids, vals, lens, ovf = _i32(ids), _f32(vals), _i32(lens), _i32(ovf)
        width = ids.shape[-1]
    else:
        ids = vals = lens = ovf = None
        width = 1
    ro = None if row_offsets is None else _i64(row_offsets)
    den = None if denominator is None else _f32(denominator)
    out = _outputs(B)
    lib().or_accept_sparse(B, V, cand, _ptr(dp), _ptr(ids), _ptr(vals), _ptr(lens), _ptr(ovf),
                           width, _i64(q_ids), _f32(q_values), _i32(verify_lens),
                           _f32(uniforms), _f32(uniform_final), _i32(prefix_lens), _ptr(ro),
                           _ptr(den), *out)
    return out


def compress_probs(p, capacity=64):
    p = _f32(p)
    rows, V = p.shape
    ids = np.empty((rows, capacity), np.int32)
    vals = np.empty((rows, capacity), np.float32)
    lens = np.empty(rows, np.int32)
    ovf = np.empty(rows, np.int32)
    lib().or_compress_probs(p, rows, V, capacity, ids, vals, lens, ovf)
    return ids, vals, lens, ovf


# ---- greedy (verification/caps.py:32-59, ragged.py:51-76) -------------------------------


def accept_greedy(candidates, top1, verify_lens, prefix_lens):
    cand = _i64(candidates)
    B = cand.shape[0]
    out = _outputs(B)
    lib().or_accept_greedy(B, cand, _i64(top1), _i32(verify_lens), _i32(prefix_lens), *out)
    return out


def argmax_rows(x):
    x = _f32(x)
    rows, V = x.shape
    out = np.empty(rows, np.int64)
    lib().or_argmax_rows(x, rows, V, V, out)
    return out


# ---- top-k (kernels/dspine.py:165-207) -------------------------------------------------


def topk_ids(x, k):
    x = _f32(x)
    rows, V = x.shape
    out = np.empty((rows, k), np.int64)
    lib().or_topk_ids(x, rows, V, V, int(k), out)
    return out


def topk_sorted(x, k):
    x = _f32(x)
    rows, V = x.shape
    vals = np.empty((rows, k), np.float32)
    ids = np.empty((rows, k), np.int64)
    lib().or_topk_sorted(x, rows, V, V, int(k), vals, ids)
    return vals, ids


def logsumexp_rows(x):
    """float64 log-sum-exp of each row (the oracle for LSE outputs, a tolerance check)."""
    x = np.asarray(x, dtype=np.float64)
    m = x.max(axis=-1, keepdims=True)
    return (m[..., 0] + np.log(np.exp(x - m).sum(axis=-1)))


# ---- RNG (sampling/random.py:22-43) ----------------------------------------------------


def uniforms(seeds, positions, width, stream):
    s = _i64(seeds).reshape(-1)
    p = _i64(positions).reshape(-1)
    out = np.empty((s.size, width), np.float32)
    lib().or_uniforms(s, p, s.size, int(width), int(stream), out)
    return out


# ---- SPS (verification/sps.py:27-99) ---------------------------------------------------


def sps_lens(raw, table, budget, boundaries=None):
    raw = _f32(raw)
    B = raw.shape[0]
    table = _f32(table)
    nb = table.shape[-1]
    bnd = None if boundaries is None else _f32(boundaries)
    lens = np.empty(B, np.int32)
    lib().or_sps_lens(B, raw, table, nb, _ptr(bnd), 0 if bnd is None else bnd.size,
                      int(budget), lens)
    return lens


def sps_index(lens, T=16):
    lens = _i32(lens)
    B = lens.size
    qo = np.empty(B + 1, np.int64)
    index = np.empty(int(lens.sum()), np.int64)
    lib().or_sps_index(B, lens, int(T), qo, index)
    return qo, index


# ---- accept-compact (restated commit contract) -----------------------------------------


def accept_compact(commit, lens, output, slots, slot_rows):
    commit = _i32(commit)
    lens = _i32(lens)
    B = commit.size
    out = _i64(output)
    slots = _i32(slots)
    rows = _i64(slot_rows)
    n = int(commit.sum())
    nfree = int(np.maximum(lens - commit, 0).sum())
    tok = np.empty(n, np.int64)
    sl = np.empty(n, np.int32)
    off = np.empty(B + 1, np.int32)
    fr = np.empty(nfree, np.int32)
    foff = np.empty(B + 1, np.int32)
    lib().or_accept_compact(B, commit, lens, out, slots, rows, tok, sl, off, fr, foff)
    return tok, sl, off, fr, foff


# ---- TP merge (sampling/tp_head.py:9-14) -----------------------------------------------


def merge_topk(values, ids, k):
    v = _f32(values)
    i = _i64(ids)
    n, m = v.shape
    ov = np.empty((n, k), np.float32)
    oi = np.empty((n, k), np.int64)
    lib().or_merge_topk(n, m, v, i, int(k), ov, oi)
    return ov, oi
