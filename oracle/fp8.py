"""CPU oracle of the FP8 coarse retrieval + BF16 rescore -- TEST INFRASTRUCTURE ONLY.

Restates, in numpy, the reference's row-scaled FP8 retrieval (paths inside the reference
project, package ``sglang_dspine``):

  e4m3_encode / decode  the float8_e4m3fn format (1 sign, 4 exponent bits with bias 7, 3
                        mantissa bits, no infinities, 448 the largest finite value) with
                        round-to-nearest-even, as torch's ``.to(torch.float8_e4m3fn)``
  quantize_rows         layers/fp8/coarse.py:41-55 (_scale, _quantize) in float32
  coarse_exact          the row-scaled FP8 GEMM of coarse.py:84-93 in float64, with the scale
                        of its fp32 accumulation error
  coarse_fp32_small     the same GEMM for inputs whose fp32 dot products are exact: (acc * sx)
                        * sw in fp32, then bf16
  lexical_topk          stable descending order, the first k (coarse.py:19-35 portable path)
  rescore_exact         layers/fp8/gather.py:7-34, 53-70 in float64
  select16              layers/fp8/gather.py:37-50, 73-79: 16 rounds of (largest score, lowest
                        token among equals; that token's scores drop to -inf), ascending

Only tests use this module, as the checker.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32


def e4m3_encode(x):
    """uint8 codes of float32 values already within [-448, 448] (NaN -> 0x7F), round to
    nearest even: a normal |v| = m 2^E (m in [1, 2)) keeps rint(8 (m - 1)) mantissa bits, a
    subnormal (|v| < 2^-6) rint(|v| 2^9) (8 of them carry into 2^-6)."""
    v = np.asarray(x, np.float32).astype(np.float64)
    a = np.abs(v)
    sign = np.where(np.signbit(v), 0x80, 0).astype(np.int64)
    frac, e = np.frexp(a)                          # a = frac 2^e, frac in [0.5, 1)
    big = e - 1                                    # a = (2 frac) 2^big
    mi = np.rint(frac * 16.0).astype(np.int64) - 8  # exact scaling, half to even
    carry = mi == 8
    big = np.where(carry, big + 1, big)
    mi = np.where(carry, 0, mi)
    sat = (big > 8) | ((big == 8) & (mi > 6))
    big = np.where(sat, 8, big)
    mi = np.where(sat, 6, mi)
    normal = sign | ((big + 7) << 3) | mi
    sub = sign | np.rint(a * 512.0).astype(np.int64)
    code = np.where(a >= 2.0 ** -6, normal, sub)
    code = np.where(np.isnan(v), 0x7F, code)
    return code.astype(np.uint8)


def e4m3_decode(codes):
    c = np.asarray(codes, np.uint8).astype(np.int64)
    sign = np.where(c & 0x80, -1.0, 1.0)
    e = (c >> 3) & 0xF
    m = c & 0x7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.exp2(e.astype(np.float64) - 7))
    val = np.where((e == 0xF) & (m == 0x7), np.nan, val)
    return sign * val


def quantize_rows(x):
    """(codes uint8 [rows, cols], scales float32 [rows]) of _scale + _quantize."""
    x = np.asarray(x, np.float32)
    amax = np.abs(x).max(axis=1)
    scale = np.where(amax > 0, (amax / F32(448.0)).astype(F32), F32(1.0)).astype(F32)
    v = np.clip((x / scale[:, None]).astype(F32), F32(-448.0), F32(448.0))
    return e4m3_encode(v), scale


def coarse_exact(xq, sx, wq, sw):
    """(float64 scores, float64 bound): scores = (xq . wq^T) sx sw exactly; bound = the scale
    of an fp32-accumulated result's error (sum of |terms| times sx sw)."""
    x = e4m3_decode(xq)
    w = e4m3_decode(wq)
    s = np.asarray(sx, np.float64)[:, None] * np.asarray(sw, np.float64)[None, :]
    return (x @ w.T) * s, (np.abs(x) @ np.abs(w).T) * s


def _bf16(x):
    """Round float32 values to bf16 (nearest even), returned as float32."""
    u = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16) << 16
    return r.astype(np.uint32).view(np.float32)


def coarse_fp32_small(xq, sx, wq, sw):
    """bf16 scores (as float32) for inputs whose dot products are exact in fp32."""
    acc = (e4m3_decode(xq) @ e4m3_decode(wq).T).astype(F32)
    return _bf16((acc * np.asarray(sx, F32)[:, None]).astype(F32) * np.asarray(sw, F32)[None, :])


def lexical_topk(scores, k):
    """ids [rows, k] by (value desc, index asc)."""
    s = np.asarray(scores, np.float64)
    out = np.empty((s.shape[0], k), np.int64)
    idx = np.arange(s.shape[1])
    for r in range(s.shape[0]):
        out[r] = np.lexsort((idx, -s[r]))[:k]     # last key primary: value desc, then index
    return out


def rescore_exact(weight, ids, hidden):
    """(float64 scores [M, C], float64 bound): W[ids] . hidden and sum |terms|."""
    w = np.asarray(weight, np.float64)
    h = np.asarray(hidden, np.float64)
    g = w[np.asarray(ids)]
    return (g * h[:, None, :]).sum(-1), (np.abs(g) * np.abs(h)[:, None, :]).sum(-1)


def select16(scores, ids):
    """int64 [M, 16] of global_top16."""
    s = np.asarray(scores, np.float64)
    t = np.asarray(ids, np.int64)
    out = np.empty((s.shape[0], 16), np.int64)
    for r in range(s.shape[0]):
        vals = s[r].copy()
        chosen = []
        for _ in range(16):
            best = vals.max()
            tok = int(t[r][vals == best].min())
            chosen.append(tok)
            vals[t[r] == tok] = -np.inf
        out[r] = sorted(chosen)
    return out
