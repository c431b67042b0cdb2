"""CPU oracle of the draft-side serial chains -- TEST INFRASTRUCTURE ONLY.

Restates, in numpy, the reference kernels that produce a block's draft tokens, q rows and
confidences (paths inside the reference project, package ``sglang_dspine``):

  sample_chain   kernels/dspine.py:616-674 _serial_sample_chain (and its test oracle
                 tests/ref_utils.py:12-50 ref_sample_chain), in fp32 with the summation orders
                 the CUDA kernel fixes (butterfly sums, Kogge-Stone prefix sums)
  table_scores   kernels/dspine.py:210-287 _serial_table: the score matrix s[n, j, c] in fp64
                 from the same bf16 inputs, with a bound on the fp32 accumulation error
  chain          kernels/dspine.py:290-324 _serial_chain
  refine_table   tests/ref_utils.py:53-76 ref_refine_table (fp64), the redone last write that
                 the greedy table approximates

Only tests and ``__graft_entry__.smoke()`` use this module, as the checker.
"""

from __future__ import annotations

import math

import numpy as np

F32 = np.float32


def _bfly_sum(v):
    """Butterfly sum of up to 64 float32 values: lane l holds v[l] + v[l + 32], then
    xor-shuffle steps 16, 8, 4, 2, 1 (every lane ends with the same value)."""
    x = np.zeros(64, F32)
    x[: len(v)] = v
    s = (x[:32] + x[32:]).astype(F32)
    lanes = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        s = (s + s[lanes ^ o]).astype(F32)
    return F32(s[0])


def _scan32(v):
    v = v.astype(F32).copy()
    for o in (1, 2, 4, 8, 16):
        v[o:] = (v[o:] + v[:-o]).astype(F32)
    return v


def _scan64(v):
    """Inclusive prefix sums of up to 64 float32 values: Kogge-Stone scans (shifts 1..16) of
    positions 0..31 and 32..63, the second half plus the total of the first."""
    x = np.zeros(64, F32)
    x[: len(v)] = v
    lo = _scan32(x[:32])
    hi = (_scan32(x[32:]) + lo[31]).astype(F32)
    return np.concatenate((lo, hi))


def sample_chain(table, inv_t, top_k, top_p, min_p, greedy, u, cand, greedy_tok, T):
    """(tok int64 [n], q f32 [n, K], conf f32 [n] with NaN where a greedy row writes nothing).

    fp32 throughout, with the summation orders the CUDA kernel fixes: butterfly sums for the
    softmax denominator and the kept mass, Kogge-Stone prefix sums for the mass ranked ahead
    (in rank order) and for the CDF (in lane order)."""
    table = np.asarray(table, F32)
    n, k, _ = table.shape
    tm1 = T - 1
    tok = np.zeros(n, np.int64)
    q_out = np.zeros((n, k), F32)
    conf = np.full(n, np.nan, F32)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        for b in range(n // tm1):
            sender = 0
            it, tk, tp, mp = F32(inv_t[b]), int(top_k[b]), F32(top_p[b]), F32(min_p[b])
            gr = bool(greedy[b])
            for i in range(tm1):
                row = b * tm1 + i
                s = (table[row, sender] * it).astype(F32)
                m = np.exp((s - s.max()).astype(F32)).astype(F32)
                total = _bfly_sum(m)
                p = (m / total).astype(F32)
                pmax = F32(p.max())
                if not gr:
                    conf[row] = pmax
                order = sorted(range(k), key=lambda c: (-float(p[c]), c))
                rank = np.empty(k, np.int64)
                rank[order] = np.arange(k)
                ahead = np.concatenate(([F32(0)], _scan64(p[order])[: k - 1]))
                before = ahead[rank]
                keep = (rank < tk) & (before <= tp) & (p >= F32(mp * pmax))
                w = np.where(keep, p, F32(0)).astype(F32)
                q = (w / _bfly_sum(w)).astype(F32)
                cdf = _scan64(q)[:k]
                thr = F32(F32(u[row]) * cdf[-1])
                choice = int((cdf <= thr).sum())
                kept = np.nonzero(keep)[0]
                choice = min(choice, int(kept.max()) if kept.size else 0)
                if gr:
                    tok[row] = greedy_tok[row]
                    q_out[row] = (cand[row] == greedy_tok[row]).astype(F32)
                else:
                    tok[row] = cand[row, choice]
                    q_out[row] = q
                sender = choice
    return tok, q_out, conf


def _sigmoid(x):
    return 1.0 / (1.0 + np.exp(-x))


def table_scores(raw, norm_w, cand, input_ids, head_rows, tg, tsv, query, rms, gate_b, T):
    """fp64 s[n, j, c] of _serial_table and bound[n, j, c] = the sum of |terms| (the scale of
    the fp32 accumulation error).  head_rows(n) -> [K, H] weight rows of drafted row n; tg,
    tsv are indexed by token id (any mapping with __getitem__ on int arrays)."""
    raw, norm_w, query = (np.asarray(x, np.float64) for x in (raw, norm_w, query))
    rms, gate_b = np.asarray(rms, np.float64), np.asarray(gate_b, np.float64)
    n, k = cand.shape
    rk = gate_b.shape[0]
    tm1 = T - 1
    s = np.zeros((n, k, k))
    bound = np.zeros((n, k, k))
    for nn in range(n):
        b, r = divmod(nn, tm1)
        row = b * T + 1 + r
        sid = np.full(k, input_ids[b * T]) if r == 0 else cand[nn - 1]
        u = raw[row] * norm_w
        w = np.asarray(head_rows(nn), np.float64)
        base = w @ u
        base_abs = np.abs(w) @ np.abs(u)
        t = np.asarray(tsv[sid], np.float64)
        m = _sigmoid(query[row, :rk][None, :] + t[:, :rk] + gate_b[None, :]) * t[:, rk:]
        g = np.asarray(tg[cand[nn]], np.float64)
        s[nn] = base[None, :] + rms[row] * (m @ g.T)
        bound[nn] = base_abs[None, :] + rms[row] * (np.abs(m) @ np.abs(g).T)
    return s, bound


def table_idx_conf(s, rms, T):
    """idx (first argmax over c) and confidence 1 / sum_c exp((s - max) / max(rms, 1e-6))."""
    n, k, _ = s.shape
    idx = s.argmax(axis=2)
    conf = np.empty((n, k))
    tm1 = T - 1
    for nn in range(n):
        b, r = divmod(nn, tm1)
        scale = max(float(rms[b * T + 1 + r]), 1e-6)
        conf[nn] = 1.0 / np.exp((s[nn] - s[nn].max(axis=1, keepdims=True)) / scale).sum(axis=1)
    return idx, conf


def chain(idx, cand, T, confidence=None):
    """Greedy walk: (out int64 [n], conf_out f32 [n] or None)."""
    n, k = cand.shape
    tm1 = T - 1
    out = np.zeros(n, np.int64)
    cout = None if confidence is None else np.zeros(n, F32)
    for b in range(n // tm1):
        j = int(idx[b * tm1, 0])
        prev = 0
        for r in range(tm1):
            nn = b * tm1 + r
            if cout is not None:
                cout[nn] = confidence[nn, prev] if 0 <= prev < k else 0.0
            out[nn] = cand[nn, j] if 0 <= j < k else 0
            prev = j
            j = int(idx[nn + 1, j]) if (r + 1 < tm1 and 0 <= j < k) else 0
    return out, cout


def refine_table(raw, rms, query, anchors, cand, codebook, pg, pv, gb, w_last, norm_w, lm, eps, T):
    """fp64 Table[n, j, c] of the redone last write (the reference's test oracle)."""
    f = lambda x: np.asarray(x, np.float64)  # noqa: E731
    raw, rms, query, codebook, pg, pv, gb, w_last, norm_w = map(
        f, (raw, rms, query, codebook, pg, pv, gb, w_last, norm_w))
    m, h = raw.shape
    n, k = cand.shape
    c_size = codebook.shape[1]
    out = np.zeros((n, k, k))
    for b in range(m // T):
        for i in range(T - 1):
            row, nn = b * T + 1 + i, b * (T - 1) + i
            senders = [int(anchors[b])] * k if i == 0 else list(cand[nn - 1])
            head = f(lm(cand[nn]))
            for j, sdr in enumerate(senders):
                e = math.sqrt(c_size) * codebook[sdr]
                gate = _sigmoid(query[row] + pg @ e + gb)
                msg = gate * (pv @ e)
                xr = raw[row] + rms[row] * (w_last @ msg)
                normalized = xr / np.sqrt(np.mean(xr * xr) + eps) * norm_w
                out[nn, j] = head @ normalized
    return out
