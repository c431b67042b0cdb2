"""Draft-side serial chains at the reference's ``sglang_dspine.kernels.dspine`` interface.

`serial_sample_chain`, `serial_table`, `serial_chain` and `topk_ids` keep the reference's
signatures, argument checks (ValueError before anything is launched) and caller-owned, in-place
outputs (kernels/dspine.py:165-207, 357-502, 677-772); each is one launch of the library's C ABI
(dsv_serial_sample_chain, dsv_serial_table, dsv_serial_chain, dsv_topk_ids).  `build_serial_tables` is the
offline table build (kernels/dspine.py:327-351): two plain bf16 library GEMMs per vocabulary
chunk, run once per weight load, not per step.
"""

from __future__ import annotations

import torch

from .. import _lib


def _stream(t) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _cuda(*tensors):
    for t in tensors:
        if t is not None and t.device.type != "cuda":
            raise ValueError("dspine_b200 runs the serial chains on CUDA tensors only")


_TOPK_CHUNK = 64
_TOPK_DTYPES = {torch.bfloat16: 0, torch.float32: 1, torch.float16: 2}


def topk_ids(logits: torch.Tensor, k: int, out: torch.Tensor = None) -> torch.Tensor:
    """logits [N, V] (contiguous rows) -> int64 [N, k] ids of the k largest values, ascending
    by id (kernels/dspine.py:165-207).  The reference's two stages (maxima of 64-wide chunks,
    then the top-k of the k chunks with the largest maxima) give the row's top-k by (value
    descending, id ascending); one launch of dsv_topk_ids, one CTA per row."""
    if logits.dim() != 2 or logits.stride(1) != 1:
        raise ValueError("topk_ids expects a row-contiguous [N, V] tensor")
    if k & k - 1 or not 1 <= k <= 64:
        raise ValueError(f"topk_ids needs a power-of-two k in [1, 64], got {k}")
    n, v = logits.shape
    nch = -(-v // _TOPK_CHUNK)
    if nch < k:
        raise ValueError(f"topk_ids needs at least k={k} chunks of {_TOPK_CHUNK}, vocab={v}")
    if logits.dtype not in _TOPK_DTYPES:
        raise ValueError(f"topk_ids supports bf16, fp16 and fp32 logits, got {logits.dtype}")
    if out is None:
        out = torch.empty((n, k), dtype=torch.int64, device=logits.device)
    elif tuple(out.shape) != (n, k) or out.dtype != torch.int64 or not out.is_contiguous():
        raise ValueError("topk_ids: out must be a contiguous int64 [N, k] tensor")
    if n == 0:
        return out
    _cuda(logits, out)
    stride = logits.stride(0) if n > 1 else v
    if torch.cuda.current_device() == logits.device.index:
        _lib.call("dsv_topk_ids", n, v, stride, _TOPK_DTYPES[logits.dtype], logits.data_ptr(), k,
                  out.data_ptr(), _stream(logits))
    else:
        with torch.cuda.device(logits.device):
            _lib.call("dsv_topk_ids", n, v, stride, _TOPK_DTYPES[logits.dtype], logits.data_ptr(),
                      k, out.data_ptr(), _stream(logits))
    return out


def build_serial_tables(lm_head_w, norm_w, write_w, pv_w, codebook, chunk: int = 8192):
    """(TG [V, R] bf16, TSV [V, 2R] bf16) with TG[v] = bf16(LmHead[v] * norm_w) @ W_last and
    TSV[v] = [G_p; A] @ bf16(sqrt(C) * Codebook[v]) (kernels/dspine.py:327-351): the per-token
    tables the serial refinement gathers by id.  Offline (once per weight load): the normed
    head rows and the scaled codebook rows are rounded to bf16 block by block and multiplied
    by the two fixed factors with library GEMMs written straight into the tables."""
    (v, h) = lm_head_w.shape
    r = write_w.shape[1]
    c = codebook.shape[1]
    if (codebook.shape[0] != v or tuple(write_w.shape) != (h, r) or tuple(pv_w.shape) != (2 * r, c)
            or norm_w.shape != (h,)):
        raise ValueError("build_serial_tables: shape contract violated")
    device = lm_head_w.device
    tg = torch.empty((v, r), device=device, dtype=torch.bfloat16)
    tsv = torch.empty((v, 2 * r), device=device, dtype=torch.bfloat16)
    w_last = write_w.to(torch.bfloat16)   # [H, R]
    gate_value = pv_w.t()                 # [C, 2R]: x @ pv_w.T
    norm = norm_w.float()
    scale = float(c) ** 0.5
    step = max(1, int(chunk))
    for lo in range(0, v, step):
        hi = min(lo + step, v)
        torch.mm((lm_head_w[lo:hi].float() * norm).to(torch.bfloat16), w_last, out=tg[lo:hi])
        torch.mm((codebook[lo:hi].float() * scale).to(torch.bfloat16), gate_value, out=tsv[lo:hi])
    return (tg, tsv)


def serial_table(raw, norm_w, cand, input_ids, lm_head_w, tg, tsv, packed, rms, gate_b,
                 block_size: int, confidence=None, candidate_head=None):
    """idx int64 [bs*(T-1), K]: idx[n, j] = the best candidate lane of row n when the previous
    row chose lane j (kernels/dspine.py:357-471).  raw [bs*T, H] bf16, cand int64 [n, K],
    input_ids [bs*T], packed [bs*T, >=R] bf16 (receiver query in columns :R), rms fp32 [bs*T];
    optional confidence fp32 [n, K] output, optional candidate_head bf16 [n, K, H]."""
    t = int(block_size)
    (m, h) = raw.shape
    (n, k) = cand.shape
    rk = tg.shape[1]
    if candidate_head is not None:
        if (candidate_head.shape != (n, k, h) or candidate_head.dtype != torch.bfloat16
                or not candidate_head.is_contiguous()):
            raise ValueError("serial_table candidate head must be contiguous BF16 [N,K,H]")
        lm_head_w = candidate_head.view(n * k, h)
    if m % t or n != m // t * (t - 1) or input_ids.numel() != m or rms.numel() != m:
        raise ValueError(f"serial_table row mismatch: raw {raw.shape}, cand {cand.shape}, T={t}")
    if (raw.dtype != torch.bfloat16 or raw.stride(1) != 1 or packed.dtype != torch.bfloat16
            or packed.stride(1) != 1):
        raise ValueError("serial_table expects row-contiguous BF16 state and query")
    if packed.shape[0] != m or packed.shape[1] < rk or rms.dtype != torch.float32 or not rms.is_contiguous():
        raise ValueError("serial_table query/rms contract violated")
    if (not cand.is_contiguous() or cand.dtype != torch.int64 or input_ids.dtype != torch.int64
            or not input_ids.is_contiguous()):
        raise ValueError("serial_table expects contiguous int64 candidates and input ids")
    if lm_head_w.stride(1) != 1 or tuple(tsv.shape) != (tg.shape[0], 2 * rk) or not (
            tg.is_contiguous() and tsv.is_contiguous()):
        raise ValueError("serial_table table layout mismatch")
    if h % 512 or rk % 128 or k & (k - 1) or not 2 <= k <= 64 or gate_b.numel() != rk or norm_w.numel() != h:
        raise ValueError("serial_table size contract violated")
    if (lm_head_w.dtype != torch.bfloat16 or tg.dtype != torch.bfloat16 or tsv.dtype != torch.bfloat16
            or norm_w.dtype != torch.bfloat16 or gate_b.dtype != torch.bfloat16):
        raise ValueError("serial_table expects BF16 weights, tables, norm and gate bias")
    idx = torch.empty((n, k), dtype=torch.int64, device=raw.device)
    if confidence is not None and (tuple(confidence.shape) != (n, k) or confidence.dtype != torch.float32
                                   or not confidence.is_contiguous()):
        raise ValueError("Confidence output must be contiguous float32 [N, K]")
    _cuda(raw, norm_w, cand, input_ids, lm_head_w, tg, tsv, packed, rms, gate_b, confidence)
    if n:
        vocab = tg.shape[0]
        if candidate_head is None and lm_head_w.shape[0] < vocab:
            vocab = lm_head_w.shape[0]  # ids must address rows of every table
        _lib.call("dsv_serial_table", m // t, t, h, rk, k, vocab, raw.data_ptr(), raw.stride(0),
                  norm_w.contiguous().data_ptr(), cand.data_ptr(), input_ids.data_ptr(),
                  lm_head_w.data_ptr(), lm_head_w.stride(0), int(candidate_head is not None),
                  tg.data_ptr(), tsv.data_ptr(), packed.data_ptr(), packed.stride(0), rms.data_ptr(),
                  gate_b.contiguous().data_ptr(), idx.data_ptr(), _lib.ptr(confidence), _stream(raw))
    return idx


def serial_chain(idx, cand, out, block_size: int, confidence=None, confidence_out=None):
    """Walk every request's greedy table: out[:bs*(T-1)] written in place (int64)
    (kernels/dspine.py:474-502)."""
    t = int(block_size)
    (n, k) = cand.shape
    if n % (t - 1) or tuple(idx.shape) != (n, k) or not (idx.is_contiguous() and cand.is_contiguous()):
        raise ValueError("serial_chain layout mismatch")
    if out.dtype != torch.int64 or out.numel() < n or idx.dtype != torch.int64:
        raise ValueError("serial_chain dtype/capacity contract violated")
    if confidence is not None and (confidence_out is None or confidence_out.dtype != torch.float32
                                   or confidence_out.numel() < n or tuple(confidence.shape) != (n, k)):
        raise ValueError("Serial confidence needs a float32 [N, K] table and [N] output")
    if not out.is_contiguous() or (confidence_out is not None and not confidence_out.is_contiguous()):
        raise ValueError("serial_chain outputs must be contiguous")
    if confidence is not None and (confidence.dtype != torch.float32 or not confidence.is_contiguous()):
        raise ValueError("Serial confidence needs a float32 [N, K] table and [N] output")
    _cuda(idx, cand, out, confidence, confidence_out)
    if n:
        conf_out = confidence_out if confidence is not None else None
        _lib.call("dsv_serial_chain", n // (t - 1), t, k, idx.data_ptr(), cand.data_ptr(),
                  out.data_ptr(), _lib.ptr(confidence), _lib.ptr(conf_out), _stream(idx))
    return out


def serial_sample_chain(table, inv_temp, top_k, top_p, min_p, greedy, u, cand, greedy_tok, out_tok,
                        out_q, block_size: int, *, confidence_out=None):
    """Sample every request's chain; fills out_tok[:n] / out_q[:n] in place
    (kernels/dspine.py:677-772).  table fp32 [n, K, K]; inv_temp fp32 [>=bs]; top_k int32
    [>=bs] (>= 1; >= K disables it); top_p fp32 [>=bs] in (0, 1]; min_p fp32 [>=bs] in [0, 1];
    greedy int32 [>=bs]; u fp32 [>=n] in [0, 1); cand int64 [n, K]; greedy_tok int64 [>=n];
    out_tok int64 [>=n]; out_q fp32 [>=n, K].  Optional confidence_out fp32 [>=n]: the maximum
    temperature-softmax probability of each sampled row before filtering (greedy rows keep
    their values)."""
    t = int(block_size)
    (n, k) = cand.shape
    if n % (t - 1) or tuple(table.shape) != (n, k, k) or not table.is_contiguous():
        raise ValueError("serial_sample_chain table layout mismatch")
    bs = n // (t - 1)
    staged = (inv_temp, top_k, top_p, min_p, greedy)
    if any(x.numel() < bs for x in staged) or u.numel() < n or greedy_tok.numel() < n:
        raise ValueError("serial_sample_chain staging buffers too small")
    if out_tok.numel() < n or out_q.shape[0] < n or out_q.shape[1] != k:
        raise ValueError("serial_sample_chain output buffers too small")
    if not (cand.is_contiguous() and out_q.is_contiguous()):
        raise ValueError("serial_sample_chain expects contiguous candidates and q")
    if confidence_out is not None and (confidence_out.dtype != torch.float32
                                       or confidence_out.numel() < n
                                       or not confidence_out.is_contiguous()
                                       or confidence_out.device != table.device):
        raise ValueError(
            "serial_sample_chain confidence needs contiguous float32 storage on the table device")
    dtypes = (table.dtype, inv_temp.dtype, top_k.dtype, top_p.dtype, min_p.dtype, greedy.dtype,
              u.dtype, cand.dtype, greedy_tok.dtype, out_tok.dtype, out_q.dtype)
    expected = (torch.float32, torch.float32, torch.int32, torch.float32, torch.float32,
                torch.int32, torch.float32, torch.int64, torch.int64, torch.int64, torch.float32)
    if dtypes != expected:
        raise ValueError(f"serial_sample_chain dtype contract violated: {dtypes}")
    if k > 64:
        raise ValueError("serial_sample_chain supports at most 64 candidates per row")
    for x in (inv_temp, top_k, top_p, min_p, greedy, u, greedy_tok, out_tok):
        if not x.is_contiguous():
            raise ValueError("serial_sample_chain expects contiguous staging and output vectors")
    _cuda(table, *staged, u, cand, greedy_tok, out_tok, out_q, confidence_out)
    if bs:
        _lib.call("dsv_serial_sample_chain", bs, t, k, table.data_ptr(), inv_temp.data_ptr(),
                  top_k.data_ptr(), top_p.data_ptr(), min_p.data_ptr(), greedy.data_ptr(),
                  u.data_ptr(), cand.data_ptr(), greedy_tok.data_ptr(), out_tok.data_ptr(),
                  out_q.data_ptr(), _lib.ptr(confidence_out), _stream(table))
    return (out_tok, out_q)
