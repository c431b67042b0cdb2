"""Sparse-q rejection and probability compression (sampling/sparse/accept.py of the reference).

`accept_sparse` and `compress_probs` keep the reference's signatures (including the leading
`torch` module argument), argument checks and caller-owned outputs; the work is one
dsv_accept_sparse / dsv_compress_probs launch (exact fixed-point residual CDF).
"""

from __future__ import annotations

from ... import _lib


def _stream(t):
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


def compress_probs(torch, p, capacity=64):
    (rows, vocab) = p.shape
    if p.device.type != "cuda" or p.dtype != torch.float32 or not p.is_contiguous():
        raise ValueError("compress_probs needs a contiguous fp32 CUDA tensor")
    ids = torch.empty((rows, capacity), device=p.device, dtype=torch.int32)
    values = torch.empty((rows, capacity), device=p.device, dtype=torch.float32)
    lengths = torch.empty(rows, device=p.device, dtype=torch.int32)
    overflow = torch.empty(rows, device=p.device, dtype=torch.int32)
    _lib.call("dsv_compress_probs", rows, vocab, int(capacity), p.data_ptr(), ids.data_ptr(),
              values.data_ptr(), lengths.data_ptr(), overflow.data_ptr(), _stream(p))
    return (ids, values, lengths, overflow)


def accept_sparse(torch, *, candidates, dense_p, packed, q_ids, q_values, verify_lens, uniforms,
                  uniform_final, prefix_lens, outputs, scratch=None, denominator=None,
                  raw_fallback=False, row_offsets=None, vocab_size=None):
    (bs, t) = candidates.shape
    if dense_p is None:
        if packed is None or type(vocab_size) is not int or vocab_size < 1:
            raise ValueError("Pure packed rejection requires packed probabilities and vocab_size")
        if raw_fallback:
            raise ValueError("Pure packed rejection requires normalized packed probabilities")
        vocab = vocab_size
    else:
        vocab = dense_p.shape[-1]
        if vocab_size is not None and vocab_size != vocab:
            raise ValueError("vocab_size differs from the dense fallback")
    if row_offsets is not None:
        if (row_offsets.shape != (bs,) or row_offsets.device != candidates.device
                or row_offsets.dtype not in (torch.int32, torch.int64)
                or not row_offsets.is_contiguous()):
            raise ValueError("row_offsets must be a contiguous device int32/int64 vector of batch size")
        row_offsets = row_offsets.to(torch.int64)
    if raw_fallback and denominator is None:
        raise ValueError("Unnormalized target probabilities require a denominator")
    if t != 16 or q_ids.shape != (bs, 15, 16) or q_values.shape != (bs, 15, 16):
        raise ValueError("Expected candidates [B,16] and sparse q [B,15,16]")
    if len(outputs) != 5:
        raise ValueError("Expected accept/commit/bonus/output/new_seq buffers")
    if candidates.device.type != "cuda":
        raise ValueError("dspine_b200 runs the sparse rejection on CUDA tensors only")
    width = 0
    ids = vals = lens = ovf = None
    if packed is not None:
        (ids, vals, lens, ovf) = packed
        width = ids.shape[-1]
        if width > 64:
            raise ValueError("packed rows wider than 64 entries are not supported")
        ids, vals = ids.contiguous(), vals.contiguous()
        lens, ovf = lens.to(torch.int32).contiguous(), ovf.to(torch.int32).contiguous()
    dense = None if dense_p is None else dense_p.reshape(-1, vocab).contiguous()
    den = denominator.reshape(-1).float().contiguous() if raw_fallback else None
    ptr = _lib.ptr
    _lib.call("dsv_accept_sparse", bs, int(vocab), int(width), candidates.contiguous().data_ptr(),
              ptr(dense), ptr(ids), ptr(vals), ptr(lens), ptr(ovf), q_ids.contiguous().data_ptr(),
              q_values.contiguous().data_ptr(), verify_lens.contiguous().data_ptr(),
              uniforms.contiguous().data_ptr(), uniform_final.contiguous().data_ptr(),
              prefix_lens.contiguous().data_ptr(), ptr(row_offsets), ptr(den),
              *(o.data_ptr() for o in outputs), _stream(candidates))
    return outputs
