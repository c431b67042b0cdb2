"""Small-support joint target P (sampling/sparse/target.py of the reference) on the GPU.

`build_sparse_target` keeps the reference's signature, its gating (None whenever the ordinary
dense path is required: another sampling backend, min-p, greedy rows, or no host-known top-k
bound in [1, capacity]) and its result type.  The whole build is one launch of
dsv_sparse_target over the logits as they are (bf16 or fp32, no cast): per row the k-th
largest p is the threshold and every tie of it stays, the mass of strictly larger p must stay
below top_p, and a row keeping more than `capacity` ids overflows to its dense row, renormalised
over p >= threshold (sampling/sparse/target.py:23-76, 156-178).  Rows map to requests through
``row_to_request``, through ``row_offsets`` (a device-side search, no host read) or, for full
blocks, through ``block_size``.  Dense rows of packed rows are left unwritten: accept_sparse
reads the dense row only where the overflow flag is set.
"""

from dataclasses import dataclass

import torch

from ... import _lib

_DTYPES = {torch.bfloat16: 0, torch.float32: 1}
MAX_CAPACITY = 64


@dataclass
class SparseTarget:
    packed: tuple
    dense_p: torch.Tensor
    denominator: torch.Tensor | None = None


def _fast_path_applies(info, capacity, sampling_backend):
    """The reference's conditions for the small-support path (sparse/target.py:106-111)."""
    max_k = getattr(info, "max_top_k", None)
    return (sampling_backend == "flashinfer"
            and not getattr(info, "need_min_p_sampling", False)
            and not getattr(info, "is_any_greedy", False)
            and isinstance(max_k, int) and 1 <= max_k <= capacity)


def _row_mapping(rows, info, row_to_request, row_offsets, block_size, device):
    """(row_request int64 [rows] or None, rows_per_request) for the kernel."""
    if row_to_request is not None:
        if row_to_request.numel() != rows:
            raise ValueError("row_to_request must cover every target row")
        return row_to_request.reshape(-1).to(device=device, dtype=torch.int64).contiguous(), 1
    if row_offsets is not None:
        # request b owns rows [row_offsets[b], row_offsets[b+1]): the number of request ends
        # at or before a row is its request
        ends = row_offsets[1:].to(device=device, dtype=torch.int64).contiguous()
        positions = torch.arange(rows, device=device, dtype=torch.int64)
        return torch.searchsorted(ends, positions, right=True), 1
    if rows != info.temperatures.numel() * block_size:
        raise ValueError("Compact target logits require row mapping")
    return None, int(block_size)


def build_sparse_target(logits, info, *, row_to_request=None, row_offsets=None, verify_lens=None,
                        block_size=16, capacity=32, sampling_backend="flashinfer"):
    """Return SparseTarget or None when the ordinary dense path is required.

    packed = (ids int32 [rows, capacity], values f32, lengths int32, overflow int32) in compact
    target-row indexing; dense_p [rows, V] f32 holds the renormalised filtered p of overflow
    rows only.  No host read of CUDA tensors.  verify_lens is accepted for the shared caller
    contract; the row mapping alone determines each row's request."""
    if not _fast_path_applies(info, capacity, sampling_backend):
        return None
    if logits.ndim != 2 or capacity < 1:
        raise ValueError("Expected [rows,vocab] logits and positive capacity")
    rows, vocab = logits.shape
    if vocab < 1 or info.max_top_k > vocab:
        return None
    if capacity > MAX_CAPACITY:
        raise ValueError(f"dspine_b200 packs at most {MAX_CAPACITY} ids per row")
    dev = logits.device
    ids = torch.empty((rows, capacity), device=dev, dtype=torch.int32)
    values = torch.empty((rows, capacity), device=dev, dtype=torch.float32)
    lengths = torch.empty(rows, device=dev, dtype=torch.int32)
    overflow = torch.empty(rows, device=dev, dtype=torch.int32)
    dense = torch.empty((rows, vocab), device=dev, dtype=torch.float32)
    request, per_request = _row_mapping(rows, info, row_to_request, row_offsets, block_size, dev)
    if rows == 0:
        return SparseTarget((ids, values, lengths, overflow), dense)
    if dev.type != "cuda":
        raise ValueError("dspine_b200 builds the sparse target on CUDA tensors only")
    if logits.dtype not in _DTYPES:
        raise ValueError(f"logits must be bf16 or fp32, got {logits.dtype}")
    if logits.stride(1) != 1:
        logits = logits.contiguous()
    temperature = info.temperatures.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    top_k = info.top_ks.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
    top_p = info.top_ps.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    with torch.cuda.device(dev):
        _lib.call("dsv_sparse_target", rows, vocab, _DTYPES[logits.dtype], logits.data_ptr(),
                  logits.stride(0), _lib.ptr(request), per_request, temperature.data_ptr(),
                  top_k.data_ptr(), top_p.data_ptr(), capacity, ids.data_ptr(),
                  values.data_ptr(), lengths.data_ptr(), overflow.data_ptr(), dense.data_ptr(),
                  torch.cuda.current_stream(dev).cuda_stream)
    return SparseTarget((ids, values, lengths, overflow), dense)
