"""Small-support joint target P (sampling/sparse/target.py of the reference) on the GPU.

`build_sparse_target` keeps the reference's signature and gating (None when min-p, greedy
rows or an unbounded top-k require the dense path) and returns a `SparseTarget` whose packed
rows are the canonical exact kept sets (ids ascending, values normalised by the kept mass)
and whose dense rows hold the filtered p (dsv_target_probs + dsv_compress_probs).
"""

from dataclasses import dataclass

import torch

from ...logits import target_probs
from .accept import compress_probs


@dataclass
class SparseTarget:
    packed: tuple
    dense_p: torch.Tensor
    denominator: torch.Tensor | None = None


def _row_indices(logits, info, row_to_request, row_offsets, block_size):
    rows = logits.shape[0]
    if row_to_request is not None:
        if row_to_request.numel() != rows:
            raise ValueError("row_to_request must cover every target row")
        return row_to_request.reshape(-1).to(device=logits.device, dtype=torch.long)
    index = torch.arange(rows, device=logits.device, dtype=torch.long)
    if row_offsets is not None:
        return torch.bucketize(index, row_offsets[1:].contiguous(), right=True)
    bs = info.temperatures.numel()
    if rows != bs * block_size:
        raise ValueError("Compact target logits require row mapping")
    return index // block_size


def build_sparse_target(logits, info, *, row_to_request=None, row_offsets=None, verify_lens=None,
                        block_size=16, capacity=32, sampling_backend="flashinfer"):
    """Return SparseTarget or None when the ordinary dense path is required."""
    max_k = getattr(info, "max_top_k", None)
    if (sampling_backend != "flashinfer" or getattr(info, "need_min_p_sampling", False)
            or getattr(info, "is_any_greedy", False)
            or not isinstance(max_k, int) or not 1 <= max_k <= capacity):
        return None
    if logits.ndim != 2 or capacity < 1:
        raise ValueError("Expected [rows,vocab] logits and positive capacity")
    rows, vocab = logits.shape
    if vocab < 1 or max_k > vocab:
        return None
    request = _row_indices(logits, info, row_to_request, row_offsets, block_size)
    if rows == 0:
        return SparseTarget((torch.empty((0, capacity), device=logits.device, dtype=torch.int32),
                             torch.empty((0, capacity), device=logits.device, dtype=torch.float32),
                             torch.empty(0, device=logits.device, dtype=torch.int32),
                             torch.empty(0, device=logits.device, dtype=torch.int32)),
                            torch.empty((0, vocab), device=logits.device, dtype=torch.float32))
    temperatures = info.temperatures.reshape(-1)[request].float()
    top_ks = info.top_ks.reshape(-1)[request].to(torch.int32)
    top_ps = info.top_ps.reshape(-1)[request].to(torch.float32)
    p = target_probs(logits.to(torch.bfloat16), temperatures, top_ks, top_ps, rows_per_request=1)
    return SparseTarget(compress_probs(torch, p, capacity), p)
