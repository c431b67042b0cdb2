"""BF16 rescore of gathered head rows and the top-16 selection (layers/fp8/gather.py:53-79).

`rescore` and `select16` keep the reference's signatures; each is one launch of
dsv_rescore_select16 (the selection alone when no weight is given).  `rescore_select16` is
the fused form retrieve_and_rescore uses: the scores and the 16 tokens in one launch.
"""

from __future__ import annotations

from ... import _lib


def _hidden_code(torch, dtype):
    if dtype == torch.bfloat16:
        return 0
    if dtype == torch.float32:
        return 1
    raise ValueError(f"rescore supports bf16 and fp32 hidden rows, got {dtype}")


def _stream(torch, t) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _check_ids(torch, ids, m):
    if ids.dim() != 2 or ids.dtype != torch.int64 or not ids.is_contiguous() or ids.shape[0] != m:
        raise ValueError("rescore expects contiguous int64 ids [M, C]")
    if not 1 <= ids.shape[1] <= 128:
        raise ValueError(f"rescore supports 1..128 candidates per row, got {ids.shape[1]}")


def rescore_select16(torch, weight, ids, hidden, *, fp32_output=False, with_top16=True):
    """(scores [M, C] in the hidden dtype (fp32 with fp32_output), top16 int64 [M, 16] or None)."""
    m, c = ids.shape
    h = hidden.shape[1]
    _check_ids(torch, ids, hidden.shape[0])
    if weight.dtype != torch.bfloat16 or weight.dim() != 2 or weight.stride(1) != 1 or weight.shape[1] != h:
        raise ValueError("rescore expects a row-contiguous bf16 weight [V, H]")
    if hidden.dim() != 2 or hidden.stride(1) != 1:
        raise ValueError("rescore expects row-contiguous hidden rows [M, H]")
    if with_top16 and c < 16:
        raise ValueError("select16 needs at least 16 candidates per row")
    out_dtype = torch.float32 if fp32_output else hidden.dtype
    scores = torch.empty((m, c), device=hidden.device, dtype=out_dtype)
    top16 = torch.empty((m, 16), device=hidden.device, dtype=torch.int64) if with_top16 else None
    if m:
        _lib.call("dsv_rescore_select16", m, c, h, weight.shape[0], weight.data_ptr(), weight.stride(0),
                  ids.data_ptr(), hidden.data_ptr(), hidden.stride(0),
                  _hidden_code(torch, hidden.dtype), scores.data_ptr(), int(out_dtype == torch.float32),
                  None if top16 is None else top16.data_ptr(), _stream(torch, hidden))
    return scores, top16


def rescore(torch, weight, ids, hidden, *, fp32_output=False):
    """scores[m, c] = W[ids[m, c]] . hidden[m] in fp32, stored in the hidden dtype
    (gather.py:53-70)."""
    return rescore_select16(torch, weight, ids, hidden, fp32_output=fp32_output, with_top16=False)[0]


def select16(torch, scores, ids):
    """int64 [M, 16]: 16 rounds of (largest score, lowest token among equals), ascending
    (gather.py:37-50, 73-79)."""
    m, c = ids.shape
    _check_ids(torch, ids, scores.shape[0])
    if tuple(scores.shape) != (m, c) or not scores.is_contiguous():
        raise ValueError("select16 expects contiguous scores shaped like ids")
    if scores.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"select16 supports bf16 and fp32 scores, got {scores.dtype}")
    if c < 16:
        raise ValueError("select16 needs at least 16 candidates per row")
    out = torch.empty((m, 16), device=ids.device, dtype=torch.int64)
    if m:
        _lib.call("dsv_rescore_select16", m, c, 0, 1, None, 0, ids.data_ptr(), None, 0, 0,
                  scores.data_ptr(), int(scores.dtype == torch.float32), out.data_ptr(),
                  _stream(torch, scores))
    return out
