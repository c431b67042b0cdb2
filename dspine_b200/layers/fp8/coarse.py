"""Row-scaled FP8 retrieval; final scores use the original BF16 head (layers/fp8/coarse.py).

`FullVFP8Coarse(torch, original_weight, tp_head=None)` keeps the reference's constructor and
`retrieve_and_rescore(hidden, *, fi_top_k, gather_ops)` its return value
(top16 ids, coarse ids [M, 128] in rank order, rescored [M, 128]).  Per step:

  1. dsv_fp8_quantize_rows   the hidden rows to e4m3 with per-row scales (_scale, _quantize)
  2. dsv_fp8_coarse_scores   the row-scaled FP8 GEMM on the tensor cores, bf16 scores
                             (torch._scaled_mm in the reference)
  3. dsv_topk_ranked         the 128 best coarse scores of each row, (value desc, id asc)
  4. dsv_rescore_select16    the BF16 head rows of those 128 dotted with the hidden row, and
                             the 16 selection rounds (gather.rescore + gather.select16)

`fi_top_k` and `gather_ops` are accepted for signature compatibility and not used: the
library's kernels are the selection and the rescore.  `stable_local_topk` is the portable
tie rule of the reference (lower index first) on the library's ranked top-k.
"""

from __future__ import annotations

from ... import _lib
from . import gather as _gather


def supports_filtered_topk(device):
    """The reference asks FlashInfer; here the ranked top-k kernel serves every device."""
    return False


def _stream(torch, t) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def _topk_dtype(torch, dtype):
    codes = {torch.bfloat16: 0, torch.float32: 1, torch.float16: 2}
    if dtype not in codes:
        raise ValueError(f"stable_local_topk supports bf16, fp16 and fp32 scores, got {dtype}")
    return codes[dtype]


def _ranked_ids(torch, scores, k):
    n, v = scores.shape
    if scores.stride(1) != 1:
        raise ValueError("stable_local_topk expects row-contiguous scores")
    if not 1 <= k <= min(128, v):
        raise ValueError(f"stable_local_topk supports 1 <= k <= min(128, columns), got k={k}")
    ids = torch.empty((n, k), dtype=torch.int64, device=scores.device)
    if n:
        _lib.call("dsv_topk_ranked", n, v, scores.stride(0) if n > 1 else v,
                  _topk_dtype(torch, scores.dtype), scores.data_ptr(), k, ids.data_ptr(),
                  _stream(torch, scores))
    return ids


def stable_local_topk(scores, k, fi_top_k=None):
    """(values, ids) of the k best scores per row, ties to the lower index, in rank order
    (coarse.py:19-35)."""
    import torch

    ids = _ranked_ids(torch, scores, int(k))
    return scores.gather(-1, ids), ids


def _quantize_rows(torch, x, q=None, scale=None):
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("FP8 quantization expects row-contiguous [rows, cols]")
    if x.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError(f"FP8 quantization supports bf16 and fp32 rows, got {x.dtype}")
    n, h = x.shape
    if q is None:
        q = torch.empty((n, h), dtype=torch.uint8, device=x.device)
    if scale is None:
        scale = torch.empty(n, dtype=torch.float32, device=x.device)
    if n:
        _lib.call("dsv_fp8_quantize_rows", n, h, x.stride(0) if n > 1 else h,
                  int(x.dtype == torch.float32), x.data_ptr(), q.data_ptr(), q.stride(0),
                  scale.data_ptr(), _stream(torch, x))
    return q, scale


def quantize_rows(x):
    """(e4m3 codes uint8 [rows, cols], fp32 scales [rows]) of _scale + _quantize."""
    import torch

    return _quantize_rows(torch, x)


def coarse_scores(xq, x_scale, wq, w_scale, err=None):
    """bf16 [M, V] = (xq . wq^T) * x_scale[:, None] * w_scale[None, :] (fp32 accumulation)."""
    import torch

    m, h = xq.shape
    v = wq.shape[0]
    if wq.shape[1] != h or h % 128:
        raise ValueError(f"coarse_scores needs hidden a multiple of 128, got {h}")
    out = torch.empty((m, v), dtype=torch.bfloat16, device=xq.device)
    own_err = err is None
    if own_err:
        err = torch.zeros(1, dtype=torch.int32, device=xq.device)
    if m:
        _lib.call("dsv_fp8_coarse_scores", m, v, h, xq.data_ptr(), xq.stride(0), x_scale.data_ptr(),
                  wq.data_ptr(), wq.stride(0), w_scale.data_ptr(), out.data_ptr(), out.stride(0),
                  err.data_ptr(), _stream(torch, xq))
    return out


class FullVFP8Coarse:
    def __init__(self, torch, original_weight, tp_head=None):
        if original_weight.dtype != torch.bfloat16 or original_weight.dim() != 2:
            raise ValueError("FullVFP8Coarse expects a bf16 head [V, H]")
        if original_weight.shape[1] % 128:
            raise ValueError("FullVFP8Coarse needs a hidden size that is a multiple of 128")
        self.torch = torch
        self.original_weight = original_weight.contiguous()
        self.tp_head = tp_head
        q, scale = _quantize_rows(torch, self.original_weight)
        self.weight8 = q.view(torch.float8_e4m3fn)
        self.weight_scale = scale.reshape(1, -1).contiguous()
        self.weight8_t = self.weight8.T
        self._err = torch.zeros(1, dtype=torch.int32, device=original_weight.device)

    def error_word(self) -> int:
        """Device error bits of the coarse GEMM since construction (bit 0: a wait timed out)."""
        return int(self._err.item())

    def retrieve_and_rescore(self, hidden, *, fi_top_k=None, gather_ops=None):
        torch = self.torch
        if hidden.dim() != 2 or hidden.shape[1] != self.original_weight.shape[1]:
            raise ValueError("retrieve_and_rescore expects hidden rows [M, H] of the head's width")
        hidden = hidden.contiguous()
        xq, sx = _quantize_rows(torch, hidden)
        wq = self.weight8.view(torch.uint8)
        coarse = coarse_scores(xq, sx, wq, self.weight_scale.reshape(-1), err=self._err)
        if self.tp_head is None:
            ids = _ranked_ids(torch, coarse, 128)
            scores, top16 = _gather.rescore_select16(torch, self.original_weight, ids, hidden)
            return top16, ids, scores
        head = self.tp_head
        coarse[:, head.num_local:].fill_(float("-inf"))
        width = min(128, coarse.shape[1])
        values, ids = stable_local_topk(coarse, width)
        ids = ids + head.start
        values = values.masked_fill(ids >= head.end, float("-inf"))
        ids = ids.masked_fill(ids >= head.end, head.global_vocab_size)
        if width < 128:
            values = torch.nn.functional.pad(values, (0, 128 - width), value=float("-inf"))
            ids = torch.nn.functional.pad(ids, (0, 128 - width), value=head.global_vocab_size)
        _, ids = head.global_topk(values, ids, 128)
        scores = head.rescore(ids, hidden)
        return _gather.select16(torch, scores, ids), ids, scores
