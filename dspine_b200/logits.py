"""Target probabilities from logits as a standalone step (C ABI: dsv_target_probs).

`target_probs` replaces runtime/worker.py:440-508 build_dspine_target_probs for bf16 and fp32
logits: temperature softmax with the filter of the batch's mode (joint top-k / top-p on the
unfiltered p; the sequential flashinfer filter with min-p; the pytorch backend's filter with
min-p), the canonical exact kept set, greedy rows one-hot at the lowest-index argmax.  Dense
fp32 output.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .verify import Workspace


def _check(cond, msg):
    if not cond:
        raise ValueError(msg)


_workspaces: dict = {}


def _workspace(requests: int, device) -> Workspace:
    """One workspace per device, grown to the largest launch (at most 1024 requests), zeroed
    again whenever the launch's layout size changes."""
    n = max(1, min(int(requests), 1024))
    index = torch.device(device).index
    ws = _workspaces.get(index)
    if ws is None or ws.batch < n:
        ws = Workspace(n, device)
        _workspaces[index] = ws
    ws.prepare(n)
    return ws


def target_probs(logits, temperature, top_k, top_p, rows_per_request=1, out=None, *,
                 min_p=None, mode=0):
    """logits [rows, V] bf16 or fp32 (rows contiguous), per-request temperature f32, top_k i32
    (>= V: off, <= 1 or T <= 0: greedy), top_p f32 (and min_p f32 with a filter mode: 0 joint,
    1 sequential, 2 pytorch backend) for each group of rows_per_request consecutive rows.
    Returns p [rows, V] fp32."""
    _check(logits.dim() == 2 and logits.dtype in (torch.bfloat16, torch.float32) and logits.is_cuda,
           "logits must be a [rows, V] bf16 or fp32 CUDA tensor")
    _check(logits.stride(1) == 1, "logit rows must be contiguous")
    rows, V = logits.shape
    rpr = int(rows_per_request)
    _check(rpr >= 1 and rows % rpr == 0, "rows must be a multiple of rows_per_request")
    R = rows // rpr
    dev = logits.device
    temperature = temperature.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    top_k = top_k.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
    top_p = top_p.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    _check(temperature.numel() == R and top_k.numel() == R and top_p.numel() == R,
           "one temperature / top_k / top_p per request")
    if min_p is not None:
        min_p = min_p.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
        _check(min_p.numel() == R, "one min_p per request")
    _check(mode in (0, 1, 2), "unknown filter mode")
    if out is None:
        out = torch.empty((rows, V), device=dev, dtype=torch.float32)
    _check(out.shape == (rows, V) and out.dtype == torch.float32 and out.is_contiguous(),
           "out must be a contiguous fp32 [rows, V] tensor")
    if rows == 0:
        return out
    ws = _workspace(R, dev)
    dtype = 0 if logits.dtype == torch.bfloat16 else 1
    with torch.cuda.device(dev):
        _lib.call("dsv_target_probs_ex", rows, V, dtype, rpr, logits.data_ptr(), logits.stride(0),
                  temperature.data_ptr(), top_k.data_ptr(), top_p.data_ptr(), _lib.ptr(min_p),
                  int(mode), out.data_ptr(), ws.buf.data_ptr(), ws.nbytes,
                  torch.cuda.current_stream(dev).cuda_stream)
    return out
