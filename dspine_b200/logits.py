"""Target probabilities from logits as a standalone step (C ABI: dsv_target_probs).

`target_probs` replaces runtime/worker.py:440-508 build_dspine_target_probs for bf16 logits:
temperature softmax with the joint top-k / top-p filter on the unfiltered p (the canonical
exact kept set), greedy rows one-hot at the lowest-index argmax.  Dense fp32 output.
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
    n = min(int(requests), 1024)
    key = (torch.device(device).index, n)
    ws = _workspaces.get(key)
    if ws is None:
        ws = Workspace(n, device)
        _workspaces[key] = ws
    return ws


def target_probs(logits, temperature, top_k, top_p, rows_per_request=1, out=None):
    """logits [rows, V] bf16 (rows contiguous), per-request temperature f32, top_k i32
    (>= V: off, <= 1 or T <= 0: greedy), top_p f32 for each group of rows_per_request (<= 16)
    consecutive rows.  Returns p [rows, V] fp32."""
    _check(logits.dim() == 2 and logits.dtype == torch.bfloat16 and logits.is_cuda,
           "logits must be a [rows, V] bf16 CUDA tensor")
    _check(logits.stride(1) == 1, "logit rows must be contiguous")
    rows, V = logits.shape
    rpr = int(rows_per_request)
    _check(1 <= rpr <= 16 and rows % rpr == 0, "rows must be a multiple of rows_per_request <= 16")
    R = rows // rpr
    dev = logits.device
    temperature = temperature.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    top_k = top_k.reshape(-1).to(device=dev, dtype=torch.int32).contiguous()
    top_p = top_p.reshape(-1).to(device=dev, dtype=torch.float32).contiguous()
    _check(temperature.numel() == R and top_k.numel() == R and top_p.numel() == R,
           "one temperature / top_k / top_p per request")
    if out is None:
        out = torch.empty((rows, V), device=dev, dtype=torch.float32)
    _check(out.shape == (rows, V) and out.dtype == torch.float32 and out.is_contiguous(),
           "out must be a contiguous fp32 [rows, V] tensor")
    ws = _workspace(R, dev)
    _lib.call("dsv_target_probs", rows, V, rpr, logits.data_ptr(), logits.stride(0),
              temperature.data_ptr(), top_k.data_ptr(), top_p.data_ptr(), out.data_ptr(),
              ws.buf.data_ptr(), ws.nbytes, torch.cuda.current_stream(dev).cuda_stream)
    return out
