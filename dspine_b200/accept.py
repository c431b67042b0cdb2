"""Host API of the per-request accept steps (C ABI: dsv_accept_greedy, dsv_accept_compact).

`accept_greedy` is verification/caps.py:32-59 `_accept_capped` on the GPU: the five accept
outputs of a greedy (argmax) verification from the target's top-1 ids.  `accept_compact`
packs accepted tokens and KV slots after any accept step (SGLang's `_commit_accept`, wrapped
at runtime/worker.py:745-777).  Argument errors raise ValueError before launch.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib
from .verify import CompactOutputs, Workspace, new_outputs, workspace_for  # noqa: F401

T = 16


def _check(cond, msg):
    if not cond:
        raise ValueError(msg)


def _stream(device) -> int:
    return torch.cuda.current_stream(torch.device(device)).cuda_stream


def accept_greedy(candidates, top1, verify_lens, prefix_lens=None, *, outputs=None):
    """candidates [B,16] int64; top1 [B,16] int64 (any stride along the last dim, e.g. column 0
    of a [B*16, k] top-k id array viewed as [B,16]); verify_lens [B] int32; prefix_lens [B]
    int32 (zeros when None).  Returns (accept, commit, bonus, output, new_seq)."""
    _check(candidates.dim() == 2 and candidates.shape[1] == T and candidates.dtype == torch.int64
           and candidates.is_contiguous(), "candidates must be contiguous int64 [B,16]")
    B = candidates.shape[0]
    dev = candidates.device
    _check(top1.shape == (B, T) and top1.dtype == torch.int64 and top1.device == dev,
           "top1 must be int64 [B,16]")
    s = top1.stride(1)
    _check(s >= 1 and top1.stride(0) == T * s, "top1 must be a uniformly strided [B,16] view")
    _check(verify_lens.shape == (B,) and verify_lens.dtype == torch.int32, "verify_lens int32 [B]")
    if prefix_lens is None:
        prefix_lens = torch.zeros(B, dtype=torch.int32, device=dev)
    _check(prefix_lens.shape == (B,) and prefix_lens.dtype == torch.int32, "prefix_lens int32 [B]")
    if outputs is None:
        outputs = new_outputs(B, dev)
    _lib.call("dsv_accept_greedy", B, candidates.data_ptr(), top1.data_ptr(), s,
              verify_lens.contiguous().data_ptr(), prefix_lens.contiguous().data_ptr(),
              *(o.data_ptr() for o in outputs), _stream(dev))
    return outputs


def accept_compact(commit, verify_lens, output, slots, slot_rows, *, compact=None,
                   workspace: Workspace | None = None):
    """Pack output[b, :commit_b] and the KV slots of positions [0, commit_b) of every request
    (and the freed slots of positions [commit_b, verify_len_b)) by the exclusive scan of commit."""
    B = commit.shape[0]
    dev = commit.device
    _check(commit.dtype == torch.int32 and verify_lens.dtype == torch.int32, "int32 commit/lens")
    _check(output.shape == (B, T) and output.dtype == torch.int64, "output int64 [B,16]")
    _check(slots.dtype == torch.int32 and slot_rows.dtype == torch.int64 and slot_rows.shape == (B,),
           "slots int32, slot_rows int64 [B]")
    if compact is None:
        compact = CompactOutputs.allocate(B, dev)
    if workspace is None:
        workspace = workspace_for(B, dev)
    c = _lib.CompactOut(slots.data_ptr(), slots.numel(), slot_rows.data_ptr(),
                        compact.tokens.data_ptr(), compact.kept_slots.data_ptr(),
                        compact.offsets.data_ptr(), compact.freed_slots.data_ptr(),
                        compact.freed_offsets.data_ptr())
    _lib.call("dsv_accept_compact", B, commit.data_ptr(), verify_lens.data_ptr(),
              output.contiguous().data_ptr(), ctypes.byref(c), workspace.buf.data_ptr(),
              _stream(dev))
    return compact
