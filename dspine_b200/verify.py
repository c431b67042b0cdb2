"""Host API of the fused verification kernel (C ABI: dsv_verify_logits).

``verify_logits`` is the one call that replaces the reference's two-step verify
(runtime/worker.py:440-508 build_dspine_target_probs, then sampling/rejection.py:12-153
sample_capped_chain_from_probs): it reads target (and draft) logits once and writes the same
five outputs (accept, commit, bonus, output, new_seq).  Argument checks raise ValueError before
anything is launched, like the reference's launchers (sampling/rejection.py:113-138).
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib

T = 16
_DTYPES = {torch.bfloat16: 0, torch.float32: 1}


class Workspace:
    """Device scratch of dsv_verify_logits (task counters and per-row decisions).

    Zeroed once at allocation; every launch leaves it zeroed.  Launches that may overlap on
    the GPU (different streams) need different workspaces."""

    def __init__(self, batch: int, device):
        size = ctypes.c_size_t()
        _lib.call("dsv_verify_workspace_size", int(batch), ctypes.byref(size))
        self.batch = int(batch)
        self.nbytes = int(size.value)
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        self.layout_batch = None  # the batch size whose layout the zeroed state follows
        self.zero()

    def zero(self):
        """Zero the whole workspace on the current stream (dsv_workspace_init)."""
        _lib.call("dsv_workspace_init", self.buf.data_ptr(), self.nbytes, _stream(self.buf.device))

    def prepare(self, batch: int):
        """A launch leaves the counters of its own batch's layout zeroed; another batch size
        lays them out elsewhere, so the workspace is zeroed again when the size changes."""
        if self.layout_batch is not None and self.layout_batch != int(batch):
            self.zero()
        self.layout_batch = int(batch)

    # error bits after which the counters and flags of the workspace may not be zero: a bulk
    # copy that timed out (bit 0), a layout check (5), a chain task or a split half that gave up
    # waiting (6, 7); the workspace is zeroed again before it is reused
    RESET_BITS = 0x1 | 0x20 | 0x40 | 0x80

    def bytes_read(self) -> int:
        """Logit bytes the streaming row kernel has read from memory through this workspace,
        summed over its launches since the workspace was last zeroed.  Verification drops rows
        that cannot change an outcome, so this is what was read, not every row of the batch.
        Synchronizes the current stream."""
        n = ctypes.c_uint64()
        _lib.call("dsv_workspace_bytes_read", self.buf.data_ptr(), ctypes.byref(n),
                  _stream(self.buf.device))
        return int(n.value)

    def error_word(self) -> int:
        """Device error bits (synchronizes the current stream); cleared after reading.  After an
        internal failure (RESET_BITS) the whole workspace is zeroed again."""
        err = ctypes.c_uint32()
        _lib.call("dsv_workspace_error", self.buf.data_ptr(), ctypes.byref(err),
                  _stream(self.buf.device))
        if err.value & self.RESET_BITS:
            self.zero()
        return int(err.value)


_workspaces: dict = {}


def workspace_for(batch: int, device) -> Workspace:
    """The device's workspace, grown to the largest batch asked for (a workspace sized for a
    larger batch serves any smaller one); one per device."""
    device = torch.device(device)
    if device.index is None:
        device = torch.device(device.type, torch.cuda.current_device())
    ws = _workspaces.get(device.index)
    if ws is None or ws.batch < int(batch):
        ws = Workspace(max(int(batch), 1), device)
        _workspaces[device.index] = ws
    return ws


def _stream(device) -> int:
    return torch.cuda.current_stream(torch.device(device)).cuda_stream


@dataclass
class CompactOutputs:
    """Packed accepted tokens / kept and freed KV slots (see dsv_compact_out)."""

    tokens: torch.Tensor
    kept_slots: torch.Tensor
    offsets: torch.Tensor
    freed_slots: torch.Tensor
    freed_offsets: torch.Tensor

    @staticmethod
    def allocate(batch: int, device) -> "CompactOutputs":
        n = batch * T
        return CompactOutputs(
            torch.empty(n, dtype=torch.int64, device=device),
            torch.empty(n, dtype=torch.int32, device=device),
            torch.empty(batch + 1, dtype=torch.int32, device=device),
            torch.empty(n, dtype=torch.int32, device=device),
            torch.empty(batch + 1, dtype=torch.int32, device=device),
        )


def new_outputs(batch: int, device):
    return (torch.empty(batch, dtype=torch.int32, device=device),
            torch.empty(batch, dtype=torch.int32, device=device),
            torch.empty(batch, dtype=torch.int64, device=device),
            torch.empty((batch, T), dtype=torch.int64, device=device),
            torch.empty(batch, dtype=torch.int32, device=device))


def _check(cond, msg):
    if not cond:
        raise ValueError(msg)


JOINT, SEQUENTIAL, TORCH = 0, 1, 2   # filter modes (dsv_filter_mode)


def filter_mode(sampling_backend: str = "flashinfer", need_min_p: bool = False) -> int:
    """The filter mode of a batch (runtime/worker.py:473-508): the pytorch backend's joint
    filter plus min-p, or the flashinfer backend, sequential when the batch has min-p."""
    if sampling_backend == "pytorch":
        return TORCH
    if sampling_backend == "flashinfer":
        return SEQUENTIAL if need_min_p else JOINT
    raise ValueError(f"DSPINE sampled verify: unsupported sampling backend {sampling_backend!r}")


def _prepare(candidates, target_logits, target_rows, temperature, top_k, top_p, verify_lens,
             uniforms, uniform_final, prefix_lens, draft_logits, draft_rows, outputs, slots,
             slot_rows, compact):
    """Validate the arguments of verify_logits (ValueError before launch, as
    sampling/rejection.py:113-138) and marshal the C-ABI arguments shared by
    dsv_verify_logits and dsv_verify_logits_noalloc (everything before the scratch)."""
    _check(candidates.dim() == 2 and candidates.shape[1] == T, "candidates must be [B,16]")
    B = candidates.shape[0]
    dev = candidates.device
    _check(dev.type == "cuda", "verify_logits runs on CUDA tensors")
    _check(target_logits.dim() == 2 and target_logits.dtype in _DTYPES,
           "target_logits must be [rows, V] bf16 or fp32")
    _check(target_logits.stride(1) == 1, "target_logits rows must be contiguous")
    V = target_logits.shape[1]
    stride = target_logits.stride(0)
    if draft_logits is not None:
        _check(draft_logits.dtype == target_logits.dtype, "draft and target dtypes differ")
        _check(draft_logits.dim() == 2 and draft_logits.shape[1] == V, "draft vocab differs")
        _check(draft_logits.stride(1) == 1 and draft_logits.stride(0) == stride,
               "draft rows must use the target row stride")
        _check(draft_rows is not None and draft_rows.shape == (B,), "draft_rows must be [B]")
    expect = {
        "candidates": (candidates, torch.int64, (B, T)),
        "target_rows": (target_rows, torch.int64, (B,)),
        "temperature": (temperature, torch.float32, (B,)),
        "top_k": (top_k, torch.int32, (B,)),
        "top_p": (top_p, torch.float32, (B,)),
        "verify_lens": (verify_lens, torch.int32, (B,)),
        "uniforms": (uniforms, torch.float32, (B, T - 1)),
        "uniform_final": (uniform_final, torch.float32, (B,)),
        "prefix_lens": (prefix_lens, torch.int32, (B,)),
    }
    if draft_rows is not None:
        expect["draft_rows"] = (draft_rows, torch.int64, (B,))
    for name, (t, dt, shape) in expect.items():
        _check(t.dtype == dt, f"{name} must be {dt}")
        _check(tuple(t.shape) == shape, f"{name} must have shape {shape}")
        _check(t.is_contiguous(), f"{name} must be contiguous")
        _check(t.device == dev, "all tensors must be on one device")
    _check(target_logits.device == dev, "all tensors must be on one device")
    if outputs is None:
        outputs = new_outputs(B, dev)
    _check(len(outputs) == 5, "Expected accept/commit/bonus/output/new_seq buffers")
    for t, (dt, shape) in zip(outputs, ((torch.int32, (B,)), (torch.int32, (B,)),
                                        (torch.int64, (B,)), (torch.int64, (B, T)),
                                        (torch.int32, (B,)))):
        _check(t.dtype == dt and tuple(t.shape) == shape and t.is_contiguous() and t.device == dev,
               "output buffers must be contiguous accept i32[B], commit i32[B], bonus i64[B], "
               "output i64[B,16], new_seq i32[B]")
    cstruct = None
    if compact is not None:
        _check(slots is not None and slot_rows is not None, "compaction needs slots and slot_rows")
        _check(slots.dtype == torch.int32 and slot_rows.dtype == torch.int64, "slot dtypes")
        _check(slot_rows.shape == (B,), "slot_rows must be [B]")
        cstruct = _lib.CompactOut(slots.data_ptr(), slots.numel(), slot_rows.data_ptr(), compact.tokens.data_ptr(),
                                  compact.kept_slots.data_ptr(), compact.offsets.data_ptr(),
                                  compact.freed_slots.data_ptr(), compact.freed_offsets.data_ptr())
    drows_n = draft_logits.shape[0] if draft_logits is not None else 0
    args = (B, V, _DTYPES[target_logits.dtype], candidates.data_ptr(),
            target_logits.data_ptr(), target_rows.data_ptr(), target_logits.shape[0],
            _lib.ptr(draft_logits), _lib.ptr(draft_rows), drows_n, stride,
            temperature.data_ptr(), top_k.data_ptr(), top_p.data_ptr(), verify_lens.data_ptr(),
            uniforms.data_ptr(), uniform_final.data_ptr(), prefix_lens.data_ptr(),
            *(o.data_ptr() for o in outputs),
            ctypes.byref(cstruct) if cstruct is not None else None)
    return B, dev, outputs, args, cstruct


def verify_logits(*, candidates, target_logits, target_rows, temperature, top_k, top_p,
                  verify_lens, uniforms, uniform_final, prefix_lens, draft_logits=None,
                  draft_rows=None, outputs=None, slots=None, slot_rows=None, compact=None,
                  workspace: Workspace | None = None, min_p=None, mode: int = JOINT):
    """Verify a ragged batch of 16-token draft blocks directly from logits.

    candidates [B,16] int64 (anchor + 15 drafts); target_logits [R,V] bf16/fp32 rows;
    target_rows [B] int64: request b's verify position s uses target row target_rows[b]+s;
    draft_logits [R',V] (same dtype) with draft_rows [B], or None for one-hot q;
    temperature [B] f32, top_k [B] i32 (>= V: off, <= 1: greedy), top_p [B] f32;
    verify_lens [B] i32 in [1,16]; uniforms [B,15] f32; uniform_final [B] f32;
    prefix_lens [B] i32.  Optional ``slots`` [*] i32 with ``slot_rows`` [B] i64 and a
    ``compact`` CompactOutputs receive the packed accepted tokens and KV slots.  ``min_p``
    [B] f32 with ``mode`` (JOINT, SEQUENTIAL or TORCH, see `filter_mode`) selects the other
    filter branches of runtime/worker.py:473-508.
    Returns (accept, commit, bonus, output, new_seq)."""
    B, dev, outputs, args, _keep = _prepare(
        candidates, target_logits, target_rows, temperature, top_k, top_p, verify_lens,
        uniforms, uniform_final, prefix_lens, draft_logits, draft_rows, outputs, slots,
        slot_rows, compact)
    if workspace is None:
        workspace = workspace_for(B, dev)
    _check(workspace.batch >= B, "workspace is too small for this batch")
    _check(mode in (JOINT, SEQUENTIAL, TORCH), "unknown filter mode")
    workspace.prepare(B)
    if min_p is not None:
        _check(min_p.dtype == torch.float32 and tuple(min_p.shape) == (B,) and
               min_p.is_contiguous() and min_p.device == dev, "min_p must be a contiguous f32 [B]")
    # dsv_verify_logits_ex takes min_p and the mode after top_p (the 14th argument)
    ex_args = args[:14] + (_lib.ptr(min_p), int(mode)) + args[14:]
    with torch.cuda.device(dev):
        _lib.call("dsv_verify_logits_ex", *ex_args, workspace.buf.data_ptr(), workspace.nbytes,
                  _stream(dev))
    return outputs


NOALLOC_MAX_BATCH = 256


def verify_logits_noalloc(*, candidates, target_logits, target_rows, temperature, top_k, top_p,
                          verify_lens, uniforms, uniform_final, prefix_lens, draft_logits=None,
                          draft_rows=None, outputs, slots=None, slot_rows=None, compact=None,
                          device_error=None):
    """verify_logits for callers that cannot allocate at verification time
    (C ABI: dsv_verify_logits_noalloc).  No workspace: the library's fixed device scratch
    serves up to NOALLOC_MAX_BATCH requests; ``outputs`` (and ``compact``) must be given.
    ``device_error`` (optional int32 [1] CUDA tensor) receives the call's device error word.
    Calls that may overlap on one device (other streams or threads) must be serialised."""
    _check(outputs is not None, "verify_logits_noalloc needs caller-owned outputs")
    B, dev, outputs, args, _keep = _prepare(
        candidates, target_logits, target_rows, temperature, top_k, top_p, verify_lens,
        uniforms, uniform_final, prefix_lens, draft_logits, draft_rows, outputs, slots,
        slot_rows, compact)
    _check(B <= NOALLOC_MAX_BATCH, f"verify_logits_noalloc serves at most {NOALLOC_MAX_BATCH} requests")
    if device_error is not None:
        _check(device_error.device == dev and device_error.numel() >= 1 and
               device_error.element_size() == 4, "device_error must be a 4-byte CUDA tensor")
    # the scratch address is looked up for the current device: make it the tensors' device
    with torch.cuda.device(dev):
        _lib.call("dsv_verify_logits_noalloc", *args, _lib.ptr(device_error), _stream(dev))
    return outputs


# ---- verification from host-resident logits -------------------------------------------------

_staging: dict = {}


def _device_rows(host: torch.Tensor, device, slot: str) -> torch.Tensor:
    """A device buffer shaped like the host logits (reused across calls; never zeroed: only
    the rows a call copies are read)."""
    key = (slot, torch.device(device), tuple(host.shape), host.dtype)
    buf = _staging.get(key)
    if buf is None:
        buf = torch.empty(host.shape, dtype=host.dtype, device=device)
        _staging[key] = buf
    return buf


@dataclass
class HostVerifyInfo:
    """What a verify_logits_host call moved: logit bytes copied to the device, bytes read back,
    and the windows (verify positions per request) of its stages."""
    h2d_bytes: int
    d2h_bytes: int
    windows: tuple


def window_stages(lens, first_window, run_stage):
    """The widening windows of verify_logits_host.  ``run_stage(pending, lo, W)`` verifies the
    requests ``pending`` with their lengths capped at W (the rows of positions [lo, W) are new
    to this stage) and returns their accepted lengths, in order, and a callable that keeps the
    results of the requests it is given (positions in ``pending``).  A request is final once
    its capped chain stops before the cap (accepted length < W - 1) or its length is at most
    W: the capped run then takes the same steps, rows and uniforms as the full one.  Returns
    the windows used."""
    pending = list(range(len(lens)))
    lo, W, windows = 0, int(first_window), []
    while pending:
        windows.append(W)
        acc, keep = run_stage(pending, lo, W)
        done = [int(a) < W - 1 or int(lens[b]) <= W for b, a in zip(pending, acc)]
        if any(done):
            keep([i for i, f in enumerate(done) if f])
        pending = [b for b, f in zip(pending, done) if not f]
        lo, W = W, 2 * W
    return tuple(windows)


def verify_logits_host(*, candidates, target_logits, target_rows, temperature, top_k, top_p,
                       verify_lens, uniforms, uniform_final, prefix_lens, device,
                       draft_logits=None, draft_rows=None, slots=None, slot_rows=None,
                       min_p=None, mode: int = JOINT, first_window: int = 2):
    """verify_logits for inputs in host memory (CPU tensors; pinned ones copy asynchronously),
    copying to the device only the logit rows the outcome can depend on.

    A chain stops at its first rejected step, so stages widen a window of verify positions:
    stage 1 copies the rows of positions [0, W) of every request (W = first_window) and
    verifies with each request's length capped at W.  A request whose chain is rejected at a
    step s < W - 1, or whose length is at most W, has its final outcome (the capped run takes
    the same steps, rows and uniforms); the others are verified again with the window doubled,
    after the rows of the new positions are copied.  The outputs equal verify_logits on the
    whole batch bit for bit; compaction (``slots`` / ``slot_rows``) runs once at the end with
    the true lengths.  Returns host tensors (accept, commit, bonus, output, new_seq), the host
    CompactOutputs (or None) and a HostVerifyInfo."""
    dev = torch.device(device)
    _check(dev.type == "cuda", "verify_logits_host needs a CUDA device")
    host = [candidates, target_logits, target_rows, temperature, top_k, top_p, verify_lens,
            uniforms, uniform_final, prefix_lens]
    _check(all(t.device.type == "cpu" for t in host) and
           (draft_logits is None or (draft_logits.device.type == "cpu" and
                                     draft_rows is not None and draft_rows.device.type == "cpu")),
           "verify_logits_host takes CPU tensors")
    _check(first_window >= 2, "the first window must hold at least two positions")
    _check(target_logits.is_contiguous() and (draft_logits is None or draft_logits.is_contiguous()),
           "host logits must be contiguous")
    _check(draft_logits is None or draft_logits.shape[1] == target_logits.shape[1],
           "draft vocab differs")
    B = candidates.shape[0]
    lens = verify_lens.numpy().astype("int64").clip(1, T)
    trow = target_rows.numpy()
    greedy = ((top_k <= 1) | ~(temperature > 0)).numpy()
    with_draft = draft_logits is not None
    drow = draft_rows.numpy() if with_draft else None

    def up(t):
        return None if t is None else t.to(dev, non_blocking=True)

    cand_d, trow_d, temp_d = up(candidates), up(target_rows), up(temperature)
    topk_d, topp_d, u_d = up(top_k), up(top_p), up(uniforms)
    uf_d, prefix_d, lens_d = up(uniform_final), up(prefix_lens), up(verify_lens)
    drow_d, mp = up(draft_rows), up(min_p)
    h2d = sum(t.numel() * t.element_size() for t in (
        candidates, target_rows, temperature, top_k, top_p, uniforms, uniform_final,
        prefix_lens, verify_lens) + ((draft_rows,) if with_draft else ()) +
        ((min_p,) if min_p is not None else ()))
    t_dev = _device_rows(target_logits, dev, "target")
    d_dev = _device_rows(draft_logits, dev, "draft") if with_draft else None
    row_bytes = target_logits.shape[1] * target_logits.element_size()
    stream = _stream(dev)
    # every stage verifies the whole batch: the requests still open with their lengths capped
    # at the window, the finished ones at length 1 (their position-0 rows are on the device;
    # those results are ignored), each stage into its own output slice
    n_stages = 1
    while first_window << (n_stages - 1) < T:
        n_stages += 1
    outs = new_outputs(B * n_stages, dev)
    stage_out = [tuple(o[k * B:(k + 1) * B] for o in outs) for k in range(n_stages)]
    cap_h = torch.ones(B, dtype=torch.int32).pin_memory()
    cap_d = torch.empty(B, dtype=torch.int32, device=dev)
    workspace = workspace_for(B, dev)
    stage_of = np.zeros(B, dtype=np.int64)
    moved = [h2d, 0]

    def copy_ranges(dst, src, first, count):
        first = np.ascontiguousarray(first, dtype=np.int64)
        count = np.ascontiguousarray(count, dtype=np.int64)
        _lib.call("dsv_copy_row_ranges", dst.data_ptr(), src.data_ptr(), row_bytes, len(first),
                  first.ctypes.data, count.ctypes.data, stream)
        moved[0] += int(count.sum()) * row_bytes

    def run_stage(pending, lo, W):
        k = len(stage_windows)
        stage_windows.append(W)
        # the rows of positions [lo, W), clipped to each request's length (drafts: length - 1)
        pb = np.asarray(pending)
        copy_ranges(t_dev, target_logits, trow[pb] + lo, np.clip(np.minimum(W, lens[pb]) - lo, 0, None))
        if with_draft:
            n_d = np.clip(np.minimum(W, lens[pb] - 1) - lo, 0, None) * (~greedy[pb])
            copy_ranges(d_dev, draft_logits, drow[pb] + lo, n_d)
        caps = cap_h.numpy()
        caps[:] = 1
        caps[pb] = np.minimum(lens[pb], W)
        cap_d.copy_(cap_h, non_blocking=True)
        moved[0] += B * 4
        verify_logits(candidates=cand_d, target_logits=t_dev, target_rows=trow_d,
                      temperature=temp_d, top_k=topk_d, top_p=topp_d, verify_lens=cap_d,
                      uniforms=u_d, uniform_final=uf_d, prefix_lens=prefix_d,
                      draft_logits=d_dev, draft_rows=drow_d, outputs=stage_out[k],
                      workspace=workspace, min_p=mp, mode=mode)
        acc = stage_out[k][0].cpu().numpy()
        moved[1] += B * 4

        def keep(positions):
            stage_of[pb[positions]] = k

        return acc[pb].tolist(), keep

    stage_windows = []
    windows = window_stages(lens, first_window, run_stage)
    h2d, d2h = moved
    # every stage's outputs to the host once; each request takes those of its last stage
    host_all = [o.to("cpu") for o in outs]
    d2h += sum(o.numel() * o.element_size() for o in host_all)
    pick = torch.from_numpy(stage_of * B + np.arange(B))
    host_out = tuple(o.index_select(0, pick) for o in host_all)
    host_compact = None
    if slots is not None:
        from .accept import accept_compact  # the compaction with the true lengths
        commit_d, output_d = up(host_out[1]), up(host_out[3])
        h2d += host_out[1].numel() * 4 + host_out[3].numel() * 8
        compact = accept_compact(commit_d, lens_d, output_d, up(slots), up(slot_rows))
        h2d += slots.numel() * slots.element_size() + slot_rows.numel() * 8
        host_compact = CompactOutputs(*(t.to("cpu") for t in (
            compact.tokens, compact.kept_slots, compact.offsets, compact.freed_slots,
            compact.freed_offsets)))
        d2h += sum(t.numel() * t.element_size() for t in (
            compact.tokens, compact.kept_slots, compact.offsets, compact.freed_slots,
            compact.freed_offsets))
    torch.cuda.current_stream(dev).synchronize()
    return host_out, host_compact, HostVerifyInfo(h2d, d2h, windows)
