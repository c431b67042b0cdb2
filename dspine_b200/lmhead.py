"""Host API of the fused draft LM head + top-k + logsumexp (C ABI: dsv_lmhead_topk, dsv_tp_merge).

`lmhead_topk` replaces the reference's materialised head product followed by its top-k
(`torch.matmul(rows, W.T)` at runtime/worker.py:283-285, then kernels/dspine.py:165-207
`topk_ids`): the [rows, vocab] logits never reach HBM.  `TPHead` mirrors
sampling/tp_head.py:17-103 (`TPHead(weight, start, end, global_vocab_size, tp_group)`,
`.global_topk`, `merge_topk`) and adds `topk_lse`, the vocab-parallel head with one all-gather.
Argument errors raise ValueError before anything is launched (as kernels/dspine.py:172-188).
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

MAX_K = 32


def _check(cond, msg):
    if not cond:
        raise ValueError(msg)


def _stream(device) -> int:
    return torch.cuda.current_stream(torch.device(device)).cuda_stream


class LmHeadWorkspace:
    """Device scratch of dsv_lmhead_topk: per-CTA partial top-k lists and the error word."""

    def __init__(self, rows: int, vocab: int, k: int, device):
        size = ctypes.c_size_t()
        _lib.call("dsv_lmhead_workspace_size", int(rows), int(vocab), int(k), ctypes.byref(size))
        self.key = (int(rows), int(vocab), int(k))
        self.nbytes = int(size.value)
        self.buf = torch.empty(self.nbytes, dtype=torch.uint8, device=device)
        _lib.call("dsv_workspace_init", self.buf.data_ptr(), self.nbytes, _stream(device))

    def error_word(self) -> int:
        """Device error word (bit 0: a pipeline wait timed out); reading it clears it."""
        err = ctypes.c_uint32()
        _lib.call("dsv_workspace_error", self.buf.data_ptr(), ctypes.byref(err),
                  _stream(self.buf.device))
        return int(err.value)


_workspaces: dict = {}


def workspace_for(rows: int, vocab: int, k: int, device) -> LmHeadWorkspace:
    device = torch.device(device)
    key = (device.index, int(rows), int(vocab), int(k))
    ws = _workspaces.get(key)
    if ws is None:
        ws = LmHeadWorkspace(rows, vocab, k, device)
        _workspaces[key] = ws
    return ws


def lmhead_topk(hidden, weight, k, *, vocab=None, id_offset=0, pad_id=None, sort_ids=False,
                out=None, workspace=None):
    """Top-k of ``hidden @ weight[:vocab].T`` per row without materialising the logits.

    hidden [rows, H] bf16, weight [>= vocab, H] bf16 (H a multiple of 64, rows contiguous).
    Returns (ids int64 [rows, k], values f32 [rows, k], lse f32 [rows]): values are the logits
    rounded to bf16 (what torch.matmul of bf16 tensors materialises), ranked descending with
    ties to the lower id; ids are column + ``id_offset`` (``pad_id`` for empty slots when
    vocab < k); lse is the logsumexp of the fp32 logits.  ``sort_ids`` orders each row's ids
    ascending instead (the order of kernels/dspine.py topk_ids)."""
    _check(hidden.dim() == 2 and weight.dim() == 2, "hidden and weight must be 2-D")
    _check(hidden.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16,
           "hidden and weight must be bf16")
    _check(hidden.is_cuda and weight.device == hidden.device, "tensors must be on one CUDA device")
    rows, H = hidden.shape
    _check(weight.shape[1] == H, "hidden size differs between hidden and weight")
    _check(H % 64 == 0 and H >= 64, "hidden size must be a multiple of 64")
    _check(hidden.stride(1) == 1 and weight.stride(1) == 1, "rows must be contiguous")
    _check(hidden.stride(0) % 8 == 0 and weight.stride(0) % 8 == 0,
           "row pitches must be multiples of 8 elements")
    vocab = weight.shape[0] if vocab is None else int(vocab)
    _check(1 <= vocab <= weight.shape[0], "vocab must be in [1, weight rows]")
    _check(1 <= int(k) <= MAX_K, f"k must be in [1, {MAX_K}]")
    k = int(k)
    pad_id = (int(id_offset) + vocab) if pad_id is None else int(pad_id)
    dev = hidden.device
    if out is None:
        out = (torch.empty(rows, k, dtype=torch.int64, device=dev),
               torch.empty(rows, k, dtype=torch.float32, device=dev),
               torch.empty(rows, dtype=torch.float32, device=dev))
    ids, vals, lse = out
    _check(ids.shape == (rows, k) and ids.dtype == torch.int64 and ids.is_contiguous(), "ids out")
    _check(vals.shape == (rows, k) and vals.dtype == torch.float32 and vals.is_contiguous(),
           "values out")
    _check(lse is None or (lse.shape == (rows,) and lse.dtype == torch.float32), "lse out")
    if workspace is None:
        workspace = workspace_for(rows, vocab, k, dev)
    _check(workspace.key == (rows, vocab, k), "workspace was sized for another shape")
    _lib.call("dsv_lmhead_topk", rows, vocab, H, k, hidden.data_ptr(), hidden.stride(0),
              weight.data_ptr(), weight.stride(0), int(id_offset), pad_id, int(bool(sort_ids)),
              ids.data_ptr(), vals.data_ptr(), _lib.ptr(lse), workspace.buf.data_ptr(),
              workspace.nbytes, _stream(dev))
    return ids, vals, lse


def merge_shards(values, ids, lse, k, *, pad_id, sort_ids=False, out=None):
    """Global top-k + logsumexp from per-shard candidates: values f32 [S, rows, k],
    ids int64 [S, rows, k] (rank order per shard), lse f32 [S, rows] (C ABI dsv_tp_merge)."""
    S, rows, kk = values.shape
    _check(ids.shape == values.shape and lse.shape == (S, rows) and kk == k, "shard shapes")
    _check(values.dtype == torch.float32 and ids.dtype == torch.int64 and lse.dtype == torch.float32,
           "shard dtypes")
    dev = values.device
    if out is None:
        out = (torch.empty(rows, k, dtype=torch.int64, device=dev),
               torch.empty(rows, k, dtype=torch.float32, device=dev),
               torch.empty(rows, dtype=torch.float32, device=dev))
    for t in (values, ids, lse):
        _check(t.stride(-1) == 1 and (t.dim() < 3 or t.stride(1) == k), "shard rows must be packed")
    _lib.call("dsv_tp_merge", rows, S, k, values.data_ptr(), values.stride(0), ids.data_ptr(),
              ids.stride(0), lse.data_ptr(), lse.stride(0), int(pad_id), int(bool(sort_ids)),
              out[0].data_ptr(), out[1].data_ptr(), _lib.ptr(out[2]), _stream(dev))
    return out


def _ordered_keys(values):
    """int32 keys ordered as torch's sort orders the values: NaN above every number, -0 equal
    to +0 (values of any float dtype, compared exactly in float32)."""
    v = values.float() + 0.0                     # -0 + 0 = +0
    bits = v.view(torch.int32)
    keys = torch.where(bits < 0, bits ^ 0x7FFFFFFF, bits)
    return torch.where(torch.isnan(v), torch.full_like(keys, 0x7FFFFFFF), keys)


def merge_topk(values, ids, k, *, max_pairs: int = 1 << 24):
    """The global top-k of candidate rows, lower token ids winning value ties
    (sampling/tp_head.py:9-14), on any device: candidate j of a row outranks candidate i when
    its value is larger, or equal with a smaller id, or equal in both and earlier in the row;
    the first min(k, width) candidates in that order are returned (values, ids).  The ranks come
    from pairwise comparisons, rows taken in blocks of at most ``max_pairs`` comparisons."""
    width = values.shape[-1]
    lead = values.shape[:-1]
    keys = _ordered_keys(values.reshape(-1, width))
    flat_ids = ids.reshape(-1, width)
    n = keys.shape[0]
    kk = min(int(k), width)
    order = torch.empty((n, kk + 1), dtype=torch.int64, device=values.device)
    position = torch.arange(width, device=values.device)
    earlier = position[None, :] < position[:, None]          # [i, j]: j before i
    step = max(1, max_pairs // max(1, width * width))
    for lo in range(0, n, step):
        hi = min(lo + step, n)
        ki, kj = keys[lo:hi, :, None], keys[lo:hi, None, :]
        ii, ij = flat_ids[lo:hi, :, None], flat_ids[lo:hi, None, :]
        beats = (kj > ki) | ((kj == ki) & ((ij < ii) | ((ij == ii) & earlier)))
        rank = beats.sum(-1).clamp_(max=kk)                   # [rows, width], distinct below kk
        order[lo:hi].scatter_(1, rank, position.expand(hi - lo, width))
    order = order[:, :kk].reshape(*lead, kk)
    return values.gather(-1, order), ids.gather(-1, order)


class TPHead:
    """Vocabulary-sharded head (sampling/tp_head.py:17-103): each rank keeps its weight shard;
    only candidates cross ranks.  ``tp_group`` provides ``world_size``,
    ``all_gather(tensor, dim)`` and ``all_reduce(tensor)`` (SGLang's GroupCoordinator;
    `TorchGroup` adapts a torch.distributed process group)."""

    def __init__(self, weight, start, end, global_vocab_size, tp_group):
        self.weight = weight
        self.start, self.end = int(start), int(end)
        self.global_vocab_size = int(global_vocab_size)
        self.group = tp_group
        self.world_size = int(tp_group.world_size)
        valid_shard = (weight.ndim == 2 and weight.dtype == torch.bfloat16
                       and weight.stride(1) == 1 and weight.shape[0] > 0
                       and 0 <= self.start <= self.end <= self.global_vocab_size
                       and self.end - self.start <= weight.shape[0])
        if not valid_shard:
            raise ValueError("Invalid DSpine vocabulary head shard")
        mine = torch.tensor([[self.start, self.end, weight.shape[0]]], device=weight.device,
                            dtype=torch.int64)
        table = self.group.all_gather(mine, dim=0).cpu()      # [world, 3], rank order
        begins, ends, allocated = table[:, 0], table[:, 1], table[:, 2]
        follows = torch.cat([begins.new_zeros(1), ends[:-1]])  # each shard starts where the last ended
        if not (torch.equal(begins, follows) and bool((ends >= begins).all())
                and bool((ends - begins <= allocated).all())):
            raise ValueError("DSpine head shards must partition the original vocabulary")
        if int(ends[-1]) != self.global_vocab_size:
            raise ValueError("DSpine head shards do not cover the original vocabulary")
        self.geometry = tuple(tuple(int(x) for x in row) for row in table.tolist())
        self.max_rows = int(allocated.max())

    @property
    def num_local(self):
        return self.end - self.start

    def global_topk(self, local_values, local_ids, k):
        """Merge equally padded local candidate blocks: the values (as their float32 bits, exact
        for bf16 / fp16 / fp32) and the ids cross ranks in ONE all-gather of an int64 block,
        then `merge_topk` on the rank-ordered concatenation (sampling/tp_head.py:76-82)."""
        if local_values.shape != local_ids.shape:
            raise ValueError("DSpine local candidate values and IDs must match")
        bits = local_values.float().view(torch.int32).to(torch.int64)
        block = torch.stack((bits, local_ids.to(torch.int64)))
        gathered = self.group.all_gather(block, dim=-1)
        values = gathered[0].to(torch.int32).view(torch.float32).to(local_values.dtype)
        return merge_topk(values, gathered[1].to(local_ids.dtype), k)

    def gather_vocab_rows(self, local):
        """The full-vocabulary table from every rank's rows (sampling/tp_head.py:58-71): shards
        padded to the largest allocation, all-gathered, each rank's real rows placed at its
        vocabulary range."""
        if local.shape[0] != self.num_local:
            raise ValueError("DSpine local vocabulary table has the wrong row count")
        padded = local.new_zeros((self.max_rows, *local.shape[1:]))
        padded[: self.num_local] = local
        blocks = self.group.all_gather(padded, dim=0).view(self.world_size, self.max_rows,
                                                           *local.shape[1:])
        full = local.new_empty((self.global_vocab_size, *local.shape[1:]))
        for rank, (begin, end, _) in enumerate(self.geometry):
            full[begin:end] = blocks[rank, : end - begin]
        return full

    def selected_rows(self, ids):
        """The bf16 head rows of global ids (sampling/tp_head.py:84-89): the owner rank
        contributes each row, the others zeros, and one all-reduce sums them."""
        local = ids - self.start
        owner = (local >= 0) & (ids < self.end)
        rows = self.weight[local.clamp(0, self.weight.shape[0] - 1)]
        rows = rows * owner[..., None].to(rows.dtype)
        return self.group.all_reduce(rows.contiguous())

    def rescore(self, ids, hidden):
        """The original BF16 head dot of global candidate ids (sampling/tp_head.py:91-103): the
        owner rank computes it (dsv_rescore_select16), the others contribute 0, one
        all-reduce sums the exchange."""
        from .layers.fp8 import gather

        owner = (ids >= self.start) & (ids < self.end)
        local_ids = (ids - self.start).clamp(0, self.weight.shape[0] - 1).contiguous()
        scores = gather.rescore(torch, self.weight, local_ids, hidden)
        scores.masked_fill_(~owner, 0)
        return self.group.all_reduce(scores)

    def topk_lse(self, hidden, k, *, sort_ids=False):
        """Global top-k ids/values and logsumexp of ``hidden @ W_full.T`` with ONE all-gather:
        the local fused head (padding rows beyond num_local excluded, ids shifted by start)
        writes straight into this rank's slot of a packed exchange block
        [ids int64 rows*k | values f32 rows*k | lse f32 rows], the block is all-gathered and
        every rank merges the same buffer, so every rank gets identical results."""
        rows = hidden.shape[0]
        words = rows * k * 3 + rows
        words += words & 1                                   # keep each block 8-byte aligned
        block = torch.empty(words, dtype=torch.int32, device=hidden.device)
        ids = block[: 2 * rows * k].view(torch.int64).view(rows, k)
        vals = block[2 * rows * k: 3 * rows * k].view(torch.float32).view(rows, k)
        lse = block[3 * rows * k: 3 * rows * k + rows].view(torch.float32)
        if self.num_local > 0:
            lmhead_topk(hidden, self.weight, k, vocab=self.num_local, id_offset=self.start,
                        pad_id=self.global_vocab_size, out=(ids, vals, lse))
        else:
            ids.fill_(self.global_vocab_size)
            vals.fill_(float("-inf"))
            lse.fill_(float("-inf"))
        gathered = self.group.all_gather(block, dim=0).view(self.world_size, words)
        g_ids = gathered[:, : 2 * rows * k].view(torch.int64).view(self.world_size, rows, k)
        g_vals = gathered[:, 2 * rows * k: 3 * rows * k].view(torch.float32).view(self.world_size, rows, k)
        g_lse = gathered[:, 3 * rows * k: 3 * rows * k + rows].view(torch.float32)
        return merge_shards(g_vals, g_ids, g_lse, k, pad_id=self.global_vocab_size,
                            sort_ids=sort_ids)


class TorchGroup:
    """`all_gather(tensor, dim)` / `all_reduce(tensor)` / `world_size` over a torch.distributed
    process group."""

    def __init__(self, group=None):
        import torch.distributed as dist
        self._dist = dist
        self.group = group
        self.world_size = dist.get_world_size(group)

    def all_reduce(self, tensor):
        self._dist.all_reduce(tensor, group=self.group)
        return tensor

    def all_gather(self, tensor, dim=0):
        """Rank blocks concatenated along ``dim`` (one output allocation; for dim != 0 the
        rank-major result is moved into place with one copy)."""
        tensor = tensor.contiguous()
        out = torch.empty((self.world_size, *tensor.shape), dtype=tensor.dtype,
                          device=tensor.device)
        self._dist.all_gather_into_tensor(out.view(-1), tensor.view(-1), group=self.group)
        if tensor.dim() == 0:
            return out
        d = dim % tensor.dim()
        if d == 0:
            return out.view(self.world_size * tensor.shape[0], *tensor.shape[1:])
        moved = out.movedim(0, d)                              # [..., world, n_d, ...]
        shape = list(tensor.shape)
        shape[d] *= self.world_size
        return moved.reshape(shape)
