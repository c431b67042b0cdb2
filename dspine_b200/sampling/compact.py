"""Request-wise logit adjustments (sampling/compact.py of the reference) on the GPU.

`adjust_logits(logits, info, row_to_request)` keeps the reference's signature and its order of
transforms (compact.py:14-79): the batch's additive penalties, its scaling penalties, each
prepared penalizer of SGLang's orchestrator in the orchestrator's order, the grammar mask, the
logit bias.  The work is a short list of in-place dsv_adjust_logits passes (`_Plan`): the
penalties, the mask and the bias share one pass when nothing else comes between them (the
usual batch: one read and one write of the rows); every penalizer of the orchestrator opens
a pass of its own, and the mask and bias join the last one.  Each step rounds to the logit
dtype exactly as the torch op it replaces.

Grammar masks: an int32 token bitmask (xgrammar's layout, bit set = allowed) or a bool mask
(True = disallowed, the outlines layout) is applied inside the pass; a grammar with any other
mask layout is applied by its own ``apply_vocab_mask``, as the reference always does.

`around_verify_logits_adjustments` is the plugin's AROUND hook for SGLang's verify-logits
adjustments (compact.py:82-116).
"""

import torch

from .. import _lib

_DTYPES = {torch.bfloat16: 0, torch.float32: 1}


def can_keep_compact(info):
    """Packed verification rows stay packed unless a custom logit processor or a sampling
    mask needs SGLang's full-batch layout (compact.py:4-10)."""
    if info is None or getattr(info, "has_custom_logit_processor", False):
        return False
    return getattr(info, "sampling_mask_batch_indices", None) is None


class _Pass:
    """One dsv_adjust_logits pass over the rows (any of its four inputs may be absent)."""

    def __init__(self, logits, row_to_request):
        rows = logits.reshape(-1, logits.shape[-1])
        if rows.stride(-1) != 1:
            raise ValueError("logit rows must be contiguous")
        if rows.dtype not in _DTYPES:
            raise ValueError("logits must be bf16 or fp32")
        self.rows = rows
        self.device = logits.device
        if row_to_request is not None:
            self.mapping = row_to_request.to(device=self.device, dtype=torch.int64).contiguous()
            self.per_request = 1
        else:  # full blocks [B, T, V]: request of row r is r // T
            self.mapping = None
            self.per_request = logits.shape[1] if logits.dim() == 3 else 1

    def _f32(self, t):
        return None if t is None else t.to(device=self.device, dtype=torch.float32).contiguous()

    def __call__(self, additive=None, scaling=None, bitmask=None, bias=None):
        add, sc, bi = self._f32(additive), self._f32(scaling), self._f32(bias)
        words = 0
        if bitmask is not None:
            bitmask = bitmask.to(device=self.device, dtype=torch.int32).contiguous()
            words = bitmask.shape[-1]
        rows = self.rows
        with torch.cuda.device(self.device):
            _lib.call("dsv_adjust_logits", rows.data_ptr(), _DTYPES[rows.dtype], rows.shape[0],
                      rows.shape[1], rows.stride(0), _lib.ptr(self.mapping), self.per_request,
                      _lib.ptr(add), _lib.ptr(sc), _lib.ptr(bitmask), words, _lib.ptr(bi),
                      torch.cuda.current_stream(self.device).cuda_stream)


class _Plan:
    """Steps gathered into as few passes as their order allows.  One pass applies its inputs in
    the order additive, scaling, mask, bias, so a step joins the open pass when nothing of the
    pass comes at or after it in that order; a penalizer stage always opens its own pass (the
    orchestrator's stages are applied one after another)."""

    ORDER = ("additive", "scaling", "bitmask", "bias")

    def __init__(self, launch):
        self.launch = launch
        self.pending = {}

    def add(self, name, tensor, own_pass=False):
        if tensor is None:
            return
        rank = self.ORDER.index(name)
        if own_pass or any(self.ORDER.index(k) >= rank for k in self.pending):
            self.flush()
        self.pending[name] = tensor

    def flush(self):
        if self.pending:
            self.launch(**self.pending)
        self.pending = {}


def _bool_mask_as_bitmask(mask, vocab):
    """A bool [B, V] mask (True = disallowed) as int32 allow-words (bit set = allowed)."""
    allowed = ~mask.to(torch.bool)
    words = (vocab + 31) // 32
    padded = torch.zeros((allowed.shape[0], words * 32), dtype=torch.int64, device=mask.device)
    padded[:, :vocab] = allowed[:, :vocab].to(torch.int64)
    weights = torch.bitwise_left_shift(torch.ones(32, dtype=torch.int64, device=mask.device),
                                       torch.arange(32, device=mask.device))
    packed = (padded.view(allowed.shape[0], words, 32) * weights).sum(-1)
    return packed.to(torch.int64).where(packed < 2**31, packed - 2**32).to(torch.int32)


def _penalizer_stages(info, vocab, device):
    """(kind, tensor) for each prepared penalizer, in the orchestrator's order: a
    multiplicative penalizer scales, any other adds the bias its apply() writes into a zeroed
    [B, V] buffer (the orchestrator's own convention)."""
    orchestrator = getattr(info, "penalizer_orchestrator", None)
    if orchestrator is None or not orchestrator.is_required:
        return
    for penalizer in orchestrator.penalizers.values():
        if not penalizer.is_prepared():
            continue
        if penalizer.is_multiplicative:
            yield "scale", penalizer.get_scaling_penalties()
        else:
            buffer = torch.zeros((len(info), vocab), device=device, dtype=torch.float32)
            penalizer.apply(buffer)
            yield "add", buffer


def adjust_logits(logits, info, row_to_request):
    """Apply native transforms to real logits, in request order.  Packed logits use
    ``row_to_request``; full blocks are [B, T, V] with no mapping."""
    if info is None:
        return
    if logits.device.type != "cuda":
        raise ValueError("dspine_b200 adjusts logits on CUDA tensors only")
    launch = _Pass(logits, row_to_request)
    vocab = logits.shape[-1]
    additive = getattr(info, "acc_additive_penalties", None)
    if additive is None:  # older DFlash callers name the same buffer "linear"
        additive = getattr(info, "acc_linear_penalties", None)
    plan = _Plan(launch)
    plan.add("additive", additive)
    plan.add("scaling", getattr(info, "acc_scaling_penalties", None))
    for kind, tensor in _penalizer_stages(info, vocab, logits.device):
        plan.add("scaling" if kind == "scale" else "additive", tensor, own_pass=True)
    grammar = getattr(info, "grammar_mask", None)
    if grammar is not None:
        mask = grammar.vocab_mask
        if mask.dtype == torch.int32:
            plan.add("bitmask", mask)
        elif mask.dtype == torch.bool:
            plan.add("bitmask", _bool_mask_as_bitmask(mask.to(logits.device), vocab))
        else:
            # an unknown layout: the grammar applies its own mask, rows mapped as the reference
            plan.flush()
            mask = mask.to(device=logits.device)
            rows_mask = (mask.index_select(0, launch.mapping) if launch.mapping is not None
                         else mask.repeat_interleave(launch.per_request, dim=0))
            grammar.grammar.apply_vocab_mask(logits=logits.reshape(-1, vocab), vocab_mask=rows_mask)
    plan.add("bias", getattr(info, "logit_bias", None))
    plan.flush()


def around_verify_logits_adjustments(original, *, next_token_logits, sampling_info,
                                     draft_token_num):
    """The AROUND hook of SGLang's apply_dflash_verify_logits_adjustments (compact.py:82-116):
    packed rounds adjust their packed rows through the controller's row mapping; full rounds
    adjust [bs, draft_token_num, V] blocks; without a DSpine worker the original runs."""
    from ..runtime import worker as module
    from ..verification.caps import active_controller

    controller = active_controller()
    if controller is None and module._active_worker is None:
        return original(next_token_logits=next_token_logits, sampling_info=sampling_info,
                        draft_token_num=draft_token_num)
    if controller is not None and getattr(controller, "compact_round", False):
        if next_token_logits is not controller.compact_logits:
            raise RuntimeError("Packed verification logits do not belong to this round")
        return adjust_logits(next_token_logits, sampling_info, controller.row_to_request)
    if sampling_info is None:
        return
    if next_token_logits.ndim != 2 or draft_token_num <= 0:
        raise ValueError("Verification needs 2D logits and a positive draft width")
    bs = len(sampling_info)
    if next_token_logits.shape[0] != bs * draft_token_num:
        raise ValueError("Verification logits do not match the request/block layout")
    if getattr(sampling_info, "has_custom_logit_processor", False):
        from sglang.srt.layers.sampler import apply_custom_logit_processor  # SGLang's own

        apply_custom_logit_processor(next_token_logits, sampling_info,
                                     num_tokens_in_batch=draft_token_num)
    return adjust_logits(next_token_logits.view(bs, draft_token_num, -1), sampling_info, None)
