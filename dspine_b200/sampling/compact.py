"""Request-wise logit adjustments (sampling/compact.py of the reference) on the GPU.

`adjust_logits(logits, info, row_to_request)` keeps the reference's signature and order of
transforms; the additive penalties, scaling penalties, grammar bitmask (xgrammar layout:
int32 words, bit set = allowed) and logit bias run as one dsv_adjust_logits pass.  Prepared
penalizers of SGLang's orchestrator are applied in their own order through the same kernel.
"""

import torch

from .. import _lib


def can_keep_compact(info):
    return (info is not None and not getattr(info, "has_custom_logit_processor", False)
            and getattr(info, "sampling_mask_batch_indices", None) is None)


def _launch(logits, mapping, rpr, additive=None, scaling=None, mask=None, bias=None):
    rows2d = logits.reshape(-1, logits.shape[-1])
    if rows2d.stride(-1) != 1:
        raise ValueError("logit rows must be contiguous")
    V = rows2d.shape[-1]
    dtype = {torch.bfloat16: 0, torch.float32: 1}.get(rows2d.dtype)
    if dtype is None:
        raise ValueError("logits must be bf16 or fp32")

    def f32(t):
        return None if t is None else t.to(device=logits.device, dtype=torch.float32).contiguous()
    m = None
    words = 0
    if mask is not None:
        m = mask.to(device=logits.device, dtype=torch.int32).contiguous()
        words = m.shape[-1]
    add, sc, bi = f32(additive), f32(scaling), f32(bias)
    _lib.call("dsv_adjust_logits", rows2d.data_ptr(), dtype, rows2d.shape[0], V, rows2d.stride(0),
              _lib.ptr(mapping), int(rpr), _lib.ptr(add), _lib.ptr(sc), _lib.ptr(m), words,
              _lib.ptr(bi), torch.cuda.current_stream(logits.device).cuda_stream)


def adjust_logits(logits, info, row_to_request):
    """Apply native transforms to real logits, in request order.  Packed logits use
    ``row_to_request``; full blocks are [B, T, V] with no mapping."""
    if info is None:
        return
    if logits.device.type != "cuda":
        raise ValueError("dspine_b200 adjusts logits on CUDA tensors only")
    if row_to_request is not None:
        mapping = row_to_request.to(device=logits.device, dtype=torch.int64).contiguous()
        rpr = 1
    else:
        mapping = None
        rpr = logits.shape[1] if logits.dim() == 3 else 1
    linear = getattr(info, "acc_additive_penalties", None)
    if linear is None:
        linear = getattr(info, "acc_linear_penalties", None)
    scaling = getattr(info, "acc_scaling_penalties", None)
    # the native buffers first (one pass), then the orchestrator's penalizers in order, then
    # the grammar mask and the bias (one pass) -- the reference's order
    if linear is not None or scaling is not None:
        _launch(logits, mapping, rpr, additive=linear, scaling=scaling)
    penalizer = getattr(info, "penalizer_orchestrator", None)
    if penalizer is not None and penalizer.is_required:
        for penalty in penalizer.penalizers.values():
            if not penalty.is_prepared():
                continue
            if penalty.is_multiplicative:
                _launch(logits, mapping, rpr, scaling=penalty.get_scaling_penalties())
            else:
                bias = torch.zeros((len(info), logits.shape[-1]), device=logits.device,
                                   dtype=torch.float32)
                penalty.apply(bias)
                _launch(logits, mapping, rpr, additive=bias)
    grammar = getattr(info, "grammar_mask", None)
    mask = None if grammar is None else grammar.vocab_mask
    bias = getattr(info, "logit_bias", None)
    if mask is not None or bias is not None:
        _launch(logits, mapping, rpr, mask=mask, bias=bias)
