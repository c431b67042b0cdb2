"""Capped chain rejection from dense probabilities (sampling/rejection.py:101-153 of the
reference) on the GPU: `sample_capped_chain_from_probs` keeps the reference's keyword-only
signature, its ValueError checks and messages, and caller-owned outputs; the work is one
dsv_chain_from_probs launch (exact fixed-point residual CDF)."""

from __future__ import annotations

import torch

from .. import _lib


def sample_capped_chain_from_probs(*, candidates, target_probs, draft_probs, verify_lens,
                                   uniforms, uniform_final, prefix_lens, outputs):
    """Launch with explicit coins, shared by the runtime and numerical tests."""
    (bs, width) = candidates.shape
    vocab = target_probs.shape[-1]
    if width != 16 or target_probs.shape != (bs, width, vocab):
        raise ValueError("Sampled ragged adapter requires target [B,16,V]")
    if draft_probs.shape != (bs, width - 1, vocab):
        raise ValueError("Sampled ragged adapter requires draft q [B,15,V]")
    if verify_lens.shape != (bs,) or uniforms.shape != (bs, width - 1):
        raise ValueError("Invalid cap or uniform layout")
    if uniform_final.shape != (bs,) or prefix_lens.shape != (bs,):
        raise ValueError("Invalid final uniform or prefix layout")
    if len(outputs) != 5:
        raise ValueError("Expected accept/commit/bonus/output/new_seq buffers")
    tensors = (candidates, target_probs, draft_probs, verify_lens, uniforms, uniform_final,
               prefix_lens, *outputs)
    if any(not t.is_contiguous() for t in tensors):
        raise ValueError("The sampled capped kernel requires contiguous tensors")
    if any(t.device != candidates.device for t in tensors):
        raise ValueError("The sampled capped kernel requires one device")
    if candidates.device.type != "cuda":
        raise ValueError("dspine_b200 runs the sampled capped kernel on CUDA tensors only")
    dtypes = ((candidates, torch.int64), (target_probs, torch.float32),
              (draft_probs, torch.float32), (verify_lens, torch.int32), (uniforms, torch.float32),
              (uniform_final, torch.float32), (prefix_lens, torch.int32),
              (outputs[0], torch.int32), (outputs[1], torch.int32), (outputs[2], torch.int64),
              (outputs[3], torch.int64), (outputs[4], torch.int32))
    if any(t.dtype != d for t, d in dtypes):
        raise ValueError("Expected int64 candidates, fp32 probabilities/uniforms, int32 caps")
    _lib.call("dsv_chain_from_probs", bs, vocab, candidates.data_ptr(), target_probs.data_ptr(),
              draft_probs.data_ptr(), verify_lens.data_ptr(), uniforms.data_ptr(),
              uniform_final.data_ptr(), prefix_lens.data_ptr(), *(o.data_ptr() for o in outputs),
              torch.cuda.current_stream(candidates.device).cuda_stream)
    return outputs
