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


def accept_sampled_prefix(controller, *, candidates, next_token_logits, sampling_info,
                          prefix_lens, bs, verify_lens, row_offsets=None, row_to_request=None):
    """Verify one shortened target call against this round's sampled chain q
    (sampling/rejection.py:156-239): the worker's TargetDistribution when it has one, else the
    dense target of the full 16-row envelope with the sparse q through dsv_accept_sparse (the
    reference scatters q into a dense buffer for sample_capped_chain_from_probs; a sparse q
    gives the same chain without that buffer)."""
    from ..runtime.worker import build_dspine_target_probs
    from .random import verification_uniforms
    from .sparse.accept import accept_sparse
    from .target import _sampling_backend

    worker = controller.worker
    if getattr(worker, "target_distribution", None) is not None:
        result = worker.target_distribution.sample_prefix(
            candidates=candidates, next_token_logits=next_token_logits,
            sampling_info=sampling_info, prefix_lens=prefix_lens, bs=bs,
            verify_lens=verify_lens, row_offsets=row_offsets, row_to_request=row_to_request)
        if result is not None:
            controller.sampled_executions += 1
            return result
    sampler = worker._dspine_sampler
    if not sampler.round_sampled or sampler.round_bs != bs:
        raise RuntimeError("Sampled caps require the current sampled proposal and q")
    width = int(worker.block_size)
    if width != 16 or candidates.shape != (bs, width):
        raise ValueError("Sampled caps require full16 proposal storage")
    if next_token_logits.shape[0] != bs * width:
        raise ValueError("Target output must retain the full16 mapped row envelope")
    target_probs = build_dspine_target_probs(
        next_token_logits=next_token_logits, sampling_info=sampling_info, block_size=width,
        bs=bs, sampling_backend=_sampling_backend(worker))
    outputs = worker._next_accept_bonus_buffers(bs)
    uniforms, final = verification_uniforms(bs, width, candidates.device, sampler.random)
    accept_sparse(torch, candidates=candidates, dense_p=target_probs.reshape(bs * width, -1),
                  packed=None, q_ids=sampler.candidate_out[:bs], q_values=sampler.q_out[:bs],
                  verify_lens=verify_lens, uniforms=uniforms, uniform_final=final,
                  prefix_lens=prefix_lens, outputs=outputs)
    controller.sampled_executions += 1
    return outputs
