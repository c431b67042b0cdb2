"""Target distributions with sparse-q chain rejection (sampling/target.py of the reference).

`TargetDistribution(worker)` keeps the reference's constructor and methods:
`dense(logits, info, bs, row_to_request=None)` is build_dspine_target_probs on the batch's
rows, and `sample_prefix(...)` (target.py:34-122) verifies a round against its sampled q:
the small-support joint target when the batch allows it (build_sparse_target), else the dense
target, packed by compress_probs when any filter is on, then dsv_accept_sparse.  Every step is
one launch of this package's kernels; the q is the draft sampler's sparse [bs, 15, 16] q,
never scattered into a dense buffer.

The worker provides ``block_size``, ``_dspine_sampler`` (``round_sampled``, ``round_bs``,
``k``, ``candidate_out``, ``q_out``, ``random``), ``_next_accept_bonus_buffers(bs)`` and
``sampling_backend`` (the reference reads SGLang's get_exec().kernel.sampling_backend, which
is used here when SGLang is importable and the worker does not name one).
"""

import copy

import torch

from .sparse import accept


def _sampling_backend(worker):
    backend = getattr(worker, "sampling_backend", None)
    if backend is not None:
        return backend
    from sglang.srt.runtime_context import get_exec  # the reference's source of truth

    return get_exec().kernel.sampling_backend


class TargetDistribution:
    def __init__(self, worker):
        self.worker = worker
        self.scratch = None  # the reference's [cap, 4096] scratch; these kernels need none

    def dense(self, logits, info, bs, row_to_request=None):
        from ..runtime.worker import build_dspine_target_probs

        width = int(self.worker.block_size)
        if row_to_request is not None:
            info = copy.copy(info)
            for name in ("temperatures", "top_ks", "top_ps", "min_ps"):
                value = getattr(info, name, None)
                if value is not None:
                    setattr(info, name, value.reshape(value.shape[0], -1)[:, 0]
                            .index_select(0, row_to_request.to(value.device)))
            bs, width = logits.shape[0], 1
        return build_dspine_target_probs(next_token_logits=logits, sampling_info=info,
                                         block_size=width, bs=bs,
                                         sampling_backend=_sampling_backend(self.worker))

    def sample_prefix(self, *, candidates, next_token_logits, sampling_info, prefix_lens, bs,
                      verify_lens, row_offsets=None, row_to_request=None):
        sampler = self.worker._dspine_sampler
        if not sampler.round_sampled or sampler.round_bs != bs:
            raise RuntimeError("Sparse rejection must consume this round's actual proposal q")
        # other block layouts keep the worker's generic rejection path
        width = int(self.worker.block_size)
        if width != 16 or sampler.k != 16:
            return None
        if candidates.shape != (bs, width):
            raise ValueError("Proposal storage does not match this decode batch")
        backend = _sampling_backend(self.worker)
        sparse = None
        if next_token_logits.device.type == "cuda":
            from .sparse.target import build_sparse_target

            sparse = build_sparse_target(next_token_logits, sampling_info,
                                         row_to_request=row_to_request, row_offsets=row_offsets,
                                         verify_lens=verify_lens, block_size=width,
                                         sampling_backend=backend)
        if sparse is None:
            p = self.dense(next_token_logits, sampling_info, bs, row_to_request)
            flat_p = p.reshape(next_token_logits.shape[0], -1)
        else:
            flat_p = sparse.dense_p
        # unfiltered p is dense anyway: keep the sparse q without compressing a support that
        # would overflow; filtered supports may pack
        filtered = any(getattr(sampling_info, name, False) for name in (
            "need_top_k_sampling", "need_top_p_sampling", "need_min_p_sampling"))
        packed = (sparse.packed if sparse is not None
                  else accept.compress_probs(torch, flat_p, capacity=32) if filtered else None)
        outputs = self.worker._next_accept_bonus_buffers(bs)
        from .random import verification_uniforms

        uniforms, final = verification_uniforms(bs, width, candidates.device, sampler.random)
        accept.accept_sparse(
            torch, candidates=candidates, dense_p=flat_p, packed=packed,
            q_ids=sampler.candidate_out[:bs], q_values=sampler.q_out[:bs],
            verify_lens=verify_lens, uniforms=uniforms, uniform_final=final,
            prefix_lens=prefix_lens, outputs=outputs, row_offsets=row_offsets,
            vocab_size=next_token_logits.shape[-1],
            denominator=sparse.denominator if sparse is not None else None)
        return outputs
