"""Capped verification acceptance (verification/caps.py of the reference) on the GPU.

`VerifyCaps.accept` keeps the reference's keyword-only signature and 5-tuple result
(caps.py:331-379).  The controller's SGLang half (shortening the target forward, CUDA-graph
replay of the capped width: caps.py:60-330) is outside this package; a controller sets
``worker``, ``full`` (the block width), ``active`` (the verified width), ``executed_width``
(the width the target forward ran) and ``sampled_round``.

- greedy rounds: the target's top-1 per row (dsv_topk_ids with k = 1: the lowest-index
  maximum, as torch.argmax) and the capped greedy accept (dsv_accept_greedy, caps.py:32-59
  `_accept_capped`);
- sampled rounds: `accept_sampled_prefix` (sampling/rejection.py) with every request capped
  at ``active``.
"""

from __future__ import annotations

import torch

from .. import accept as _accept
from ..kernels.dspine import topk_ids


def target_top1(next_token_logits, bs, full):
    """[bs, full] int64 top-1 ids of the verify rows (lowest index among equal maxima)."""
    logits = next_token_logits if next_token_logits.stride(-1) == 1 else next_token_logits.contiguous()
    return topk_ids(logits, 1).view(bs, full)


class VerifyCaps:
    def __init__(self, worker, *, full=16, active=None):
        self.worker = worker
        self.full = int(full)
        self.active = int(active if active is not None else full)
        self.executed_width = self.active
        self.sampled_round = False
        self.sampled_executions = 0
        self._sampled_cap_lens = {}

    def accept(self, *, candidates, next_token_logits, sampling_info, draft_input, prefix_lens,
               bs):
        if self.executed_width != self.active:
            raise RuntimeError("Capped acceptance requires a confirmed shortened target forward")
        if self.sampled_round:
            from ..sampling.rejection import accept_sampled_prefix

            key = (bs, self.active)
            if key not in self._sampled_cap_lens:
                self._sampled_cap_lens[key] = torch.full(
                    (bs,), self.active, device=candidates.device, dtype=torch.int32)
            return accept_sampled_prefix(
                self, candidates=candidates, next_token_logits=next_token_logits,
                sampling_info=sampling_info, prefix_lens=prefix_lens, bs=bs,
                verify_lens=self._sampled_cap_lens[key])
        top1 = target_top1(next_token_logits, bs, self.full)
        outputs = self.worker._next_accept_bonus_buffers(bs)
        key = (bs, self.active, "greedy")
        if key not in self._sampled_cap_lens:
            self._sampled_cap_lens[key] = torch.full(
                (bs,), self.active, device=candidates.device, dtype=torch.int32)
        return _accept.accept_greedy(candidates, top1, self._sampled_cap_lens[key],
                                     prefix_lens.to(torch.int32), outputs=outputs)


def active_controller():
    from ..runtime import worker as module

    current = module._active_worker
    return getattr(current, "verify_caps", None) if current is not None else None
