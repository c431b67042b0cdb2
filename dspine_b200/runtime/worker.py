"""The verification seams of the reference's runtime/worker.py on the GPU.

The reference's DSpine worker (runtime/worker.py:680-1115) is an SGLang DFlashWorkerV2
subclass; its SGLang side (scheduling, CUDA-graph runners, the draft model) is outside this
package.  What plugs into it keeps the reference's module path, names and signatures:

- `build_dspine_target_probs` (worker.py:440-470): the [bs, T, V] fp32 target distribution,
  one dsv_target_probs_ex launch over the logits as they are (bf16 or fp32), with the filter of
  the batch (the sampling backend and its need_* flags, worker.py:473-508) and greedy rows
  one-hot at the lowest-index argmax (worker.py:461-469).
- `dspine_accept_sampling` (worker.py:511-581): chain rejection of the drafted block against
  the sparse q the drafts were drawn from, returning (accept_len int32, bonus int64).  The
  reference scatters q into a zeroed dense [bs, T-1, V] buffer and runs SGLang's chain kernel;
  here the sparse q goes straight into dsv_accept_sparse (q of a token = the sum of its
  entries), so `dense_q` is accepted for the contract and never touched.
- `accept_dspine_sampled_round` (worker.py:1092-1115): seam C, the plugin's AROUND hook target,
  delegating to the active worker's `_accept_sampled_round`.
- `DSpineVerifier`: the worker-side half of seam C (worker.py:1016-1090, `_accept_sampled_round`
  and `_dspine_verify`) for a worker that owns a draft sampler (`candidate_out`, `q_out`,
  `random`, `round_sampled`, `round_bs`), with SGLang's double-buffered accept outputs
  (`_next_accept_bonus_buffers`).  An SGLang worker composes it and sets `_active_worker`.
"""

from __future__ import annotations

import torch

from .. import logits as _logits
from .. import verify as _verify
from ..sampling import random as _random
from ..sampling.sparse import accept as _accept
from ..sampling.target import TargetDistribution

_active_worker = None
TOPK_ALL = 1 << 30


def set_active_worker(worker):
    """Install the worker that seam C delegates to (the reference sets the module global in
    DSpineWorkerV2.__init__)."""
    global _active_worker
    _active_worker = worker


def _flag(info, name):
    return bool(getattr(info, name, False))


def filter_params(sampling_info, bs, device):
    """Per-request (temperature, top_k, top_p, min_p, mode) of a batch as the kernels read them:
    a filter whose need_* flag is off is switched off (top_k all, top_p 1, min_p 0), as the
    reference applies only the flagged filters; greedy requests (top_k <= 1) stay greedy."""
    temperature = sampling_info.temperatures.reshape(-1)[:bs].to(device=device, dtype=torch.float32)
    top_k = sampling_info.top_ks.reshape(-1)[:bs].to(device=device, dtype=torch.int32)
    top_p = sampling_info.top_ps.reshape(-1)[:bs].to(device=device, dtype=torch.float32)
    min_ps = getattr(sampling_info, "min_ps", None)
    need_k = _flag(sampling_info, "need_top_k_sampling")
    need_p = _flag(sampling_info, "need_top_p_sampling")
    need_min_p = _flag(sampling_info, "need_min_p_sampling")
    if not need_k:
        top_k = torch.where(top_k <= 1, top_k, torch.full_like(top_k, TOPK_ALL))
    if not need_p:
        top_p = torch.ones_like(top_p)
    min_p = None
    if need_min_p and min_ps is not None:
        min_p = min_ps.reshape(-1)[:bs].to(device=device, dtype=torch.float32).contiguous()
    return (temperature.contiguous(), top_k.contiguous(), top_p.contiguous(), min_p,
            need_min_p)


def build_dspine_target_probs(*, next_token_logits, sampling_info, block_size: int, bs: int,
                              sampling_backend: str) -> torch.Tensor:
    """[bs, T, V] fp32: the distribution SGLang's ordinary sampler draws from for each verify
    row (runtime/worker.py:440-470): softmax(logits / temperature), then the backend's filter
    (flashinfer: joint top-k / top-p, or top-k -> top-p -> min-p when the batch has min-p;
    pytorch: joint top-k / top-p and min-p), renormalised; greedy rows one-hot at the
    lowest-index argmax.  Exact canonical kept sets (dsv_target_probs_ex)."""
    t = int(block_size)
    logits = next_token_logits
    if logits.dim() != 2 or logits.shape[0] != bs * t:
        raise ValueError("DSPINE target probabilities need [bs * block_size, V] logits")
    mode = _verify.filter_mode(sampling_backend, _flag(sampling_info, "need_min_p_sampling"))
    temperature, top_k, top_p, min_p, _ = filter_params(sampling_info, bs, logits.device)
    probs = _logits.target_probs(logits.contiguous(), temperature, top_k, top_p,
                                 rows_per_request=t, min_p=min_p, mode=mode)
    return probs.view(bs, t, -1)


def dspine_accept_sampling(*, target_probs=None, candidates: torch.Tensor,
                           target_logits: torch.Tensor, candidate_ids: torch.Tensor,
                           q_rows: torch.Tensor, sampling_info, sampling_backend: str,
                           dense_q: torch.Tensor | None = None, random_state=None):
    """Chain rejection of the drafted block (runtime/worker.py:511-581): candidates [bs, T] =
    [anchor, T-1 drafts]; candidate_ids / q_rows [bs, T-1, K] the sparse q each draft was
    sampled from.  Returns (accept_len int32 [bs], bonus int64 [bs])."""
    (bs, block) = candidates.shape
    gamma = block - 1
    if (tuple(candidate_ids.shape[:2]) != (bs, gamma)
            or candidate_ids.shape != q_rows.shape):
        raise RuntimeError("DSPINE verify: candidate / q layout mismatch")
    if block != 16 or candidate_ids.shape[2] != 16:
        raise RuntimeError("DSPINE verify on the GPU needs 16-token blocks with K = 16 q entries")
    device = candidates.device
    if target_probs is None:
        target_probs = build_dspine_target_probs(
            next_token_logits=target_logits, sampling_info=sampling_info, block_size=block,
            bs=bs, sampling_backend=sampling_backend)
    uniforms, uniform_final = _random.verification_uniforms(bs, block, device, random_state)
    outputs = _verify.new_outputs(bs, device)
    _accept.accept_sparse(
        torch, candidates=candidates.contiguous(), dense_p=target_probs.reshape(bs * block, -1),
        packed=None, q_ids=candidate_ids.to(torch.int64).contiguous(),
        q_values=q_rows.to(torch.float32).contiguous(),
        verify_lens=torch.full((bs,), block, device=device, dtype=torch.int32),
        uniforms=uniforms.contiguous(), uniform_final=uniform_final.contiguous(),
        prefix_lens=torch.zeros(bs, device=device, dtype=torch.int32), outputs=outputs)
    return outputs[0], outputs[2]


class DSpineVerifier:
    """The worker-side half of seam C (runtime/worker.py:1016-1090).

    ``sampler`` is the draft sampler of the round (the reference's DSpineDraftSampler: its
    ``candidate_out`` / ``q_out`` [max_bs, T-1, K] hold the sampled chain's q, ``random`` the
    request RNG, ``round_sampled`` / ``round_bs`` the round state).  ``sampling_backend`` is
    SGLang's configured backend (the reference reads get_exec().kernel.sampling_backend)."""

    def __init__(self, sampler, *, block_size: int = 16, sampling_backend: str = "flashinfer",
                 use_target_distribution: bool = True):
        self._dspine_sampler = sampler
        self.block_size = int(block_size)
        self.sampling_backend = sampling_backend
        self.target_distribution = TargetDistribution(self) if use_target_distribution else None
        self._accept_buffers = {}
        self._accept_parity = {}

    def _next_accept_bonus_buffers(self, bs: int):
        """Caller-visible accept outputs, double-buffered per batch size so that a round's
        results stay valid while the next round is verified (SGLang's
        _next_accept_bonus_buffers; tests/test_tp_accept.py:174-181)."""
        device = self._dspine_sampler.candidate_out.device
        key = (device, int(bs))
        if key not in self._accept_buffers:
            self._accept_buffers[key] = (_verify.new_outputs(bs, device),
                                         _verify.new_outputs(bs, device))
            self._accept_parity[key] = 0
        parity = self._accept_parity[key]
        self._accept_parity[key] = parity ^ 1
        return self._accept_buffers[key][parity]

    def _accept_sampled_round(self, *, candidates, next_token_logits, sampling_info,
                              max_top_k=None, uniform_top_k_value=None):
        """Verify a round with a sampled request against the q its drafts were drawn from; a
        round whose sampled chain never ran is refused (runtime/worker.py:1016-1044)."""
        sampler = self._dspine_sampler
        bs = int(candidates.shape[0])
        if not sampler.round_sampled:
            raise RuntimeError(
                "DSPINE sampled verify reached without this round's sampled draft chain")
        if bs != sampler.round_bs:
            raise RuntimeError(
                f"DSPINE sampled verify for batch {bs} while the staged round has batch "
                f"{sampler.round_bs}")
        return self._dspine_verify(candidates=candidates, next_token_logits=next_token_logits,
                                   candidate_ids=sampler.candidate_out[:bs],
                                   q_rows=sampler.q_out[:bs], sampling_info=sampling_info,
                                   max_top_k=max_top_k, uniform_top_k_value=uniform_top_k_value)

    def _dspine_verify(self, *, candidates, next_token_logits, candidate_ids, q_rows,
                       sampling_info, max_top_k=None, uniform_top_k_value=None):
        bs = candidates.shape[0]
        target_probs = None
        if self.target_distribution is not None:
            outputs = self.target_distribution.sample_prefix(
                candidates=candidates, next_token_logits=next_token_logits,
                sampling_info=sampling_info,
                prefix_lens=torch.zeros(bs, device=candidates.device, dtype=torch.int32), bs=bs,
                verify_lens=torch.full((bs,), self.block_size, device=candidates.device,
                                       dtype=torch.int32))
            if outputs is not None:
                return outputs[0], outputs[2]
            target_probs = self.target_distribution.dense(next_token_logits, sampling_info, bs)
        return dspine_accept_sampling(
            target_probs=target_probs, candidates=candidates, target_logits=next_token_logits,
            candidate_ids=candidate_ids, q_rows=q_rows, sampling_info=sampling_info,
            sampling_backend=self.sampling_backend, dense_q=None,
            random_state=getattr(self._dspine_sampler, "random", None))


def accept_dspine_sampled_round(*, candidates, next_token_logits, sampling_info, max_top_k=None,
                                uniform_top_k_value=None, **_dflash_only_arguments):
    """Seam C under DSPINE (called by the plugin's AROUND hook in place of DFlash's
    compute_dflash_sampling_correct_drafts_and_bonus): (accept_len int32 [bs], bonus int64
    [bs]).  Sampling follows the request's ordinary AR target distribution."""
    worker = _active_worker
    if worker is None:
        raise RuntimeError("DSPINE sampled verify reached before the DSpine worker exists")
    return worker._accept_sampled_round(candidates=candidates,
                                        next_token_logits=next_token_logits,
                                        sampling_info=sampling_info, max_top_k=max_top_k,
                                        uniform_top_k_value=uniform_top_k_value)
