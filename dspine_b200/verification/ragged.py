"""Ragged verification acceptance (verification/ragged.py of the reference) on the GPU.

`RaggedVerifyCaps.accept` keeps the reference's signature and 5-tuple (ragged.py:282-335):
per-request verify lengths from the round's layout (``layout.verify_lens``).  Greedy rounds
take the target's top-1 of the full 16-row envelope (the controller's prepare step pads the
packed rows back to it) and dsv_accept_greedy with those lengths (ragged.py:51-76 `_accept`);
sampled rounds go to `accept_sampled_prefix`, with the compact row mapping when the round
verified packed rows.  The controller's SGLang half (attention backends and CUDA-graph
runners of the ragged target forward) is outside this package; a controller sets
``ragged_round``, ``batch_size``, ``tokens`` / ``executed_tokens``, ``layout``,
``compact_round``, ``row_offsets`` and ``row_to_request``.

The data steps around that forward are here: `compact_window` (ragged.py:192-200: the verify
input's draft tokens, positions and KV slots gathered to the SPS window, the layout attached,
the originals kept for `restore_window`) and `expand_rows` (ragged.py:257-266: packed target
rows scattered back into the full [bs * 16, V] envelope over neutral padding rows, and the
packed row -> request mapping of compact rounds).
"""

from __future__ import annotations

import torch

from .. import accept as _accept
from ..sampling.padding import logits_padding
from .caps import VerifyCaps, target_top1


def compact_window(verify_input, batch, window_index, layout):
    """Gather the verify input to the SPS window (flat request * full + position indices) and
    attach the ragged layout; returns what `restore_window` needs."""
    saved = (verify_input, verify_input.draft_token, verify_input.positions,
             getattr(verify_input, "ragged_verify_layout", None),
             getattr(verify_input, "kv_loc_cols", None), batch, batch.out_cache_loc)
    verify_input.draft_token = verify_input.draft_token.index_select(0, window_index)
    verify_input.positions = verify_input.positions.index_select(0, window_index)
    verify_input.ragged_verify_layout = layout
    verify_input.kv_loc_cols = window_index
    batch.out_cache_loc = batch.out_cache_loc.index_select(0, window_index)
    return saved


def restore_window(saved):
    (verify_input, verify_input.draft_token, verify_input.positions,
     verify_input.ragged_verify_layout, verify_input.kv_loc_cols, batch,
     batch.out_cache_loc) = saved


def expand_rows(controller, packed, window_index, bs, full=16, logits=True):
    """Packed rows of the window back at their (request, position) rows of the full envelope;
    the other rows neutral (logits: one-point padding rows, other tensors: zeros)."""
    shape = (bs * full, packed.shape[-1])
    rows = logits_padding(controller, packed, shape) if logits else packed.new_zeros(shape)
    rows.index_copy_(0, window_index, packed)
    return rows


def window_requests(window_index, full=16):
    """The request of every packed row (compact rounds' row -> request mapping)."""
    return window_index.div(full, rounding_mode="floor")


class RaggedVerifyCaps(VerifyCaps):
    def __init__(self, worker, *, full=16, active=None):
        super().__init__(worker, full=full, active=active)
        self.ragged_round = False
        self.compact_round = False
        self.batch_size = 0
        self.tokens = self.executed_tokens = 0
        self.layout = None
        self.row_offsets = self.row_to_request = None

    def accept(self, *, candidates, next_token_logits, sampling_info, draft_input, prefix_lens,
               bs):
        if not self.ragged_round:
            return super().accept(candidates=candidates, next_token_logits=next_token_logits,
                                  sampling_info=sampling_info, draft_input=draft_input,
                                  prefix_lens=prefix_lens, bs=bs)
        if bs != self.batch_size or self.executed_tokens != self.tokens:
            raise RuntimeError("Ragged acceptance requires confirmed packed verification")
        if self.sampled_round:
            from ..sampling.rejection import accept_sampled_prefix

            return accept_sampled_prefix(
                self, candidates=candidates, next_token_logits=next_token_logits,
                sampling_info=sampling_info, prefix_lens=prefix_lens, bs=bs,
                verify_lens=self.layout.verify_lens,
                row_offsets=self.row_offsets if self.compact_round else None,
                row_to_request=self.row_to_request if self.compact_round else None)
        top1 = target_top1(next_token_logits, bs, self.full)
        outputs = self.worker._next_accept_bonus_buffers(bs)
        return _accept.accept_greedy(candidates, top1,
                                     self.layout.verify_lens.to(torch.int32).contiguous(),
                                     prefix_lens.to(torch.int32), outputs=outputs)
