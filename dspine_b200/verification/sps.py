"""SPS verify-length allocation (verification/sps.py:27-99 of the reference) on the GPU.

`allocate_verify_lens` keeps the reference's signature and validation and returns the same
lengths (one dsv_sps_plan launch); `sps_plan` also returns qo_indptr and the token index
that the reference's device_plan builds.
"""

from __future__ import annotations

import torch

from .. import _lib

T = 16


def _table(probabilities, depth, gamma):
    """The [gamma, nbins] conditional table the reference indexes as probabilities[depth, bins];
    depth must select the same row for every request (the reference passes arange(gamma))."""
    depth = torch.as_tensor(depth, device=probabilities.device)
    if depth.dim() == 0:
        depth = depth.expand(gamma)
    if depth.dim() == 2:
        if not bool((depth == depth[:1]).all()):
            raise ValueError("per-request depth rows are not supported")
        depth = depth[0]
    if depth.shape != (gamma,):
        raise ValueError("depth must index one table row per draft depth")
    return probabilities[depth.long()].float().contiguous()


def sps_plan(raw, probabilities, depth, budget, boundaries=None):
    bs, gamma = raw.shape
    full = gamma + 1
    if not bs <= budget <= bs * full:
        raise ValueError("SPS budget must include every root and fit the draft block")
    if full != T:
        raise ValueError("dspine_b200 plans 16-token draft blocks")
    if raw.device.type != "cuda":
        raise ValueError("dspine_b200 plans on CUDA tensors only")
    table = _table(probabilities, depth, gamma)
    raw = raw.float().contiguous()
    bnd = None if boundaries is None else boundaries.float().contiguous()
    dev = raw.device
    lens = torch.empty(bs, dtype=torch.int32, device=dev)
    qo = torch.empty(bs + 1, dtype=torch.int64, device=dev)
    index = torch.empty(int(budget), dtype=torch.int64, device=dev)
    _lib.call("dsv_sps_plan", bs, raw.data_ptr(), table.data_ptr(), table.shape[-1],
              _lib.ptr(bnd), 0 if bnd is None else bnd.numel(), int(budget), lens.data_ptr(),
              qo.data_ptr(), index.data_ptr(), torch.cuda.current_stream(dev).cuda_stream)
    return lens, qo, index


def allocate_verify_lens(raw, probabilities, depth, budget, boundaries=None):
    """Keep the highest-survival prefixes, including one root per request."""
    return sps_plan(raw, probabilities, depth, budget, boundaries)[0]


class RaggedVerifyLayout:
    """The device half of SGLang's RaggedVerifyLayout that the ragged verify path reads:
    per-request verify lengths, their exclusive scan (qo_indptr_device [B+1]) and the token
    budget.  When SGLang is importable, `device_plan` returns SGLang's own layout instead."""

    def __init__(self, verify_lens, qo_indptr_device, graph_num_tokens, total_verify_tokens):
        self.verify_lens = verify_lens
        self.qo_indptr_device = qo_indptr_device
        self.graph_num_tokens = int(graph_num_tokens)
        self.total_verify_tokens = int(total_verify_tokens)

    @classmethod
    def _assemble_device(cls, *, verify_lens, graph_num_tokens, total_verify_tokens,
                         qo_indptr=None):
        if qo_indptr is None:
            qo_indptr = torch.zeros(verify_lens.numel() + 1, device=verify_lens.device,
                                    dtype=torch.int64)
            qo_indptr[1:] = verify_lens.to(torch.int64).cumsum(0)
        return cls(verify_lens, qo_indptr, graph_num_tokens, total_verify_tokens)


def _layout_class():
    try:
        from sglang.srt.speculative.ragged_verify import RaggedVerifyLayout as sglang_layout
    except ImportError:
        return None
    return sglang_layout


def device_plan(raw, probabilities, depth, budget, cfg, graph_tokens=None, boundaries=None, *,
                tp=None):
    """(layout, index) of one SPS round (verification/sps.py:61-99): the verify lengths of
    allocate_verify_lens, their layout and index[qo[b] + t] = b * 16 + t, from one
    dsv_sps_plan launch.  Under TP the lengths are synchronised from the leader and the index
    is rebuilt on the device from the synchronised lengths (no host read)."""
    if cfg.min_verify_len != 1 or cfg.survival_eps != 0.0:
        raise ValueError("DSpine SPS requires one root per request and no survival cutoff")
    bs, gamma = raw.shape
    full = gamma + 1
    if graph_tokens is None:
        graph_tokens = budget
    if graph_tokens != budget:
        raise ValueError("SPS graph tier must equal the verified token budget")
    lens, qo, index = sps_plan(raw, probabilities, depth, budget, boundaries)
    if tp is not None:
        tp.sync_tensor(lens)
        qo = torch.zeros_like(qo)
        qo[1:] = lens.to(torch.int64).cumsum(0)
        token = torch.arange(budget, device=raw.device)
        row = torch.searchsorted(qo[1:], token, right=True)
        index = row * full + token - qo[row]
    sglang_layout = _layout_class()
    if sglang_layout is not None:
        layout = sglang_layout._assemble_device(verify_lens=lens, graph_num_tokens=graph_tokens,
                                                total_verify_tokens=budget)
    else:
        layout = RaggedVerifyLayout._assemble_device(verify_lens=lens,
                                                     graph_num_tokens=graph_tokens,
                                                     total_verify_tokens=budget, qo_indptr=qo)
    return layout, index
