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
