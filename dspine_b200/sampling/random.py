"""Request-seeded uniforms (sampling/random.py:22-118 of the reference) on the GPU.

`seeded_uniforms` keeps the reference's signature, validation and results: CUDA tensors go
through dsv_uniforms (bit-exact with the reference's `_cpu_uniforms`); CPU tensors are
refused, since this package has no CPU path.
"""

from __future__ import annotations

import torch

from .. import _lib

DRAFT, ACCEPT, BONUS, PREFILL = range(4)


def seeded_uniforms(seeds, positions, width, stream):
    if seeds.ndim != 1 or positions.shape != seeds.shape:
        raise ValueError("Seeds and positions must be matching request vectors")
    if seeds.dtype != torch.int64 or positions.dtype not in (torch.int32, torch.int64):
        raise ValueError("Expected int64 seeds and integer positions")
    if seeds.device != positions.device or not 0 < width < 65536 or stream not in range(4):
        raise ValueError("Invalid seeded uniform layout")
    if seeds.device.type != "cuda":
        raise ValueError("dspine_b200 draws uniforms on CUDA tensors only")
    seeds, positions = seeds.contiguous(), positions.contiguous()
    out = torch.empty((seeds.numel(), width), device=seeds.device, dtype=torch.float32)
    _lib.call("dsv_uniforms", seeds.numel(), int(width), seeds.data_ptr(), positions.data_ptr(),
              int(positions.dtype == torch.int64), int(stream), out.data_ptr(),
              torch.cuda.current_stream(seeds.device).cuda_stream)
    return out


class RequestRNG:
    def __init__(self, tp=None):
        self.seeds = self.positions = None
        self.tp = tp

    def stage(self, seeds, positions):
        self.seeds = seeds
        self.positions = positions.clone() if seeds is not None else None

    def draw(self, width, stream):
        return seeded_uniforms(self.seeds, self.positions, width, stream)


def verification_uniforms(bs, width, device, random_state=None):
    """(accept uniforms [bs, width-1], bonus uniforms [bs]) as the reference's
    verification_uniforms: seeded draws when a request order is staged, else torch.rand."""
    if random_state is None or random_state.seeds is None:
        tp = getattr(random_state, "tp", None)
        if tp is not None and tp.enabled:
            return tp.uniforms((bs, width - 1), device), tp.uniforms((bs,), device)
        return (torch.rand((bs, width - 1), device=device, dtype=torch.float32),
                torch.rand((bs,), device=device, dtype=torch.float32))
    if random_state.seeds.numel() != bs:
        raise RuntimeError("Seeded verification request order was not staged")
    return random_state.draw(width - 1, ACCEPT), random_state.draw(1, BONUS).view(bs)
