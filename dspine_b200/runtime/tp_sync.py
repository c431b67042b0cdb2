"""Tensor-parallel sharing of acceptance buffers (runtime/tp_sync.py:67-106 of the reference).

With the vocab-parallel head of this package every rank computes identical accept decisions
from the same gathered candidates (dspine_b200.lmhead.TPHead.topk_lse), so no broadcast is
needed on that path.  `TpCoordinator.sync_accept` is kept for callers that decide on one rank:
it packs the buffers into one int64 packet, broadcasts it from the group's first rank and
copies it back in place (the buffers keep their storage, so CUDA-graph pointers stay valid).
"""

import torch


class TpCoordinator:
    def __init__(self, group=None, enabled=True):
        import torch.distributed as dist
        self._dist = dist
        self.group = group
        self.enabled = bool(enabled) and dist.is_initialized() and dist.get_world_size(group) > 1
        self._accept_packets = {}

    def sync_tensor(self, tensor):
        src = self._dist.get_global_rank(self.group, 0) if self.group is not None else 0
        self._dist.broadcast(tensor, src=src, group=self.group)

    def sync_accept(self, *values):
        """Share existing acceptance buffers in place, before cache updates."""
        self._sync_values(tuple(v for v in values if v is not None), self._accept_packets)
        return values

    def _sync_values(self, values, packets):
        if not self.enabled or not values:
            return
        size = sum(v.numel() for v in values)
        key = (values[0].device, size)
        packet = packets.get(key)
        if packet is None:
            packet = torch.empty(size, device=values[0].device, dtype=torch.int64)
            packets[key] = packet
        offset = 0
        for v in values:
            end = offset + v.numel()
            packet[offset:end].copy_(v.reshape(-1))
            offset = end
        self.sync_tensor(packet)
        offset = 0
        for v in values:
            end = offset + v.numel()
            v.copy_(packet[offset:end].view_as(v))
            offset = end
