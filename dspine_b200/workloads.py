"""Seeded synthetic workloads of the benchmark configurations (no dataset is involved).

Config 0: 4 requests x 16, vocab 151936, fp32 logits; requests 0-1 greedy, 2-3 temperature 1.
Config 1: 64 requests, verify length U{1..16}, vocab 151936, bf16 logits; temperature
          U[0, 1.5] with 25% exactly 0; top_k from {off, 1, 20, 50}; top_p U[0.8, 1];
          KV slots a random permutation of 0..65535 (page size 1).
Config 4: 256 requests, draft length U{1..16} capped by an SPS width table (batch-size bucket
          -> width, seeded ints 4..16) and by an early stop at the first draft position whose
          draft-token probability is below 0.3; temperatures half 0, half 1; 131072 KV slots.

Target logits ~ N(0, 2.5^2) plus +8 at one seeded token per row; draft logits = target +
N(0, 1).  Drafted tokens are sampled from the draft distribution (greedy requests: its
argmax); "off" top-k is encoded as 1 << 30 like SGLang.  Everything is generated with
torch.Generator seeds on the host, so the CPU oracle and the GPU see identical inputs.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np
import torch

T = 16
VOCAB = 151936
TOPK_OFF = 1 << 30


@dataclass
class Batch:
    """Inputs of one verification call; tensors live on `device`."""

    V: int
    candidates: torch.Tensor
    target_logits: torch.Tensor
    target_rows: torch.Tensor
    draft_logits: torch.Tensor | None
    draft_rows: torch.Tensor | None
    temperature: torch.Tensor
    top_k: torch.Tensor
    top_p: torch.Tensor
    verify_lens: torch.Tensor
    uniforms: torch.Tensor
    uniform_final: torch.Tensor
    prefix_lens: torch.Tensor
    slots: torch.Tensor | None = None
    slot_rows: torch.Tensor | None = None
    meta: dict = field(default_factory=dict)

    @property
    def B(self) -> int:
        return int(self.candidates.shape[0])

    def kwargs(self) -> dict:
        return dict(candidates=self.candidates, target_logits=self.target_logits,
                    target_rows=self.target_rows, draft_logits=self.draft_logits,
                    draft_rows=self.draft_rows, temperature=self.temperature, top_k=self.top_k,
                    top_p=self.top_p, verify_lens=self.verify_lens, uniforms=self.uniforms,
                    uniform_final=self.uniform_final, prefix_lens=self.prefix_lens)

    def to(self, device) -> "Batch":
        def mv(t):
            return None if t is None else t.to(device)
        return Batch(self.V, *(mv(getattr(self, n)) for n in (
            "candidates", "target_logits", "target_rows", "draft_logits", "draft_rows",
            "temperature", "top_k", "top_p", "verify_lens", "uniforms", "uniform_final",
            "prefix_lens", "slots", "slot_rows")), meta=dict(self.meta))

    def algorithmic_bytes(self) -> int:
        """Bytes the verification must read: every verify row of the target, and every draft
        row of a sampled request that can be consulted (positions < len-1)."""
        esz = self.target_logits.element_size()
        lens = self.verify_lens.cpu().long()
        greedy = _greedy_mask(self.temperature.cpu(), self.top_k.cpu())
        rows = int(lens.sum())
        if self.draft_logits is not None:
            rows += int(((lens - 1).clamp_min(0) * (~greedy)).sum())
        return rows * self.V * esz

    def deciding_bytes(self, accept) -> int:
        """Bytes of the rows the outcome depends on, given the accepted lengths: target rows
        0..accept and, for sampled requests with draft logits, draft rows 0..min(accept,
        len - 2) (a chain stops at its first rejected step; later rows are never consulted)."""
        esz = self.target_logits.element_size()
        lens = self.verify_lens.cpu().long()
        acc = torch.as_tensor(accept).cpu().long()
        greedy = _greedy_mask(self.temperature.cpu(), self.top_k.cpu())
        rows = int((acc + 1).sum())
        if self.draft_logits is not None:
            rows += int(((torch.minimum(acc + 1, lens - 1)).clamp_min(0) * (~greedy)).sum())
        return rows * self.V * esz

    def verified_tokens(self) -> int:
        return int(self.verify_lens.sum())


def _greedy_mask(temperature, top_k):
    return (top_k <= 1) | ~(temperature > 0)


def _filtered_probs(logits: torch.Tensor, T: torch.Tensor, k: torch.Tensor, p: torch.Tensor):
    """Approximate filtered softmax used only to draw the synthetic drafts (fp32, torch)."""
    x = logits.float() / T.clamp_min(1e-6)[:, None]
    probs = torch.softmax(x, -1)
    sp, si = probs.sort(-1, descending=True)
    ahead = sp.cumsum(-1) - sp
    rank = torch.arange(probs.shape[-1])[None, :]
    keep = (rank < k.clamp_max(probs.shape[-1])[:, None]) & (ahead <= p[:, None])
    keep[:, 0] = True
    sp = torch.where(keep, sp, torch.zeros_like(sp))
    out = torch.zeros_like(probs).scatter_(-1, si, sp)
    return out / out.sum(-1, keepdim=True)


def _logits(rows: int, V: int, g: torch.Generator):
    x = torch.randn(rows, V, generator=g) * 2.5
    spike = torch.randint(0, V, (rows,), generator=g)
    x[torch.arange(rows), spike] += 8.0
    return x


def build(lens, temperature, top_k, top_p, V=VOCAB, dtype=torch.bfloat16, seed=0,
          with_draft=True, slots_space=65536, device="cpu") -> Batch:
    """Assemble a batch: packed target rows (sum lens) and packed draft rows (sum lens-1)."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.as_tensor(lens, dtype=torch.int32)
    B = lens.numel()
    temperature = torch.as_tensor(temperature, dtype=torch.float32)
    top_k = torch.as_tensor(top_k, dtype=torch.int32)
    top_p = torch.as_tensor(top_p, dtype=torch.float32)
    tgt_rows = torch.zeros(B, dtype=torch.int64)
    tgt_rows[1:] = lens.long().cumsum(0)[:-1]
    nd = (lens.long() - 1).clamp_min(0)
    drf_rows = torch.zeros(B, dtype=torch.int64)
    drf_rows[1:] = nd.cumsum(0)[:-1]
    R = int(lens.sum())
    target = _logits(R, V, g)
    draft = None
    if with_draft:
        draft = torch.empty(max(int(nd.sum()), 1), V)
        for b in range(B):
            n = int(nd[b])
            if n:
                t0, d0 = int(tgt_rows[b]), int(drf_rows[b])
                draft[d0:d0 + n] = target[t0:t0 + n] + torch.randn(n, V, generator=g)
    target = target.to(dtype)
    if draft is not None:
        draft = draft.to(dtype)
    greedy = _greedy_mask(temperature, top_k)
    cand = torch.zeros(B, T, dtype=torch.int64)
    cand[:, 0] = torch.randint(0, V, (B,), generator=g)
    for b in range(B):
        n = int(nd[b])
        if n == 0:
            continue
        src = draft[int(drf_rows[b]):int(drf_rows[b]) + n] if draft is not None else \
            target[int(tgt_rows[b]):int(tgt_rows[b]) + n]
        if bool(greedy[b]):
            cand[b, 1:1 + n] = src.float().argmax(-1)
        else:
            q = _filtered_probs(src, temperature[b].expand(n), top_k[b].expand(n), top_p[b].expand(n))
            cand[b, 1:1 + n] = torch.multinomial(q, 1, generator=g)[:, 0]
    uniforms = torch.rand(B, T - 1, generator=g)
    uniform_final = torch.rand(B, generator=g)
    prefix = torch.randint(0, 4096, (B,), generator=g, dtype=torch.int32)
    slots = torch.randperm(slots_space, generator=g)[:B * T].to(torch.int32)
    slot_rows = torch.arange(B, dtype=torch.int64) * T
    batch = Batch(V, cand, target, tgt_rows, draft, drf_rows if draft is not None else None,
                  temperature, top_k, top_p, lens, uniforms, uniform_final, prefix, slots,
                  slot_rows, meta={"seed": seed})
    return batch.to(device)


def config0(seed=0, device="cpu", V=VOCAB) -> Batch:
    lens = [16, 16, 16, 16]
    return build(lens, [0.0, 0.0, 1.0, 1.0], [1, 1, TOPK_OFF, TOPK_OFF], [1.0] * 4, V=V,
                 dtype=torch.float32, seed=seed, device=device)


def config1_params(B=64, seed=1):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, T + 1, (B,), generator=g, dtype=torch.int32)
    temperature = torch.rand(B, generator=g) * 1.5
    temperature[torch.rand(B, generator=g) < 0.25] = 0.0
    choices = torch.tensor([TOPK_OFF, 1, 20, 50], dtype=torch.int32)
    top_k = choices[torch.randint(0, 4, (B,), generator=g)]
    top_p = 0.8 + 0.2 * torch.rand(B, generator=g)
    return lens, temperature, top_k, top_p


def config1(seed=1, device="cpu", V=VOCAB, B=64) -> Batch:
    lens, temperature, top_k, top_p = config1_params(B, seed)
    return build(lens, temperature, top_k, top_p, V=V, dtype=torch.bfloat16, seed=seed + 100,
                 device=device)


def subset(batch: Batch, requests) -> Batch:
    """The requests `requests` of `batch` (in that order) as a batch of their own: their
    target and draft rows repacked, every per-request tensor indexed.  The rows are the very
    rows of the parent batch, so results on a subset equal the parent's for those requests."""
    idx = torch.as_tensor(list(requests), dtype=torch.int64)
    lens = batch.verify_lens.cpu()[idx]
    nd = (lens.long() - 1).clamp_min(0)

    def rows_of(src, starts, counts):
        parts = [src[int(s):int(s) + int(n)] for s, n in zip(starts, counts)]
        return torch.cat(parts) if parts else src[:0]

    tgt = rows_of(batch.target_logits.cpu(), batch.target_rows.cpu()[idx], lens)
    tgt_rows = torch.zeros(idx.numel(), dtype=torch.int64)
    tgt_rows[1:] = lens.long().cumsum(0)[:-1]
    draft = draft_rows = None
    if batch.draft_logits is not None:
        draft = rows_of(batch.draft_logits.cpu(), batch.draft_rows.cpu()[idx], nd)
        if draft.shape[0] == 0:
            draft = batch.draft_logits.cpu()[:1]
        draft_rows = torch.zeros(idx.numel(), dtype=torch.int64)
        draft_rows[1:] = nd.cumsum(0)[:-1]
    slots = slot_rows = None
    if batch.slots is not None:
        slots = rows_of(batch.slots.cpu(), batch.slot_rows.cpu()[idx], lens)
        slot_rows = tgt_rows.clone()

    def pick(t):
        return t.cpu()[idx].contiguous()
    sub = Batch(batch.V, pick(batch.candidates), tgt, tgt_rows, draft, draft_rows,
                pick(batch.temperature), pick(batch.top_k), pick(batch.top_p), lens.contiguous(),
                pick(batch.uniforms), pick(batch.uniform_final), pick(batch.prefix_lens), slots,
                slot_rows, meta=dict(batch.meta, subset=idx.tolist()))
    return sub.to(batch.candidates.device)


def config1_subset(n=16, seed=1, device="cpu") -> Batch:
    """The first n requests of the config 1 batch (the benchmark's own rows)."""
    return subset(config1(seed=seed), range(n)).to(device)


def fingerprint(batch: Batch) -> str:
    """SHA-256 of the raw bytes of the logits, candidates and uniforms: a check that a
    regenerated batch is bit for bit the one a fixture was made from."""
    import hashlib

    h = hashlib.sha256()
    for t in (batch.target_logits, batch.draft_logits, batch.candidates, batch.uniforms,
              batch.uniform_final):
        if t is not None:
            h.update(t.detach().cpu().contiguous().view(torch.uint8).numpy().tobytes())
    return h.hexdigest()


def config4(seed=4, device="cpu", V=VOCAB, B=256) -> Batch:
    """Dynamic-verification stress; verify lengths come from an SPS width table and an early
    stop on draft confidence (restated rule: no such rule exists in the reference)."""
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, T + 1, (B,), generator=g, dtype=torch.int32)
    buckets = [1, 2, 4, 8, 16, 32, 64, 128, 256]
    widths = {bs: int(w) for bs, w in zip(buckets, torch.randint(4, 17, (len(buckets),), generator=g))}
    # the verify width of the batch's bucket from an SPS policy holding that table (the
    # reference's DSpineSpsPolicy.width, verification/policy.py)
    from dspine_b200.verification.policy import SpsPolicy
    policy = SpsPolicy(verify_widths=widths)
    width = policy.width(min(bk for bk in buckets if bk >= B)) if B <= 256 else 16
    temperature = torch.where(torch.arange(B) % 2 == 0, torch.zeros(B), torch.ones(B))
    top_k = torch.where(temperature == 0, torch.ones(B, dtype=torch.int32),
                        torch.full((B,), TOPK_OFF, dtype=torch.int32))
    top_p = torch.ones(B)
    caps = torch.minimum(lens, torch.full_like(lens, width))
    batch = build(lens, temperature, top_k, top_p, V=V, dtype=torch.bfloat16, seed=seed + 100,
                  slots_space=131072, device="cpu")
    # early stop: draft-token probability under its own (approximate) draft distribution
    conf = torch.ones(B, T - 1)
    for b in range(B):
        n = int(lens[b]) - 1
        if n <= 0:
            continue
        d0 = int(batch.draft_rows[b])
        q = _filtered_probs(batch.draft_logits[d0:d0 + n].float(), temperature[b].expand(n).clamp_min(1e-6)
                            if temperature[b] > 0 else torch.ones(n), top_k[b].expand(n), top_p[b].expand(n))
        if temperature[b] == 0:
            conf[b, :n] = 1.0
        else:
            conf[b, :n] = q.gather(1, batch.candidates[b, 1:1 + n, None])[:, 0]
    stop = torch.full((B,), T, dtype=torch.int32)
    for b in range(B):
        low = (conf[b] < 0.3).nonzero()
        if low.numel():
            stop[b] = int(low[0, 0]) + 1
    batch.verify_lens = torch.minimum(caps, stop).clamp_min(1).to(torch.int32)
    batch.meta.update({"sps_width": width, "early_stop": 0.3})
    return batch.to(device)
