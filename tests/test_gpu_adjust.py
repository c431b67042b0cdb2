"""Parity of the fused logit adjustments (dsv_adjust_logits) with the reference's torch ops
(sampling/compact.py:14-79: add_, torch.where(l < 0, l * s, l / s), masked -inf, add_) on
the same tensors, bf16 and fp32, packed (row_to_request) and full-block layouts: bitwise."""

from types import SimpleNamespace

import pytest
import torch

from dspine_b200.sampling.compact import adjust_logits

pytestmark = pytest.mark.gpu

DEV = "cuda"


def reference(logits, info, row_to_request):
    def mapped(v):
        v = v.to(logits.device)
        return v.index_select(0, row_to_request) if row_to_request is not None else v[:, None, :]
    logits.add_(mapped(info.acc_additive_penalties))
    s = mapped(info.acc_scaling_penalties)
    logits.copy_(torch.where(logits < 0, logits * s, logits / s))
    words = info.grammar_mask.vocab_mask
    V = logits.shape[-1]
    bits = ((words[:, :, None] >> torch.arange(32, device=words.device)) & 1).reshape(words.shape[0], -1)[:, :V].bool()
    allowed = bits.index_select(0, row_to_request) if row_to_request is not None else bits[:, None, :]
    logits.masked_fill_(~allowed, float("-inf"))
    logits.add_(mapped(info.logit_bias))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("packed", [False, True])
def test_adjust_logits_matches_torch(dtype, packed):
    g = torch.Generator(device=DEV).manual_seed(7)
    B, T, V = 6, 16, 4099
    words = (V + 31) // 32
    info = SimpleNamespace(
        acc_additive_penalties=torch.randn(B, V, generator=g, device=DEV),
        acc_scaling_penalties=1.0 + torch.rand(B, V, generator=g, device=DEV),
        grammar_mask=SimpleNamespace(vocab_mask=torch.randint(-2**31, 2**31 - 1, (B, words), generator=g,
                                                              device=DEV, dtype=torch.int64).to(torch.int32)),
        logit_bias=torch.randn(B, V, generator=g, device=DEV) * 0.5)
    if packed:
        rows = 37
        r2r = torch.randint(0, B, (rows,), generator=g, device=DEV)
        x = (torch.randn(rows, V, generator=g, device=DEV) * 3).to(dtype)
    else:
        r2r = None
        x = (torch.randn(B, T, V, generator=g, device=DEV) * 3).to(dtype)
    want = x.clone()
    reference(want, info, r2r)
    adjust_logits(x, info, r2r)
    torch.cuda.synchronize()
    assert torch.equal(x.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                       want.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))
