"""Parity of the logit adjustments (dsv_adjust_logits behind sampling/compact.py adjust_logits)
with the reference's own adjust_logits (sampling/compact.py:14-79, pure torch), run on CPU
tensors by tests/golden/make_golden.py (adjust.npz): additive and scaling penalties, an
orchestrator with a multiplicative, an idle and an additive penalizer, a grammar bitmask
applied through the grammar's own apply_vocab_mask (xgrammar semantics) and a logit bias; full
[B, T, V] blocks and packed rows with row_to_request; bf16 and fp32 logits.  Bitwise."""

from pathlib import Path
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from dspine_b200.sampling.compact import adjust_logits

pytestmark = pytest.mark.gpu

DEV = "cuda"
FIX = np.load(Path(__file__).resolve().parent / "golden" / "adjust.npz")


class Info(SimpleNamespace):
    def __len__(self):
        return self.acc_additive_penalties.shape[0]


def case_info(ci, grammar_mask):
    def t(name):
        return torch.from_numpy(FIX[f"c{ci}_{name}"]).to(DEV)
    pen_scale, pen_add = t("pen_scale"), t("pen_add")
    mult = SimpleNamespace(is_prepared=lambda: True, is_multiplicative=True,
                           get_scaling_penalties=lambda: pen_scale)
    addp = SimpleNamespace(is_prepared=lambda: True, is_multiplicative=False,
                           apply=lambda b: b.add_(pen_add))
    idle = SimpleNamespace(is_prepared=lambda: False, is_multiplicative=False)
    return Info(acc_additive_penalties=t("add"), acc_scaling_penalties=t("scl"),
                penalizer_orchestrator=SimpleNamespace(is_required=True,
                                                       penalizers={"m": mult, "i": idle, "a": addp}),
                grammar_mask=grammar_mask(t("mask")), logit_bias=t("bias"))


def run_case(ci, grammar_mask):
    dtype = torch.bfloat16 if bool(FIX[f"c{ci}_bf16"]) else torch.float32
    x = torch.from_numpy(FIX[f"c{ci}_x"]).to(dtype).to(DEV)
    r2r = FIX[f"c{ci}_r2r"]
    r2r = torch.from_numpy(r2r).to(DEV) if r2r.size else None
    adjust_logits(x, case_info(ci, grammar_mask), r2r)
    torch.cuda.synchronize()
    want = torch.from_numpy(FIX[f"c{ci}_y"]).to(dtype)
    return x.cpu(), want


@pytest.mark.parametrize("ci", range(int(FIX["n"])))
def test_adjust_logits_matches_reference(ci):
    got, want = run_case(ci, lambda m: SimpleNamespace(vocab_mask=m))
    assert torch.equal(got.float().view(torch.int32), want.float().view(torch.int32))


@pytest.mark.parametrize("ci", range(int(FIX["n"])))
def test_bool_grammar_mask_matches_the_bitmask(ci):
    """A bool mask (True = disallowed) packs to the same allow-bits inside the pass."""
    def as_bool(words):
        V = FIX[f"c{ci}_x"].shape[-1]
        shifts = torch.arange(32, device=DEV, dtype=torch.int32)
        bits = ((words[:, :, None] >> shifts) & 1).reshape(words.shape[0], -1)[:, :V]
        return SimpleNamespace(vocab_mask=bits == 0)
    got, want = run_case(ci, as_bool)
    assert torch.equal(got.float().view(torch.int32), want.float().view(torch.int32))


def test_other_mask_layouts_use_the_grammars_own_apply():
    """A mask of another layout goes to grammar.apply_vocab_mask with rows mapped as the
    reference maps them (repeat_interleave over full blocks)."""
    seen = {}

    def apply(logits, vocab_mask):
        seen["rows"] = vocab_mask.shape[0]
        logits[vocab_mask > 0.5] = float("-inf")

    B, T, V = 2, 16, 97
    x = torch.zeros(B, T, V, device=DEV)
    mask = torch.zeros(B, V, device=DEV, dtype=torch.float16)
    mask[1, 5] = 1
    info = SimpleNamespace(grammar_mask=SimpleNamespace(vocab_mask=mask,
                                                        grammar=SimpleNamespace(apply_vocab_mask=apply)))
    adjust_logits(x, info, None)
    assert seen["rows"] == B * T
    assert torch.isinf(x[1, :, 5]).all() and not torch.isinf(x[0]).any()


@pytest.mark.parametrize("ci", range(int(FIX["n"])))
def test_around_hook_adjusts_full_and_packed_rounds(ci):
    """The plugin's AROUND hook (sampling/compact.py:82-116): without a DSpine worker the
    original runs untouched; with one, a full round adjusts the [bs * T, V] logits as
    [bs, T, V] blocks and a packed round adjusts the controller's packed rows through its row
    mapping; both equal the reference's own adjust_logits."""
    from dspine_b200.runtime import worker as W
    from dspine_b200.sampling.compact import around_verify_logits_adjustments

    dtype = torch.bfloat16 if bool(FIX[f"c{ci}_bf16"]) else torch.float32
    x = torch.from_numpy(FIX[f"c{ci}_x"]).to(dtype).to(DEV)
    r2r = FIX[f"c{ci}_r2r"]
    info = case_info(ci, lambda m: SimpleNamespace(vocab_mask=m))
    want = torch.from_numpy(FIX[f"c{ci}_y"]).to(dtype)
    calls = []

    def original(**kw):
        calls.append(kw)

    rows = x.reshape(-1, x.shape[-1])
    T = x.shape[1] if x.dim() == 3 else 16
    previous = W._active_worker
    try:
        W.set_active_worker(None)
        around_verify_logits_adjustments(original, next_token_logits=rows, sampling_info=info,
                                         draft_token_num=T)
        assert len(calls) == 1 and calls[0]["next_token_logits"] is rows
        if r2r.size:
            ctl = SimpleNamespace(compact_round=True, compact_logits=rows,
                                  row_to_request=torch.from_numpy(r2r).to(DEV))
            W.set_active_worker(SimpleNamespace(verify_caps=ctl))
        else:
            W.set_active_worker(SimpleNamespace(verify_caps=None))
        around_verify_logits_adjustments(original, next_token_logits=rows, sampling_info=info,
                                         draft_token_num=T)
    finally:
        W.set_active_worker(previous)
    torch.cuda.synchronize()
    assert len(calls) == 1
    got = rows.view_as(x).cpu()
    assert torch.equal(got.float().view(torch.int32), want.float().view(torch.int32))


def test_scaling_matches_the_ieee_quotient_for_every_bf16_logit():
    """The scaling step's l / s (l >= 0) takes a reciprocal product away from bf16 rounding
    midpoints; across every finite bf16 logit of both signs and penalties from tiny to huge, the
    result must equal the reference's rule (compact.py:32-34: fp32 l / s or l * s, then bf16)."""
    pos = torch.arange(0, 0x7F80, dtype=torch.int32)                 # +0 .. largest finite
    bits = torch.cat([pos, pos | 0x8000]).to(torch.int16)            # and every negative
    V = bits.numel()
    g = torch.Generator().manual_seed(5)
    B = 12
    logits = bits.view(torch.bfloat16).repeat(B, 1).view(B, 1, V).contiguous()
    scales = torch.empty(B, V)
    for b in range(B - 4):  # random penalties over [0.25, 8)
        scales[b] = torch.exp2(torch.rand(V, generator=g) * 5 - 2)
    scales[B - 4] = 3.0
    scales[B - 3] = 1.0
    scales[B - 2] = 1e-30  # outside the reciprocal's range: the division itself
    scales[B - 1] = 7e29
    want = torch.where(logits.float() < 0, logits.float() * scales[:, None, :],
                       logits.float() / scales[:, None, :]).to(torch.bfloat16)
    x = logits.to(DEV)
    adjust_logits(x, SimpleNamespace(acc_scaling_penalties=scales.to(DEV)), None)
    got = x.cpu()
    same = got.view(torch.int16) == want.view(torch.int16)
    both_nan = torch.isnan(got.float()) & torch.isnan(want.float())
    assert bool((same | both_nan).all())
