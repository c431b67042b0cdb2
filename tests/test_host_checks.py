"""Argument checks of the host modules, on the CPU: each mirror raises the reference's
ValueError (same message) before anything is launched, and valid CPU tensors are refused
with a ValueError instead of running anywhere else (there is no CPU fallback).

Reference checks: sampling/rejection.py:113-138 (sample_capped_chain_from_probs),
sampling/random.py:72-81 (seeded_uniforms), verification/sps.py:39-40 (allocate_verify_lens
budget), kernels/dspine.py:172-188 (topk_ids).  The "16-token draft blocks" and "CUDA tensors
only" checks are this library's own."""

import pytest
import torch

from dspine_b200.kernels import dspine as K
from dspine_b200.sampling import random as R
from dspine_b200.sampling.rejection import sample_capped_chain_from_probs
from dspine_b200.verification import sps


def _chain_args(bs=2, V=50, **override):
    a = dict(
        candidates=torch.zeros(bs, 16, dtype=torch.int64),
        target_probs=torch.zeros(bs, 16, V),
        draft_probs=torch.zeros(bs, 15, V),
        verify_lens=torch.ones(bs, dtype=torch.int32),
        uniforms=torch.zeros(bs, 15),
        uniform_final=torch.zeros(bs),
        prefix_lens=torch.zeros(bs, dtype=torch.int32),
        outputs=(torch.zeros(bs, dtype=torch.int32), torch.zeros(bs, dtype=torch.int32),
                 torch.zeros(bs, dtype=torch.int64), torch.zeros(bs, 16, dtype=torch.int64),
                 torch.zeros(bs, dtype=torch.int32)),
    )
    a.update(override)
    return a


@pytest.mark.parametrize("override,message", [
    (dict(candidates=torch.zeros(2, 15, dtype=torch.int64)), "requires target \\[B,16,V\\]"),
    (dict(target_probs=torch.zeros(2, 16, 50)[:, :, :49]), "requires draft q \\[B,15,V\\]"),
    (dict(draft_probs=torch.zeros(2, 14, 50)), "requires draft q \\[B,15,V\\]"),
    (dict(verify_lens=torch.ones(3, dtype=torch.int32)), "Invalid cap or uniform layout"),
    (dict(uniforms=torch.zeros(2, 16)), "Invalid cap or uniform layout"),
    (dict(uniform_final=torch.zeros(3)), "Invalid final uniform or prefix layout"),
    (dict(outputs=()), "Expected accept/commit/bonus/output/new_seq buffers"),
    (dict(target_probs=torch.zeros(2, 50, 16).transpose(1, 2)), "requires contiguous tensors"),
    ({}, "on CUDA tensors only"),
])
def test_sample_capped_chain_checks(override, message):
    with pytest.raises(ValueError, match=message):
        sample_capped_chain_from_probs(**_chain_args(**override))


def test_seeded_uniform_checks():
    s = torch.zeros(4, dtype=torch.int64)
    with pytest.raises(ValueError, match="matching request vectors"):
        R.seeded_uniforms(s, torch.zeros(3, dtype=torch.int64), 16, 0)
    with pytest.raises(ValueError, match="int64 seeds and integer positions"):
        R.seeded_uniforms(s.int(), torch.zeros(4, dtype=torch.int64), 16, 0)
    with pytest.raises(ValueError, match="Invalid seeded uniform layout"):
        R.seeded_uniforms(s, torch.zeros(4, dtype=torch.int64), 0, 0)
    with pytest.raises(ValueError, match="on CUDA tensors only"):
        R.seeded_uniforms(s, torch.zeros(4, dtype=torch.int64), 16, 0)


def test_sps_plan_checks():
    raw = torch.zeros(4, 15)
    probs = torch.full((15, 16), 0.5)
    depth = torch.arange(15)
    with pytest.raises(ValueError, match="budget must include every root"):
        sps.sps_plan(raw, probs, depth, 3)
    with pytest.raises(ValueError, match="16-token draft blocks"):
        sps.sps_plan(torch.zeros(4, 7), probs, depth, 8)
    with pytest.raises(ValueError, match="on CUDA tensors only"):
        sps.sps_plan(raw, probs, depth, 8)


def test_topk_ids_refuses_cpu_tensors():
    with pytest.raises(ValueError, match="on CUDA tensors only"):
        K.topk_ids(torch.zeros(2, 4096), 4)
