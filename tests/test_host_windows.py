"""The widening windows of verify_logits_host, checked on the CPU oracle: verifying the
requests still pending with their lengths capped at W = 2, 4, 8, 16 and keeping each request
once its capped chain stops before the cap (or its length fits the window) gives the outputs
of one verification of the whole batch, bit for bit.  The device call uses the same driver
(`verify.window_stages`); its GPU test is in test_gpu_verify.py."""

import numpy as np
import pytest
import torch

from dspine_b200 import verify, workloads
from tests.helpers import NAMES, oracle_verify


def _batch(seed, B=24, V=1031, accept_all=False):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(1, 17, (B,), generator=g, dtype=torch.int32)
    temperature = torch.rand(B, generator=g) * 1.5
    temperature[torch.rand(B, generator=g) < 0.25] = 0.0
    top_k = torch.tensor([workloads.TOPK_OFF, 1, 20, 50], dtype=torch.int32)[
        torch.randint(0, 4, (B,), generator=g)]
    top_p = 0.8 + 0.2 * torch.rand(B, generator=g)
    batch = workloads.build(lens, temperature, top_k, top_p, V=V, dtype=torch.bfloat16, seed=seed)
    if accept_all:
        batch.draft_logits = batch.target_logits.clone()
        batch.draft_rows = batch.target_rows.clone()
        am = batch.target_logits.float().argmax(dim=1)
        for b in range(B):
            n = int(lens[b])
            r0 = int(batch.target_rows[b])
            batch.candidates[b, 1:n] = am[r0:r0 + n - 1]
    return batch


@pytest.mark.parametrize("seed,accept_all,first", [(1, False, 2), (2, False, 2), (3, True, 2),
                                                   (4, False, 4)])
def test_windows_give_the_outputs_of_the_whole_batch(seed, accept_all, first):
    batch = _batch(seed, accept_all=accept_all)
    want = oracle_verify(batch)
    lens = batch.verify_lens.numpy()
    got = [np.zeros_like(w) for w in want]

    def run_stage(pending, lo, W):
        sub = workloads.subset(batch, pending)
        sub.verify_lens = sub.verify_lens.clamp(max=W)
        res = oracle_verify(sub)

        def keep(positions):
            for full, part in zip(got, res):
                full[np.asarray(pending)[positions]] = part[positions]

        return res[0].tolist(), keep

    windows = verify.window_stages(lens, first, run_stage)
    for name, g, w in zip(NAMES, got, want):
        assert np.array_equal(g, w), name
    assert windows[0] == first and windows[-1] <= 16 * 2
    if accept_all:  # every step accepted: the windows grow until the longest request fits
        assert windows[-1] >= int(lens.max())


def _host_kwargs(batch):
    return {k: v for k, v in batch.kwargs().items() if v is not None}


@pytest.mark.parametrize("case", ["cpu_device", "first_window", "non_contiguous", "vocab"])
def test_host_call_rejects_bad_arguments_before_any_copy(case):
    """verify_logits_host raises ValueError on its argument checks before touching a device,
    like the reference's launchers (sampling/rejection.py:113-138)."""
    batch = _batch(7, B=4, V=257)
    kw = _host_kwargs(batch)
    device = "cuda"
    extra = {}
    if case == "cpu_device":
        device = "cpu"
    elif case == "first_window":
        extra["first_window"] = 1
    elif case == "non_contiguous":
        kw["target_logits"] = kw["target_logits"].t().contiguous().t()
    elif case == "vocab":
        kw["draft_logits"] = kw["draft_logits"][:, :-1].contiguous()
    with pytest.raises(ValueError):
        verify.verify_logits_host(**kw, device=device, **extra)
