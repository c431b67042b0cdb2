"""Host-side pieces of rows a9 and a10: the neutral padding rows (sampling/padding.py:4-12) and
the SPS width / budget policy (verification/policy.py:9-114).  CPU only."""

import json

import numpy as np
import pytest
import torch

import oracle as O
from dspine_b200.sampling.padding import logits_padding
from dspine_b200.verification.policy import SpsPolicy, execution_identity


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_padding_rows_are_a_one_point_distribution(dtype):
    value = torch.zeros(3, dtype=dtype)
    rows = logits_padding(None, value, (2, 16, 97))
    assert rows.shape == (2, 16, 97) and rows.dtype == dtype and rows.device == value.device
    assert bool((rows[..., 0] == 0).all()) and bool(torch.isinf(rows[..., 1:]).all())
    assert bool((rows[..., 1:] < 0).all())
    # every filter keeps it normalised at token 0 (the oracle's target rows)
    x = rows.reshape(-1, 97)[:2].float().numpy()
    for mode in (O.JOINT, O.SEQUENTIAL, O.TORCH):
        p = O.target_probs(x, [0.7, 1.3], [5, 1 << 30], [0.9, 0.5], rows_per_request=1,
                           min_p=[0.2, 0.0], mode=mode)
        assert np.array_equal(p[:, 0], np.ones(2, np.float32)) and not p[:, 1:].any()


def test_policy_width_budget_and_defaults():
    pol = SpsPolicy({1: 6, 2: 9}, {8: 48})
    assert pol.width(1) == 6 and pol.width(2) == 9 and pol.width(3) == 16
    assert pol.width(2, full=8) == 8
    assert pol.budget(8) == 48 and pol.budget(4) == 64 and pol.budget(8, full=4) == 32
    assert SpsPolicy.from_dict(pol.to_dict()) == pol


@pytest.mark.parametrize("widths,budgets", [({0: 4}, {}), ({1: 17}, {}), ({1: 0}, {}),
                                            ({}, {4: 3}), ({}, {4: 65}), ({2: 4}, {2: 8}),
                                            ({1: 4.0}, {})])
def test_policy_rejects_bad_entries(widths, budgets):
    with pytest.raises(ValueError):
        SpsPolicy(widths, budgets)


def test_policy_profiles(tmp_path):
    hw = {"name": "NVIDIA B200", "capability": [10, 0], "memory_bytes": 1}
    v2 = {"format": "dspine-sps-v2", "hardware": hw, "execution": execution_identity(1, 1),
          "policy": {"token_budgets": {"8": 64}},
          "mode_policies": {"greedy": {"verify_widths": {"1": 12}}}}
    path = tmp_path / "sps.json"
    path.write_text(json.dumps(v2))
    base, modes = SpsPolicy.load_with_modes(str(path), hw, execution_identity(1, 1))
    assert base.budget(8) == 64 and modes["greedy"].width(1) == 12
    assert SpsPolicy.load(None, hw) == SpsPolicy()
    with pytest.raises(ValueError):
        SpsPolicy.load(str(path), dict(hw, name="other"))
    with pytest.raises(ValueError):
        SpsPolicy.load(str(path), hw, execution_identity(2, 1))
    v1 = {"format": "dspine-sps-v1", "hardware": hw,
          "policy": {"uniform_widths": [16, 12, 10, 8, 8, 6, 4], "batch8_tokens": 48}}
    path.write_text(json.dumps(v1))
    legacy = SpsPolicy.load(str(path), hw)
    assert legacy.width(3) == 10 and legacy.budget(8) == 48
    v1["policy"]["batch8_tokens"] = 50
    path.write_text(json.dumps(v1))
    with pytest.raises(ValueError):
        SpsPolicy.load(str(path), hw)


def test_ragged_window_compaction_and_expansion():
    from types import SimpleNamespace

    from dspine_b200.verification import ragged

    bs, full, V = 3, 4, 11
    window = torch.tensor([0, 1, 4, 8, 9, 10])
    vi = SimpleNamespace(draft_token=torch.arange(100, 112), positions=torch.arange(12) * 2,
                         ragged_verify_layout=None, kv_loc_cols=None)
    batch = SimpleNamespace(out_cache_loc=torch.arange(50, 62, dtype=torch.int32))
    saved = ragged.compact_window(vi, batch, window, "layout")
    assert vi.draft_token.tolist() == [100, 101, 104, 108, 109, 110]
    assert vi.positions.tolist() == [0, 2, 8, 16, 18, 20]
    assert batch.out_cache_loc.tolist() == [50, 51, 54, 58, 59, 60]
    assert vi.ragged_verify_layout == "layout" and vi.kv_loc_cols is window
    ragged.restore_window(saved)
    assert vi.draft_token.tolist() == list(range(100, 112)) and vi.kv_loc_cols is None
    assert batch.out_cache_loc.tolist() == list(range(50, 62))
    packed = torch.randn(window.numel(), V)
    rows = ragged.expand_rows(None, packed, window, bs, full)
    assert torch.equal(rows[window], packed)
    rest = torch.ones(bs * full, dtype=torch.bool)
    rest[window] = False
    assert bool((rows[rest][:, 0] == 0).all()) and bool(torch.isinf(rows[rest][:, 1:]).all())
    hidden = ragged.expand_rows(None, packed, window, bs, full, logits=False)
    assert not hidden[rest].any()
    assert ragged.window_requests(window, full).tolist() == [0, 0, 1, 2, 2, 2]
