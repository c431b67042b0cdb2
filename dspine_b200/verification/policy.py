"""Verification widths and token budgets per batch size (verification/policy.py of the reference).

`SpsPolicy` keeps the reference's fields, checks and methods (policy.py:9-114): a batch size
maps either to a fixed verify width (1..16 rows per request) or to a token budget for the
SPS allocator (bs..16 bs tokens), never both; a batch size without an entry verifies the full
block.  `width(bs, full)` / `budget(bs, full)` (policy.py:31-35) are what the controllers read
every round; `load_with_modes` reads a tuned profile (format "dspine-sps-v1" or "-v2") and
refuses one measured on other hardware or another execution layout.  Host-side configuration:
nothing here runs on the GPU.
"""

from __future__ import annotations

import json
from dataclasses import dataclass, field
from pathlib import Path

_FORMATS = ("dspine-sps-v1", "dspine-sps-v2")
_NAMES = ("verify_widths", "token_budgets")


def _check(mapping, name):
    if not isinstance(mapping, dict):
        raise ValueError(f"SPS {name} must map positive batch sizes to integers")
    for bs, value in mapping.items():
        if type(bs) is not int or bs < 1 or type(value) is not int:
            raise ValueError(f"SPS {name} requires positive integer batch sizes")
        lo, hi = (1, 16) if name == "verify_widths" else (bs, 16 * bs)
        if value < lo or value > hi:
            raise ValueError(f"SPS {name}[{bs}] must be in [{lo}, {hi}]")


@dataclass(frozen=True)
class SpsPolicy:
    verify_widths: dict = field(default_factory=dict)
    token_budgets: dict = field(default_factory=dict)

    def __post_init__(self):
        _check(self.verify_widths, "verify_widths")
        _check(self.token_budgets, "token_budgets")
        if set(self.verify_widths) & set(self.token_budgets):
            raise ValueError("SPS batch sizes must use either a width or a token budget")

    def width(self, bs, full=16):
        """Rows verified per request at batch size bs (the full block when unmeasured)."""
        return min(full, self.verify_widths.get(bs, full))

    def budget(self, bs, full=16):
        """Tokens the SPS allocator may verify at batch size bs (every row when unmeasured)."""
        return min(bs * full, self.token_budgets.get(bs, bs * full))

    def to_dict(self):
        return {name: {str(bs): v for bs, v in sorted(getattr(self, name).items())}
                for name in _NAMES}

    @classmethod
    def from_dict(cls, policy):
        unknown = set(policy) - set(_NAMES)
        if unknown:
            raise ValueError("Unknown fields in DSpine SPS policy")
        return cls(**{name: {int(bs): v for bs, v in policy.get(name, {}).items()}
                      for name in _NAMES})

    @classmethod
    def load(cls, path, hardware, execution=None):
        return cls.load_with_modes(path, hardware, execution)[0]

    @classmethod
    def load_with_modes(cls, path, hardware, execution=None):
        """(fallback policy, {mode: policy}) from a tuned profile; no path: the full block."""
        if not path:
            return cls(), {}
        data = json.loads(Path(path).read_text())
        if data.get("format") not in _FORMATS:
            raise ValueError("Expected a DSpine SPS profile from scripts/tune_sps.py")
        if data.get("hardware") != hardware:
            raise ValueError("SPS profile hardware differs; rerun scripts/tune_sps.py on this GPU")
        if execution is not None:
            _check_execution(data.get("execution"), execution)
        policy = data["policy"]
        if data["format"] == "dspine-sps-v1":
            return _legacy(cls, policy), {}
        modes = data.get("mode_policies", {})
        if not isinstance(modes, dict) or not set(modes) <= {"greedy", "sampled"}:
            raise ValueError("SPS mode_policies only supports greedy and sampled")
        return cls.from_dict(policy), {m: cls.from_dict(p) for m, p in modes.items()}


def _check_execution(recorded, expected):
    """The profile's TP layout must match; attention backends only where both name one."""
    if recorded is None:
        if expected["tp_size"] != 1 or expected["draft_tp_size"] != 1:
            raise ValueError("SPS profile has no TP layout; retune for this deployment")
        return
    for name in ("tp_size", "draft_tp_size", "attention_backend", "draft_attention_backend"):
        want, have = expected.get(name), recorded.get(name)
        both = want is not None and have is not None
        if (name.endswith("tp_size") or both) and want != have:
            raise ValueError("SPS profile execution layout differs; retune for this deployment")


def _legacy(cls, policy):
    """v1 profiles: widths for batch sizes 1..7 and one token budget at batch size 8."""
    widths, budget = policy["uniform_widths"], policy["batch8_tokens"]
    ok = (len(widths) == 7 and all(type(w) is int and 2 <= w <= 16 for w in widths)
          and type(budget) is int and budget in range(16, 129, 16))
    if not ok:
        raise ValueError("Invalid legacy DSpine SPS profile")
    return cls({bs: w for bs, w in enumerate(widths, 1)}, {8: budget})


def hardware_identity(device):
    import torch

    props = torch.cuda.get_device_properties(device)
    return {"name": props.name, "capability": [props.major, props.minor],
            "memory_bytes": props.total_memory}


def execution_identity(tp_size, draft_tp_size, attention_backend=None,
                       draft_attention_backend=None):
    return {"tp_size": int(tp_size), "draft_tp_size": int(draft_tp_size),
            "attention_backend": attention_backend,
            "draft_attention_backend": draft_attention_backend}
