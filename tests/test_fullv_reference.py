"""The benchmark configurations at the full vocabulary (V = 151936), pinned to the reference.

tests/golden/fullv.npz holds the outputs of the reference's own sample_capped_chain_from_probs
(sampling/rejection.py:101-153, run under the Triton interpreter) over target and draft rows
built by the reference's test definition of the target distribution (tests/ref_utils.py:79-108
ref_target_row, float64; greedy rows one-hot at the lowest-index argmax,
runtime/worker.py:461-469), for configs 0, 1 and 4 of dspine_b200.workloads
(tests/golden/make_golden.py fullv).  The inputs are regenerated here from the same seeds
and checked against a stored fingerprint first.

CPU: the oracle equals the reference on configs 0 and 1.  GPU: dsv_verify_logits equals the
reference on configs 0, 1 and 4 (accept, commit, bonus, output, new_seq bit for bit).
"""

from pathlib import Path

import numpy as np
import pytest
import torch

from dspine_b200 import workloads
from helpers import NAMES, oracle_verify

FIX = np.load(Path(__file__).resolve().parent / "golden" / "fullv.npz")
BUILDERS = {"config0": workloads.config0, "config1": workloads.config1,
            "config4": workloads.config4}


def _batch(name):
    batch = BUILDERS[name]()
    fp = str(FIX[f"{name}_fingerprint"])
    assert workloads.fingerprint(batch) == fp, (
        f"{name}: regenerated inputs differ from the fixture's (torch RNG changed?)")
    return batch


def _compare(name, got):
    for key, g in zip(NAMES, got):
        g = g.detach().cpu().numpy() if isinstance(g, torch.Tensor) else np.asarray(g)
        want = FIX[f"{name}_{key}"]
        if not np.array_equal(g, want):
            bad = np.argwhere(g != want)[:8].tolist()
            margin = FIX[f"{name}_margin"]
            raise AssertionError(
                f"{name} {key} differs from the reference at {bad}; bonus-draw margins of those "
                f"requests (distance of u*M from the nearest CDF step / M): "
                f"{[float(margin[i[0]]) for i in bad]}")


@pytest.mark.parametrize("name", ["config0", "config1"])
def test_oracle_matches_reference_full_vocab(name):
    _compare(name, oracle_verify(_batch(name)))


@pytest.mark.gpu
@pytest.mark.parametrize("name", ["config0", "config1", "config4"])
def test_gpu_matches_reference_full_vocab(name):
    from dspine_b200 import verify

    dev = torch.device("cuda", 0)
    batch = _batch(name).to(dev)
    got = verify.verify_logits(**batch.kwargs())
    torch.cuda.synchronize(dev)
    assert verify.workspace_for(batch.B, dev).error_word() == 0
    _compare(name, got)
