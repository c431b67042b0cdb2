"""Shared test helpers: run the CPU oracle on a workload Batch."""

import numpy as np
import torch

import oracle as O


def np_f32(t):
    return t.detach().float().cpu().numpy()


def np_i(t):
    return t.detach().cpu().numpy()


def oracle_verify(batch, nthreads=None):
    """The oracle's five outputs for a workloads.Batch (any device)."""
    return O.verify_logits(
        np_i(batch.candidates), np_f32(batch.target_logits), np_i(batch.target_rows),
        None if batch.draft_logits is None else np_f32(batch.draft_logits),
        None if batch.draft_rows is None else np_i(batch.draft_rows),
        np_f32(batch.temperature), np_i(batch.top_k), np_f32(batch.top_p),
        np_i(batch.verify_lens), np_f32(batch.uniforms), np_f32(batch.uniform_final),
        np_i(batch.prefix_lens), nthreads=nthreads)


NAMES = ("accept", "commit", "bonus", "output", "new_seq")


def assert_same(got, expected, tag=""):
    for name, g, e in zip(NAMES, got, expected):
        g = g.detach().cpu().numpy() if isinstance(g, torch.Tensor) else np.asarray(g)
        if not np.array_equal(g, e):
            bad = np.argwhere(g != e)[:8]
            raise AssertionError(f"{tag} {name} differs at {bad.tolist()}: got {g[tuple(bad.T)]} "
                                 f"expected {e[tuple(bad.T)]}")
