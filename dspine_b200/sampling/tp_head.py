"""Vocabulary-sharded head (sampling/tp_head.py of the reference): see dspine_b200.lmhead."""

from ..lmhead import TPHead, TorchGroup, merge_topk  # noqa: F401
