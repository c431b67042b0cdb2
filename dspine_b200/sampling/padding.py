"""Neutral target rows for positions outside a request's verified prefix (sampling/padding.py).

`logits_padding(controller, value, shape)` keeps the reference's signature (padding.py:4-12).
Rows of the full 16-row envelope that no verified position fills must not emit a token and
must survive every filter: a one-point distribution (-inf everywhere, 0.0 at token 0) stays
normalised under temperature, top-k, top-p and min-p, so the target kernels give it
probability 1 at token 0 without a uniform full-vocabulary dummy row.  One device fill in the
dtype and on the device of `value`.
"""

import torch


def logits_padding(controller, value, shape):
    rows = torch.full(tuple(shape), float("-inf"), dtype=value.dtype, device=value.device)
    rows.narrow(-1, 0, 1).zero_()  # the single point: token 0
    return rows
