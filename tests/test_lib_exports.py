"""The C-ABI library builds, loads without a GPU, and exports every declared entry point."""

import ctypes

import pytest

from dspine_b200 import _lib, build


@pytest.fixture(scope="module")
def lib():
    build.build()
    return _lib.load()


def test_every_declared_symbol_is_exported(lib):
    names = _lib.declared_symbols()
    assert "dsv_verify_logits" in names
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_every_declared_symbol_has_a_binding():
    assert set(_lib.declared_symbols()) <= set(_lib._SIGNATURES)


def test_version_and_status_strings(lib):
    assert lib.dsv_version().startswith(b"dspine_b200")
    assert lib.dsv_status_string(0) == b"ok"
    assert lib.dsv_status_string(6) == b"workspace too small"


def test_host_validation_rejects_before_launch(lib):
    size = ctypes.c_size_t()
    assert lib.dsv_verify_workspace_size(64, ctypes.byref(size)) == 0
    assert size.value >= 64 * 16 * 16
    assert lib.dsv_verify_workspace_size(-1, ctypes.byref(size)) == 1
    # bad shape / dtype / null pointers are refused without touching the device

    def args(batch, vocab, dtype, target_rows=1, stride=None):
        a = [None] * 27
        a[0], a[1], a[2] = batch, vocab, dtype
        a[6] = target_rows       # target_rows
        a[9] = 0                 # draft_rows
        a[10] = stride if stride is not None else max(vocab, 1)
        a[25] = 0                # workspace_bytes
        return a

    assert lib.dsv_verify_logits(*args(4, 0, 0)) == 1      # vocab < 1
    assert lib.dsv_verify_logits(*args(4, 100, 7)) == 2    # unknown dtype
    assert lib.dsv_verify_logits(*args(4, 100, 0)) == 3    # null pointers
    assert lib.dsv_verify_logits(*args(4, 100, 0, stride=50)) == 1  # stride < vocab
    assert lib.dsv_verify_logits(*args(0, 100, 0)) == 0    # empty batch is a no-op


def test_topk_ids_validation(lib):
    """kernels/dspine.py:172-189: shape, k and out checks raise before any launch; the C ABI
    refuses the same shapes, an unknown dtype and null pointers without touching the device."""
    import torch

    from dspine_b200.kernels import dspine as K

    x = torch.zeros(2, 4096)
    with pytest.raises(ValueError, match="row-contiguous"):
        K.topk_ids(x.t(), 4)
    with pytest.raises(ValueError, match="power-of-two"):
        K.topk_ids(x, 3)
    with pytest.raises(ValueError, match="power-of-two"):
        K.topk_ids(x, 128)
    with pytest.raises(ValueError, match="at least k=64 chunks"):
        K.topk_ids(torch.zeros(2, 4000), 64)
    with pytest.raises(ValueError, match="out must be"):
        K.topk_ids(x, 4, out=torch.empty(2, 4, dtype=torch.int32))
    assert tuple(K.topk_ids(torch.zeros(0, 4096), 4).shape) == (0, 4)
    assert lib.dsv_topk_ids(2, 4096, 4096, 0, None, 4, None, None) == 3       # null pointers
    assert lib.dsv_topk_ids(2, 4096, 4096, 5, None, 4, None, None) == 2       # unknown dtype
    assert lib.dsv_topk_ids(2, 4096, 4096, 0, None, 3, None, None) == 1       # k not a power of 2
    assert lib.dsv_topk_ids(2, 4096, 100, 0, None, 4, None, None) == 1        # stride < vocab
    assert lib.dsv_topk_ids(2, 262145, 262145, 0, None, 4, None, None) == 1   # vocab too large
    assert lib.dsv_topk_ids(2, 4000, 4000, 0, None, 64, None, None) == 1      # fewer chunks than k
    assert lib.dsv_topk_ids(0, 4096, 4096, 0, None, 4, None, None) == 0       # no rows: no-op
