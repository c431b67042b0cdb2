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


def test_fp8_entry_validation(lib):
    """The FP8 retrieval entries refuse bad shapes, dtypes, pointers and alignments before any
    launch; the host modules raise ValueError as the reference's argument checks do."""
    import torch

    from dspine_b200.layers.fp8 import coarse as C
    from dspine_b200.layers.fp8 import gather as G

    # dsv_topk_ranked: any k in [1, min(128, vocab)]
    assert lib.dsv_topk_ranked(2, 100, 100, 0, None, 100, None, None) == 3    # shape ok, null pointers
    assert lib.dsv_topk_ranked(2, 100, 100, 0, None, 101, None, None) == 1    # k > vocab
    assert lib.dsv_topk_ranked(2, 4096, 4096, 0, None, 129, None, None) == 1  # k > 128
    assert lib.dsv_topk_ranked(2, 4096, 4096, 3, None, 16, None, None) == 2   # dtype
    # dsv_fp8_quantize_rows
    assert lib.dsv_fp8_quantize_rows(2, 64, 64, 0, None, None, 64, None, None) == 3
    assert lib.dsv_fp8_quantize_rows(2, 64, 32, 0, None, None, 64, None, None) == 1
    assert lib.dsv_fp8_quantize_rows(2, 64, 64, 2, None, None, 64, None, None) == 2
    assert lib.dsv_fp8_quantize_rows(0, 64, 64, 0, None, None, 64, None, None) == 0
    # dsv_fp8_coarse_scores: hidden a multiple of 128, 16-byte TMA alignment
    cs = lib.dsv_fp8_coarse_scores
    assert cs(4, 512, 100, None, 100, None, None, 100, None, None, 512, None, None) == 1
    assert cs(4, 512, 512, None, 512, None, None, 512, None, None, 512, None, None) == 3
    assert cs(4, 512, 512, 16, 520, 16, 16, 512, 16, 16, 512, 16, None) == 4  # pitch not 16-byte multiple
    assert cs(0, 512, 512, None, 512, None, None, 512, None, None, 512, None, None) == 0
    # dsv_rescore_select16
    rs = lib.dsv_rescore_select16
    assert rs(4, 129, 512, 1000, None, 512, None, None, 512, 0, None, 0, None, None) == 1  # > 128 candidates
    assert rs(4, 8, 512, 1000, 16, 512, 16, 16, 512, 0, 16, 0, 16, None) == 1            # top-16 of 8
    assert rs(4, 128, 500, 1000, 16, 512, 16, 16, 512, 0, 16, 0, None, None) == 1         # hidden % 8
    assert rs(4, 128, 512, 1000, 16, 512, 16, 16, 512, 2, 16, 0, None, None) == 2         # hidden dtype
    assert rs(4, 128, 0, 1, None, 0, 16, None, 0, 0, 16, 0, None, None) == 3              # selection needs out16
    # host modules
    with pytest.raises(ValueError, match="multiple of 128"):
        C.FullVFP8Coarse(torch, torch.zeros(64, 100, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="bf16 head"):
        C.FullVFP8Coarse(torch, torch.zeros(64, 128))
    with pytest.raises(ValueError, match="1 <= k"):
        C.stable_local_topk(torch.zeros(2, 100), 101)
    with pytest.raises(ValueError, match="1..128 candidates"):
        G.rescore(torch, torch.zeros(10, 64, dtype=torch.bfloat16), torch.zeros(2, 129, dtype=torch.int64),
                  torch.zeros(2, 64, dtype=torch.bfloat16))
    with pytest.raises(ValueError, match="at least 16"):
        G.select16(torch, torch.zeros(2, 8), torch.zeros(2, 8, dtype=torch.int64))
    with pytest.raises(ValueError, match="multiple of 128"):
        C.coarse_scores(torch.zeros(2, 100, dtype=torch.uint8), torch.ones(2),
                        torch.zeros(8, 100, dtype=torch.uint8), torch.ones(8))


def test_copy_row_ranges_and_bytes_read_validation(lib):
    """Argument errors of the staged row copier and of the bytes-read query are refused before
    any CUDA call (a negative count, a negative or null range, a null workspace)."""
    first = (ctypes.c_int64 * 2)(0, 3)
    count = (ctypes.c_int64 * 2)(2, 1)
    bad = (ctypes.c_int64 * 2)(-1, 3)
    buf = ctypes.create_string_buffer(64)
    assert lib.dsv_copy_row_ranges(buf, buf, 8, -1, first, count, None) == 1   # n < 0
    assert lib.dsv_copy_row_ranges(buf, buf, 8, 0, None, None, None) == 0      # nothing to copy
    assert lib.dsv_copy_row_ranges(None, buf, 8, 2, first, count, None) == 3   # null destination
    assert lib.dsv_copy_row_ranges(buf, buf, 8, 2, None, count, None) == 3     # null ranges
    assert lib.dsv_copy_row_ranges(buf, buf, 8, 2, bad, count, None) == 1      # negative row
    n = ctypes.c_uint64()
    assert lib.dsv_workspace_bytes_read(None, ctypes.byref(n), None) == 3
