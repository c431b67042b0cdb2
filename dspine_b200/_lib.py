"""ctypes binding of libdspine_b200.so (the C ABI in include/dspine_b200.h).

The library is built in-tree by ``dspine_b200.build``.  There is no fallback: if the library
is missing every operator raises, so a CUDA run can never silently take another path.
"""

from __future__ import annotations

import ctypes
import os
import re
import threading
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE / "_lib" / "libdspine_b200.so"
HEADER = _HERE.parent / "include" / "dspine_b200.h"

_lock = threading.Lock()
_lib = None

STATUS = {
    0: "ok",
    1: "bad shape",
    2: "bad dtype",
    3: "bad pointer",
    4: "bad alignment",
    5: "kernel launch failed",
    6: "workspace too small",
    7: "device wait timed out",
    8: "unsupported configuration",
}

c_void_p = ctypes.c_void_p
c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_size_t = ctypes.c_size_t


class CompactOut(ctypes.Structure):
    _fields_ = [
        ("slots", c_void_p),
        ("slots_len", c_int64),
        ("slot_row", c_void_p),
        ("tokens", c_void_p),
        ("kept_slots", c_void_p),
        ("offsets", c_void_p),
        ("freed_slots", c_void_p),
        ("freed_offsets", c_void_p),
    ]


# argument types of every entry point (restype is int unless listed in _RESTYPES)
_SIGNATURES = {
    "dsv_version": [],
    "dsv_launch_count": [],
    "dsv_status_string": [c_int32],
    "dsv_verify_workspace_size": [c_int32, ctypes.POINTER(c_size_t)],
    "dsv_workspace_init": [c_void_p, c_size_t, c_void_p],
    "dsv_workspace_error": [c_void_p, ctypes.POINTER(ctypes.c_uint32), c_void_p],
    "dsv_workspace_bytes_read": [c_void_p, ctypes.POINTER(ctypes.c_uint64), c_void_p],
    "dsv_copy_row_ranges": [c_void_p, c_void_p, ctypes.c_size_t, ctypes.c_int32, c_void_p, c_void_p,
                            c_void_p],
    "dsv_verify_logits": [c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int64,
                          c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                          c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                          c_void_p, c_void_p, ctypes.POINTER(CompactOut), c_void_p, c_size_t,
                          c_void_p],
    "dsv_verify_logits_ex": [c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_int64,
                             c_void_p, c_void_p, c_int64, c_int64, c_void_p, c_void_p, c_void_p,
                             c_void_p, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             ctypes.POINTER(CompactOut), c_void_p, c_size_t, c_void_p],
    "dsv_target_probs_ex": [c_int64, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p,
                            c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_size_t,
                            c_void_p],
    "dsv_lmhead_workspace_size": [c_int32, c_int32, c_int32, ctypes.POINTER(c_size_t)],
    "dsv_lmhead_topk": [c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_int64,
                        c_int64, c_int64, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                        c_size_t, c_void_p],
    "dsv_tp_merge": [c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_int64, c_void_p,
                     c_int64, c_int64, c_int32, c_void_p, c_void_p, c_void_p, c_void_p],
    "dsv_chain_from_probs": [c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                             c_void_p],
    "dsv_target_probs": [c_int64, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p,
                         c_void_p, c_void_p, c_void_p, c_size_t, c_void_p],
    "dsv_accept_sparse": [c_int32, c_int32, c_int32] + [c_void_p] * 19 + [c_void_p],
    "dsv_sparse_target": [c_int64, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_int32,
                          c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p, c_void_p,
                          c_void_p, c_void_p, c_void_p],
    "dsv_compress_probs": [c_int64, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                           c_void_p, c_void_p],
    "dsv_adjust_logits": [c_void_p, c_int32, c_int64, c_int32, c_int64, c_void_p, c_int32,
                          c_void_p, c_void_p, c_void_p, c_int32, c_void_p, c_void_p],
    "dsv_accept_greedy": [c_int32, c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p,
                          c_void_p, c_void_p, c_void_p, c_void_p, c_void_p],
    "dsv_uniforms": [c_int32, c_int32, c_void_p, c_void_p, c_int32, c_int32, c_void_p, c_void_p],
    "dsv_sps_plan": [c_int32, c_void_p, c_void_p, c_int32, c_void_p, c_int32, c_int32, c_void_p,
                     c_void_p, c_void_p, c_void_p],
    "dsv_accept_compact": [c_int32, c_void_p, c_void_p, c_void_p, ctypes.POINTER(CompactOut),
                           c_void_p, c_void_p],
    "dsv_topk_ids": [c_int64, c_int32, c_int64, c_int32, c_void_p, c_int32, c_void_p, c_void_p],
    "dsv_topk_ranked": [c_int64, c_int32, c_int64, c_int32, c_void_p, c_int32, c_void_p, c_void_p],
    "dsv_fp8_quantize_rows": [c_int64, c_int32, c_int64, c_int32, c_void_p, c_void_p, c_int64,
                              c_void_p, c_void_p],
    "dsv_fp8_coarse_scores": [c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p, c_void_p,
                              c_int64, c_void_p, c_void_p, c_int64, c_void_p, c_void_p],
    "dsv_rescore_select16": [c_int32, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p,
                             c_void_p, c_int64, c_int32, c_void_p, c_int32, c_void_p, c_void_p],
    "dsv_serial_sample_chain": [c_int32, c_int32, c_int32] + [c_void_p] * 13,
    "dsv_serial_table": [c_int32, c_int32, c_int32, c_int32, c_int32, c_int64, c_void_p, c_int64,
                         c_void_p, c_void_p, c_void_p, c_void_p, c_int64, c_int32, c_void_p,
                         c_void_p, c_void_p, c_int64, c_void_p, c_void_p, c_void_p, c_void_p,
                         c_void_p],
    "dsv_serial_chain": [c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p, c_void_p,
                         c_void_p, c_void_p],
    "dsv_verify_logits_noalloc": [c_int32, c_int32, c_int32, c_void_p, c_void_p, c_void_p,
                                  c_int64, c_void_p, c_void_p, c_int64, c_int64, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  c_void_p, c_void_p, c_void_p, c_void_p, c_void_p,
                                  ctypes.POINTER(CompactOut), c_void_p, c_void_p],
}
_RESTYPES = {"dsv_version": ctypes.c_char_p, "dsv_status_string": ctypes.c_char_p,
             "dsv_launch_count": ctypes.c_uint64}


class DSVError(RuntimeError):
    """A dsv_* entry point returned a non-zero status."""

    def __init__(self, fn: str, status: int):
        self.status = status
        super().__init__(f"{fn}: {STATUS.get(status, 'status %d' % status)}")


def declared_symbols() -> list[str]:
    """Entry points declared in include/dspine_b200.h."""
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|uint64_t|const char\*)\s+(dsv_\w+)\s*\(", text, re.M)))


def load():
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        # DSV_LIBRARY selects another build of the same C ABI (e.g. the index-checking one)
        path = Path(os.environ.get("DSV_LIBRARY", LIB_PATH))
        if not path.exists():
            raise RuntimeError(
                f"{path} is missing: build it with `python -m dspine_b200.build` "
                "(the CUDA library is required; there is no CPU fallback)")
        lib = ctypes.CDLL(str(path))
        for name, argtypes in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = _RESTYPES.get(name, c_int32)
        _lib = lib
    return _lib


def call(name: str, *args) -> None:
    status = getattr(load(), name)(*args)
    if status != 0:
        if status in (1, 2, 3, 4, 6):
            raise ValueError(f"{name}: {STATUS.get(status, status)}")
        raise DSVError(name, status)


def ptr(t) -> int | None:
    """Device pointer of a tensor (or None)."""
    return None if t is None else t.data_ptr()
