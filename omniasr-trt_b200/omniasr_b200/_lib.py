"""ctypes binding of the C ABI in ``include/omniasr_b200.h`` (``lib/libomniasr_b200.so``).

The library is built in-tree (``make -C omniasr-trt_b200/csrc`` or ``__graft_entry__.build()``); there
is no other implementation behind these functions, so a missing library is an error, never a fallback.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent.parent / "lib" / "libomniasr_b200.so"

BF16, F32 = 0, 1
OK, ERR_ARGUMENT, ERR_UNSUPPORTED, ERR_WORKSPACE, ERR_CUDA, ERR_DEVICE = range(6)
DECODE, DRAFT, BEAM = 0, 1, 2

_p = ctypes.c_void_p
_i = ctypes.c_int
_i64 = ctypes.c_int64
_f = ctypes.c_float
_sz = ctypes.c_size_t

# name -> (restype, argtypes); the order of include/omniasr_b200.h.
SIGNATURES = {
    "omniasr_abi_version": (_i, []),
    "omniasr_last_error": (ctypes.c_char_p, []),
    "omniasr_device_supported": (_i, [_i]),
    "omniasr_splits_for": (_i, [_i, _i, _i, _i, _i, ctypes.POINTER(_i), ctypes.POINTER(_i)]),
    "omniasr_attention_workspace": (_sz, [_i, _i, _i, _i, _i, _i, _i64, _i64]),
    "omniasr_rope_kv": (_i, [_p, _i64, _p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i, _i, _i,
                             _i, _p, _p]),
    "omniasr_decode_attention": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _i, _i, _i, _i, _f, _i, _p,
                                      _sz, _p, _p]),
    "omniasr_draft_attention": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _i, _i, _i, _i, _i, _f, _i,
                                     _p, _sz, _p, _p]),
    "omniasr_beam_attention": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _p, _i64, _i64, _i64, _i64,
                                    _i64, _p, _i64, _p, _p, _i, _i, _i, _i, _i, _f, _i, _p, _sz, _p, _p]),
    "omniasr_prefill_attention": (_i, [_p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64, _i64, _i64, _p, _i64,
                                       _i64, _i64, _i, _i, _i, _i, _f, _i, _p, _p]),
    "omniasr_prefill_grouped_workspace": (_sz, [_i, _i, _i, _i]),
    "omniasr_prefill_attention_grouped": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _i, _i, _i, _i, _f, _i,
                                               _p, _sz, _p, _p]),
    "omniasr_reorder_gather": (_i, [_p, _i64, _i64, _p, _i64, _p, _i, _i, _i64, _p, _p]),
    "omniasr_decode_attention_noalloc": (_i, [_p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p, _p, _i, _i, _i, _i, _f,
                                              _i, _p, _p]),
    "omniasr_noalloc_scratch_bytes": (_sz, []),
    "omniasr_noalloc_reset": (_i, [_p]),
    "omniasr_selftest_wait_timeout": (_i, [_i64, _p, _p, _p]),
    "omniasr_propose": (_i, [_p, _i64, _i64, _p, _i64, _i64, _p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p, _i,
                             _i, _p, _p]),
    "omniasr_beam_select": (_i, [_p, _i64, _i, _p, _p, _p, _p, _p, _i64, _i64, _p, _i64, _i64, _p, _p, _p, _i, _i, _i,
                                 _i, _i64, _i64, _i64, _p, _p]),
    "omniasr_decode_gemm_rope": (_i, [_p, _i64, _i, _p, _i64, _i, _p, _i64, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64,
                                      _i64, _i64, _i, _i, _p, _sz, _p, _p]),
    "omniasr_accept": (_i, [_p, _p, _p, _i64, _i64, _p, _p, _p, _p, _p, _p, _i, _i, _i64, _i64, _p, _p]),
    "omniasr_decode_gemm_workspace": (_sz, [_i, _i, _i, _i]),
    "omniasr_decode_gemm": (_i, [_p, _i64, _i, _p, _i64, _i, _i, _i, _p, _i64, _p, _i64, _p, _sz, _p, _p]),
}

_lib = None
_lock = threading.Lock()


class KernelError(RuntimeError):
    """A C ABI call returned an error code."""

    def __init__(self, fn: str, code: int, message: str):
        super().__init__(f"{fn} failed ({code}): {message}")
        self.code = code


def load() -> ctypes.CDLL:
    """The shared library with every declared symbol bound (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(f"{LIB_PATH} is missing: build it with `make -C omniasr-trt_b200/csrc` "
                                   "or `python -c 'import __graft_entry__ as g; g.build()'`")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name: str, *args) -> None:
    """Calls ``name`` and raises :class:`KernelError` with the library's message on a non-zero code."""
    lib = load()
    code = getattr(lib, name)(*args)
    if code != OK:
        msg = lib.omniasr_last_error().decode(errors="replace")
        if code in (ERR_ARGUMENT, ERR_UNSUPPORTED, ERR_WORKSPACE):
            raise ValueError(f"{name}: {msg}")
        raise KernelError(name, code, msg)
