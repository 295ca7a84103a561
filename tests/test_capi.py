"""The C ABI library without a GPU: it loads, exports every symbol of include/omniasr_b200.h, and its host-only
functions agree with the oracle."""

import ctypes
import re

import numpy as np
import pytest

from conftest import ROOT
from omniasr_b200 import _lib
from oracle import splits

HEADER = ROOT / "include" / "omniasr_b200.h"


def declared():
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    return sorted(set(re.findall(r"\b(omniasr_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared()
    assert len(names) >= 9
    for name in names:
        assert hasattr(lib, name), name
    assert set(names) == set(_lib.SIGNATURES), "the ctypes table and the header disagree"


def test_exported_symbols_in_the_shared_object():
    import subprocess

    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (omniasr_\w+)", out))
    assert set(declared()) <= exported


def test_abi_version_and_no_error_message():
    lib = _lib.load()
    assert lib.omniasr_abi_version() == 2
    assert isinstance(lib.omniasr_last_error(), bytes)


def test_splits_for_matches_reference(golden):
    lib = _lib.load()
    s, c = ctypes.c_int(), ctypes.c_int()
    for rows, heads, keys, block, programs, ws, wc in golden("splits")["cases"]:
        assert lib.omniasr_splits_for(int(rows), int(heads), int(keys), int(block), int(programs), ctypes.byref(s),
                                      ctypes.byref(c)) == 0
        assert (s.value, c.value) == (ws, wc) == splits.splits_for(int(rows), int(heads), int(keys), int(block),
                                                                   int(programs))


def test_splits_for_rejects_bad_arguments():
    from omniasr_b200 import kernels

    with pytest.raises(ValueError, match="splits_for"):
        kernels.splits_for(0, 8, 256)


def test_workspace_sizes():
    lib = _lib.load()
    for kind, per in ((_lib.DECODE, 1), (_lib.DRAFT, 5), (_lib.BEAM, 5)):
        for dtype in (_lib.BF16, _lib.F32):
            n = lib.omniasr_attention_workspace(kind, dtype, 8, per, 32, 128, 2048, 512)
            rows = 8 * per
            assert n >= rows * 32 * (128 + 2) * 4  # at least one split of partials per (row, head)
            assert n % 16 == 0
    assert lib.omniasr_attention_workspace(_lib.DECODE, _lib.BF16, 8, 1, 32, 96, 2048, 0) == 0  # unsupported D
    assert lib.omniasr_attention_workspace(_lib.DECODE, 7, 8, 1, 32, 128, 2048, 0) == 0


def test_decode_and_draft_workspaces_start_with_the_unit_counters():
    """ABI version 2: decode / draft workspaces hold OMNIASR_ATTENTION_COUNTER_BYTES (64 KB) of per-(row, head)
    counters before the split partials, on the tensor-core path (bf16, head_dim 128) and the CUDA-core path alike."""
    lib = _lib.load()
    counters = 65536
    header = (ROOT / "include" / "omniasr_b200.h").read_text()
    assert f"#define OMNIASR_ATTENTION_COUNTER_BYTES {counters}" in header
    for kind, per in ((_lib.DECODE, 1), (_lib.DRAFT, 5)):
        for dtype, dim in ((_lib.BF16, 128), (_lib.F32, 128), (_lib.BF16, 64)):
            n = lib.omniasr_attention_workspace(kind, dtype, 8, per, 32, dim, 2048, 0)
            assert n >= counters + 8 * per * 32 * (dim + 2) * 4, (kind, dtype, dim, n)
    # The beam workspace carries no counters: one split of partials per (row, head) suffices for a tiny shape.
    n = lib.omniasr_attention_workspace(_lib.BEAM, _lib.BF16, 1, 1, 1, 128, 128, 0)
    assert 0 < n < counters


def test_no_device_is_an_error_not_a_fallback():
    """Without a GPU the compute entry points return an error code (no CPU path behind them)."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    code = lib.omniasr_reorder_gather(None, 0, 0, None, 0, None, 0, 1, 16, None, None)
    assert code == _lib.ERR_DEVICE
    assert b"device" in lib.omniasr_last_error()


def test_available_is_false_on_cpu():
    import torch

    from omniasr_b200 import kernels

    assert kernels.available(torch.device("cpu")) is False


def test_build_flags_target_sm100a():
    mk = (ROOT / "omniasr-trt_b200" / "csrc" / "Makefile").read_text()
    assert "arch=compute_100a,code=sm_100a" in mk
    assert np.all([p.suffix in (".cu", ".cuh") for p in (ROOT / "omniasr-trt_b200" / "csrc").glob("*.cu*")])
