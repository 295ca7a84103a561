"""The no-allocation decode entry point (omniasr_decode_attention_noalloc), through the C ABI.

Some callers cannot allocate device memory: a host whose GPU memory belongs to another allocator (a serving engine
that reserves HBM for its own pool), or a plugin boundary that passes only input and output buffers. For them the
library keeps the split partials in its own device array. These tests check that entry point against the float64
oracle and against the regular entry point on consecutive calls whose units are split over different numbers of CTAs
(the array keeps the previous call's contents, and its counters must come back to zero after every call), that the
reset entry point leaves the array usable, that an invalid call is reported as an argument error before any scratch
check, and that a shape too large for the array is refused without touching the GPU.

This file is collected last, so that a run stopping at its first failure has already run every other test.
"""

import ctypes

import pytest
import torch

from gpu_util import check_attention, randn
from oracle import attention as oatt

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


def _noalloc(lib, q, kc, vc, lengths, keys, scale, out, status, batch=None):
    return lib.omniasr_decode_attention_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kc.data_ptr()), ctypes.c_void_p(vc.data_ptr()), kc.size(0),
        kc.size(2), kc.stride(0), kc.stride(1), kc.stride(2), ctypes.c_void_p(lengths.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), q.size(0) if batch is None else batch, q.size(1), q.size(2), keys, scale,
        0 if q.dtype == torch.bfloat16 else 1, ctypes.c_void_p(status.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


# Three shapes whose (row, head) units the pass cuts between CTAs differently: 8 full rows (about 1.7 CTAs per
# unit), ragged rows with empty and one-key rows, and 2 long rows (many CTAs per unit).
CALLS = ((8, 32, 1024, [1024] * 8), (5, 32, 1024, [1, 0, 700, 129, 1024]), (2, 8, 4096, [4096, 3001]))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_oracle_and_regular_entry_point_on_consecutive_calls(dtype):
    from omniasr_b200 import _lib, kernels

    lib = _lib.load()
    assert lib.omniasr_noalloc_scratch_bytes() == 8 << 20
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    d = 128
    for call, (b, h, s, lens) in enumerate(CALLS + CALLS[:1]):  # the first shape again after the others
        q = randn((b, h, d), dtype, 300 + call)
        kc = randn((b, h, s, d), dtype, 310 + call)
        vc = randn((b, h, s, d), dtype, 320 + call)
        lengths = torch.tensor(lens)
        out = torch.empty_like(q).cuda()
        qd, kd, vd, ld = q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda()
        assert _noalloc(lib, qd, kd, vd, ld, s, d**-0.5, out, status) == 0, lib.omniasr_last_error()
        regular = kernels.decode_attention(qd, kd, vd, ld, s, d**-0.5)
        torch.cuda.synchronize()
        want = oatt.decode_attention(q, kc, vc, lengths, d**-0.5)
        check_attention(out, want, dtype, 2e-5, f"no-alloc call {call} against the oracle")
        check_attention(out, regular.float(), dtype, 2e-5, f"no-alloc call {call} against the regular entry point")
        assert (out[lengths.cuda() == 0] == 0).all(), "a row of length 0 gets zeros"
        assert int(status.item()) == 0


def test_noalloc_reset_then_call():
    from omniasr_b200 import _lib

    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.omniasr_noalloc_reset(stream) == 0, lib.omniasr_last_error()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    b, h, s, d = 4, 16, 2048, 128
    q, kc, vc = randn((b, h, d), torch.bfloat16, 41), randn((b, h, s, d), torch.bfloat16, 42), \
        randn((b, h, s, d), torch.bfloat16, 43)
    lengths = torch.tensor([2048, 1500, 17, 900])
    out = torch.empty(b, h, d, dtype=torch.bfloat16, device="cuda")
    for _ in range(2):
        assert _noalloc(lib, q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), s, d**-0.5, out, status) == 0
        assert lib.omniasr_noalloc_reset(stream) == 0
    torch.cuda.synchronize()
    check_attention(out, oatt.decode_attention(q, kc, vc, lengths, d**-0.5), torch.bfloat16, 2e-5, "after reset")
    assert int(status.item()) == 0


def test_noalloc_reports_bad_arguments_before_scratch():
    from omniasr_b200 import _lib

    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    b, h, d, s = 64, 32, 128, 8192  # would need ~69 MB of partials, but keys > cache length is the error
    q = torch.zeros(b, h, d, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(8, dtype=torch.bfloat16, device="cuda")
    big = torch.empty(b, h, 16, d, dtype=torch.bfloat16, device="meta")
    lengths = torch.zeros(b, dtype=torch.long, device="cuda")
    out = torch.empty_like(q)
    code = lib.omniasr_decode_attention_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kc.data_ptr()), ctypes.c_void_p(kc.data_ptr()), b, 16,
        big.stride(0), big.stride(1), big.stride(2), ctypes.c_void_p(lengths.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), b, h, d, s, d**-0.5, 0, ctypes.c_void_p(status.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code == _lib.ERR_ARGUMENT
    assert b"keys" in lib.omniasr_last_error()


def test_noalloc_refuses_shapes_beyond_its_scratch():
    from omniasr_b200 import _lib

    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    b, h, d, s = 64, 32, 128, 8192  # ~69 MB of partials, far past the 8 MiB array
    q = torch.zeros(b, h, d, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(8, dtype=torch.bfloat16, device="cuda")  # never read: the call is refused first
    big = torch.empty(b, h, s, d, dtype=torch.bfloat16, device="meta")
    lengths = torch.zeros(b, dtype=torch.long, device="cuda")
    out = torch.empty_like(q)
    code = lib.omniasr_decode_attention_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kc.data_ptr()), ctypes.c_void_p(kc.data_ptr()), b, s,
        big.stride(0), big.stride(1), big.stride(2), ctypes.c_void_p(lengths.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), b, h, d, s, d**-0.5, 0, ctypes.c_void_p(status.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert code == _lib.ERR_WORKSPACE
    assert b"no-alloc" in lib.omniasr_last_error()
