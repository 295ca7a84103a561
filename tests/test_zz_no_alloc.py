"""The no-allocation decode entry point (omniasr_decode_attention_noalloc) against the regular one.

Some callers cannot allocate device memory: a host whose GPU memory belongs to another allocator (a serving engine
that reserves HBM for its own pool), or a plugin boundary that passes only input and output buffers. For them the
library keeps the split partials in its own device array; these tests call that entry point through the C ABI and
check that it gives the regular entry point's output, twice in a row (the array keeps the previous call's contents),
and that a shape too large for the array is refused without touching the GPU.
"""

import ctypes

import pytest
import torch

from gpu_util import check_attention, randn

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


def _noalloc(lib, q, kc, vc, lengths, keys, scale, out, status):
    return lib.omniasr_decode_attention_noalloc(
        ctypes.c_void_p(q.data_ptr()), ctypes.c_void_p(kc.data_ptr()), ctypes.c_void_p(vc.data_ptr()), kc.size(0),
        kc.size(2), kc.stride(0), kc.stride(1), kc.stride(2), ctypes.c_void_p(lengths.data_ptr()),
        ctypes.c_void_p(out.data_ptr()), q.size(0), q.size(1), q.size(2), keys, scale,
        0 if q.dtype == torch.bfloat16 else 1, ctypes.c_void_p(status.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_regular_entry_point_twice(dtype):
    from omniasr_b200 import _lib, kernels

    lib = _lib.load()
    assert lib.omniasr_noalloc_scratch_bytes() == 8 << 20
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    h, d, s = 32, 128, 1024
    for call, (b, lens) in enumerate(((8, [1024] * 8), (5, [1, 0, 700, 129, 1024]))):
        q = randn((b, h, d), dtype, 300 + call).cuda()
        kc = randn((b, h, s, d), dtype, 310 + call).cuda()
        vc = randn((b, h, s, d), dtype, 320 + call).cuda()
        lengths = torch.tensor(lens, device="cuda")
        out = torch.empty_like(q)
        assert _noalloc(lib, q, kc, vc, lengths, s, d**-0.5, out, status) == 0, lib.omniasr_last_error()
        want = kernels.decode_attention(q, kc, vc, lengths, s, d**-0.5)
        torch.cuda.synchronize()
        check_attention(out, want.float(), dtype, 2e-5, f"no-alloc call {call}")
        assert int(status.item()) == 0


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
