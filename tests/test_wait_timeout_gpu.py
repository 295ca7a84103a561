"""The bounded device wait of every kernel here, made to run out on purpose (no fault, no hang).

omniasr_selftest_wait_timeout runs one kernel that waits, through the same mbar_wait every kernel of the library uses,
on an mbarrier that nothing completes. With a 1 ms limit the wait must give up, OR the timeout bit (2) into the status
word and return; the context must stay usable, so a regular kernel call right after it gives correct results.
"""

import ctypes

import pytest
import torch

from gpu_util import check_attention, randn
from oracle import attention as oatt

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


def test_bounded_wait_gives_up_and_sets_status_bit_2():
    from omniasr_b200 import _lib, kernels

    lib = _lib.load()
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    waited = torch.zeros(1, dtype=torch.int64, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    limit_ns = 1_000_000
    assert lib.omniasr_selftest_wait_timeout(limit_ns, ctypes.c_void_p(status.data_ptr()),
                                             ctypes.c_void_p(waited.data_ptr()), stream) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 2, "the wait did not report that it gave up"
    assert limit_ns <= int(waited.item()) < 100 * limit_ns, f"waited {int(waited.item())} ns"

    # The context is still usable: a decode call right after gives the oracle's result.
    q, kc, vc = randn((2, 4, 128), torch.bfloat16, 7), randn((2, 4, 300, 128), torch.bfloat16, 8), \
        randn((2, 4, 300, 128), torch.bfloat16, 9)
    lengths = torch.tensor([300, 77])
    out = kernels.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), 300, 128**-0.5)
    check_attention(out, oatt.decode_attention(q, kc, vc, lengths, 128**-0.5), torch.bfloat16, what="after timeout")
    assert kernels.read_status() == 0


def test_selftest_rejects_long_limits():
    from omniasr_b200 import _lib

    lib = _lib.load()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.omniasr_selftest_wait_timeout(10**9, None, None, stream) == _lib.ERR_ARGUMENT
