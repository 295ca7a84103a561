"""The request-sharded launcher (``omniasr_b200.launch.run_sharded``) on the CPU: worker processes with a ``gloo``
start barrier, as on the GPUs of one box but with the host as the device.

* Real decoding: two workers each run the reference's GreedyDecoder (the small random model of its own tests,
  tests/test_decode.py:17-28, float64) on their shard of contexts; the gathered token sequences equal a
  single-process run, in request order.
* Failure detection: a worker that exits, raises, or never finishes is reported by the parent with its rank and the
  reason, the other workers are stopped, and nothing waits forever (the start barrier has a short group timeout).
"""

import os
import sys
import time

import pytest
import torch

from conftest import ROOT
from omniasr_b200.launch import WorkerFailed, run_sharded


def _reference_src() -> str:
    """The reference package, as __graft_entry__.build() places it in baseline/_ref."""
    p = ROOT / "baseline" / "_ref"
    if os.path.exists(os.path.join(str(p), "omniasr_trt", "decode.py")):
        return str(p)
    pytest.fail("the reference package is missing (run __graft_entry__.build())")


def _small_model(modeling, seed=0, vocab=12):
    torch.manual_seed(seed)
    enc = modeling.EncoderConfig(model_dim=16, num_layers=2, num_heads=2, ffn_dim=32, feature_dim=8,
                                 conv_layers=((8, 10, 5), (8, 3, 2), (8, 2, 2)), pos_kernel=4, pos_groups=2)
    dec = modeling.DecoderConfig(model_dim=32, num_layers=2, num_heads=2, ffn_dim=24, vocab_size=vocab, num_langs=5,
                                 max_seq_len=8192)
    m = modeling.LLMModel(enc, dec).double().eval()
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0, 0.5)
        m.final_proj.weight.mul_(4)
    return m


def _contexts():
    g = torch.Generator().manual_seed(1)
    lens = [int(x) for x in torch.randint(3, 40, (7,), generator=g)]
    return [torch.randn(n, 32, generator=g, dtype=torch.float64) for n in lens]


def greedy_factory(rank, device, src=None):
    """Worker side: the reference's GreedyDecoder on its small model; returns shard -> token lists."""
    src = src or _reference_src()
    if src not in sys.path:
        sys.path.insert(0, src)
    from omniasr_trt import decode, modeling

    m = _small_model(modeling)
    dec = decode.GreedyDecoder(m, max_batch=4, sync_every=5, graphs=False, reserve=32)
    return lambda shard: dec.generate(shard)


def exiting_factory(rank, device):
    if rank == 1:
        os._exit(3)  # dies without a word
    return lambda shard: [x * 2 for x in shard]


def raising_factory(rank, device):
    def fn(shard):
        if rank == 1:
            raise ValueError("planted failure in rank 1")
        return [x * 2 for x in shard]

    return fn


def hanging_factory(rank, device):
    def fn(shard):
        if rank == 0:
            time.sleep(600)  # never finishes within the parent's deadline
        return [x * 2 for x in shard]

    return fn


def doubling_factory(rank, device):
    return lambda shard: [x * 2 for x in shard]


def test_two_workers_decode_their_shards_in_request_order():
    ctxs = _contexts()
    want = greedy_factory(0, torch.device("cpu"))(ctxs)
    assert any(len(t) > 3 for t in want)
    got = run_sharded(greedy_factory, ctxs, 2, device_type="cpu", backend="gloo", timeout_s=300)
    assert got == want


@pytest.mark.parametrize("world", [1, 3])
def test_results_in_order_for_any_world(world):
    assert run_sharded(doubling_factory, list(range(8)), world, device_type="cpu", timeout_s=120) == \
        [2 * x for x in range(8)]


def test_worker_that_exits_is_reported():
    t0 = time.monotonic()
    with pytest.raises(WorkerFailed) as e:
        run_sharded(exiting_factory, list(range(6)), 2, device_type="cpu", backend="gloo", timeout_s=120,
                    group_timeout_s=10)
    assert e.value.rank == 1 and "exited with code 3" in e.value.reason
    assert time.monotonic() - t0 < 60


def test_worker_that_raises_is_reported_with_its_traceback():
    with pytest.raises(WorkerFailed) as e:
        run_sharded(raising_factory, list(range(6)), 2, device_type="cpu", backend="gloo", timeout_s=120)
    assert e.value.rank == 1 and "planted failure in rank 1" in e.value.reason


def test_worker_that_never_finishes_times_out():
    t0 = time.monotonic()
    with pytest.raises(WorkerFailed) as e:
        run_sharded(hanging_factory, list(range(6)), 2, device_type="cpu", timeout_s=15)
    assert e.value.rank == 0 and "timed out" in e.value.reason
    assert time.monotonic() - t0 < 60  # the hanging worker was terminated, not waited for
