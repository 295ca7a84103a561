"""Request-sharded transcription over the GPUs of one box: one worker process per GPU, no collective on the data path.

Every input's result depends only on that input (the reference's llm.py:7-9), so a list of requests is cut into
contiguous shards (:func:`omniasr_b200.shard.shard_bounds`), worker ``r`` runs shard ``r`` on ``cuda:r`` through its
own decoder (typically ``OmniASRLLM.transcribe`` with these kernels dropped in), and the parent puts the results back
in request order. Workers share nothing but an optional start barrier (a ``torch.distributed`` group over
127.0.0.1, ``gloo`` or ``nccl``); results come back through one pipe per worker.

Failure detection is on the host: the parent watches every worker's pipe and process sentinel against a deadline. A
worker that raises, exits without a result, or is still running at the deadline is reported as
:class:`WorkerFailed` with its rank and the reason (the traceback, the exit code, or the timeout); the other workers
are then stopped. A worker that dies before the start barrier makes the others' barrier end with an error after the
group's timeout, so no rank waits forever.

    def factory(rank, device):                      # runs in the worker, once
        from omniasr_b200 import dropin; dropin.install()
        from omniasr_trt import OmniASRLLM
        model = OmniASRLLM.from_pretrained(path, device=device)
        return lambda shard: model.transcribe([a for a, _ in shard], [l for _, l in shard])

    texts = run_sharded(factory, list(zip(audio, langs)), world=8)
"""

from __future__ import annotations

import datetime
import multiprocessing as mp
import socket
import time
import traceback
from multiprocessing.connection import wait
from typing import Any, Callable, Sequence

from .shard import shard_bounds


class WorkerFailed(RuntimeError):
    """A worker raised, exited without a result, or did not finish before the deadline."""

    def __init__(self, rank: int, reason: str):
        super().__init__(f"worker {rank}: {reason}")
        self.rank = rank
        self.reason = reason


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, factory: Callable, requests: Sequence[Any], conn, device_type: str,
            backend: str | None, port: int, group_timeout_s: float) -> None:
    group = False
    try:
        import torch

        if device_type == "cuda":
            torch.cuda.set_device(rank)
            device = torch.device("cuda", rank)
        else:
            device = torch.device("cpu")
        if backend and world > 1:
            import torch.distributed as dist

            kw = {"device_id": device} if backend == "nccl" else {}
            dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                    timeout=datetime.timedelta(seconds=group_timeout_s), **kw)
            group = True
            dist.barrier()  # start together; a rank that never arrives ends this with an error after the timeout
        fn = factory(rank, device)
        results = list(fn(list(requests)))
        if len(results) != len(requests):
            raise RuntimeError(f"{len(results)} results for {len(requests)} requests")
        conn.send(("ok", results))
    except BaseException:  # noqa: BLE001 -- every failure goes back to the parent
        try:
            conn.send(("error", traceback.format_exc()))
        except Exception:  # noqa: BLE001 -- the parent then sees the exit code
            pass
        raise SystemExit(1)
    finally:
        if group:
            import torch.distributed as dist

            dist.destroy_process_group()
        conn.close()


def run_sharded(factory: Callable, requests: Sequence[Any], world: int, *, device_type: str = "cuda",
                backend: str | None = None, timeout_s: float = 3600.0, group_timeout_s: float = 60.0,
                start_method: str = "spawn") -> list:
    """Runs ``factory(rank, device)(shard)`` in one process per rank over contiguous shards of ``requests`` and
    returns every result in request order.

    ``factory`` must be picklable (a module-level function): it builds the worker's decoder once and returns a
    function from a list of requests to the list of their results. ``device_type`` "cuda" puts rank r on
    ``cuda:r``; "cpu" runs the workers on the host. ``backend`` ("gloo" / "nccl" / None) adds a start barrier.
    Raises :class:`WorkerFailed` when a worker raises, exits without its results, or is still running
    ``timeout_s`` seconds after the start; the other workers are then terminated."""
    if world <= 0:
        raise ValueError(f"world {world}")
    total = len(requests)
    ctx = mp.get_context(start_method)
    port = _free_port()
    procs, conns = [], []
    for rank in range(world):
        a, b = shard_bounds(total, world, rank)
        parent, child = ctx.Pipe(duplex=False)
        p = ctx.Process(target=_worker, args=(rank, world, factory, list(requests[a:b]), child, device_type,
                                              backend, port, group_timeout_s), daemon=True)
        p.start()
        child.close()
        procs.append(p)
        conns.append(parent)
    results: list = [None] * world
    pending = set(range(world))
    deadline = time.monotonic() + timeout_s
    try:
        while pending:
            left = deadline - time.monotonic()
            if left <= 0:
                rank = min(pending)
                raise WorkerFailed(rank, f"no result within {timeout_s:g} s (timed out)")
            ready = wait([conns[r] for r in pending] + [procs[r].sentinel for r in pending], timeout=left)
            for r in sorted(pending):
                if conns[r] in ready or conns[r].poll():
                    try:
                        kind, payload = conns[r].recv()
                    except EOFError:
                        procs[r].join(5)
                        raise WorkerFailed(r, f"exited with code {procs[r].exitcode} before sending results")
                    if kind != "ok":
                        raise WorkerFailed(r, f"raised:\n{payload}")
                    results[r] = payload
                    pending.discard(r)
                elif procs[r].sentinel in ready:
                    procs[r].join(5)
                    if conns[r].poll():  # the result arrived just before the exit
                        continue
                    raise WorkerFailed(r, f"exited with code {procs[r].exitcode} before sending results")
    finally:
        for p in procs:
            if p.is_alive() and pending:
                p.terminate()
        for p in procs:
            p.join(10)
            if p.is_alive():
                p.kill()
                p.join(5)
        for c in conns:
            c.close()
    out: list = []
    for rank, part in enumerate(results):
        a, b = shard_bounds(total, world, rank)
        if len(part) != b - a:
            raise WorkerFailed(rank, f"{len(part)} results for {b - a} requests")
        out.extend(part)
    return out


def visible_gpus() -> int:
    """Number of GPUs this process may use (CUDA_VISIBLE_DEVICES honoured)."""
    import torch

    return torch.cuda.device_count() if torch.cuda.is_available() else 0


__all__ = ["WorkerFailed", "run_sharded", "visible_gpus"]
