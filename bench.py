#!/usr/bin/env python
"""Benchmark of the omniASR-LLM decoder-attention hot path on B200.

One step is the attention part of one speculative (spec-4) decoder step over a batch of 8 rows, for all 12 decoder
layers: per layer the fused RoPE + KV-cache append of the 40 new tokens (``kernels.rope_kv``) and the verify attention
of their 5 queries per row over the cache (``kernels.draft_attention``), 32 heads x 128, bf16, cache capacity 4096,
cached lengths U[200, 2000] (seed 0). Every layer has its own cache, so a step reads 12 x ~145 MB of K/V, far more
than the 126 MB L2; no flush is needed between steps.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]

Under torchrun (N > 1) every rank runs its own batch of 8 rows (request-sharded data parallel, weak scaling, no
collective on the path); the timed region is bracketed by a barrier and a device synchronisation, and the slowest
rank's time is reported. ``--impl reference`` times the CPU port of the reference's algorithm (the oracle) on the
host cores, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import shutil
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "omniasr-trt_b200"))
sys.path.insert(0, str(ROOT))

import numpy as np  # noqa: E402
import torch  # noqa: E402

B, T, H, D, CAP, LAYERS = 8, 5, 32, 128, 4096, 12
METRIC = "decode-attn HBM GB/s (spec-4 verify + fused RoPE/KV append, batch 8, 12 layers)"
NOMINAL_HBM_GBS = 8000.0


def peaks() -> tuple[float, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return float(json.loads(path.read_text())["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def workload_lengths() -> torch.Tensor:
    """Cached keys per row before the step, U[200, 2000] from the seed-0 CPU generator (drawn first)."""
    return torch.randint(200, 2001, (B,), generator=torch.Generator().manual_seed(0))


def keys_bucket(lengths: torch.Tensor) -> int:
    """The decoders' key bucket: the last query's keys rounded up to 256 (decode.py:349)."""
    return int((int(lengths.max()) + T + 255) // 256 * 256)


def algorithmic_bytes(lengths: torch.Tensor) -> dict:
    """Unique HBM bytes one layer must move (bf16): K/V of every key the last query of a row sees, the new qkv rows,
    their cos/sin rows, the appended K/V, the rotated q (written, then read) and the output."""
    kv_read = int((16384 * (lengths + T)).sum())  # 2 (K, V) x H x D x 2 B per key
    qkv = B * T * 3 * H * D * 2
    cs = B * T * (D // 2) * 2 * 4
    append = B * T * 2 * H * D * 2
    q_rw = 2 * B * T * H * D * 2
    out = B * T * H * D * 2
    attention = kv_read + B * T * H * D * 2 + out  # what draft_attention itself must move
    return {"layer": kv_read + qkv + cs + append + q_rw + out, "attention": attention, "kv_read": kv_read}


# --------------------------------------------------------------------------------------------------------- GPU arm


class Step:
    """The 12-layer attention step, captured once as a CUDA graph through the public API."""

    def __init__(self, device: torch.device, seed: int):
        from omniasr_b200 import kernels
        from oracle.rope import rope_table

        self.K = kernels
        assert kernels.available(device), "needs a B200 (compute capability 10.0) and the built library"
        self.device = device
        lengths = workload_lengths()
        self.lengths_cpu = lengths
        self.keys = keys_bucket(lengths)
        gen = torch.Generator(device=device).manual_seed(seed)
        self.kc = [torch.randn(B, H, CAP, D, generator=gen, device=device, dtype=torch.bfloat16) for _ in range(LAYERS)]
        self.vc = [torch.randn(B, H, CAP, D, generator=gen, device=device, dtype=torch.bfloat16) for _ in range(LAYERS)]
        self.qkv = torch.randn(LAYERS, B * T, 3 * H * D, generator=gen, device=device, dtype=torch.bfloat16)
        self.cs = rope_table(D, CAP).to(device)
        j = torch.arange(T)
        self.pos = (lengths[:, None] + j).reshape(-1).to(device)  # input positions of the 5 fed tokens
        self.slots = torch.arange(B).repeat_interleave(T).to(device)
        self.att_len = (lengths + 1).to(device)  # query i of a row sees lengths + 1 + i keys (spec.py:95)
        self.scale = D**-0.5
        self.graph = None
        self.outs = None
        self.ev = None

    def run(self, timed_events: bool = False):
        outs = []
        for i in range(LAYERS):
            q = self.K.rope_kv(self.qkv[i], self.cs, self.pos, self.kc[i], self.vc[i], H, self.slots)
            if timed_events:
                self.ev[i][0].record()
            outs.append(self.K.draft_attention(q, self.kc[i], self.vc[i], self.att_len, T, self.keys, self.scale))
            if timed_events:
                self.ev[i][1].record()
        return outs

    def capture(self):
        self.ev = [(torch.cuda.Event(enable_timing=True, external=True),
                    torch.cuda.Event(enable_timing=True, external=True)) for _ in range(LAYERS)]
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.run()  # warm-up outside the capture (the appended K/V are rewritten identically)
            torch.cuda.synchronize(self.device)
            self.graph = torch.cuda.CUDAGraph()
            self.graph.capture_begin()
            self.outs = self.run(timed_events=True)
            self.graph.capture_end()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)

    def attention_ms(self) -> list[float]:
        """Per-layer duration of the verify attention in the last replay (CUDA events inside the graph)."""
        return [a.elapsed_time(b) for a, b in self.ev]


class Clocks:
    """nvidia-smi samples during the timed region (SM clock, throttle reasons)."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.proc = None
        self.path = None
        if shutil.which("nvidia-smi") is None:
            return
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.f = open(self.path, "w")
        self.proc = subprocess.Popen(["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f,
                                     stderr=subprocess.DEVNULL)
        time.sleep(0.3)

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.2)
        self.proc.terminate()
        self.proc.wait()
        self.f.close()
        rows = [ln.split(",") for ln in Path(self.path).read_text().splitlines() if ln.strip()]
        os.unlink(self.path)
        sm = [float(r[1]) for r in rows if len(r) >= 9 and r[1].strip().replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if len(r) >= 9 and r[2].strip().replace(".", "").isdigit()]
        reasons = set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for r in rows:
            if len(r) >= 9:
                for name, v in zip(names, r[5:9]):
                    if v.strip() == "Active":
                        reasons.add(name)
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def traffic_per_launch() -> float | None:
    """DRAM bytes per verify-attention call from the committed ncu summary, if one is present."""
    path = ROOT / "profiles" / "roofline_traffic.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("draft_attention_config2_bytes_per_call="):
            return float(line.split("=", 1)[1])
    return None


def cpu_baseline(seconds: float = 10.0) -> dict:
    """The CPU port of the reference's path (oracle) on one layer of the same workload, on all host cores."""
    from oracle import attention as oatt
    from oracle import rope as orope

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    lengths = workload_lengths()
    keys = keys_bucket(lengths)
    g = torch.Generator().manual_seed(1)
    kc = torch.randn(B, H, keys, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, H, keys, D, generator=g).to(torch.bfloat16)
    qkv = torch.randn(B * T, 3 * H * D, generator=g).to(torch.bfloat16)
    cs = orope.rope_table(D, CAP).numpy()
    pos = (lengths[:, None] + torch.arange(T)).reshape(-1).numpy()
    slots = np.repeat(np.arange(B), T)
    kn = kc.view(torch.int16).numpy().view(np.uint16)
    vn = vc.view(torch.int16).numpy().view(np.uint16)
    qkv_raw = qkv.view(torch.int16).numpy().view(np.uint16)
    nbytes = algorithmic_bytes(lengths)["layer"]

    def one():
        qn = orope.rope_kv(qkv_raw, cs, pos, kn, vn, H, slots, None, True)
        q = torch.from_numpy(qn.astype(np.int16)).view(torch.bfloat16)
        oatt.draft_attention_model_dtype(q, kc, vc, lengths + 1, T, D**-0.5)

    one()
    reps, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or reps < 3:
        one()
        reps += 1
    dt = (time.perf_counter() - t0) / reps
    return {"value": nbytes / dt / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"1 of the 12 layers of a step (B=8, T=5, 32x128, same lengths), {reps} repetitions over "
                      f"{seconds:.0f} s: oracle RoPE/append (numpy) + model-dtype verify attention (torch CPU)"}


def run_gpu(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch.distributed as dist

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    step = Step(device, seed=1000 + rank)
    step.capture()
    nbytes = algorithmic_bytes(step.lengths_cpu)
    step_bytes = nbytes["layer"] * LAYERS

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # --- device-resident timing (value) ---
    for _ in range(args.warmup):
        step.graph.replay()
    torch.cuda.synchronize(device)
    clocks = Clocks(device.index) if rank == 0 else None
    barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        step.graph.replay()
    end.record()
    torch.cuda.synchronize(device)
    barrier()
    clock = clocks.stop() if clocks else None
    ms = max_over_ranks(start.elapsed_time(end))
    att_ms = step.attention_ms()  # the last timed step's per-layer verify attention
    att_ms = max_over_ranks(float(np.mean(att_ms)))

    # --- end to end through the public API: host qkv in, outputs back to the host, every step ---
    qkv_host = torch.empty_like(step.qkv, device="cpu").pin_memory()
    qkv_host.copy_(step.qkv.cpu())
    out_host = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in step.outs]
    stream = torch.cuda.current_stream(device)

    def e2e_step():
        step.qkv.copy_(qkv_host, non_blocking=True)
        step.graph.replay()
        for h, o in zip(out_host, step.outs):
            h.copy_(o, non_blocking=True)

    for _ in range(args.warmup):
        e2e_step()
    barrier()
    torch.cuda.synchronize(device)
    s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e2.record(stream)
    torch.cuda.synchronize(device)
    barrier()
    e2e_ms = max_over_ranks(s2.elapsed_time(e2))

    if rank != 0:
        return None
    peak, peak_kind = peaks()
    ms_step = ms / args.steps
    value = world * step_bytes / (ms_step * 1e-3) / 1e9
    achieved = nbytes["attention"] / (att_ms * 1e-3) / 1e9
    traffic = traffic_per_launch()
    line = {
        "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic (seeded N(0,1) bf16 caches and qkv; lengths seed 0)",
        "pct_of_8tbs": round(100 * value / world / NOMINAL_HBM_GBS, 1),
        "config": {"workload": "BASELINE config 2: spec-4 verify attention + fused RoPE/KV append, batch 8 per GPU, "
                               "T=5, 32x128 heads, lengths U[200,2000], cache 4096, 12 layers per step",
                   "global_batch": B * world, "q_len": T, "heads": H, "head_dim": D, "layers": LAYERS,
                   "keys_bucket": step.keys, "bytes_per_step_per_gpu": step_bytes,
                   "l2": "inputs larger than L2: each step reads 12 distinct layer caches (~1.7 GB)",
                   "parallelism": f"request-sharded dp{world} (no collective)"},
        "e2e": {"value": round(world * step_bytes / (e2e_ms / args.steps * 1e-3) / 1e9, 1), "unit": "GB/s",
                "ms_per_step": round(e2e_ms / args.steps, 4),
                "h2d_bytes_per_step": int(qkv_host.numel() * qkv_host.element_size()),
                "d2h_bytes_per_step": int(sum(o.numel() * o.element_size() for o in out_host)),
                "path": "kernels.rope_kv + kernels.draft_attention captured in a CUDA graph; pinned host qkv copied "
                        "in and every layer's output copied out each step"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 3), "peak_kind": peak_kind,
                     "kernel": "draft_attention (split + combine launches of one layer)",
                     "traffic": traffic, "bytes_per_launch": nbytes["attention"],
                     "us_per_launch": round(att_ms * 1e3, 2)},
        "gpu_launches": 3 * LAYERS * args.steps,
        "clocks": clock,
    }
    if world == 1:
        line["cpu_baseline"] = cpu_baseline()
    return line


# --------------------------------------------------------------------------------------------------- reference arm


def run_reference(args, rank: int) -> dict | None:
    """The CPU port of the reference's algorithm (oracle), on all host cores, rank 0 only."""
    if rank != 0:
        return None
    from oracle import attention as oatt
    from oracle import rope as orope

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    lengths = workload_lengths()
    keys = keys_bucket(lengths)
    g = torch.Generator().manual_seed(1)
    kc = torch.randn(B, H, keys, D, generator=g).to(torch.bfloat16)
    vc = torch.randn(B, H, keys, D, generator=g).to(torch.bfloat16)
    qkv = torch.randn(B * T, 3 * H * D, generator=g).to(torch.bfloat16)
    cs = orope.rope_table(D, CAP).numpy()
    pos = (lengths[:, None] + torch.arange(T)).reshape(-1).numpy()
    slots = np.repeat(np.arange(B), T)
    kn = kc.view(torch.int16).numpy().view(np.uint16)
    vn = vc.view(torch.int16).numpy().view(np.uint16)
    qkv_raw = qkv.view(torch.int16).numpy().view(np.uint16)

    def one_layer():
        qn = orope.rope_kv(qkv_raw, cs, pos, kn, vn, H, slots, None, True)
        q = torch.from_numpy(qn.astype(np.int16)).view(torch.bfloat16)
        return oatt.draft_attention_model_dtype(q, kc, vc, lengths + 1, T, D**-0.5)

    for _ in range(args.warmup):
        one_layer()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        one_layer()
    dt = (time.perf_counter() - t0) / args.steps
    value = algorithmic_bytes(lengths)["layer"] / dt / 1e9
    sample = "one layer of the step per timed iteration (B=8, T=5, 32x128, same lengths); GB/s is size-independent"
    return {"impl": "reference", "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "BASELINE config 2 (one layer per step on the CPU)", "global_batch": B,
                       "q_len": T, "heads": H, "head_dim": D},
            "cpu_baseline": {"value": round(value, 2), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 2), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    args = p.parse_args()
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        line = run_reference(args, rank)
        if line:
            print(json.dumps(line), flush=True)
        return
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        line = run_gpu(args, rank, world, local_rank)
        if line:
            print(json.dumps(line), flush=True)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
