#!/usr/bin/env python
"""Benchmark of the omniASR-LLM decoder-attention hot path on B200.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference] [--workload NAME] [--layers L]

The default workload (``verify``) is the headline: one step is the attention part of one
speculative (spec-4) decoder step over a batch of 8 rows, for all 12 decoder layers -- per layer the fused RoPE +
KV-cache append of the 40 new tokens (``kernels.rope_kv``) and the verify attention of their 5 queries per row over
the cache (``kernels.draft_attention``), 32 heads x 128, bf16, cache capacity 4096, cached lengths U[200, 2000]
(seed 0). Every layer has its own cache, so a step reads 12 x ~145 MB of K/V, far more than the 126 MB L2; no flush
is needed between steps. The other BASELINE configs are their own workloads, each printing one line of the same form:

    decode   config 1: q_len-1 decode attention, batch 8, 1024 keys per row, 12 layers
    beam     config 3: beam attention, 8 inputs x 5 beams, context U[300, 1800] shared per input, 12 layers
    gather   config 3: the K/V-cache reorder of the beam step by int32 parents (bit-exact row gather)
    prefill  config 4: causal prefill attention, 8 rows x 1500 frames, 12 layers (tensor-bound: TFLOP/s)
    sweep    config 5: 64 rows sharded over the ranks, q_len 1 and 5, lengths 512 / 2048 / 8192

Under torchrun (N > 1) every rank runs its own shard (request-sharded data parallel, no collective on the path);
the timed region is bracketed by a barrier and a device synchronisation, and the slowest rank's time is reported.
``--impl reference`` times the CPU port of the reference's algorithm (the oracle) on the host cores, rank 0 only.
``--layers`` shrinks a workload (for profiling captures); the line then says so in ``config``.
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

H, D, LAYERS = 32, 128, 12
NOMINAL_HBM_GBS = 8000.0
KV_TOKEN = 2 * H * D * 2  # K + V bytes of one token in one layer (bf16)


def peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        d = json.loads(path.read_text())
        return {"hbm": float(d["hbm_gbs"]), "tensor": float(d["bf16_tflops"]), "kind": "measured"}
    return {"hbm": 6650.0, "tensor": 1590.0, "kind": "fallback"}


def traffic_per_launch(key: str) -> float | None:
    """DRAM bytes per launch of a workload's dominant kernel from the committed ncu summary, if present. Head
    geometries other than 32 x 128 have their own lines (suffix `_d<head_dim>`)."""
    path = ROOT / "profiles" / "roofline_traffic.txt"
    if not path.exists():
        return None
    if D != 128:
        key = f"{key}_d{D}"
    for line in path.read_text().splitlines():
        if line.startswith(f"{key}="):
            return float(line.split("=", 1)[1])
    return None


def cpu_gen(seed: int = 0) -> torch.Generator:
    return torch.Generator().manual_seed(seed)


def rope_table(positions: int, theta: float = 10_000.0) -> torch.Tensor:
    """The decoder's cos/sin input table [positions, D/2, 2] float32 (the reference's modeling.py:293-298)."""
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float32) / D))
    angles = torch.outer(torch.arange(positions, dtype=torch.float32), inv)
    return torch.stack([torch.cos(angles), torch.sin(angles)], -1)


def keys_bucket(n: int) -> int:
    """The decoders' key bucket: rounded up to 256 (decode.py:349)."""
    return (n + 255) // 256 * 256


# ------------------------------------------------------------------------------------------------------ workloads


class Workload:
    """One step of a BASELINE config through the public API (``omniasr_b200.kernels``), captured as a CUDA graph.

    A step is ``layers`` layers (or cases); ``layer(i, ev)`` issues layer i's launches and returns the results a
    caller reads back, with ``ev`` (a pair of events) recorded around the dominant (roofline) call, and
    ``layer_in(i)`` names the device inputs layer i takes from the host in the end-to-end step. ``step_units`` is the
    algorithmic bytes (or FLOPs) of one step on this rank and ``roof_units`` those of one roofline call."""

    name = ""
    metric = ""
    unit = "GB/s"
    bound = "hbm"
    roof_kernel = ""
    traffic_key = ""
    calls_per_layer = 1
    # How the roofline call's duration is taken: "whole" -- a step is nothing but the dominant calls, so one call is
    # the event-free step time / layers; "difference" -- the step minus the same step without the dominant calls
    # (both event-free graphs); "events" -- CUDA events around each dominant call in a second graph.
    roof_timing = "whole"
    dominant_per_layer = 1  # dominant (roofline) calls per layer
    skip_dominant = False  # set while capturing the step without its dominant calls ("difference")
    gpu_reference_unavailable = None  # why the reference's GPU kernels are not timed on this workload, if so

    def __init__(self, device: torch.device, rank: int, world: int, layers: int):
        from omniasr_b200 import kernels

        self.K = kernels
        assert kernels.available(device), "needs a B200 (compute capability 10.0) and the built library"
        self.device, self.rank, self.world, self.layers = device, rank, world, layers
        self.gen = torch.Generator(device=device).manual_seed(1000 + rank)
        self.d2h: list[list[torch.Tensor]] = []  # per layer, the results read back in the end-to-end step

    def randn(self, *shape):
        return torch.randn(*shape, generator=self.gen, device=self.device, dtype=torch.bfloat16)

    def layer(self, i: int, ev=None) -> list[torch.Tensor]:
        raise NotImplementedError

    def layer_in(self, i: int) -> list[torch.Tensor]:
        return []

    def run(self, ev=None):
        self.d2h = [self.layer(i, ev[i] if ev else None) for i in range(self.layers)]

    def config(self) -> dict:
        raise NotImplementedError

    def launches_per_step(self) -> int:
        return self.calls_per_layer * self.layers


class Verify(Workload):
    """fused RoPE/KV append + spec-4 verify attention, batch 8, 12 layers."""

    name = "verify"
    metric = "decode-attn HBM GB/s (spec-4 verify + fused RoPE/KV append, batch 8, 12 layers)"
    roof_kernel = "draft_attention (the pass of one layer, split units merged inside it)"
    traffic_key = "draft_attention_config2_bytes_per_call"
    B, T, CAP = 8, 5, 4096
    calls_per_layer = 2  # rope_kv, attention pass (it merges split units itself)
    roof_timing = "difference"

    @classmethod
    def lengths(cls) -> torch.Tensor:
        """Cached keys per row before the step, U[200, 2000] from the seed-0 CPU generator (drawn first)."""
        return torch.randint(200, 2001, (cls.B,), generator=cpu_gen(0))

    @classmethod
    def bytes(cls, lengths: torch.Tensor) -> dict:
        """Unique HBM bytes one layer must move (bf16): K/V of every key the last query of a row sees, the new qkv
        rows, their cos/sin rows, the appended K/V, the rotated q (written, then read) and the output."""
        B, T = cls.B, cls.T
        kv_read = int((KV_TOKEN * (lengths + T)).sum())
        qkv = B * T * 3 * H * D * 2
        cs = B * T * (D // 2) * 2 * 4
        append = B * T * 2 * H * D * 2
        q_rw = 2 * B * T * H * D * 2
        out = B * T * H * D * 2
        attention = kv_read + B * T * H * D * 2 + out  # what draft_attention itself must move
        return {"layer": kv_read + qkv + cs + append + q_rw + out, "attention": attention}

    def __init__(self, *a):
        super().__init__(*a)
        B, T, CAP = self.B, self.T, self.CAP
        lengths = self.lengths()
        self.lengths_cpu = lengths
        self.keys = keys_bucket(int(lengths.max()) + T)
        self.kc = [self.randn(B, H, CAP, D) for _ in range(self.layers)]
        self.vc = [self.randn(B, H, CAP, D) for _ in range(self.layers)]
        self.qkv = self.randn(self.layers, B * T, 3 * H * D)
        self.cs = rope_table(CAP).to(self.device)
        self.pos = (lengths[:, None] + torch.arange(T)).reshape(-1).to(self.device)  # positions of the 5 tokens
        self.slots = torch.arange(B).repeat_interleave(T).to(self.device)
        self.att_len = (lengths + 1).to(self.device)  # query i of a row sees lengths + 1 + i keys (spec.py:95)
        nb = self.bytes(lengths)
        self.step_units = nb["layer"] * self.layers
        self.roof_units = nb["attention"]

    def layer_in(self, i):
        return [self.qkv[i]]

    def layer(self, i, ev=None):
        q = self.K.rope_kv(self.qkv[i], self.cs, self.pos, self.kc[i], self.vc[i], H, self.slots)
        if self.skip_dominant:
            return [q]
        if ev:
            ev[0].record()
        o = self.K.draft_attention(q, self.kc[i], self.vc[i], self.att_len, self.T, self.keys, D**-0.5)
        if ev:
            ev[1].record()
        return [o]

    def config(self):
        return {"workload": "BASELINE config 2: spec-4 verify attention + fused RoPE/KV append, batch 8 per GPU, "
                            "T=5, 32x128 heads, lengths U[200,2000], cache 4096, 12 layers per step",
                "global_batch": self.B * self.world, "q_len": self.T, "heads": H, "head_dim": D,
                "layers": self.layers, "keys_bucket": self.keys, "bytes_per_step_per_gpu": self.step_units,
                "l2": "inputs larger than L2: each step reads 12 distinct layer caches (~1.7 GB)"}

    @classmethod
    def cpu_sampler(cls):
        from oracle import attention as oatt
        from oracle import rope as orope

        B, T = cls.B, cls.T
        lengths = cls.lengths()
        keys = keys_bucket(int(lengths.max()) + T)
        g = cpu_gen(1)
        kc = torch.randn(B, H, keys, D, generator=g).to(torch.bfloat16)
        vc = torch.randn(B, H, keys, D, generator=g).to(torch.bfloat16)
        qkv = torch.randn(B * T, 3 * H * D, generator=g).to(torch.bfloat16)
        cs = orope.rope_table(D, cls.CAP).numpy()
        pos = (lengths[:, None] + torch.arange(T)).reshape(-1).numpy()
        slots = np.repeat(np.arange(B), T)
        kn = kc.view(torch.int16).numpy().view(np.uint16)
        vn = vc.view(torch.int16).numpy().view(np.uint16)
        qkv_raw = qkv.view(torch.int16).numpy().view(np.uint16)

        def one():
            qn = orope.rope_kv(qkv_raw, cs, pos, kn, vn, H, slots, None, True)
            q = torch.from_numpy(qn.astype(np.int16)).view(torch.bfloat16)
            oatt.draft_attention_model_dtype(q, kc, vc, lengths + 1, T, D**-0.5)
            return cls.bytes(lengths)["layer"]

        return one, ("1 of the 12 layers of a step (B=8, T=5, 32x128, same lengths): oracle RoPE/append (numpy) + "
                     "model-dtype verify attention (torch CPU)")


class Decode(Workload):
    """q_len-1 decode attention, batch 8, 1024 keys per row (12 layer caches, > L2)."""

    name = "decode"
    metric = "decode-attn HBM GB/s (q_len 1, batch 8, 1024 keys, 12 layers)"
    roof_kernel = "decode_attention (the pass of one layer, split units merged inside it)"
    traffic_key = "decode_attention_config1_bytes_per_call"
    B, L = 8, 1024
    calls_per_layer = 1

    def __init__(self, *a):
        super().__init__(*a)
        B, L = self.B, self.L
        self.kc = [self.randn(B, H, L, D) for _ in range(self.layers)]
        self.vc = [self.randn(B, H, L, D) for _ in range(self.layers)]
        self.q = self.randn(self.layers, B, H, D)
        self.lengths = torch.full((B,), L, dtype=torch.int64, device=self.device)
        self.roof_units = B * L * KV_TOKEN + 2 * B * H * D * 2
        self.step_units = self.roof_units * self.layers

    def layer_in(self, i):
        return [self.q[i]]

    def layer(self, i, ev=None):
        if ev:
            ev[0].record()
        o = self.K.decode_attention(self.q[i], self.kc[i], self.vc[i], self.lengths, self.L, D**-0.5)
        if ev:
            ev[1].record()
        return [o]

    def config(self):
        return {"workload": "BASELINE config 1: decode attention, batch 8 per GPU, q_len 1, 32x128 heads, 1024 keys "
                            "per row, scale 1/sqrt(128), 12 layer caches per step",
                "global_batch": self.B * self.world, "q_len": 1, "heads": H, "head_dim": D, "layers": self.layers,
                "bytes_per_step_per_gpu": self.step_units, "l2": "inputs larger than L2 (12 x 134 MB per step)"}

    @classmethod
    def cpu_sampler(cls):
        from oracle import attention as oatt

        g = cpu_gen(0)
        q = torch.randn(cls.B, H, D, generator=g).to(torch.bfloat16)
        kc = torch.randn(cls.B, H, cls.L, D, generator=g).to(torch.bfloat16)
        vc = torch.randn(cls.B, H, cls.L, D, generator=g).to(torch.bfloat16)
        lengths = torch.full((cls.B,), cls.L, dtype=torch.int64)

        def one():
            oatt.draft_attention_model_dtype(q, kc, vc, lengths, 1, D**-0.5)
            return cls.B * cls.L * KV_TOKEN + 2 * cls.B * H * D * 2

        return one, "one decode-attention call (B=8, 1024 keys, 32x128): model-dtype masked softmax (torch CPU)"


class Beam(Workload):
    """BASELINE config 3 (attention): 8 inputs x 5 beams; the context is read once per input."""

    name = "beam"
    metric = "beam-attn HBM GB/s (8 inputs x 5 beams, context U[300,1800], 12 layers)"
    roof_kernel = "beam_attention (context pass and combine of one layer; the combine attends the generated keys)"
    traffic_key = "beam_attention_config3_bytes_per_call"
    S, N, CAP, G, GEN = 8, 5, 2048, 64, 32
    calls_per_layer = 2  # context pass (tensor cores), combine (with the generated keys)

    @classmethod
    def draw(cls):
        g = cpu_gen(0)
        ctx = torch.randint(300, 1801, (cls.S,), generator=g)
        picks = torch.randint(0, cls.N, (cls.S * cls.N, cls.G), generator=g, dtype=torch.int32)
        ptr = (torch.arange(cls.S * cls.N, dtype=torch.int32)[:, None] // cls.N) * cls.N + picks
        return ctx, ptr

    @classmethod
    def bytes(cls, ctx: torch.Tensor) -> int:
        rows = cls.S * cls.N
        return int(KV_TOKEN * ctx.sum()) + rows * cls.GEN * KV_TOKEN + rows * cls.GEN * 4 + 2 * rows * H * D * 2

    def __init__(self, *a):
        super().__init__(*a)
        S, N, rows = self.S, self.N, self.S * self.N
        ctx, ptr = self.draw()
        self.ctx_keys = keys_bucket(int(ctx.max()))
        self.kc = [self.randn(S, H, self.CAP, D) for _ in range(self.layers)]
        self.vc = [self.randn(S, H, self.CAP, D) for _ in range(self.layers)]
        self.kg = [self.randn(rows, H, self.G, D) for _ in range(self.layers)]
        self.vg = [self.randn(rows, H, self.G, D) for _ in range(self.layers)]
        self.q = self.randn(self.layers, rows, H, D)
        self.ctx = ctx.to(self.device)
        self.ptr = ptr.to(self.device)
        self.gen_len = torch.full((rows,), self.GEN, dtype=torch.int64, device=self.device)
        self.roof_units = self.bytes(ctx)
        self.step_units = self.roof_units * self.layers

    def layer_in(self, i):
        return [self.q[i]]

    def layer(self, i, ev=None):
        if ev:
            ev[0].record()
        o = self.K.beam_attention(self.q[i], self.kc[i], self.vc[i], self.ctx, self.kg[i], self.vg[i], self.ptr,
                                  self.gen_len, self.N, self.ctx_keys, D**-0.5)
        if ev:
            ev[1].record()
        return [o]

    def config(self):
        return {"workload": "BASELINE config 3 (attention): 8 inputs x 5 beams = 40 rows per GPU, q_len 1, 32x128, "
                            "context U[300,1800] shared per input (read once per input), 32 generated keys per row "
                            "through int32 pointers, 12 layers",
                "global_batch": self.S * self.N * self.world, "heads": H, "head_dim": D, "layers": self.layers,
                "bytes_per_step_per_gpu": self.step_units, "l2": "inputs larger than L2 (12 layers, ~1.5 GB)"}

    @classmethod
    def cpu_sampler(cls):
        from oracle import attention as oatt

        ctx, ptr = cls.draw()
        rows = cls.S * cls.N
        g = cpu_gen(1)
        q = torch.randn(rows, H, D, generator=g).to(torch.bfloat16)
        keys = keys_bucket(int(ctx.max()))
        kc = torch.randn(cls.S, H, keys, D, generator=g).to(torch.bfloat16)
        vc = torch.randn(cls.S, H, keys, D, generator=g).to(torch.bfloat16)
        kg = torch.randn(rows, H, cls.G, D, generator=g).to(torch.bfloat16)
        vg = torch.randn(rows, H, cls.G, D, generator=g).to(torch.bfloat16)
        gen_len = torch.full((rows,), cls.GEN, dtype=torch.int64)

        def one():
            oatt.beam_attention(q, kc, vc, ctx, kg, vg, ptr.long(), gen_len, cls.N, D**-0.5, dtype=torch.float32)
            return cls.bytes(ctx)

        return one, "one beam-attention call (40 rows, same lengths): per-row fp32 masked softmax (torch CPU)"


class Gather(Workload):
    """BASELINE config 3 (reorder): out[r] = src[parent[r]] over a layer's K and V cache rows, bit-exact."""

    name = "gather"
    metric = "beam KV reorder HBM GB/s (read + write, 40 rows x [32, 2048, 128] bf16, K and V)"
    roof_kernel = "reorder_gather (one launch per K or V tensor)"
    traffic_key = "reorder_gather_config3_bytes_per_call"
    S, N, CAP = 8, 5, 2048
    COPIES = 3  # distinct source layers cycled through, so a step never finds its source in L2

    @classmethod
    def parents(cls) -> torch.Tensor:
        picks = torch.randint(0, cls.N, (cls.S * cls.N,), generator=cpu_gen(0), dtype=torch.int32)
        return (torch.arange(cls.S * cls.N, dtype=torch.int32) // cls.N) * cls.N + picks

    def __init__(self, device, rank, world, layers):
        super().__init__(device, rank, world, min(layers, self.COPIES))
        rows = self.S * self.N
        self.src = [(self.randn(rows, H, self.CAP, D), self.randn(rows, H, self.CAP, D)) for _ in range(self.layers)]
        self.dst = (torch.empty_like(self.src[0][0]), torch.empty_like(self.src[0][1]))
        self.parent = self.parents().to(self.device)
        self.row_bytes = H * self.CAP * D * 2
        self.roof_units = 2 * rows * self.row_bytes  # read + write of one tensor
        self.step_units = 2 * self.roof_units * self.layers
        self.calls_per_layer = 2
        self.dominant_per_layer = 2

    def layer_in(self, i):
        return [self.parent] if i == 0 else []

    def layer(self, i, ev=None):
        for t in range(2):
            if ev and t == 0:
                ev[0].record()
            self.K.reorder_gather(self.src[i][t], self.parent, self.dst[t])
            if ev and t == 0:
                ev[1].record()
        # a few bytes of each gathered row after the last source: the step's visible result
        return [self.dst[0][:, 0, 0, :8]] if i == self.layers - 1 else []

    def config(self):
        return {"workload": "BASELINE config 3 (reorder): K and V cache rows [40, 32, 2048, 128] bf16 gathered by "
                            "int32 parents U[0,5) within each input's 5 beams",
                "rows": self.S * self.N, "row_bytes": self.row_bytes, "source_layers": self.layers,
                "bytes_per_step_per_gpu": self.step_units,
                "l2": f"inputs larger than L2 ({self.layers} distinct 671 MB sources per step)"}

    @classmethod
    def cpu_sampler(cls):
        from oracle import gather as og

        rows = cls.S * cls.N
        src = np.random.default_rng(0).integers(0, 65535, (rows, H * cls.CAP * D // 8), dtype=np.uint16)
        parent = cls.parents().numpy()

        def one():
            og.reorder_gather(src, parent)
            return 2 * src.nbytes

        return one, "the reorder of one 40-row tensor at 1/8 of the row length (numpy fancy indexing)"


class Prefill(Workload):
    """BASELINE config 4 (prefill): causal attention of 8 rows x 1500 frames, 12 layers, tensor-bound."""

    name = "prefill"
    metric = "prefill-attn TFLOP/s (causal, 8 x 1500 frames, 32x128, 12 layers)"
    unit = "TFLOP/s"
    bound = "tensor"
    roof_kernel = "prefill_attention (one launch per layer)"
    traffic_key = "prefill_attention_config4_bytes_per_call"
    B, W, CAP = 8, 1500, 2048

    def __init__(self, *a):
        super().__init__(*a)
        B, W = self.B, self.W
        # q as rope_kv returns it ([B*W, H, D]) and k/v as the prefill reads them: cache views (decode.py:156-158)
        self.q = self.randn(self.layers, B * W, H, D)
        self.kc = [self.randn(B, H, self.CAP, D) for _ in range(self.layers)]
        self.vc = [self.randn(B, H, self.CAP, D) for _ in range(self.layers)]
        self.roof_units = 4 * (W * (W + 1) // 2) * D * B * H  # QK^T and PV over the causal half (incl. diagonal)
        self.step_units = self.roof_units * self.layers

    def layer_in(self, i):
        return [self.q[i]]

    def layer(self, i, ev=None):
        q = self.q[i].view(self.B, self.W, H, D).transpose(1, 2)
        if ev:
            ev[0].record()
        o = self.K.prefill_attention(q, self.kc[i][:, :, :self.W], self.vc[i][:, :, :self.W], D**-0.5)
        if ev:
            ev[1].record()
        return [o]

    def config(self):
        return {"workload": "BASELINE config 4 (prefill attention): 8 rows x 1500 frames per GPU, causal, 32x128 "
                            "heads, q [B*W,H,D] and K/V cache views of capacity 2048, 12 layers",
                "global_batch": self.B * self.world, "width": self.W, "heads": H, "head_dim": D,
                "layers": self.layers, "flops_per_step_per_gpu": self.step_units,
                "l2": "inputs larger than L2 (12 layers x 294 MB of q/k/v per step)"}

    @classmethod
    def cpu_sampler(cls):
        g = cpu_gen(1)
        W = cls.W
        q = torch.randn(1, 8, W, D, generator=g).to(torch.bfloat16)
        k = torch.randn(1, 8, W, D, generator=g).to(torch.bfloat16)
        v = torch.randn(1, 8, W, D, generator=g).to(torch.bfloat16)

        def one():
            torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True)
            return 4 * (W * (W + 1) // 2) * D * 8

        return one, "one row x 8 heads x 1500 frames: torch SDPA (causal, bf16) on the CPU, the reference's call"


class Sweep(Workload):
    """64 rows sharded over the ranks; q_len 1 and 5 at lengths 512, 2048 and 8192."""

    name = "sweep"
    roof_timing = "events"  # the roofline call is the largest case (q5, 8192 keys, ~1 ms): events cost nothing there
    # The reference's Triton split kernel forms its cache offsets in 32-bit arithmetic (kernels.py:172-173,
    # b * s_kb + h * s_kh): with 64 rows x 32 heads x 8200 positions x 128 dims (2.15e9 elements) they overflow, and on
    # a B200 it raised an illegal memory access on this workload, so it is not run here.
    gpu_reference_unavailable = ("the reference's Triton kernels overflow 32-bit cache offsets at 64 rows x 8192 keys "
                                 "(kernels.py:172-173) and raised an illegal memory access on this workload")
    metric = "decode-attn HBM GB/s, whole box (64 rows sharded, q_len 1/5, lengths 512/2048/8192)"
    roof_kernel = "draft_attention (q_len 5, 8192 keys)"
    traffic_key = "draft_attention_config5_bytes_per_call"
    ROWS, CASES = 64, [(1, 512), (1, 2048), (1, 8192), (5, 512), (5, 2048), (5, 8192)]
    calls_per_layer = 1

    def __init__(self, device, rank, world, layers):
        super().__init__(device, rank, world, len(self.CASES))
        from omniasr_b200 import shard

        a, b = shard.shard_bounds(self.ROWS, world, rank)  # this rank's contiguous shard of the 64 rows
        self.rows = b - a
        self.keys = [L if t == 1 else keys_bucket(L + t) for t, L in self.CASES]
        cap = max(self.keys)
        self.kc = self.randn(self.rows, H, cap, D)
        self.vc = self.randn(self.rows, H, cap, D)
        self.q = {t: self.randn(self.rows * t, H, D) for t in (1, 5)}
        self.case_bytes = [self.rows * KV_TOKEN * (L + t - 1) + 2 * self.rows * t * H * D * 2 for t, L in self.CASES]
        self.roof_units = self.case_bytes[-1]
        self.step_units = sum(self.case_bytes)
        self.n = {L: torch.full((self.rows,), L, dtype=torch.int64, device=self.device) for _, L in self.CASES}

    def layer_in(self, i):
        t = self.CASES[i][0]
        first = next(j for j, c in enumerate(self.CASES) if c[0] == t)
        return [self.q[t]] if i == first else []

    def layer(self, i, ev=None):
        t, L = self.CASES[i]
        n, keys = self.n[L], self.keys[i]
        if ev:
            ev[0].record()
        if t == 1:
            o = self.K.decode_attention(self.q[1], self.kc, self.vc, n, keys, D**-0.5)
        else:
            o = self.K.draft_attention(self.q[5], self.kc, self.vc, n, t, keys, D**-0.5)
        if ev:
            ev[1].record()
        return [o]

    def config(self):
        return {"workload": "BASELINE config 5: 64 rows in all, sharded evenly over the GPUs, 32x128 heads; cases "
                            "q_len {1,5} x cached length {512, 2048, 8192}, one call each per step",
                "rows_per_gpu": self.rows, "cases": [f"q{t}_L{L}" for t, L in self.CASES],
                "bytes_per_step_per_gpu": self.step_units, "l2": "inputs larger than L2 (every case > 126 MB at 8 "
                                                                 "rows/GPU except 512 keys: 67 MB, 5 cases after it)"}

    @classmethod
    def cpu_sampler(cls):
        from oracle import attention as oatt

        g = cpu_gen(0)
        rows, L = 8, 2048
        q = torch.randn(rows * 5, H, D, generator=g).to(torch.bfloat16)
        kc = torch.randn(rows, H, L + 8, D, generator=g).to(torch.bfloat16)
        vc = torch.randn(rows, H, L + 8, D, generator=g).to(torch.bfloat16)
        n = torch.full((rows,), L, dtype=torch.int64)

        def one():
            oatt.draft_attention_model_dtype(q, kc, vc, n, 5, D**-0.5)
            return rows * KV_TOKEN * (L + 4) + 2 * rows * 5 * H * D * 2

        return one, "8 rows, q_len 5, 2048 keys (one case of the sweep): model-dtype masked softmax (torch CPU)"


class Gemm(Workload):
    """The decoder step's four weight GEMMs for 40 token rows (BASELINE config 4's batch 8 x spec-4 + 1), 12 layers:
    QKV, the output projection + residual, gate/inner + SwiGLU, the FFN output + residual (kernels.decode_gemm)."""

    name = "gemm"
    roof_timing = "events"
    metric = "decode GEMM weight-streaming GB/s (QKV, out+res, SwiGLU, FFN-out+res; 40 tokens; 12 layers)"
    roof_kernel = "decode_gemm (QKV: 12288 x 4096)"
    traffic_key = "decode_gemm_qkv_bytes_per_call"
    M, D_MODEL, FFN = 40, 4096, 11008
    calls_per_layer = 4

    def __init__(self, *a):
        super().__init__(*a)
        M, Dm, Fn = self.M, self.D_MODEL, self.FFN
        w = lambda r, c: (torch.randn(r, c, generator=self.gen, device=self.device) * 0.02).to(torch.bfloat16)  # noqa
        self.w = [(w(3 * Dm, Dm), w(Dm, Dm), w(2 * Fn, Dm), w(Dm, Fn)) for _ in range(self.layers)]
        self.x = self.randn(M, Dm)
        self.o = self.randn(M, Dm)
        self.h = self.randn(M, Dm)
        self.g = self.randn(M, Fn)
        per_layer = 2 * (3 * Dm * Dm + Dm * Dm + 2 * Fn * Dm + Dm * Fn)
        self.roof_units = 2 * 3 * Dm * Dm
        self.step_units = per_layer * self.layers

    def layer_in(self, i):
        return [self.x] if i == 0 else []

    def layer(self, i, ev=None):
        qkv_w, out_w, gi_w, ffo_w = self.w[i]
        if ev:
            ev[0].record()
        self.K.decode_gemm(self.x, qkv_w)
        if ev:
            ev[1].record()
        self.K.decode_gemm(self.o, out_w, "residual", residual=self.h)
        self.K.decode_gemm(self.x, gi_w, "swiglu")
        last = self.K.decode_gemm(self.g, ffo_w, "residual", residual=self.h)
        return [last] if i == self.layers - 1 else []

    def run_library(self):
        """torch.matmul / addmm (cuBLAS) and the SwiGLU elementwise, as the reference's decoder step computes them."""
        outs = []
        for i in range(self.layers):
            qkv_w, out_w, gi_w, ffo_w = self.w[i]
            outs.append(self.x @ qkv_w.t())
            outs.append(torch.addmm(self.h, self.o, out_w.t()))
            gate, inner = (self.x @ gi_w.t()).chunk(2, -1)
            outs.append(inner * torch.nn.functional.silu(gate))
            outs.append(torch.addmm(self.h, self.g, ffo_w.t()))
        return outs

    def config(self):
        return {"workload": "the decoder step's weight GEMMs (BASELINE config 4 model), 40 token rows, 12 layers of "
                            "distinct weights (~4.8 GB per step, far above L2)",
                "rows": self.M, "layers": self.layers, "bytes_per_step_per_gpu": self.step_units}

    @classmethod
    def cpu_sampler(cls):
        g = cpu_gen(0)
        x = torch.randn(cls.M, cls.D_MODEL, generator=g).to(torch.bfloat16)
        w = (torch.randn(cls.D_MODEL, cls.D_MODEL, generator=g) * 0.02).to(torch.bfloat16)

        def one():
            x @ w.t()
            return 2 * cls.D_MODEL * cls.D_MODEL

        return one, "the output projection (4096 x 4096, 40 rows) in torch on the CPU"


class QkvRope(Workload):
    """Row f1: the decoder step's QKV product with RoPE and the KV-cache append in its epilogue
    (kernels.decode_gemm_rope), for config 2's 8 rows x 5 tokens, 12 layers of distinct weights."""

    name = "qkvrope"
    roof_timing = "whole"
    metric = "QKV + RoPE/append weight-streaming GB/s (40 tokens, 4096 -> 3 x 32 x 128, 12 layers)"
    roof_kernel = "decode_gemm_rope (12288 x 4096, RoPE + cache append in the epilogue)"
    traffic_key = "decode_gemm_rope_bytes_per_call"
    B, T, D_MODEL, CAP = 8, 5, 4096, 4096

    def __init__(self, *a):
        super().__init__(*a)
        n, Dm = self.B * self.T, self.D_MODEL
        w = lambda r, c: (torch.randn(r, c, generator=self.gen, device=self.device) * 0.02).to(torch.bfloat16)  # noqa
        self.w = [w(3 * Dm, Dm) for _ in range(self.layers)]
        self.x = self.randn(n, Dm)
        from oracle import rope as orope

        self.cs = orope.rope_table(D, self.CAP + 8).contiguous().to(self.device)
        g = cpu_gen(0)
        base = torch.randint(200, 2001, (self.B,), generator=g)
        self.pos = (base[:, None] + torch.arange(self.T)[None]).reshape(-1).to(self.device)
        self.slots = torch.arange(self.B).repeat_interleave(self.T).to(self.device)
        self.kc = self.randn(self.B, H, self.CAP, D)
        self.vc = self.randn(self.B, H, self.CAP, D)
        self.roof_units = 2 * 3 * Dm * Dm + n * Dm * 2 + 3 * n * H * D * 2  # weights, x, q + k + v written
        self.step_units = self.roof_units * self.layers

    def layer_in(self, i):
        return [self.x] if i == 0 else []

    def layer(self, i, ev=None):
        if ev:
            ev[0].record()
        q = self.K.decode_gemm_rope(self.x, self.w[i], self.cs, self.pos, self.kc, self.vc, H, slots=self.slots)
        if ev:
            ev[1].record()
        return [q] if i == self.layers - 1 else []

    def run_library(self):
        """The reference's sequence: the product by torch (cuBLAS), then RoPE + append (this library's rope_kv)."""
        outs = []
        for i in range(self.layers):
            qkv = self.x @ self.w[i].t()
            outs.append(self.K.rope_kv(qkv, self.cs, self.pos, self.kc, self.vc, H, slots=self.slots))
        return outs

    def config(self):
        return {"workload": "row f1: QKV product + RoPE + KV append for config 2's 40 tokens (8 rows x spec-4 + 1), "
                            "32 x 128 heads, d_model 4096, 12 layers of distinct weights (1.2 GB per step)",
                "rows": self.B * self.T, "layers": self.layers, "bytes_per_step_per_gpu": self.step_units,
                "l2": "inputs larger than L2 (12 distinct 100 MB weight matrices per step)"}

    @classmethod
    def cpu_sampler(cls):
        g = cpu_gen(0)
        x = torch.randn(cls.B * cls.T, cls.D_MODEL, generator=g).to(torch.bfloat16)
        w = (torch.randn(3 * cls.D_MODEL, cls.D_MODEL, generator=g) * 0.02).to(torch.bfloat16)

        def one():
            x @ w.t()
            return 2 * 3 * cls.D_MODEL * cls.D_MODEL

        return one, "the QKV product (12288 x 4096, 40 rows) in torch on the CPU (RoPE left out)"


class Select(Workload):
    """BASELINE config 3 (beam step after the LM head): per input, the best 5 of 5 x 10288 candidates, then the rows
    follow their parents (pointer / history rows, scores, counts, flags), in place -- beam.py:161-187."""

    name = "select"
    metric = "beam selection HBM GB/s (8 inputs x 5 beams x 10288 vocab, bf16 log-probs, history 1024, 128 searches)"
    roof_kernel = "beam_select (one launch per search)"
    traffic_key = "beam_select_config3_bytes_per_call"
    S, N, V, G = 8, 5, 10288, 1024
    SEARCHES = 128  # independent searches per step: 128 x 1.5 MB of state, more than L2

    def __init__(self, device, rank, world, layers):
        super().__init__(device, rank, world, self.SEARCHES)
        r = self.S * self.N
        self.logp = [torch.log_softmax(self.randn(r, self.V).float() * 3, -1).to(torch.bfloat16)
                     for _ in range(self.layers)]
        g = torch.Generator(device=device).manual_seed(2000 + rank)
        dev = device
        self.state = []
        for _ in range(self.layers):
            self.state.append({
                "score": -torch.rand(r, generator=g, device=dev) * 20,
                "ended": torch.zeros(r, dtype=torch.bool, device=dev),
                "count": torch.randint(1, 50, (r,), generator=g, device=dev),
                "tok": torch.randint(3, self.V, (r,), generator=g, device=dev),
                "hist": torch.randint(3, self.V, (r, self.G + 1), generator=g, device=dev, dtype=torch.int32),
                "ptr": (torch.arange(r, device=dev)[:, None] // self.N * self.N
                        + torch.randint(0, self.N, (r, self.G), generator=g, device=dev)).to(torch.int32),
                "k_step": torch.full((self.S,), 64, dtype=torch.long, device=dev),
                "ctx": torch.randint(300, 1801, (self.S,), generator=g, device=dev),
                "gdone": torch.zeros(self.S, dtype=torch.bool, device=dev),
            })
        # logp once + the pointer and history rows read and written + the per-row / per-group scalars
        self.roof_units = (r * self.V * 2 + 2 * r * (2 * self.G + 1) * 4 + 2 * r * (4 + 1 + 8 + 8)
                           + 2 * self.S * (8 + 8 + 1))
        self.step_units = self.roof_units * self.layers

    def layer_in(self, i):
        return [self.logp[i]]

    def layer(self, i, ev=None):
        st = self.state[i]
        if ev:
            ev[0].record()
        self.K.beam_select(self.logp[i], st["score"], st["ended"], st["count"], st["tok"], st["hist"], st["ptr"],
                           st["k_step"], st["ctx"], st["gdone"], self.N, True, 2, 1, 8188)
        if ev:
            ev[1].record()
        return [st["tok"]]

    def config(self):
        return {"workload": "BASELINE config 3 (beam step): 8 inputs x 5 beams, bf16 log-probabilities over 10288 "
                            "tokens, length normalisation, history / pointer rows of 1024 positions; 128 independent "
                            "searches per step (the state advances one step per replay: k_step 64 + replays)",
                "rows": self.S * self.N, "vocab": self.V, "history": self.G, "searches": self.layers,
                "bytes_per_step_per_gpu": self.step_units,
                "l2": f"inputs larger than L2 ({self.layers} distinct searches, {self.step_units / 1e6:.0f} MB)"}

    @classmethod
    def cpu_sampler(cls):
        from oracle import beam as ob

        rng = np.random.default_rng(0)
        r = cls.S * cls.N
        logp = np.log(rng.dirichlet(np.ones(cls.V), r)).astype(np.float32)
        st = {"score": -rng.random(r).astype(np.float32) * 20, "ended": np.zeros(r, bool),
              "count": rng.integers(1, 50, r), "tok": rng.integers(3, cls.V, r),
              "hist": rng.integers(3, cls.V, (r, cls.G + 1)).astype(np.int32),
              "ptr": (np.arange(r)[:, None] // cls.N * cls.N + rng.integers(0, cls.N, (r, cls.G))).astype(np.int32),
              "k_step": np.full(cls.S, 64), "ctx": rng.integers(300, 1801, cls.S), "gdone": np.zeros(cls.S, bool)}
        units = r * cls.V * 2 + 2 * r * (2 * cls.G + 1) * 4

        def one():
            ob.beam_select(logp, **{k: v.copy() for k, v in st.items()}, beams=cls.N, length_norm=True, eos=2, pad=1,
                           limit=8188)
            return units

        return one, "one selection step of the 8 x 5 beams (numpy oracle, fp32 log-probabilities)"


WORKLOADS = {w.name: w for w in (Verify, Decode, Beam, Gather, Prefill, Sweep, Gemm, Select, QkvRope)}


# ------------------------------------------------------------------------------- the reference's own GPU kernels


def reference_beam_select(logp, score, ended, count, tok, hist, ptr, k_step, ctx, gdone, n, length_norm, eos, pad,
                          limit):
    """The reference's selection after the LM head as it runs it: the torch operations of BeamDecoder.step_beam,
    beam.py:161-187, on the first logp.size(0) rows (the reference has no kernel of its own for them)."""
    r, vocab = logp.shape
    s = r // n
    dev = logp.device
    tok, score, ended, count = tok[:r], score[:r], ended[:r], count[:r]
    k_step, ctx, gdone = k_step[:s], ctx[:s], gdone[:s]
    hist, ptr = hist[:r], ptr[:r]
    rows = torch.arange(r, device=dev)
    group = rows // n
    live = ~gdone[group]
    k = k_step[group]
    if length_norm:
        first = count[group * n][:, None]
        c = count[:, None]
        cand = torch.where(first > 0, (score[:, None] * c + logp) / (c + 1), score[:, None] + logp)
    else:
        cand = score[:, None] + logp
    cand = cand.masked_fill(ended[:, None], float("-inf"))
    cand[:, eos] = torch.where(ended, score, cand[:, eos])
    top, pick = cand.view(s, n * vocab).topk(n, dim=-1, sorted=True)
    parent = (pick // vocab + torch.arange(s, device=dev)[:, None] * n).view(-1)
    parent = torch.where(live, parent, rows)
    new = torch.where(live, (pick % vocab).view(-1), tok)
    ptr.copy_(ptr[parent])
    hist.copy_(hist[parent])
    p_ended, p_score, p_count = ended[parent], score[parent], count[parent]
    new = torch.where(p_ended, eos, new)
    hist.scatter_(1, k[:, None], torch.where(live, new, hist.gather(1, k[:, None])[:, 0].long())[:, None]
                  .to(hist.dtype))
    score.copy_(torch.where(live & ~p_ended, top.view(-1), p_score))
    count.copy_(p_count + (live & ~p_ended & (new != pad) & (new != eos)).long())
    ended.copy_(torch.where(live, new == eos, p_ended))
    tok.copy_(new)
    all_ended = ended.view(s, n).all(-1)
    k_step.copy_(k_step + (~gdone).long())
    gdone |= all_ended | (ctx - 1 + k_step - 1 >= limit)


def reference_gpu_kernels():
    """The reference's own GPU path for these workloads, unmodified: its Triton kernels (``omniasr_trt.kernels``:
    rope_kv, decode_attention, draft_attention, beam_attention, kernels.py:294-423) from baseline/_ref, torch's SDPA
    for the prefill exactly as decode.py:171 calls it, and ``index_select`` for the K/V reorder (llm.py:237-238).
    Returns (namespace, None) or (None, why not)."""
    import types

    ref = ROOT / "baseline" / "_ref"
    if not (ref / "omniasr_trt" / "kernels.py").exists():
        return None, "the reference package is not in baseline/_ref"
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    try:
        from omniasr_trt import kernels as rk
    except Exception as e:  # noqa: BLE001
        return None, f"importing the reference's kernels failed: {e!r}"
    if getattr(rk, "__omniasr_b200__", False):
        return None, "the reference's kernel module was replaced in this process"
    if not rk.available(torch.device("cuda")):
        return None, "the reference's Triton kernels are not available on this device"

    def prefill_attention(q, k, v, scale=None):
        return torch.nn.functional.scaled_dot_product_attention(q, k, v, is_causal=True, scale=scale)

    def reorder_gather(src, parent, out=None):
        return torch.index_select(src, 0, parent, out=out)

    ns = types.SimpleNamespace(rope_kv=rk.rope_kv, decode_attention=rk.decode_attention,
                               draft_attention=rk.draft_attention, beam_attention=rk.beam_attention,
                               prefill_attention=prefill_attention, reorder_gather=reorder_gather,
                               beam_select=reference_beam_select)
    return ns, None


def graph_ms(side: torch.cuda.Stream, device, fn, steps: int, warmup: int) -> float:
    """Captures ``fn`` (warmed up once outside the capture) in a CUDA graph on ``side`` and returns the mean replay
    time in ms over ``steps`` replays after ``warmup``, timed with CUDA events, no events inside the graph."""
    with torch.cuda.stream(side):
        fn()
        torch.cuda.synchronize(device)
        g = torch.cuda.CUDAGraph()
        g.capture_begin()
        fn()
        g.capture_end()
    torch.cuda.synchronize(device)
    for _ in range(warmup):
        g.replay()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(device)
    s.record()
    for _ in range(steps):
        g.replay()
    e.record()
    torch.cuda.synchronize(device)
    return s.elapsed_time(e) / steps


# --------------------------------------------------------------------------------------------------------- timing


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


def cpu_time(wl, seconds: float) -> dict:
    """The CPU port of the reference's path (oracle) on a bounded sample of the workload, on all host cores."""
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    one, sample = wl.cpu_sampler()
    one()
    reps, units, t0 = 0, 0.0, time.perf_counter()
    while time.perf_counter() - t0 < seconds or reps < 3:
        units += one()
        reps += 1
    dt = time.perf_counter() - t0
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    return {"value": round(units / dt / scale, 3), "unit": wl.unit, "cores": threads, "kind": "port",
            "sample": f"{sample}; {reps} repetitions in {dt:.1f} s"}


def run_gpu(args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch.distributed as dist

    from omniasr_b200 import shard

    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    wl = WORKLOADS[args.workload](device, rank, world, args.layers)
    n_ev = wl.layers
    ev = [(torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
          for _ in range(n_ev)]
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        wl.run()  # warm-up outside the capture (plans, tensor maps, appended rows rewritten identically)
        torch.cuda.synchronize(device)
        # The timed graph has no event nodes (they would split the kernels' programmatic-launch chain); a second
        # graph with events around the dominant calls gives the per-call durations for the roofline.
        graph_ev = torch.cuda.CUDAGraph()
        graph_ev.capture_begin()
        wl.run(ev)
        graph_ev.capture_end()
        graph = torch.cuda.CUDAGraph()
        graph.capture_begin()
        wl.run()
        graph.capture_end()
    torch.cuda.current_stream(device).wait_stream(side)
    torch.cuda.synchronize(device)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        return shard.max_over_ranks(x, device=device)

    # --- device-resident timing (value) ---
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize(device)
    clocks = Clocks(device.index) if rank == 0 else None
    barrier()
    torch.cuda.synchronize(device)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record()
    for _ in range(args.steps):
        graph.replay()
    end.record()
    torch.cuda.synchronize(device)
    barrier()
    clock = clocks.stop() if clocks else None
    ms = max_over_ranks(start.elapsed_time(end))
    per_call = []
    for _ in range(3):  # the instrumented graph, after the timed region
        graph_ev.replay()
        torch.cuda.synchronize(device)
        per_call.append([a.elapsed_time(b) for a, b in ev])
    per_call = list(np.median(np.array(per_call), axis=0))  # per dominant call, median of 3 replays
    isolated_ms = max_over_ranks(float(np.mean(per_call)) if args.workload != "sweep" else per_call[-1])
    case_ms = [max_over_ranks(x) for x in per_call] if args.workload == "sweep" else None
    # The roofline call's duration inside the event-free step, so that layers x per call <= ms_per_step.
    if wl.roof_timing == "whole":
        roof_ms = max_over_ranks(ms / args.steps / (wl.layers * wl.dominant_per_layer))
    elif wl.roof_timing == "difference":
        wl.skip_dominant = True
        minus_ms = graph_ms(side, device, wl.run, args.steps, args.warmup)
        wl.skip_dominant = False
        roof_ms = max_over_ranks((ms / args.steps - minus_ms) / (wl.layers * wl.dominant_per_layer))
    else:
        roof_ms = isolated_ms
    roof_how = {"whole": "event-free step time / dominant calls per step (a step is only the dominant calls)",
                "difference": "(event-free step - the same step without the dominant calls) / dominant calls per step",
                "events": "CUDA events around each dominant call, in a second graph replayed after the timed region "
                          "(median of 3)"}[wl.roof_timing]

    # The reference's own GPU kernels (Triton; SDPA / index_select where it calls torch) on the same workload, the
    # same graph timing; the same inputs (the appended rows are rewritten with identical values).
    gpu_ref = None
    if hasattr(wl, "run_library"):
        gpu_ref_why = "this workload's library comparison is cuBLAS (library_baseline)"
    elif wl.gpu_reference_unavailable:
        gpu_ref_why = wl.gpu_reference_unavailable
    else:
        ref_ns, gpu_ref_why = reference_gpu_kernels()
        if ref_ns is not None:
            ours = wl.K
            wl.K = ref_ns
            try:
                ref_ms = max_over_ranks(graph_ms(side, device, wl.run, args.steps, args.warmup))
            finally:
                wl.K = ours
            gpu_ref = {"ms_per_step": ref_ms}

    # --- end to end through the public API: inputs from pinned host memory, results back, every step ---
    # One graph per step: layer i's inputs are copied in on an input copy stream, its launches run on the capture
    # stream once they have arrived, and its results are copied out on an output copy stream, so the copies of
    # other layers overlap the kernels (two copy engines, one per direction). Replays are stream-ordered: a step
    # starts after the previous step's last result has reached the host.
    hosts_in = [[torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in wl.layer_in(i)] for i in range(wl.layers)]
    for i, hs in enumerate(hosts_in):
        for h, t in zip(hs, wl.layer_in(i)):
            h.copy_(t.cpu())
    hosts_out = [[torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in outs] for outs in wl.d2h]
    stream = torch.cuda.current_stream(device)
    copy_in, copy_out = torch.cuda.Stream(device), torch.cuda.Stream(device)
    graph_e2e = torch.cuda.CUDAGraph()
    with torch.cuda.stream(side):
        graph_e2e.capture_begin()
        copy_in.wait_stream(side)
        copy_out.wait_stream(side)
        arrived = []
        with torch.cuda.stream(copy_in):
            for i, hs in enumerate(hosts_in):
                for h, t in zip(hs, wl.layer_in(i)):
                    t.copy_(h, non_blocking=True)
                arrived.append(torch.cuda.Event())
                arrived[-1].record(copy_in)
        e2e_outs = []
        for i in range(wl.layers):
            side.wait_event(arrived[i])
            outs = wl.layer(i)
            e2e_outs.append(outs)
            done = torch.cuda.Event()
            done.record(side)
            copy_out.wait_event(done)
            with torch.cuda.stream(copy_out):
                for h, t in zip(hosts_out[i], outs):
                    h.copy_(t, non_blocking=True)
        side.wait_stream(copy_in)
        side.wait_stream(copy_out)
        graph_e2e.capture_end()
    stream.wait_stream(side)
    torch.cuda.synchronize(device)

    def e2e_step():
        graph_e2e.replay()

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
    pk = peaks()
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    peak = pk["tensor"] if wl.bound == "tensor" else pk["hbm"]
    ms_step = ms / args.steps
    value = world * wl.step_units / (ms_step * 1e-3) / scale
    achieved = wl.roof_units / (roof_ms * 1e-3) / scale
    line = {
        "metric": wl.metric + ("" if (H, D) == (32, 128) else f" [{H} heads x {D}]"), "value": round(value, 1),
        "unit": wl.unit, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True,
        "scaling": "strong" if args.workload == "sweep" else "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 tensors; lengths and parents from the seed-0 CPU generator)",
        "config": dict(wl.config(), parallelism=f"request-sharded dp{world} (no collective)"),
        "e2e": {"value": round(world * wl.step_units / (e2e_ms / args.steps * 1e-3) / scale, 1), "unit": wl.unit,
                "ms_per_step": round(e2e_ms / args.steps, 4),
                "h2d_bytes_per_step": int(sum(t.numel() * t.element_size() for hs in hosts_in for t in hs)),
                "d2h_bytes_per_step": int(sum(t.numel() * t.element_size() for hs in hosts_out for t in hs)),
                "path": "omniasr_b200.kernels calls captured in one CUDA graph per step: every layer's inputs copied "
                        "in from pinned host memory and its results copied out, on two copy streams overlapping the "
                        "other layers' kernels; steps do not overlap"},
        "roofline": {"bound": wl.bound, "achieved": round(achieved, 1), "peak": peak,
                     "unit": "TFLOP/s" if wl.bound == "tensor" else "GB/s", "frac": round(achieved / peak, 3),
                     "peak_kind": pk["kind"], "kernel": wl.roof_kernel, "traffic": traffic_per_launch(wl.traffic_key),
                     "timing": roof_how,
                     ("flops_per_launch" if wl.bound == "tensor" else "bytes_per_launch"): wl.roof_units,
                     "us_per_launch": round(roof_ms * 1e3, 2),
                     "us_per_launch_isolated": round(isolated_ms * 1e3, 2)},
        "gpu_launches": wl.launches_per_step() * args.steps,
        "clocks": clock,
    }
    if wl.unit == "GB/s":
        line["pct_of_8tbs"] = round(100 * value / world / NOMINAL_HBM_GBS, 1)
    if gpu_ref is not None:
        tv = world * wl.step_units / (gpu_ref["ms_per_step"] * 1e-3) / scale
        line["triton_value"] = round(tv, 1)
        line["gpu_reference"] = {"value": round(tv, 1), "unit": wl.unit, "ms_per_step": round(gpu_ref["ms_per_step"], 4),
                                 "speedup": round(value / tv, 3),
                                 "what": "the reference's own GPU path, unmodified, on this B200: its Triton kernels "
                                         "(rope_kv / decode / draft / beam attention), torch SDPA (is_causal) for the "
                                         "prefill, index_select for the reorder; same inputs, same graph timing"}
    elif not hasattr(wl, "run_library"):
        line["triton_value"] = None
        line["gpu_reference"] = {"unavailable": gpu_ref_why}
    if case_ms is not None:
        line["cases"] = {f"q{t}_L{L}": {"per_gpu_gbs": round(b / (c * 1e-3) / 1e9, 1),
                                        "box_gbs": round(world * b / (c * 1e-3) / 1e9, 1), "us": round(c * 1e3, 1)}
                         for (t, L), b, c in zip(wl.CASES, wl.case_bytes, case_ms)}
    if args.layers != LAYERS and args.workload not in ("sweep", "gather"):
        line["config"]["reduced"] = f"{args.layers} of {LAYERS} layers (profiling case, not a headline number)"
    if hasattr(wl, "run_library"):  # the same work through torch / cuBLAS, graph-timed the same way
        lib_graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            wl.run_library()
            torch.cuda.synchronize(device)
            lib_graph.capture_begin()
            wl.run_library()
            lib_graph.capture_end()
        torch.cuda.synchronize(device)
        for _ in range(args.warmup):
            lib_graph.replay()
        s3, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s3.record()
        for _ in range(args.steps):
            lib_graph.replay()
        e3.record()
        torch.cuda.synchronize(device)
        lib_ms = s3.elapsed_time(e3) / args.steps
        line["library_baseline"] = {"value": round(wl.step_units / (lib_ms * 1e-3) / scale, 1), "unit": wl.unit,
                                    "ms_per_step": round(lib_ms, 4),
                                    "what": (wl.run_library.__doc__ or "").strip().replace("\n", " ")
                                    or "the same work through torch / cuBLAS"}
    if world == 1 and args.cpu_seconds > 0:
        line["cpu_baseline"] = cpu_time(WORKLOADS[args.workload], args.cpu_seconds)
    return line



# ------------------------------------------------------------------------------------- full decoder step (config 4)

STEP_B, STEP_W, STEP_STEPS, STEP_SYNC = 8, 1500, 256, 8


def reference_modules(ours: bool, gemm: bool = False):
    """The reference package (Wataru-Nakata/omniasr-trt) from baseline/_ref, with this library's kernels in place of
    its ``omniasr_trt.kernels`` when ``ours`` (the drop-in; with ``gemm`` also the step's weight products);
    (modules, None) or (None, why not)."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "omniasr_trt" / "spec.py").exists():
        return None, "the reference package is not installed in baseline/_ref"
    if str(ref) not in sys.path:
        sys.path.insert(0, str(ref))
    if ours:
        from omniasr_b200 import dropin

        dropin.install(gemm=gemm)
    from omniasr_trt import decode, llm, modeling, spec

    return {"decode": decode, "llm": llm, "modeling": modeling, "spec": spec}, None


def step_model(mods, device, seed: int = 0, dtype=torch.bfloat16):
    """BASELINE config 4's decoder: 12 layers, d 4096, 32 x 128 heads, SwiGLU 11008, vocab 10288, RMSNorm; weights
    N(0, 0.02) in bf16, norm weights 1, a 1-layer stand-in encoder (never run). The LM head's EOS row is zero, so
    no row stops early and every step runs the full batch."""
    modeling = mods["modeling"]
    enc = modeling.EncoderConfig(model_dim=16, num_layers=1, num_heads=2, ffn_dim=32, feature_dim=8,
                                 conv_layers=((8, 10, 5),), pos_kernel=4, pos_groups=2)
    dec = modeling.DecoderConfig(model_dim=4096, num_layers=12, num_heads=32, ffn_dim=11008, vocab_size=10288)
    with torch.device(device):
        m = modeling.LLMModel(enc, dec)
    m = m.to(dtype).eval()
    g = torch.Generator(device=device).manual_seed(seed)
    with torch.no_grad():
        for name, prm in m.named_parameters():
            if name.endswith("layer_norm.weight"):
                prm.fill_(1.0)
            else:
                prm.normal_(0.0, 0.02, generator=g)
        m.final_proj.weight[mods["llm"].EOS].zero_()
    m.rope = modeling.rope_table(dec, device)
    return m


def step_bytes(m, lengths_mean: float, b: int, width: int) -> int:
    """Unique HBM bytes of one decoder step: every decoder weight and the LM head once, plus the K/V of every key
    the rows' last queries see (12 layers x 16,384 B per key), at the run's mean cached length."""
    w = sum(p.numel() * p.element_size() for p in m.llama_decoder.parameters())
    w += m.final_proj.weight.numel() * m.final_proj.weight.element_size()
    kv = LAYERS * KV_TOKEN // 2 * m.final_proj.weight.element_size()  # K + V of one key, every layer
    return int(w + kv * b * (lengths_mean + width))


def decode_run(mods, dec, ctxs, steps: int, timed: bool):
    """Prefill ``ctxs`` into slots 0..B-1 and run ``steps`` drafted decoder steps through the reference's own step
    graphs (dec.runner), checking positions on the host every STEP_SYNC steps as its decode loop does; returns
    (prefill ms, steps ms, first / last positions) when timed."""
    llm, dlib = mods["llm"], mods["decode"]
    b, dev = len(ctxs), dec.device
    dec.done[:b] = True
    dec.last[:b] = 0
    dec.tok[:b] = 0
    dec.ensure_capacity(max(max(c.size(0) for c in ctxs), dec.context_floor) + dec.reserve)
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(3)]
    torch.cuda.synchronize(dev)
    ev[0].record()
    first = dec.prefill(ctxs, list(range(b)))
    ev[1].record()
    idx = torch.arange(b, device=dev)
    pos = torch.tensor([c.size(0) - 1 for c in ctxs], device=dev)
    dec.out[idx] = llm.PAD
    dec.out[idx, pos] = first.to(torch.int32)
    dec.tok[idx] = first
    dec.last[idx] = pos
    dec.done[idx] = (first == llm.EOS) | (pos >= dlib.LIMIT)
    dec.filled(list(range(b)), list(range(b)))
    start_pos = pos.clone()
    for _ in range(steps // STEP_SYNC):
        last = dec.last[:b].cpu()
        need = int(last.max()) + STEP_SYNC * dec.step_tokens + 2
        if need > dec.capacity:
            dec.ensure_capacity(need + dec.reserve)
        keys = min(dec.capacity, -(-need // dlib.KEY_BUCKET) * dlib.KEY_BUCKET)
        run = dec.runner(b, keys)
        for _ in range(STEP_SYNC):
            run()
    ev[2].record()
    torch.cuda.synchronize(dev)
    return ev[0].elapsed_time(ev[1]), ev[1].elapsed_time(ev[2]), start_pos.cpu(), dec.last[:b].cpu()


def run_step(args, rank: int, world: int, local_rank: int, ours: bool) -> dict | None:
    """the reference's SpecDecoder (spec-4, batch 8, CUDA graphs) on a random-init decoder, with
    this library's kernels dropped in (``ours``) or the reference's own Triton kernels."""
    import hashlib

    from omniasr_b200 import shard

    impl = "b200" if ours else "reference"
    device = torch.device("cuda", local_rank)
    torch.cuda.set_device(device)
    mods, why = reference_modules(ours, gemm=ours and args.step_gemm == "b200")
    if mods is None:
        return {"impl": impl, "unavailable": why} if rank == 0 else None
    torch.manual_seed(0)
    dtype = torch.float32 if args.dtype == "f32" else torch.bfloat16
    m = step_model(mods, device, dtype=dtype)
    steps = args.decode_steps
    g = torch.Generator().manual_seed(1 + rank)
    ctx_host = [torch.randn(STEP_W, 4096, generator=g).to(dtype).pin_memory() for _ in range(STEP_B)]
    ctxs = [c.to(device) for c in ctx_host]
    dec = mods["spec"].SpecDecoder(m, draft_tokens=4, max_batch=STEP_B, sync_every=STEP_SYNC, reserve=1536)
    with torch.inference_mode():
        decode_run(mods, dec, ctxs, steps, timed=False)  # captures every key bucket's step graph
        for _ in range(max(0, args.warmup - 3)):
            decode_run(mods, dec, ctxs, steps, timed=False)
        clocks = Clocks(device.index) if rank == 0 else None
        if world > 1:
            import torch.distributed as dist

            dist.barrier()
        runs = [decode_run(mods, dec, ctxs, steps, timed=True) for _ in range(3)]
        clock = clocks.stop() if clocks else None
        pre_ms = float(np.median([r[0] for r in runs]))
        steps_ms = float(np.median([r[1] for r in runs]))
        p0, p1 = runs[-1][2], runs[-1][3]
        tokens = dec.out[:STEP_B].cpu()
        # end to end: contexts from pinned host memory, tokens back to the host (median of 3)
        e2e = []
        for _ in range(3):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize(device)
            e0.record()
            ctx_dev = [c.to(device, non_blocking=True) for c in ctx_host]
            decode_run(mods, dec, ctx_dev, steps, timed=True)
            out_host = dec.out[:STEP_B].to("cpu", non_blocking=True)
            e1.record()
            torch.cuda.synchronize(device)
            e2e.append(e0.elapsed_time(e1))
        e2e_ms = float(np.median(e2e))
    if args.tokens_out and rank == 0:
        np.save(args.tokens_out, tokens[:, STEP_W - 1:].numpy())
    steps_ms = shard.max_over_ranks(steps_ms, device=device)
    pre_ms = shard.max_over_ranks(pre_ms, device=device)
    e2e_ms = shard.max_over_ranks(e2e_ms, device=device)
    if rank != 0:
        return None
    gen = (p1 - p0).tolist()
    mean_len = float((p0.float() + p1.float()).mean() / 2)
    nbytes = step_bytes(m, mean_len, STEP_B, dec.step_tokens)
    pk = peaks()
    steps_s = steps / (steps_ms * 1e-3)
    digest = hashlib.sha256(tokens[:, STEP_W - 1:].numpy().tobytes()).hexdigest()[:16]
    assert torch.equal(out_host[:, STEP_W - 1:], tokens[:, STEP_W - 1:]), "the decoder is not deterministic"
    line = {
        "metric": "decoder steps/s (spec-4, batch 8, 12 layers, CUDA graphs)", "value": round(world * steps_s, 2),
        "unit": "steps/s", "n_gpus": world, "steps": steps, "warmup": max(args.warmup, 3) - 2,
        "ms_per_step": round(steps_ms / steps, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": args.dtype, "impl": impl,
        "data": "synthetic: N(0,1) bf16 prefix embeddings (8 x 1500 frames), decoder weights N(0,0.02), LM-head EOS row "
                "zeroed so every row runs all steps; no draft text (proposals from the rows' own tokens)",
        "config": {"workload": "BASELINE config 4: the reference's SpecDecoder (draft_tokens 4, batch 8 per GPU, "
                               "sync_every 8) on a 12-layer d4096 32x128 SwiGLU-11008 vocab-10288 decoder; prefill "
                               "of 8 x 1500 frames, then 256 steps",
                   "kernels": ("omniasr_b200 (drop-in: attention, RoPE/append, prefill, propose, accept"
                               + (", the step's weight products)" if args.step_gemm == "b200" else ")")) if ours
                   else "the reference's Triton kernels",
                   "global_batch": STEP_B * world, "prefill_ms": round(pre_ms, 3), "timing": "median of 3 runs",
                   "prefill_frames_per_s": round(world * STEP_B * STEP_W / (pre_ms * 1e-3), 1),
                   "tokens_generated": gen, "tokens_per_s": round(world * sum(gen) / (steps_ms * 1e-3), 1),
                   "tokens_digest": digest, "parallelism": f"request-sharded dp{world} (no collective)"},
        "e2e": {"value": round(world * steps / (e2e_ms * 1e-3), 2), "unit": "steps/s",
                "ms_total": round(e2e_ms, 3),
                "h2d_bytes_per_step": int(STEP_B * STEP_W * 4096 * ctx_host[0].element_size() / steps),
                "d2h_bytes_per_step": int(tokens.numel() * 4 / steps),
                "path": "contexts copied from pinned host memory, prefill + 256 steps, tokens copied back (per-step "
                        "bytes are the totals / 256)"},
        "roofline": {"bound": "hbm", "achieved": round(nbytes / (steps_ms / steps * 1e-3) / 1e9, 1),
                     "peak": pk["hbm"], "unit": "GB/s",
                     "frac": round(nbytes / (steps_ms / steps * 1e-3) / 1e9 / pk["hbm"], 3),
                     "peak_kind": pk["kind"], "kernel": "whole decoder step (weights + K/V read once)",
                     "traffic": None, "bytes_per_step": nbytes},
        "gpu_launches": (2 * LAYERS + 2) * steps if ours else 0,  # rope_kv, pass per layer; propose, accept
        "clocks": clock,
    }
    return line

# --------------------------------------------------------------------------------------------------- reference arm


def run_reference(args, rank: int) -> dict | None:
    """The CPU port of the reference's algorithm (oracle), on all host cores, rank 0 only."""
    if rank != 0:
        return None
    wl = WORKLOADS[args.workload]
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    one, sample = wl.cpu_sampler()
    for _ in range(args.warmup):
        one()
    units, t0 = 0.0, time.perf_counter()
    for _ in range(args.steps):
        units += one()
    dt = time.perf_counter() - t0
    scale = 1e12 if wl.unit == "TFLOP/s" else 1e9
    value = units / dt / scale
    return {"impl": "reference", "metric": wl.metric, "value": round(value, 3), "unit": wl.unit, "n_gpus": 1,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"{wl.name}: bounded CPU sample per step ({sample})"},
            "cpu_baseline": {"value": round(value, 3), "unit": wl.unit, "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(value, 3), "unit": wl.unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    global H, D
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=50)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["b200", "reference"], default="b200")
    p.add_argument("--workload", choices=sorted(WORKLOADS) + ["step"], default="verify")
    p.add_argument("--layers", type=int, default=LAYERS)
    p.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample length (0: none)")
    p.add_argument("--tokens-out", default=None, help="step workload: save the generated tokens (.npy)")
    p.add_argument("--decode-steps", type=int, default=STEP_STEPS, help="step workload: decoder steps per run")
    p.add_argument("--dtype", choices=["bf16", "f32"], default="bf16", help="step workload: model dtype")
    p.add_argument("--step-gemm", choices=["cublas", "b200"], default="cublas",
                   help="step workload, this library's arm: the decoder's weight products on cuBLAS (as the reference "
                        "runs them) or on this library's decode GEMM (dropin.install(gemm=True))")
    p.add_argument("--heads", type=int, default=H, help="attention workloads: heads (heads x head_dim = 4096)")
    p.add_argument("--head-dim", type=int, default=D,
                   help="attention workloads: head_dim; 512 with 8 heads is the shipped model's geometry")
    args = p.parse_args()
    if args.heads * args.head_dim != H * D:
        p.error(f"heads x head_dim must be {H * D} (the decoder's model width)")
    H, D = args.heads, args.head_dim
    args.warmup = max(args.warmup, 3)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.workload == "step":  # both arms on the GPU: this library's kernels, or the reference's own
        if world > 1:
            import datetime

            import torch.distributed as dist

            torch.cuda.set_device(local_rank)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                    device_id=torch.device("cuda", local_rank))
        try:
            line = run_step(args, rank, world, local_rank, ours=args.impl == "b200")
            if line:
                print(json.dumps(line), flush=True)
        finally:
            if world > 1:
                import torch.distributed as dist

                dist.destroy_process_group()
        return
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
