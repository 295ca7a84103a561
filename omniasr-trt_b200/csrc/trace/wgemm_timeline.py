"""Per-CTA timeline of the decode GEMM on the decoder step's four products (BASELINE config 4 model, 40 token rows,
12 layers of distinct weights, one CUDA graph per step), from the tracing build:

    make -C omniasr-trt_b200/csrc trace
    python omniasr-trt_b200/csrc/trace/wgemm_timeline.py

Prints, for the last layer's QKV / output / gate-inner (SwiGLU) / FFN-output calls, the min / median / max over CTAs
of each pipeline event (microseconds from the QKV call's first CTA entry; the events are listed in wgemm_trace.cu),
the median per-CTA weight-stream rate, and the tail from the last MMA issued to the CTA's exit. The step time is
the graph's, taken with CUDA events around whole steps."""

import ctypes
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
PKG = HERE.parent.parent
sys.path.insert(0, str(PKG))
from omniasr_b200 import _lib  # noqa: E402

_lib.LIB_PATH = PKG / "lib" / "libomniasr_b200_trace.so"
from omniasr_b200 import kernels  # noqa: E402

EVENTS = {0: "entry", 1: "waited", 2: "load1", 3: "full1", 4: "lastmma", 6: "epi", 7: "exit"}
NAMES = ("qkv", "out", "swiglu", "ffn")


def main() -> None:
    lib = _lib.load()
    lib.omni_wg_trace_read.argtypes = [ctypes.c_void_p]
    dev = "cuda"
    rows, d, f, layers = 40, 4096, 11008, 12
    g = torch.Generator(device=dev).manual_seed(0)
    w = lambda r, c: (torch.randn(r, c, generator=g, device=dev) * 0.02).to(torch.bfloat16)  # noqa: E731
    weights = [(w(3 * d, d), w(d, d), w(2 * f, d), w(d, f)) for _ in range(layers)]
    x, o, h = (torch.randn(rows, d, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
    gg = torch.randn(rows, f, generator=g, device=dev).to(torch.bfloat16)

    def step():
        for qkv_w, out_w, gi_w, ffo_w in weights:
            kernels.decode_gemm(x, qkv_w)
            kernels.decode_gemm(o, out_w, "residual", residual=h)
            kernels.decode_gemm(x, gi_w, "swiglu")
            kernels.decode_gemm(gg, ffo_w, "residual", residual=h)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for _ in range(3):
        graph.replay()
    times = []
    for _ in range(10):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        times.append(e0.elapsed_time(e1))
    ms = float(np.median(times))
    nbytes = layers * 2 * (3 * d * d + d * d + 2 * f * d + d * f)
    lib.omni_wg_trace_clear()
    graph.replay()
    torch.cuda.synchronize()
    buf = np.zeros((4, 256, 16), dtype=np.uint64)
    lib.omni_wg_trace_read(ctypes.c_void_p(buf.ctypes.data))
    print(f"step {ms:.3f} ms, {nbytes / ms / 1e6:.0f} GB/s over the four GEMMs; status {kernels.read_status()}")
    wbytes = (2 * 3 * d * d, 2 * d * d, 2 * 2 * f * d, 2 * d * f)
    t0 = None
    for s, name in enumerate(NAMES):
        ev = buf[s].astype(np.int64)
        ev = ev[ev[:, 0] > 0]
        if not len(ev):
            continue
        t0 = ev[:, 0].min() if t0 is None else t0
        r = (ev - t0) / 1000.0
        cols = " | ".join(f"{EVENTS[c]} {r[:, c].min():6.2f} {np.median(r[:, c]):6.2f} {r[:, c].max():6.2f}"
                          for c in EVENTS)
        stream = np.median(r[:, 4] - r[:, 3])
        tail = r[:, 7] - r[:, 4]
        print(f"{name:6s} {len(ev):3d} CTAs | {cols}")
        print(f"       stream {stream:.2f} us median, {wbytes[s] / len(ev) / stream / 1e3:.1f} GB/s per CTA; "
              f"tail (last MMA -> exit) median {np.median(tail):.2f} max {tail.max():.2f} us; "
              f"span {r[:, 7].max() - r[:, 0].min():.2f} us (weights at 6.44 TB/s: {wbytes[s] / 6.4441e6:.2f} us)")


if __name__ == "__main__":
    main()
