"""Golden vectors of the speculative acceptance rule, produced by the reference's own GPU kernel.

    python tests/golden/make_accept_golden.py --out tests/golden/accept.npz

The reference states its acceptance rule only as a Triton kernel (``_accept``, omniasr_trt/kernels.py:271-291,
called through ``kernels.accept``, :380-391, by ``SpecDecoder.step``, spec.py:108), so this script must run on a
CUDA GPU with the reference package importable (``baseline/_ref``, placed there by ``__graft_entry__.build()``). It
imports the reference's ``omniasr_trt.kernels`` unmodified (no drop-in), runs ``accept`` on seeded inputs and stores
the inputs and the in-place results. ``tests/test_oracle.py`` pins the CPU restatement to these vectors, and
``tests/test_spec_gpu.py`` the CUDA kernel.

Inputs are drawn like the reference's spec tests draw their states: few token symbols (so that fed tokens often equal
the argmax before them), leading runs of matches of every length, EOS inside the runs, positions near the length
limit, finished rows, both draft sources.
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent

WIDTHS = (1, 2, 5, 9)
ROWS, CAP, EOS, LIMIT = 64, 300, 2, 260


def draw(width: int, seed: int) -> dict:
    rng = np.random.default_rng(seed)
    tokens = rng.integers(2, 6, (ROWS, width)).astype(np.int64)
    nxt = rng.integers(2, 6, (ROWS, width)).astype(np.int64)
    for r in range(ROWS):  # leading runs of matches of every length
        n = r % (width + 1)
        nxt[r, :max(0, n - 1)] = tokens[r, 1:n]
    nxt[5::11, min(1, width - 1)] = EOS
    last = rng.integers(200, 270, ROWS).astype(np.int64)  # some at or past the limit
    return {
        "tokens": tokens, "nxt": nxt, "last": last,
        "out": rng.integers(3, 9, (ROWS, CAP)).astype(np.int32),
        "tok": rng.integers(3, 9, ROWS).astype(np.int64),
        "done": rng.random(ROWS) < 0.15,
        "draft_next": rng.integers(0, 50, ROWS).astype(np.int64),
        "start": rng.integers(0, 50, ROWS).astype(np.int64),
        "use_draft": rng.random(ROWS) < 0.5,
    }


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--out", default=str(HERE / "accept.npz"))
    p.add_argument("--reference", default=str(ROOT / "baseline" / "_ref"), help="directory holding omniasr_trt")
    args = p.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    from omniasr_trt import kernels as ref  # the reference's own module (Triton kernels)

    assert ref.available(torch.device("cuda")), "the reference's Triton kernels need a CUDA GPU"
    dev = torch.device("cuda")
    save = {"widths": np.array(WIDTHS), "rows": ROWS, "cap": CAP, "eos": EOS, "limit": LIMIT}
    for width in WIDTHS:
        x = draw(width, 80 + width)
        t = {k: torch.as_tensor(v.copy(), device=dev) for k, v in x.items()}
        ref.accept(t["tokens"], t["nxt"], t["out"], t["tok"], t["last"], t["done"], t["draft_next"], t["start"],
                   t["use_draft"], LIMIT, EOS)
        torch.cuda.synchronize()
        for k, v in x.items():
            save[f"w{width}_{k}"] = v
        for k in ("out", "tok", "last", "done", "draft_next"):
            save[f"w{width}_{k}_after"] = t[k].cpu().numpy()
    Path(args.out).parent.mkdir(parents=True, exist_ok=True)
    np.savez_compressed(args.out, **save)
    print("wrote", args.out)


if __name__ == "__main__":
    main()
