"""Golden vectors of the order torch.topk(sorted=True) returns on a CUDA tensor when values tie.

    python tests/golden/make_topk_golden.py --out tests/golden/topk_ties.npz      (on a CUDA GPU)

The reference's beam search takes each group's best candidates with ``cand.view(s, n * vocab).topk(n, dim=-1,
sorted=True)`` (omniasr_trt/beam.py:171) on the GPU, and the order of equal candidates decides which beam row gets
which of them. torch.topk on the CPU orders ties differently (in no fixed way), so these vectors come from the GPU:
rows whose values are all equal (k = 1..32) and rows drawn from two to four distinct values, some with half their
entries -inf, of lengths 12 to 51440 (the beam search's 5 x 10288), k = 2..16. ``tests/test_oracle.py`` pins
``oracle.beam.topk_order`` to them; ``tests/test_beam_select_gpu.py`` checks the CUDA kernel against torch directly.
"""

from __future__ import annotations

import argparse
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--out", default=str(HERE / "topk_ties.npz"))
    args = p.parse_args()
    out = {}
    for k in range(1, 33):
        out[f"eq_k{k}"] = torch.zeros(1, 40, device="cuda").topk(k, sorted=True).indices.cpu().numpy()[0]
    g = torch.Generator().manual_seed(0)
    n = 120
    for i in range(n):
        length = [12, 40, 100, 1000, 51440][i % 5]
        k = min(length, int(torch.randint(2, 17, (1,), generator=g)))
        nv = int(torch.randint(2, 5, (1,), generator=g))
        x = torch.randint(0, nv, (1, length), generator=g).float()
        if i % 3 == 0:
            x[0, torch.randperm(length, generator=g)[: length // 2]] = float("-inf")
        idx = x.cuda().topk(k, sorted=True).indices.cpu().numpy()[0]
        # store the row compactly: its values as int8 codes (-1 for -inf)
        out[f"case{i}_x"] = np.where(np.isinf(x.numpy()[0]), -1, x.numpy()[0]).astype(np.int8)
        out[f"case{i}_i"] = idx
    out["n"] = np.array(n)
    np.savez_compressed(args.out, **out)
    print(f"{n} cases -> {args.out}")


if __name__ == "__main__":
    main()
