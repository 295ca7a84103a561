"""The reference's key-split rule (test infrastructure only): omniasr_trt/kernels.py:393-400 (``splits_for``)."""

from __future__ import annotations


def splits_for(rows: int, heads: int, keys: int, block: int = 64, programs: int = 264) -> tuple[int, int]:
    want = max(1, programs // (rows * heads))
    splits = 1
    while splits * 2 <= want and splits * 2 * block <= keys:
        splits *= 2
    chunk = -(-keys // splits)
    return splits, -(-chunk // block) * block
