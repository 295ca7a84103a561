"""Beam reorder gather, byte-exact, in numpy (test infrastructure only).

``dst[r] = src[parent[r]]``: the reference's K/V reorder ``kv.index_select(0, parent)`` (omniasr_trt/llm.py:237-238)
and its pointer / history reorder ``ptr.copy_(ptr[parent])``, ``hist.copy_(hist[parent])`` (omniasr_trt/beam.py:175-176).
"""

from __future__ import annotations

import numpy as np


def reorder_gather(src: np.ndarray, parent: np.ndarray) -> np.ndarray:
    parent = np.asarray(parent, dtype=np.int64)
    if parent.size and (parent.min() < 0 or parent.max() >= src.shape[0]):
        raise IndexError("parent outside src rows")
    return src[parent].copy()


def beam_parents(groups: int, beams: int, picks: np.ndarray) -> np.ndarray:
    """Global parent rows of a beam step: input g's beam b follows row g*beams + picks[g, b] (beam.py:280)."""
    return (np.arange(groups)[:, None] * beams + picks).reshape(-1)
