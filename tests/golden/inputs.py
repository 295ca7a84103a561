"""Seeded inputs of the golden cases (shared by ``make_golden.py`` and the tests).

Values come from ``numpy.random.default_rng(seed)`` as float32 N(0, 1) and are rounded to bfloat16 for the bf16
cases; each golden file stores the sha256 of its inputs so that a change of generator shows up as a failure, not as
a silent mismatch.
"""

from __future__ import annotations

import hashlib

import numpy as np

from oracle import bf16


def normal(rng: np.random.Generator, shape, is_bf16: bool) -> np.ndarray:
    x = rng.standard_normal(shape, dtype=np.float32)
    return bf16.from_float32(x) if is_bf16 else x


def values(a: np.ndarray, is_bf16: bool) -> np.ndarray:
    """Raw arrays (uint16 bf16 bits or float32) -> float64 values."""
    return (bf16.to_float32(a) if is_bf16 else a).astype(np.float64)


def digest(*arrays: np.ndarray) -> str:
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


# ----------------------------------------------------------------------------------------------- attention cases

DECODE = dict(seed=11, b=3, h=2, d=128, s=200, rows=4, lengths=[200, 37, 0], keys=200)
DRAFT = dict(seed=12, b=3, t=5, h=2, d=128, s=300, rows=4, lengths=[250, 17, 1], keys=256)
BEAM = dict(seed=13, groups=3, beams=3, h=2, d=128, c=160, g=24, ctx_len=[160, 33, 0], ctx_keys=160)


def decode_inputs(is_bf16: bool, c=DECODE):
    rng = np.random.default_rng(c["seed"])
    q = normal(rng, (c["b"], c["h"], c["d"]), is_bf16)
    k = normal(rng, (c["rows"], c["h"], c["s"], c["d"]), is_bf16)
    v = normal(rng, (c["rows"], c["h"], c["s"], c["d"]), is_bf16)
    return q, k, v, np.array(c["lengths"], dtype=np.int64)


def draft_inputs(is_bf16: bool, c=DRAFT):
    rng = np.random.default_rng(c["seed"])
    q = normal(rng, (c["b"] * c["t"], c["h"], c["d"]), is_bf16)
    k = normal(rng, (c["rows"], c["h"], c["s"], c["d"]), is_bf16)
    v = normal(rng, (c["rows"], c["h"], c["s"], c["d"]), is_bf16)
    return q, k, v, np.array(c["lengths"], dtype=np.int64)


def beam_inputs(is_bf16: bool, c=BEAM):
    rng = np.random.default_rng(c["seed"])
    r = c["groups"] * c["beams"]
    q = normal(rng, (r, c["h"], c["d"]), is_bf16)
    kc = normal(rng, (c["groups"] + 1, c["h"], c["c"], c["d"]), is_bf16)
    vc = normal(rng, (c["groups"] + 1, c["h"], c["c"], c["d"]), is_bf16)
    kg = normal(rng, (r + 2, c["h"], c["g"], c["d"]), is_bf16)
    vg = normal(rng, (r + 2, c["h"], c["g"], c["d"]), is_bf16)
    gen_len = rng.integers(0, c["g"] + 1, r).astype(np.int64)
    gen_len[-c["beams"]:] = 0  # the last input is finished: no keys at all
    ptr = rng.integers(0, r, (r, c["g"])).astype(np.int32)
    return q, kc, vc, np.array(c["ctx_len"], dtype=np.int64), kg, vg, ptr, gen_len


PREFILL = dict(seed=14, b=2, h=1, w=160, d=128)
PREFILL_D512 = dict(seed=15, b=1, h=1, w=70, d=512)


def prefill_inputs(is_bf16: bool, c=PREFILL):
    """q, k, v [B, H, W, D] of a right-padded prefill (the decoder's views at decode.py:158-171)."""
    rng = np.random.default_rng(c["seed"])
    shape = (c["b"], c["h"], c["w"], c["d"])
    return normal(rng, shape, is_bf16), normal(rng, shape, is_bf16), normal(rng, shape, is_bf16)
