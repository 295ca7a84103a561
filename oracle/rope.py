"""RoPE + KV-cache append, bit-exact, in numpy (test infrastructure only).

Restates ``omniasr_trt.kernels.rope_kv`` (kernels.py:294-306, kernel :31-54) with the arithmetic of
``modeling.apply_rope`` (modeling.py:301-306): for each interleaved pair (re, im) = (x[2j], x[2j+1]) and table
entry (c, s) = cs[pos, j], in float32 with every product and sum rounded separately (numpy float32 ops do not
contract into FMAs):  re' = re*c - im*s,  im' = re*s + im*c;  then cast back to the input dtype (bf16: round to
nearest even). v is copied unchanged.
"""

from __future__ import annotations

import numpy as np

from . import bf16


def rotate(x: np.ndarray, cs_rows: np.ndarray) -> np.ndarray:
    """float32 ``x`` [..., D] rotated with ``cs_rows`` [..., D/2, 2] (broadcast) -> float32 [..., D]."""
    x = x.astype(np.float32, copy=False)
    re, im = x[..., 0::2], x[..., 1::2]
    c, s = cs_rows[..., 0].astype(np.float32), cs_rows[..., 1].astype(np.float32)
    out = np.empty_like(x)
    out[..., 0::2] = (re * c) - (im * s)
    out[..., 1::2] = (re * s) + (im * c)
    return out


def rope_kv(qkv: np.ndarray, cs: np.ndarray, pos: np.ndarray, k_cache: np.ndarray, v_cache: np.ndarray, heads: int,
            slots: np.ndarray | None = None, cache_pos: np.ndarray | None = None, is_bf16: bool = True) -> np.ndarray:
    """In place on ``k_cache``/``v_cache`` [rows, H, S, D]; returns q [N, H, D].

    Arrays hold raw values: uint16 bf16 bit patterns when ``is_bf16``, else float32.
    """
    n = qkv.shape[0]
    d = qkv.shape[1] // (3 * heads)
    parts = qkv.reshape(n, 3, heads, d)
    rows = np.arange(n) if slots is None else slots
    cpos = pos if cache_pos is None else cache_pos
    cs_rows = cs[pos][:, None]  # [N, 1, D/2, 2]
    if is_bf16:
        qf, kf = bf16.to_float32(parts[:, 0]), bf16.to_float32(parts[:, 1])
        q = bf16.from_float32(rotate(qf, cs_rows))
        k = bf16.from_float32(rotate(kf, cs_rows))
    else:
        q = rotate(parts[:, 0], cs_rows)
        k = rotate(parts[:, 1], cs_rows)
    # Two tokens writing one (row, position) are unordered in the reference's kernel (and in the CUDA one); here
    # the later token wins, so tests compare only positions written once.
    for t in range(n):
        k_cache[rows[t], :, cpos[t]] = k[t]
        v_cache[rows[t], :, cpos[t]] = parts[t, 2]
    return q


def rope_table(head_dim: int, positions: int, theta: float = 10_000.0):
    """cos/sin of every position, ``[positions, head_dim / 2, 2]`` float32, computed on the CPU in torch as the
    reference's ``rope_table`` does (modeling.py:293-298). It is an input of the kernel and of :func:`rope_kv`."""
    import torch

    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.float32) / head_dim))
    angles = torch.outer(torch.arange(positions, dtype=torch.float32), inv)
    return torch.stack([torch.cos(angles), torch.sin(angles)], -1)
