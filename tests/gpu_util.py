"""Helpers of the GPU tests: raw golden arrays to device tensors, seeded torch inputs, tolerances."""

from __future__ import annotations

import numpy as np
import torch

# north_star tolerances for bf16 attention against an fp64/fp32 reference (written into every bf16 check).
BF16_MAX_ABS = 2e-2
BF16_MEAN_ABS = 2e-3


def dev(a: np.ndarray, is_bf16: bool, device="cuda") -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(a).astype(np.int16)).view(torch.bfloat16) if is_bf16 \
        else torch.from_numpy(np.ascontiguousarray(a))
    return t.to(device)


def raw(t: torch.Tensor) -> np.ndarray:
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().astype(np.uint16)
    return t.numpy()


def randn(shape, dtype, seed: int) -> torch.Tensor:
    """N(0, 1) drawn on the CPU in fp32 with a seeded generator, cast to ``dtype`` (the BASELINE recipe)."""
    g = torch.Generator().manual_seed(seed)
    return torch.randn(shape, generator=g, dtype=torch.float32).to(dtype)


def check_attention(got: torch.Tensor, want: torch.Tensor, dtype: torch.dtype, fp32_tol: float = 2e-5,
                    what: str = "") -> tuple[float, float]:
    """bf16: max-abs <= 2e-2 and mean-abs <= 2e-3; fp32: |got - want| <= fp32_tol * (1 + |want|)."""
    g = got.detach().double().cpu()
    w = want.double().cpu()
    diff = (g - w).abs()
    mx, mean = (float(diff.max()), float(diff.mean())) if diff.numel() else (0.0, 0.0)
    if dtype == torch.bfloat16:
        assert mx <= BF16_MAX_ABS and mean <= BF16_MEAN_ABS, f"{what}: max-abs {mx:.3g}, mean-abs {mean:.3g}"
    else:
        bad = diff > fp32_tol * (1 + w.abs())
        assert not bool(bad.any()), f"{what}: max-abs {mx:.3g} (fp32 tol {fp32_tol})"
    return mx, mean
