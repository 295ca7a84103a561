"""Put these kernels in place of the reference's ``omniasr_trt.kernels`` (Wataru-Nakata/omniasr-trt).

After :func:`install`, ``import omniasr_trt.kernels`` (and the ``from . import kernels`` of ``decode``, ``spec``,
``beam`` and ``llm``) yields a module whose path functions -- ``available``, ``rope_kv``, ``decode_attention``,
``draft_attention``, ``beam_attention``, ``splits_for``, ``ATTN``, ``DRAFT_ATTN`` -- are this package's CUDA
kernels. The speculative decoder's control kernels ``propose`` / ``accept`` are not on this path and stay the
reference's own. Nothing else of the reference changes: its decoders, CUDA-graph capture, ``OmniASRLLM.transcribe``
and ``compat.Pipeline`` run unchanged on top.
"""

from __future__ import annotations

import importlib
import sys
import types

PATH_FUNCTIONS = ("available", "rope_kv", "decode_attention", "draft_attention", "beam_attention", "splits_for",
                  "ATTN", "DRAFT_ATTN")


def install(package: str = "omniasr_trt") -> types.ModuleType:
    """Swaps ``<package>.kernels`` for a module with this package's path functions; returns that module."""
    from . import kernels as ours

    pkg = importlib.import_module(package)
    ref = importlib.import_module(f"{package}.kernels")
    if getattr(ref, "__omniasr_b200__", False):
        return ref
    merged = types.ModuleType(f"{package}.kernels", ours.__doc__)
    for name in dir(ref):  # the reference's other names (propose, accept, ...) first
        if not name.startswith("__"):
            setattr(merged, name, getattr(ref, name))
    for name in PATH_FUNCTIONS:
        setattr(merged, name, getattr(ours, name))
    merged.reorder_gather = ours.reorder_gather
    merged.__omniasr_b200__ = True
    merged.reference = ref
    sys.modules[f"{package}.kernels"] = merged
    pkg.kernels = merged
    for sub in ("decode", "spec", "beam", "llm"):  # modules that already bound the old one
        mod = sys.modules.get(f"{package}.{sub}")
        if mod is not None and getattr(mod, "kernels", None) is ref:
            mod.kernels = merged
    return merged
