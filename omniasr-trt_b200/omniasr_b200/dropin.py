"""Put these kernels in place of the reference's ``omniasr_trt.kernels`` (Wataru-Nakata/omniasr-trt).

After :func:`install`, ``import omniasr_trt.kernels`` (and the ``from . import kernels`` of ``decode``, ``spec``,
``beam`` and ``llm``) yields a module whose path functions -- ``available``, ``rope_kv``, ``decode_attention``,
``draft_attention``, ``beam_attention``, ``splits_for``, ``ATTN``, ``DRAFT_ATTN`` and the speculative decoder's
control kernels ``propose`` / ``accept`` -- are this package's CUDA kernels, and the prefill's causal
``F.scaled_dot_product_attention`` in ``decode.py`` (decode.py:171) runs
:func:`omniasr_b200.kernels.prefill_attention`. No Triton kernel of the reference remains on these decoders' path.
Nothing else of the reference changes: its decoders, CUDA-graph capture, ``OmniASRLLM.transcribe`` and
``compat.Pipeline`` run unchanged on top.
"""

from __future__ import annotations

import importlib
import sys
import types

PATH_FUNCTIONS = ("available", "rope_kv", "decode_attention", "draft_attention", "beam_attention", "splits_for",
                  "ATTN", "DRAFT_ATTN", "propose", "accept")


class _Functional(types.ModuleType):
    """``torch.nn.functional`` as ``decode.py`` sees it, with the prefill's causal attention routed to these kernels
    (every other name is torch's own)."""

    def __init__(self, prefill):
        super().__init__("torch.nn.functional")
        import torch.nn.functional as torch_f

        self._torch_f = torch_f
        self._prefill = prefill

    def __getattr__(self, name):
        return getattr(self._torch_f, name)

    def scaled_dot_product_attention(self, q, k, v, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
                                     **kw):
        if is_causal and attn_mask is None and dropout_p == 0.0 and not kw and q.is_cuda and q.dim() == 4 \
                and k.shape == q.shape and v.shape == q.shape:
            return self._prefill(q, k, v, scale)
        return self._torch_f.scaled_dot_product_attention(q, k, v, attn_mask=attn_mask, dropout_p=dropout_p,
                                                          is_causal=is_causal, scale=scale, **kw)


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
    decode = importlib.import_module(f"{package}.decode")  # its prefill attention (decode.py:171)
    if not isinstance(decode.F, _Functional):
        decode.F = _Functional(ours.prefill_attention)
    return merged
