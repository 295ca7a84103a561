"""Put these kernels in place of the reference's ``omniasr_trt.kernels`` (Wataru-Nakata/omniasr-trt).

After :func:`install`, ``import omniasr_trt.kernels`` (and the ``from . import kernels`` of ``decode``, ``spec``,
``beam`` and ``llm``) yields a module whose path functions -- ``available``, ``rope_kv``, ``decode_attention``,
``draft_attention``, ``beam_attention``, ``splits_for``, ``ATTN``, ``DRAFT_ATTN`` and the speculative decoder's
control kernels ``propose`` / ``accept`` -- are this package's CUDA kernels, and the prefill's causal
``F.scaled_dot_product_attention`` in ``decode.py`` (decode.py:171) runs
:func:`omniasr_b200.kernels.prefill_attention`. No Triton kernel of the reference remains on these decoders' path.
The beam decoder's selection after the LM head (beam.py:161-187: candidates, per-group top-k, the pointer / history
reorder and the state updates, some thirty small torch kernels) runs as one kernel,
:func:`omniasr_b200.kernels.beam_select`, through :func:`_beam_step`. Nothing else of the reference changes: its
decoders, CUDA-graph capture, ``OmniASRLLM.transcribe`` and ``compat.Pipeline`` run unchanged on top.
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


def _beam_step(self, s: int, ckeys: int, gkeys: int) -> None:
    """``BeamDecoder.step_beam`` (beam.py:127-187) with its selection as one kernel.

    The step up to the log-probabilities is the reference's own sequence of operations (beam.py:130-160: the pointer
    of the token fed now, then per layer the QKV product, ``rope_kv``, the beam attention, the output projection and
    the SwiGLU FFN, then the final norm, the LM head and the log-softmax) -- it must be, for the same tokens; the
    candidates, per-group top-k, parents and reorder that follow are :func:`kernels.beam_select`. Shapes and dtypes
    the kernel does not take (the PyTorch path, an fp64 model, more than 16 beams) run the reference's own method."""
    import torch
    import torch.nn.functional as F

    from . import kernels as ours

    if not self.fused or self.score.dtype != torch.float32 or self.dtype not in (torch.bfloat16, torch.float32) \
            or self.beams > 16:
        return _beam_step.reference(self, s, ckeys, gkeys)
    m, n = self.m, self.beams
    r = s * n
    rows = torch.arange(r, device=self.device)
    gdone, ctx = self.gdone[:s], self.ctx[:s]
    live = ~gdone[self.group[:r]]
    k = self.k_step[:s][self.group[:r]]  # the token fed now was chosen at step k - 1
    pos = ctx[self.group[:r]] - 1 + k  # its input position
    j = (k - 1).clamp(min=0)  # its generated-cache position
    ctx_len = torch.where(gdone, 0, ctx)
    gen_len = torch.where(live, k, 0)
    ptr = self.ptr[:r]
    kept = ptr.gather(1, j[:, None])[:, 0].long()
    ptr.scatter_(1, j[:, None], torch.where(live, rows, kept)[:, None].to(ptr.dtype))
    h = m.text_frontend.weight[self.tok[:r]]
    for i, layer in enumerate(m.llama_decoder.layers):
        qkv_w, out_w, gi_w, ffo_w = self.layers[i]
        qkv = layer.self_attn_layer_norm(h) @ qkv_w.t()
        q = ours.rope_kv(qkv, m.rope, pos, self.kg[i], self.vg[i], self.heads, cache_pos=j)
        o = self.attention(i, q, ctx_len, gen_len, s, ckeys, gkeys).reshape(r, -1)
        h = torch.addmm(h, o, out_w.t())
        gate, inner = (layer.ffn_layer_norm(h) @ gi_w.t()).chunk(2, -1)
        h = torch.addmm(h, inner * F.silu(gate), ffo_w.t())
    logp = F.log_softmax(m.final_proj(m.llama_decoder.layer_norm(h)), dim=-1)
    ours.beam_select(logp, self.score, self.ended, self.count, self.tok, self.hist, self.ptr, self.k_step, self.ctx,
                     self.gdone, n, self.length_norm, EOS, PAD, LIMIT)


EOS, PAD, LIMIT = 2, 1, 8188  # set from the reference's llm / decode modules by install()

_WEIGHT_CLASS = None


def _weight_class():
    """A view class for the decoders' weights (``fuse_projections``' tuples, decode.py:34-54): ``x @ w.t()`` and
    ``torch.addmm(h, x, w.t())`` with at most 64 bf16 token rows run :func:`kernels.decode_gemm` (store / residual);
    every other use of the weight, and every other shape or dtype (the prefill's thousands of rows, an fp32 model),
    is torch's own operation on the plain tensor."""
    global _WEIGHT_CLASS
    if _WEIGHT_CLASS is not None:
        return _WEIGHT_CLASS
    import torch

    from . import kernels as ours

    def plain(t):
        return t.as_subclass(torch.Tensor) if isinstance(t, DecodeWeight) else t

    def fits(x, w) -> bool:
        return (x.is_cuda and x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2
                and 1 <= x.size(0) <= 64 and x.stride(1) == 1 and x.stride(0) % 8 == 0 and x.data_ptr() % 16 == 0
                and w.dim() == 2 and w.stride(1) == 1 and w.stride(0) % 8 == 0 and w.data_ptr() % 16 == 0
                and x.size(1) == w.size(1) and x.size(1) % 8 == 0 and x.device == w.device)

    class DecodeWeight(torch.Tensor):
        _base = None  # on the view returned by .t(): the weight [n, k] itself

        @classmethod
        def __torch_function__(cls, func, types, args=(), kwargs=None):
            kwargs = kwargs or {}
            if func is torch.Tensor.t and len(args) == 1 and isinstance(args[0], DecodeWeight):
                with torch._C.DisableTorchFunctionSubclass():
                    w = plain(args[0])
                    view = w.t().as_subclass(DecodeWeight)
                view._base = w
                return view
            if func in (torch.matmul, torch.Tensor.matmul, torch.Tensor.__matmul__) and len(args) == 2 and not kwargs:
                x, wt = args
                if isinstance(wt, DecodeWeight) and wt._base is not None and not isinstance(x, DecodeWeight) \
                        and fits(x, wt._base):
                    return ours.decode_gemm(x, wt._base)
            if func is torch.addmm and len(args) == 3 and not kwargs:
                h, x, wt = args
                if isinstance(wt, DecodeWeight) and wt._base is not None and not isinstance(x, DecodeWeight) \
                        and not isinstance(h, DecodeWeight) and fits(x, wt._base) and h.dtype == torch.bfloat16 \
                        and h.shape == (x.size(0), wt._base.size(0)) and h.stride(1) == 1 and h.stride(0) % 8 == 0 \
                        and h.data_ptr() % 16 == 0:
                    return ours.decode_gemm(x, wt._base, "residual", residual=h)
            with torch._C.DisableTorchFunctionSubclass():
                return func(*[plain(a) for a in args], **{k: plain(v) for k, v in kwargs.items()})

    _WEIGHT_CLASS = DecodeWeight
    return DecodeWeight


def _routed_projections(fuse):
    """``decode.fuse_projections`` whose tuples hold weight views that route the decode step's products."""

    def fuse_projections(model):
        cls = _weight_class()
        return [tuple(w.as_subclass(cls) for w in layer) for layer in fuse(model)]

    fuse_projections.reference = fuse
    return fuse_projections


def _route_products(package: str, gemm: bool) -> None:
    decode = importlib.import_module(f"{package}.decode")
    routed = getattr(decode.fuse_projections, "reference", None) is not None
    if gemm and not routed:
        decode.fuse_projections = _routed_projections(decode.fuse_projections)
    elif not gemm and routed:
        decode.fuse_projections = decode.fuse_projections.reference


def install(package: str = "omniasr_trt", gemm: bool = False) -> types.ModuleType:
    """Swaps ``<package>.kernels`` for a module with this package's path functions; returns that module. With
    ``gemm``, decoders built afterwards also run their step's weight products with at most 64 bf16 token rows
    (decode.py:201-205, spec.py:100-107, beam.py:148-154: the QKV, output, gate/inner and FFN-output projections) on
    :func:`kernels.decode_gemm` instead of cuBLAS."""
    from . import kernels as ours

    pkg = importlib.import_module(package)
    ref = importlib.import_module(f"{package}.kernels")
    if getattr(ref, "__omniasr_b200__", False):
        _route_products(package, gemm)
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
    _route_products(package, gemm)
    beam = importlib.import_module(f"{package}.beam")  # its selection after the LM head (beam.py:161-187)
    llm = importlib.import_module(f"{package}.llm")
    global EOS, PAD, LIMIT
    EOS, PAD, LIMIT = llm.EOS, llm.PAD, decode.LIMIT
    if beam.BeamDecoder.step_beam is not _beam_step:
        _beam_step.reference = beam.BeamDecoder.step_beam
        beam.BeamDecoder.step_beam = _beam_step
    return merged
