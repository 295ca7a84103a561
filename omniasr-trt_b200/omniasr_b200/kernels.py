"""B200 (sm_100a) kernels behind the Python API of ``omniasr_trt.kernels`` (Wataru-Nakata/omniasr-trt).

Same names, arguments, results and edge semantics as the reference module
(``omniasr_trt/kernels.py:25-423``), so its decoders (``decode.py``, ``spec.py``, ``beam.py``) and their
CUDA-graph capture run on these kernels unchanged:

* :func:`rope_kv` -- RoPE of q and k at each token's position and the KV-cache append, bit-exact with
  ``modeling.apply_rope`` (``kernels.py:294-306``);
* :func:`decode_attention` -- one query per row, split-KV flash-decode (``kernels.py:406-423``);
* :func:`draft_attention` -- a row's 1 + k draft queries, causal within them (``kernels.py:338-358``);
* :func:`beam_attention` -- beams over their input's shared context plus their own generated keys through
  the pointer history (``kernels.py:309-332``);
* :func:`prefill_attention` -- causal attention of prefilled contexts, the prefill's
  ``F.scaled_dot_product_attention(is_causal=True)`` (``decode.py:171``);
* :func:`reorder_gather` -- the beam reorder ``dst[r] = src[parent[r]]``, byte-exact (``llm.py:237-238``,
  ``beam.py:175-176``).

Each call is a launch (or two) of hand-written CUDA through the C ABI of ``include/omniasr_b200.h`` on the
current stream; outputs and the beam search's split workspace are allocated with ``torch.empty`` on the caller's
device (from the graph pool during a capture); decode and draft calls reuse one zeroed workspace per stream, whose
leading unit counters let the pass merge split units itself. There is no other code path: on a CUDA device without
the built library every function raises.
"""

from __future__ import annotations

import ctypes

import torch

from . import _lib

ATTN = {"block": 64, "warps": 8, "stages": 2, "programs": 264}  # accepted and ignored (reference launch knobs)
DRAFT_ATTN = {"block": 32, "warps": 4, "stages": 2, "programs": 264}

_DTYPES = {torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}
_status: dict[int, torch.Tensor] = {}


def available(device: torch.device) -> bool:
    """True on a CUDA device these kernels run on (compute capability 10.0).

    Raises on a CUDA device when the library is missing: the product path has no silent fallback.
    """
    device = torch.device(device)
    if device.type != "cuda" or not torch.cuda.is_available():
        return False
    lib = _lib.load()
    index = device.index if device.index is not None else torch.cuda.current_device()
    return bool(lib.omniasr_device_supported(index))


def status_word(device: torch.device | int | None = None) -> torch.Tensor:
    """The device's status word (int32; bit 1: an index outside its tensor was skipped, bit 2: a bounded wait
    gave up). Kernels OR into it; it is never cleared by them."""
    index = torch.device("cuda", torch.cuda.current_device() if device is None else
                         (device if isinstance(device, int) else torch.device(device).index or 0)).index
    word = _status.get(index)
    if word is None:
        with torch.inference_mode(False):  # a normal tensor, so it can be cleared inside or outside inference mode
            word = _status[index] = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", index))
    return word


def read_status(device=None, clear: bool = True) -> int:
    """Synchronises, returns the status word and clears it. After a wait that gave up (bit 2) the unit counters of
    the decode / draft workspaces and the split-tile counters of the GEMM workspaces may be left non-zero,
    so those workspaces are dropped (the next call zeroes a new one)."""
    word = status_word(device)
    value = int(word.item())
    if clear:
        word.zero_()
    if value & 2:
        index = word.device.index
        for key in [k for k in _ATTN_WS if k[0] == index]:
            _ATTN_WS_RETIRED.append(_ATTN_WS.pop(key))
        for key in [k for k in _GEMM_WS if k[0] == index]:
            _GEMM_WS_RETIRED.append(_GEMM_WS.pop(key))
    return value


def _ptr(t: torch.Tensor | None) -> ctypes.c_void_p | None:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _dtype(t: torch.Tensor, name: str) -> int:
    code = _DTYPES.get(t.dtype)
    if code is None:
        raise ValueError(f"{name}: dtype {t.dtype} (supported: bfloat16, float32)")
    return code


def _index(t: torch.Tensor) -> torch.Tensor:
    """int64, contiguous (the reference's index tensors are torch.long)."""
    if t.dtype != torch.int64:
        t = t.to(torch.int64)
    return t.contiguous()


def _cache(k: torch.Tensor, v: torch.Tensor, name: str) -> tuple:
    if k.dim() != 4 or v.shape != k.shape or v.stride() != k.stride():
        raise ValueError(f"{name}: k and v caches must be [rows, H, S, D] views with the same strides")
    if k.stride(3) != 1:
        raise ValueError(f"{name}: cache head_dim stride must be 1")
    if v.dtype != k.dtype:
        raise ValueError(f"{name}: k / v dtypes differ")
    return k.size(0), k.size(2), k.stride(0), k.stride(1), k.stride(2)


def _workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    return torch.empty(max(int(nbytes), 16), dtype=torch.uint8, device=device)


_ATTN_WS: dict = {}  # (device, stream) -> decode / draft workspace; its unit counters start zero and stay zero
_ATTN_WS_RETIRED: list = []  # outgrown workspaces, kept alive for CUDA graphs that captured them


def _attn_workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """The decode / draft workspace of the current stream: zeroed once when allocated (its leading unit counters
    must be zero on entry, and every call leaves them zero), reused by the stream's calls in order."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _ATTN_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        if ws is not None:
            _ATTN_WS_RETIRED.append(ws)
        with torch.inference_mode(False):
            ws = torch.zeros(max(int(nbytes), 1 << 20), dtype=torch.uint8, device=device)
        _ATTN_WS[key] = ws
    return ws


def rope_kv(qkv: torch.Tensor, cs: torch.Tensor, pos: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor,
            heads: int, slots: torch.Tensor | None = None, cache_pos: torch.Tensor | None = None) -> torch.Tensor:
    """``qkv`` [N, 3*H*D] (q|k|v of N tokens), ``cs`` [P, D/2, 2] fp32, ``pos`` [N]; ``k_cache``/``v_cache``
    [rows, H, S, D] with unit stride in D. Rotates at ``pos[n]`` and writes token n's k, v at cache row
    ``slots[n]`` (default n), position ``cache_pos[n]`` (default ``pos[n]``); returns the rotated q [N, H, D]."""
    n = qkv.size(0)
    dim = qkv.size(1) // (3 * heads)
    q = torch.empty(n, heads, dim, device=qkv.device, dtype=qkv.dtype)
    if n == 0:
        return q
    if qkv.stride(1) != 1:
        raise ValueError("rope_kv: qkv must have unit inner stride")
    if k_cache.dtype != qkv.dtype:
        raise ValueError("rope_kv: cache dtype differs from qkv")
    cs = cs if cs.dtype == torch.float32 and cs.is_contiguous() else cs.float().contiguous()
    rows, length, s_row, s_head, s_pos = _cache(k_cache, v_cache, "rope_kv")
    pos = _index(pos)
    slots = None if slots is None else _index(slots)
    cache_pos = None if cache_pos is None else _index(cache_pos)
    _lib.call("omniasr_rope_kv", _ptr(qkv), qkv.stride(0), _ptr(cs), cs.size(0), _ptr(pos), _ptr(slots),
              _ptr(cache_pos), _ptr(q), _ptr(k_cache), _ptr(v_cache), rows, length, s_row, s_head, s_pos, n, heads,
              dim, _dtype(qkv, "rope_kv"), _ptr(status_word(qkv.device)), _stream(qkv.device))
    return q


def decode_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lengths: torch.Tensor,
                     keys: int, scale: float, block: int | None = None, warps: int | None = None,
                     stages: int | None = None, programs: int | None = None) -> torch.Tensor:
    """``q`` [B, H, D]; ``k_cache``/``v_cache`` [>=B, H, S, D]; row r attends to keys [0, lengths[r]) (all
    within the first ``keys``, which fixes the launch grid). Returns [B, H, D] in q's dtype; a row of length 0
    gets zeros. ``block``/``warps``/``stages``/``programs`` are accepted for API compatibility and ignored."""
    b, heads, dim = q.shape
    out = torch.empty_like(q)
    if b == 0:
        return out
    if not q.is_contiguous():
        raise ValueError("decode_attention: q must be contiguous [B, H, D]")
    dtype = _dtype(q, "decode_attention")
    rows, length, s_row, s_head, s_pos = _cache(k_cache, v_cache, "decode_attention")
    lengths = _index(lengths)
    lib = _lib.load()
    nbytes = lib.omniasr_attention_workspace(_lib.DECODE, dtype, b, 1, heads, dim, keys, 0)
    ws = _attn_workspace(nbytes, q.device)
    _lib.call("omniasr_decode_attention", _ptr(q), _ptr(k_cache), _ptr(v_cache), rows, length, s_row, s_head, s_pos,
              _ptr(lengths), _ptr(out), b, heads, dim, int(keys), float(scale), dtype, _ptr(ws), ws.numel(),
              _ptr(status_word(q.device)), _stream(q.device))
    return out


def draft_attention(q: torch.Tensor, k_cache: torch.Tensor, v_cache: torch.Tensor, lengths: torch.Tensor,
                    tokens: int, keys: int, scale: float, **launch) -> torch.Tensor:
    """Draft verification: ``q`` [B*T, H, D], row b's T queries at rows b*T .. b*T+T-1; query i of row b attends
    to keys [0, lengths[b] + i) of cache row b (``k_cache``/``v_cache`` [>=B, H, S, D], all within the first
    ``keys``). Returns [B*T, H, D] in q's dtype. ``launch`` (reference launch knobs) is ignored."""
    rows_q, heads, dim = q.shape
    out = torch.empty_like(q)
    if rows_q == 0:
        return out
    if rows_q % tokens:
        raise ValueError(f"draft_attention: {rows_q} query rows is not a multiple of tokens={tokens}")
    if not q.is_contiguous():
        raise ValueError("draft_attention: q must be contiguous [B*T, H, D]")
    b = rows_q // tokens
    dtype = _dtype(q, "draft_attention")
    rows, length, s_row, s_head, s_pos = _cache(k_cache, v_cache, "draft_attention")
    lengths = _index(lengths)
    lib = _lib.load()
    nbytes = lib.omniasr_attention_workspace(_lib.DRAFT, dtype, b, tokens, heads, dim, keys, 0)
    ws = _attn_workspace(nbytes, q.device)
    _lib.call("omniasr_draft_attention", _ptr(q), _ptr(k_cache), _ptr(v_cache), rows, length, s_row, s_head, s_pos,
              _ptr(lengths), _ptr(out), b, int(tokens), heads, dim, int(keys), float(scale), dtype, _ptr(ws),
              ws.numel(), _ptr(status_word(q.device)), _stream(q.device))
    return out


def beam_attention(q: torch.Tensor, kc: torch.Tensor, vc: torch.Tensor, ctx_len: torch.Tensor, kg: torch.Tensor,
                   vg: torch.Tensor, ptr: torch.Tensor, gen_len: torch.Tensor, beams: int, ctx_keys: int,
                   scale: float) -> torch.Tensor:
    """Beam rows ``q`` [S*N, H, D] (input g's beams are rows g*N .. g*N+N-1): attention over input g's context
    ``kc``/``vc`` [>=S, H, C, D] (first ``ctx_len[g]`` keys, all within ``ctx_keys``) and row r's generated keys
    ``kg``/``vg`` [>=S*N, H, G, D], position j taken from row ``ptr[r, j]`` (first ``gen_len[r]``)."""
    rows_q, heads, dim = q.shape
    out = torch.empty_like(q)
    if rows_q == 0:
        return out
    if rows_q % beams:
        raise ValueError(f"beam_attention: {rows_q} rows is not a multiple of beams={beams}")
    if not q.is_contiguous():
        raise ValueError("beam_attention: q must be contiguous [S*N, H, D]")
    if ptr.dtype != torch.int32 or ptr.dim() != 2 or ptr.stride(1) != 1:
        raise ValueError("beam_attention: ptr must be int32 [R, G] with unit inner stride")
    groups = rows_q // beams
    dtype = _dtype(q, "beam_attention")
    c_rows, c_len, c_row, c_head, c_pos = _cache(kc, vc, "beam_attention")
    g_rows, g_len, g_row, g_head, g_pos = _cache(kg, vg, "beam_attention")
    if ptr.size(0) < rows_q or ptr.size(1) < g_len:
        raise ValueError("beam_attention: ptr must cover [rows, generated length]")
    ctx_len, gen_len = _index(ctx_len), _index(gen_len)
    lib = _lib.load()
    nbytes = lib.omniasr_attention_workspace(_lib.BEAM, dtype, groups, beams, heads, dim, ctx_keys, g_len)
    ws = _workspace(nbytes, q.device)
    _lib.call("omniasr_beam_attention", _ptr(q), _ptr(kc), _ptr(vc), c_rows, c_len, c_row, c_head, c_pos,
              _ptr(ctx_len), _ptr(kg), _ptr(vg), g_rows, g_len, g_row, g_head, g_pos, _ptr(ptr), ptr.stride(0),
              _ptr(gen_len), _ptr(out), groups, int(beams), heads, dim, int(ctx_keys), float(scale), dtype, _ptr(ws),
              ws.numel(), _ptr(status_word(q.device)), _stream(q.device))
    return out


def prefill_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float | None = None) -> torch.Tensor:
    """Causal attention of prefilled contexts: ``q``/``k``/``v`` [B, H, W, D] (any strides, unit stride in D; k and
    v typically cache views); query w sees keys [0, w]. Returns [B, H, W, D] in q's dtype -- a view of a
    [B, W, H, D] buffer, so the caller's ``o.transpose(1, 2).reshape(B * W, -1)`` costs nothing. This is the
    reference's ``F.scaled_dot_product_attention(q, k, v, is_causal=True)`` (decode.py:171): bf16 head_dim 128 and
    512 run on the tensor-core prefill kernels; other dtypes / head dims run as a drafted verify with W queries per
    row on the CUDA cores. :func:`prefill_attention_grouped` is the head_dim-512 alternative on the decode pass."""
    b, heads, width, dim = q.shape
    scale = dim**-0.5 if scale is None else float(scale)
    out = torch.empty(b, width, heads, dim, dtype=q.dtype, device=q.device)
    if b == 0 or width == 0:
        return out.transpose(1, 2)
    if k.shape != q.shape or v.shape != q.shape or q.stride(3) != 1 or k.stride(3) != 1 or v.stride(3) != 1:
        raise ValueError("prefill_attention: q, k, v must be [B, H, W, D] with unit stride in D")
    if q.dtype == torch.bfloat16 and dim in (128, 512):
        _lib.call("omniasr_prefill_attention", _ptr(q), q.stride(0), q.stride(1), q.stride(2), _ptr(k), k.stride(0),
                  k.stride(1), k.stride(2), _ptr(v), v.stride(0), v.stride(1), v.stride(2), _ptr(out), out.stride(0),
                  out.stride(2), out.stride(1), b, heads, width, dim, scale, _lib.BF16,
                  _ptr(status_word(q.device)), _stream(q.device))
        return out.transpose(1, 2)
    # Every row's W queries as one draft of W tokens over its own keys: query w sees 1 + w keys.
    if k.stride() != v.stride():  # the draft pass reads k and v through one set of strides
        k, v = k.contiguous(), v.contiguous()
    qq = q.transpose(1, 2).reshape(b * width, heads, dim)
    ones = torch.ones(b, dtype=torch.int64, device=q.device)
    o = draft_attention(qq, k, v, ones, width, width, scale)
    return o.view(b, width, heads, dim).transpose(1, 2)


_PREFILL_GROUP = 16  # query positions per group of the grouped prefill


def prefill_attention_grouped(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                              scale: float | None = None) -> torch.Tensor:
    """bf16 head_dim 512: every row's queries as groups of 16 consecutive positions on the tensor-core decode pass
    (omniasr_prefill_attention_grouped), the queries padded to a multiple of 16 positions; rows are split into calls
    of at most 16384 (group, head) units. The same result as :func:`prefill_attention` (within bf16 rounding)."""
    b, heads, width, dim = q.shape
    if q.dtype != torch.bfloat16 or dim != 512 or q.stride(3) != 1 or k.shape != q.shape or v.shape != q.shape:
        raise ValueError("prefill_attention_grouped: bf16 [B, H, W, 512] q, k, v with unit stride in D")
    scale = dim**-0.5 if scale is None else float(scale)
    if b == 0 or width == 0:
        return torch.empty(b, width, heads, dim, dtype=q.dtype, device=q.device).transpose(1, 2)
    wp = -(-width // _PREFILL_GROUP) * _PREFILL_GROUP
    if k.stride() != v.stride() or k.stride(3) != 1:
        k, v = k.contiguous(), v.contiguous()
    qp = torch.zeros(b, wp, heads, dim, dtype=q.dtype, device=q.device)
    qp[:, :width] = q.transpose(1, 2)
    outp = torch.empty_like(qp)
    rows_per_call = max(1, 16384 // ((wp // _PREFILL_GROUP) * heads))
    lib = _lib.load()
    for r0 in range(0, b, rows_per_call):
        rb = min(rows_per_call, b - r0)
        nbytes = lib.omniasr_prefill_grouped_workspace(rb, heads, width, dim)
        ws = _attn_workspace(nbytes, q.device)
        kk, vv = k[r0:r0 + rb], v[r0:r0 + rb]
        _lib.call("omniasr_prefill_attention_grouped", _ptr(qp[r0:r0 + rb]), _ptr(kk), _ptr(vv), kk.size(0),
                  kk.size(2), kk.stride(0), kk.stride(1), kk.stride(2), _ptr(outp[r0:r0 + rb]), rb, heads, width, dim,
                  float(scale), _lib.BF16, _ptr(ws), ws.numel(), _ptr(status_word(q.device)), _stream(q.device))
    return outp[:, :width].transpose(1, 2)


def _vec(t: torch.Tensor, dtype: torch.dtype, name: str) -> torch.Tensor:
    if t.dtype != dtype or not t.is_contiguous():
        raise ValueError(f"{name} must be a contiguous {dtype} tensor")
    return t


def propose(out: torch.Tensor, draft: torch.Tensor, draft_len: torch.Tensor, last: torch.Tensor,
            first: torch.Tensor, nxt: torch.Tensor, start: torch.Tensor, tokens: int, ngram: int, behind: int,
            ahead: int, reach: tuple, self_window: int, self_min: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Drafted decoding's proposals of rows 0..B-1 (B = ``last.numel()``): ``tokens`` ids each [B, k] (int64) and
    whether they come from the draft [B] (bool); ``start`` [B] (int64) gets the draft position of the first one.
    ``out`` [>=B, S] / ``draft`` [>=B, C] int32 token rows (unit inner stride); ``draft_len``, ``last``, ``first``,
    ``nxt`` int64 [B]; ``reach`` 4 (distance, matching tokens) pairs. Bit-exact with the reference's ``propose``
    (kernels.py:361-377)."""
    b = last.numel()
    prop = torch.empty(b, tokens, device=out.device, dtype=torch.long)
    use_draft = torch.empty(b, device=out.device, dtype=torch.bool)
    if b == 0:
        return prop, use_draft
    if out.dtype != torch.int32 or draft.dtype != torch.int32 or out.stride(1) != 1 or draft.stride(1) != 1:
        raise ValueError("propose: out and draft must be int32 with unit inner stride")
    for t, name in ((draft_len, "draft_len"), (last, "last"), (first, "first"), (nxt, "nxt"), (start, "start")):
        _vec(t, torch.int64, name)
    pairs = [int(x) for pair in reach for x in pair]
    if len(pairs) != 8:
        raise ValueError("propose: reach must hold 4 (distance, tokens) pairs")
    creach = (ctypes.c_int * 8)(*pairs)
    _lib.call("omniasr_propose", _ptr(out), out.stride(0), out.size(1), _ptr(draft), draft.stride(0), draft.size(1),
              _ptr(draft_len), _ptr(last), _ptr(first), _ptr(nxt), _ptr(start), _ptr(prop), _ptr(use_draft), b,
              int(tokens), int(ngram), int(behind), int(ahead), ctypes.cast(creach, ctypes.c_void_p),
              int(self_window), int(self_min), _ptr(status_word(out.device)), _stream(out.device))
    return prop, use_draft


def accept(tokens: torch.Tensor, nxt: torch.Tensor, out: torch.Tensor, tok: torch.Tensor, last: torch.Tensor,
           done: torch.Tensor, draft_next: torch.Tensor, start: torch.Tensor, use_draft: torch.Tensor, limit: int,
           eos: int) -> None:
    """In place on rows 0..B-1 after a drafted step: ``tokens`` fed [B, T] (the newest token, then the proposal) and
    ``nxt`` the argmax after each [B, T] (int64); ``out`` [>=B, S] int32; ``tok`` / ``last`` / ``draft_next`` /
    ``start`` [B] int64, ``done`` / ``use_draft`` [B] bool. Bit-exact with the reference's ``accept``
    (kernels.py:380-391)."""
    b, width = tokens.shape
    if b == 0:
        return
    _vec(tokens, torch.int64, "tokens")
    _vec(nxt, torch.int64, "nxt")
    for t, name in ((tok, "tok"), (last, "last"), (draft_next, "draft_next"), (start, "start")):
        _vec(t, torch.int64, name)
    _vec(done, torch.bool, "done")
    _vec(use_draft, torch.bool, "use_draft")
    if out.dtype != torch.int32 or out.stride(1) != 1:
        raise ValueError("accept: out must be int32 with unit inner stride")
    _lib.call("omniasr_accept", _ptr(tokens), _ptr(nxt), _ptr(out), out.stride(0), out.size(1), _ptr(tok),
              _ptr(last), _ptr(done), _ptr(draft_next), _ptr(start), _ptr(use_draft), b, width, int(limit),
              int(eos), _ptr(status_word(out.device)), _stream(out.device))


def beam_select(logp: torch.Tensor, score: torch.Tensor, ended: torch.Tensor, count: torch.Tensor, tok: torch.Tensor,
                hist: torch.Tensor, ptr: torch.Tensor, k_step: torch.Tensor, ctx: torch.Tensor, gdone: torch.Tensor,
                beams: int, length_norm: bool, eos: int, pad: int, limit: int) -> None:
    """Beam search's selection step after the LM head, in place: ``logp`` [S * beams, V] (bf16 or fp32) selects, per
    group of ``beams`` rows, the group's best ``beams`` candidates over beams x V and every row of a group that is
    not done follows its parent. State: ``score`` [R] fp32, ``ended`` [R] bool, ``count`` / ``tok`` [R] int64,
    ``hist`` [R, G + 1] / ``ptr`` [R, G] int32 (unit inner stride), ``k_step`` / ``ctx`` [S] int64, ``gdone`` [S]
    bool, R >= S * beams. Bit-exact with BeamDecoder.step_beam after its log-softmax (beam.py:161-187)."""
    rows, vocab = logp.shape
    groups = rows // beams
    if rows != groups * beams:
        raise ValueError("beam_select: logp rows must be groups x beams")
    if logp.dtype not in (torch.bfloat16, torch.float32) or logp.stride(1) != 1:
        raise ValueError("beam_select: logp must be bf16 or fp32 with unit inner stride")
    if groups == 0:
        return
    _vec(score, torch.float32, "score")
    _vec(ended, torch.bool, "ended")
    for t, name in ((count, "count"), (tok, "tok"), (k_step, "k_step"), (ctx, "ctx")):
        _vec(t, torch.int64, name)
    _vec(gdone, torch.bool, "gdone")
    for t, name in ((hist, "hist"), (ptr, "ptr")):
        if t.dtype != torch.int32 or t.dim() != 2 or (t.size(1) > 1 and t.stride(1) != 1):
            raise ValueError(f"beam_select: {name} must be int32 [rows, width] with unit inner stride")
    _lib.call("omniasr_beam_select", _ptr(logp), logp.stride(0), int(logp.dtype == torch.float32), _ptr(score),
              _ptr(ended), _ptr(count), _ptr(tok), _ptr(hist), hist.stride(0), hist.size(1), _ptr(ptr), ptr.stride(0),
              ptr.size(1), _ptr(k_step), _ptr(ctx), _ptr(gdone), groups, beams, vocab, int(bool(length_norm)),
              int(eos), int(pad), int(limit), _ptr(status_word(logp.device)), _stream(logp.device))


GEMM_MODES = {"store": 0, "residual": 1, "swiglu": 2}
_GEMM_WS: dict = {}  # (device, stream) -> zero-initialised workspace; the kernel leaves its counters zero
_GEMM_WS_RETIRED: list = []  # outgrown workspaces, kept alive for CUDA graphs that captured them


def _gemm_workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    key = (device.index, torch.cuda.current_stream(device).cuda_stream)
    ws = _GEMM_WS.get(key)
    if ws is None or ws.numel() < nbytes:
        if ws is not None:
            _GEMM_WS_RETIRED.append(ws)
        with torch.inference_mode(False):
            ws = torch.zeros(max(int(nbytes), 1 << 20), dtype=torch.uint8, device=device)
        _GEMM_WS[key] = ws
    return ws


def decode_gemm(x: torch.Tensor, w: torch.Tensor, mode: str = "store", residual: torch.Tensor | None = None,
                out: torch.Tensor | None = None) -> torch.Tensor:
    """The decoder step's weight GEMMs for at most 64 token rows (bf16): ``x @ w.t()`` ("store"),
    ``torch.addmm(residual, x, w.t())`` ("residual"), or with ``w`` the concatenated [gate; inner] weights
    ``inner * F.silu(gate)`` of ``(x @ w.t()).chunk(2, -1)`` ("swiglu", each half rounded to bf16 first, as the
    reference computes it). Rows of x and w must be contiguous with 16-byte aligned strides. The kernel requests its
    first weight tiles before waiting for the kernel launched before it on the stream, so ``w`` must not be written
    by that kernel (decoder weights are not); x and the residual may be."""
    rows, k = x.shape
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16:
        raise ValueError("decode_gemm: bf16 x and w")
    if x.stride(1) != 1 or w.stride(1) != 1 or w.size(1) != k:
        raise ValueError("decode_gemm: x [rows, k] and w [n, k] with unit inner stride")
    m = GEMM_MODES[mode]
    n = w.size(0) // 2 if mode == "swiglu" else w.size(0)
    if out is None:
        out = torch.empty(rows, n, dtype=x.dtype, device=x.device)
    if rows == 0 or n == 0:
        return out
    if mode == "residual":
        if residual is None or residual.shape != (rows, n) or residual.stride(1) != 1:
            raise ValueError("decode_gemm: residual [rows, n] with unit inner stride")
    lib = _lib.load()
    ws = _gemm_workspace(lib.omniasr_decode_gemm_workspace(rows, n, k, m), x.device)
    _lib.call("omniasr_decode_gemm", _ptr(x), x.stride(0), rows, _ptr(w), w.stride(0), n, k, m,
              _ptr(residual) if residual is not None else None, residual.stride(0) if residual is not None else 0,
              _ptr(out), out.stride(0), _ptr(ws), ws.numel(), _ptr(status_word(x.device)), _stream(x.device))
    return out


def decode_gemm_rope(x: torch.Tensor, w: torch.Tensor, cs: torch.Tensor, pos: torch.Tensor, k_cache: torch.Tensor,
                     v_cache: torch.Tensor, heads: int, slots: torch.Tensor | None = None,
                     cache_pos: torch.Tensor | None = None) -> torch.Tensor:
    """``rope_kv(x @ w.t(), cs, pos, k_cache, v_cache, heads, slots, cache_pos)`` in one kernel (bf16, at most 64
    token rows, head_dim a multiple of 128): the QKV product's epilogue rotates q and k and appends k and v to the
    caches; returns q [N, heads, D]. The product is rounded to bf16 before the rotation, as the GEMM's output is.
    As for :func:`decode_gemm`, ``w`` must not be written by the kernel launched just before on the stream."""
    rows, k = x.shape
    n = w.size(0)
    dim = n // (3 * heads)
    if x.dtype != torch.bfloat16 or w.dtype != torch.bfloat16 or w.size(1) != k or n != 3 * heads * dim:
        raise ValueError("decode_gemm_rope: bf16 x [rows, k], w [3 * heads * D, k]")
    if x.stride(1) != 1 or w.stride(1) != 1:
        raise ValueError("decode_gemm_rope: unit inner strides")
    q = torch.empty(rows, heads, dim, dtype=x.dtype, device=x.device)
    if rows == 0:
        return q
    if k_cache.dtype != x.dtype:
        raise ValueError("decode_gemm_rope: cache dtype differs from x")
    cs = cs if cs.dtype == torch.float32 and cs.is_contiguous() else cs.float().contiguous()
    crows, length, s_row, s_head, s_pos = _cache(k_cache, v_cache, "decode_gemm_rope")
    pos = _index(pos)
    slots = None if slots is None else _index(slots)
    cache_pos = None if cache_pos is None else _index(cache_pos)
    lib = _lib.load()
    ws = _gemm_workspace(lib.omniasr_decode_gemm_workspace(rows, n, k, GEMM_MODES["store"]), x.device)
    _lib.call("omniasr_decode_gemm_rope", _ptr(x), x.stride(0), rows, _ptr(w), w.stride(0), k, _ptr(cs), cs.size(0),
              _ptr(pos), _ptr(slots), _ptr(cache_pos), _ptr(q), _ptr(k_cache), _ptr(v_cache), crows, length, s_row,
              s_head, s_pos, heads, dim, _ptr(ws), ws.numel(), _ptr(status_word(x.device)), _stream(x.device))
    return q


def reorder_gather(src: torch.Tensor, parent: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
    """``out[r] = src[parent[r]]`` along dim 0, byte-exact (``torch.index_select(src, 0, parent)``); each row of
    ``src`` / ``out`` must be contiguous. ``out`` (optional) must not overlap ``src``."""
    rows = parent.numel()
    if out is None:
        out = torch.empty((rows,) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
    if rows == 0:
        return out
    if out.shape[1:] != src.shape[1:] or out.size(0) < rows or out.dtype != src.dtype:
        raise ValueError("reorder_gather: out must be [len(parent), *src.shape[1:]] of src's dtype")
    if not (src[0].is_contiguous() and out[0].is_contiguous()):
        raise ValueError("reorder_gather: rows of src and out must be contiguous")
    if parent.dtype not in (torch.int32, torch.int64):
        raise ValueError("reorder_gather: parent must be int32 or int64")
    parent = parent.contiguous()
    row_bytes = src[0].numel() * src.element_size()
    _lib.call("omniasr_reorder_gather", _ptr(src), src.stride(0) * src.element_size(), src.size(0), _ptr(out),
              out.stride(0) * out.element_size(), _ptr(parent), int(parent.dtype == torch.int64), rows, row_bytes,
              _ptr(status_word(src.device)), _stream(src.device))
    return out


def splits_for(rows: int, heads: int, keys: int, block: int = 64, programs: int = 264) -> tuple[int, int]:
    """Key splits (a power of two, about ``programs`` programs in all) and the keys each split covers -- the
    reference's rule (``kernels.py:393-400``), kept for its scripts; these kernels plan their own splits."""
    s, c = ctypes.c_int(), ctypes.c_int()
    _lib.call("omniasr_splits_for", int(rows), int(heads), int(keys), int(block), int(programs), ctypes.byref(s),
              ctypes.byref(c))
    return s.value, c.value
