"""Decoder attention restated in torch on the CPU (test infrastructure only).

Plain masked softmax attention, computed in float64 by default from the kernels' exact input values, as the
reference's PyTorch paths compute it:

* decode (q_len 1): ``softmax(q K[:n]^T * scale) V[:n]`` per row -- omniasr_trt/decode.py:206-214 (fallback
  step) and the formula of the reference's kernel test, tests/test_kernels.py:52-55;
* draft verify: query i of row b sees ``lengths[b] + i`` keys -- the ``tril(past)`` mask of
  omniasr_trt/modeling.py:400-403 and tests/test_spec.py:103-108;
* beam: a row sees its input's context ``[0, ctx_len[g])`` and its generated keys ``j < gen_len[r]`` read from
  row ``ptr[r, j]`` -- omniasr_trt/beam.py:221-233 and tests/test_kernels.py:115-126; a row with no keys gets 0;
* prefill: causal attention of right-padded rows -- omniasr_trt/decode.py:171 / modeling.py:398-399.

Tensors are ``torch`` CPU tensors; results are float64 (or ``dtype``).
"""

from __future__ import annotations

import torch


def _masked(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, allowed: torch.Tensor, scale: float) -> torch.Tensor:
    """q [..., Q, D], k/v [..., K, D], allowed [..., Q, K] -> [..., Q, D]; rows with no key -> 0."""
    scores = (q @ k.transpose(-1, -2)) * scale
    scores = scores.masked_fill(~allowed, float("-inf"))
    w = torch.softmax(scores, dim=-1).nan_to_num(0.0)
    return w @ v


def decode_attention(q, k_cache, v_cache, lengths, scale, dtype=torch.float64):
    """q [B, H, D]; caches [>=B, H, S, D]; row b attends to keys [0, lengths[b])."""
    b = q.size(0)
    s = k_cache.size(2)
    k = k_cache[:b].to(dtype)
    v = v_cache[:b].to(dtype)
    allowed = torch.arange(s)[None, :] < lengths.reshape(b, 1).cpu()  # [B, S]
    out = _masked(q.to(dtype)[:, :, None, :], k, v, allowed[:, None, None, :], scale)
    return out[:, :, 0]


def draft_attention(q, k_cache, v_cache, lengths, tokens, scale, dtype=torch.float64):
    """q [B*T, H, D]; query i of row b attends to keys [0, lengths[b] + i) of cache row b."""
    rows, h, d = q.shape
    b = rows // tokens
    s = k_cache.size(2)
    k = k_cache[:b].to(dtype)  # [B, H, S, D]
    v = v_cache[:b].to(dtype)
    qq = q.to(dtype).view(b, tokens, h, d).transpose(1, 2)  # [B, H, T, D]
    lim = lengths.reshape(b, 1).cpu() + torch.arange(tokens)[None, :]  # [B, T]
    allowed = torch.arange(s)[None, None, :] < lim[:, :, None]  # [B, T, S]
    out = _masked(qq, k, v, allowed[:, None], scale)  # [B, H, T, D]
    return out.transpose(1, 2).reshape(rows, h, d)


def beam_attention(q, kc, vc, ctx_len, kg, vg, ptr, gen_len, beams, scale, dtype=torch.float64):
    """q [S*N, H, D]; context kc/vc [>=S, H, C, D]; generated kg/vg [>=S*N, H, G, D] through ptr [R, G]."""
    rows, h, d = q.shape
    out = torch.zeros(rows, h, d, dtype=dtype)
    for r in range(rows):
        g = r // beams
        nc, ng = int(ctx_len[g]), int(gen_len[r])
        if nc + ng == 0:
            continue
        j = torch.arange(ng)
        src = ptr[r, :ng].long()
        k = torch.cat([kc[g, :, :nc], kg[src, :, j].transpose(0, 1)], 1).to(dtype)  # [H, nc+ng, D]
        v = torch.cat([vc[g, :, :nc], vg[src, :, j].transpose(0, 1)], 1).to(dtype)
        w = torch.softmax((q[r].to(dtype)[:, None, :] @ k.transpose(-1, -2)) * scale, dim=-1)
        out[r] = (w @ v)[:, 0]
    return out


def prefill_attention(q, k, v, scale=None, dtype=torch.float64):
    """Causal attention: q/k/v [B, H, W, D] -> [B, H, W, D]; query t sees keys [0, t]."""
    w = q.size(2)
    scale = q.size(-1) ** -0.5 if scale is None else scale
    allowed = torch.ones(w, w, dtype=torch.bool).tril()
    return _masked(q.to(dtype), k.to(dtype), v.to(dtype), allowed, scale)


def prefill_attention_rows(q, k, v, positions, scale=None, dtype=torch.float64):
    """The causal prefill at selected query positions only: q/k/v [B, H, W, D], positions [P] -> [B, H, P, D]; query
    t sees keys [0, t] (the rows of prefill_attention at those positions, for shapes too large to compute whole)."""
    w = q.size(2)
    scale = q.size(-1) ** -0.5 if scale is None else scale
    pos = torch.as_tensor(positions, dtype=torch.long)
    allowed = torch.arange(w)[None, :] <= pos[:, None]  # [P, W]
    return _masked(q[:, :, pos].to(dtype), k.to(dtype), v.to(dtype), allowed, scale)


def error_stats(got: torch.Tensor, want: torch.Tensor) -> tuple[float, float]:
    """(max-abs, mean-abs) difference in float64."""
    diff = (got.double() - want.double()).abs()
    return float(diff.max()) if diff.numel() else 0.0, float(diff.mean()) if diff.numel() else 0.0


def draft_attention_model_dtype(q, k_cache, v_cache, lengths, tokens, scale):
    """The reference's CPU arithmetic for the verify step, used to time the CPU baseline: scores from a matmul in the
    model dtype, softmax in float32, then the probabilities cast back to the model dtype for the value matmul
    (omniasr_trt/decode.py:211-214, with the ``len + i`` keys of query i, modeling.py:400-403)."""
    rows, h, d = q.shape
    b = rows // tokens
    keys = k_cache.size(2)
    qq = q.view(b, tokens, h, d).transpose(1, 2)  # [B, H, T, D]
    lim = lengths.reshape(b, 1) + torch.arange(tokens)[None, :]
    bias = torch.zeros(b, 1, tokens, keys, dtype=torch.float32)
    bias.masked_fill_(~(torch.arange(keys)[None, None, :] < lim[:, :, None])[:, None], float("-inf"))
    scores = (qq @ k_cache[:b].transpose(-1, -2)).float() * scale + bias
    out = torch.softmax(scores, dim=-1).to(q.dtype) @ v_cache[:b]
    return out.transpose(1, 2).reshape(rows, h, d)
