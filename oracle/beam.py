"""Beam search's selection step after the LM head, restated in numpy (test infrastructure only).

The tail of the reference's ``BeamDecoder.step_beam`` (omniasr_trt/beam.py:161-187), on the first ``groups``
groups of ``beams`` rows:

* candidates (beam.py:161-170): ``score + logp``, or with length normalisation when the group's row 0 has counted
  tokens ``(score * count + logp) / (count + 1)``, every operation rounded to float32 as torch's elementwise
  kernels round it; an ended row offers only EOS, at its score (everything else -inf);
* the group's best ``beams`` of its beams x vocab candidates (beam.py:171), ordered as ``torch.topk(sorted=True)``
  on a CUDA tensor orders them: value descending, equal values by flat index ascending (torch.topk on the CPU
  breaks ties in no fixed order, so golden vectors made on the CPU avoid ties at the selection);
* parents, new tokens and the rows' reorder (beam.py:172-187).

Arrays are numpy and are updated in place: ``logp`` [R, V] float32 (bf16 values widened), ``score`` [R] float32,
``ended`` [R] bool, ``count`` / ``tok`` [R] int64, ``hist`` [R, G + 1] / ``ptr`` [R, G] int32, ``k_step`` / ``ctx``
[S] int64, ``gdone`` [S] bool.
"""

from __future__ import annotations

import numpy as np


def topk_order(values: np.ndarray, k: int) -> np.ndarray:
    """Indices of the ``k`` largest values, value descending and index ascending among equal values."""
    v = values.astype(np.float32)
    v = np.where(v == 0, np.float32(0), v)  # -0 and +0 compare equal
    v = np.where(np.isnan(v), np.float32(np.inf), v)
    nan_first = np.isnan(values)  # NaN counts as larger than +inf
    return np.lexsort((np.arange(v.size), -v, ~nan_first))[:k]


def candidates(logp: np.ndarray, score: np.ndarray, ended: np.ndarray, count: np.ndarray, beams: int,
               length_norm: bool, eos: int) -> np.ndarray:
    """[R, V] float32 candidates of beam.py:161-170."""
    f32 = np.float32
    r = logp.shape[0]
    sc = score[:r].astype(f32)[:, None]
    lp = logp.astype(f32)
    if length_norm:
        first = count[(np.arange(r) // beams) * beams][:, None]
        c = count[:r][:, None]
        normed = ((sc * c.astype(f32)).astype(f32) + lp).astype(f32) / (c + 1).astype(f32)
        cand = np.where(first > 0, normed.astype(f32), (sc + lp).astype(f32))
    else:
        cand = (sc + lp).astype(f32)
    cand = cand.astype(f32).copy()
    e = ended[:r]
    cand[e] = -np.inf
    cand[e, eos] = score[:r][e]
    return cand


def beam_select(logp, score, ended, count, tok, hist, ptr, k_step, ctx, gdone, beams: int, length_norm: bool,
                eos: int, pad: int, limit: int) -> None:
    r, vocab = logp.shape
    s = r // beams
    rows = np.arange(r)
    group = rows // beams
    live = ~gdone[:s][group]
    k = k_step[:s][group].copy()
    cand = candidates(logp, score, ended, count, beams, length_norm, eos)
    flat = cand.reshape(s, beams * vocab)
    pick = np.stack([topk_order(flat[g], beams) for g in range(s)])  # [S, N]
    top = np.take_along_axis(flat, pick, 1).reshape(-1)
    parent = (pick // vocab + np.arange(s)[:, None] * beams).reshape(-1)
    parent = np.where(live, parent, rows)
    new = np.where(live, (pick % vocab).reshape(-1), tok[:r])
    ptr[:r] = ptr[:r][parent]
    hist[:r] = hist[:r][parent]
    p_ended, p_score, p_count = ended[:r][parent].copy(), score[:r][parent].copy(), count[:r][parent].copy()
    new = np.where(p_ended, eos, new)
    write = live & (k >= 0) & (k < hist.shape[1])  # a position outside the row is skipped (the kernels report it)
    hist[rows[write], k[write]] = new[write].astype(np.int32)
    grow = live & ~p_ended
    score[:r] = np.where(grow, top, p_score).astype(np.float32)
    count[:r] = p_count + (grow & (new != pad) & (new != eos)).astype(np.int64)
    ended[:r] = np.where(live, new == eos, p_ended)
    tok[:r] = new
    all_ended = ended[:r].reshape(s, beams).all(-1)
    k_step[:s] = k_step[:s] + (~gdone[:s]).astype(np.int64)
    gdone[:s] = gdone[:s] | all_ended | (ctx[:s] - 1 + k_step[:s] - 1 >= limit)
