"""Beam search's selection step after the LM head, restated in numpy (test infrastructure only).

The tail of the reference's ``BeamDecoder.step_beam`` (omniasr_trt/beam.py:161-187), on the first ``groups``
groups of ``beams`` rows:

* candidates (beam.py:161-170): ``score + logp``, or with length normalisation when the group's row 0 has counted
  tokens ``(score * count + logp) / (count + 1)``, every operation rounded to float32 as torch's elementwise
  kernels round it; an ended row offers only EOS, at its score (everything else -inf);
* the group's best ``beams`` of its beams x vocab candidates (beam.py:171), in the order ``torch.topk(sorted=True)``
  returns them for a CUDA tensor (:func:`topk_order`; torch.topk on the CPU orders ties in no fixed way, so golden
  vectors made on the CPU avoid ties at the selection);
* parents, new tokens and the rows' reorder (beam.py:172-187).

Arrays are numpy and are updated in place: ``logp`` [R, V] float32 (bf16 values widened), ``score`` [R] float32,
``ended`` [R] bool, ``count`` / ``tok`` [R] int64, ``hist`` [R, G + 1] / ``ptr`` [R, G] int32, ``k_step`` / ``ctx``
[S] int64, ``gdone`` [S] bool.
"""

from __future__ import annotations

import numpy as np


def _order_key(values: np.ndarray) -> np.ndarray:
    """Float32 values as order-preserving integers (int64): -0 counts as +0, NaN as larger than +inf."""
    v = values.astype(np.float32)
    v = np.where(v == 0, np.float32(0), v).astype(np.float32)
    b = v.view(np.uint32).astype(np.int64)
    b = np.where(np.isnan(v), 0x7FC00000, b)
    return np.where(b & 0x80000000, (~b) & 0xFFFFFFFF, b | 0x80000000)


def topk_order(values: np.ndarray, k: int) -> np.ndarray:
    """Indices of the ``k`` <= 32 largest values in the order ``torch.topk(sorted=True)`` returns them for a CUDA
    tensor (pinned by tests/golden/topk_ties.npz, made with torch on a GPU): the values above the k-th largest, then
    those equal to it, each in index order; then a bitonic sorting network over 32 slots (unused slots last) whose
    compare-exchange keeps a pair only when the first entry is the larger, so equal values move with their slots."""
    key = _order_key(values)
    order = np.lexsort((np.arange(key.size), -key))
    kth = key[order[k - 1]]
    above = np.sort(order[:k][key[order[:k]] > kth])
    equal = np.nonzero(key == kth)[0][: k - above.size]
    pre = list(above) + list(equal)
    size_p = 32
    kv = [int(key[i]) for i in pre] + [0] * (size_p - k)
    ix = pre + [-1] * (size_p - k)
    ok = [True] * k + [False] * (size_p - k)

    def exchange(a: int, b: int, direction: bool):
        s = (kv[a] > kv[b] and ok[a]) or not ok[b]
        if s == direction:
            kv[a], kv[b] = kv[b], kv[a]
            ix[a], ix[b] = ix[b], ix[a]
            ok[a], ok[b] = ok[b], ok[a]

    size = 2
    while size < size_p:
        stride = size // 2
        while stride:
            for t in range(size_p // 2):
                pos = 2 * t - (t & (stride - 1))
                exchange(pos, pos + stride, (t & (size // 2)) != 0)
            stride //= 2
        size *= 2
    stride = size_p // 2
    while stride:
        for t in range(size_p // 2):
            pos = 2 * t - (t & (stride - 1))
            exchange(pos, pos + stride, False)
        stride //= 2
    return np.array(ix[:k], dtype=np.int64)


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
