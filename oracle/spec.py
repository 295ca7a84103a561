"""Speculative decoding's control steps, restated in numpy with per-row loops (test infrastructure only).

* ``propose``: a row's next ``tokens`` proposed tokens -- the reference's ``_propose`` (omniasr_trt/kernels.py:214-262,
  wrapper :361-377), whose PyTorch statement is the reference's own kernel check ``reference_propose``
  (tests/test_spec.py:43-92). The draft position whose preceding tokens match the row's newest ones best (a match
  must be longer the farther it lies from the expected position: the ``reach`` table), or else the latest earlier
  place of the row's own tokens that does (prompt lookup), continued periodically.
* ``accept``: after a drafted step, keep the fed tokens equal to the argmax before them -- the reference's ``_accept``
  (omniasr_trt/kernels.py:264-291, wrapper :380-391).

Arrays are numpy; ``out`` / ``draft`` int32 rows, per-row scalars int64, flags bool. ``propose`` uses
``next_pow2(self_window)`` own candidates and ``next_pow2(behind + ahead + 1)`` draft slots, as the Triton launch does
(kernels.py:372-373); the reference's constants (256, and 64 + 160 + 1) make both the PyTorch statement's ranges.
"""

from __future__ import annotations

import numpy as np


def _next_pow2(n: int) -> int:
    return 1 << max(0, int(n) - 1).bit_length()


def _need(dist: int, ngram: int, reach) -> int:
    for r, n in reach:
        if dist <= r:
            return n
    return ngram


def propose(out, draft, draft_len, last, first, nxt, tokens: int, ngram: int, behind: int, ahead: int, reach,
            self_window: int, self_min: int):
    """Proposals [B, tokens] int64, from-draft flags [B] bool and start positions [B] int64 of rows 0..B-1."""
    b = len(last)
    prop = np.zeros((b, tokens), dtype=np.int64)
    use_draft = np.zeros(b, dtype=bool)
    start = np.zeros(b, dtype=np.int64)
    sw = _next_pow2(self_window)
    for r in range(b):
        lst, fst, nx, dl = int(last[r]), int(first[r]), int(nxt[r]), int(draft_len[r])
        hist = [int(out[r, lst - t]) if lst - t >= fst else -1 for t in range(ngram)]
        hv = [lst - t >= fst for t in range(ngram)]
        # The draft: candidate anchors (draft position of the newest token) around the expected one.
        best_rank, best_off, best_score = -1, None, 0
        for off in range(-behind, ahead + 1):
            anchor = nx - 1 + off
            alive = anchor < dl
            score = 0
            for t in range(ngram):
                at = anchor - t
                alive = alive and at >= 0 and hv[t] and int(draft[r, at]) == hist[t]
                score += alive
            dist = abs(off)
            rank = score * 256 - dist if score >= _need(dist, ngram, reach) else -1
            if rank > best_rank:  # strictly greater: the first (leftmost) maximum wins
                best_rank, best_off, best_score = rank, off, score
        found = best_rank >= 0
        drafted = best_score if found else 0
        st = nx + best_off if found else nx
        # The row's own tokens: latest earlier position first.
        mine, mine_i = -1, 0
        for i in range(sw):
            back = lst - 1 - i
            alive = back >= fst
            score = 0
            for t in range(ngram):
                at = back - t
                alive = alive and at >= 0 and hv[t] and int(out[r, at]) == hist[t]
                score += alive
            if score > mine:
                mine, mine_i = score, i
        j = lst - 1 - mine_i
        period = max(lst - j, 1)
        ud = mine < self_min or mine <= drafted
        for k in range(tokens):
            if ud:
                at = st + k
                prop[r, k] = int(draft[r, at]) if at < dl else 0
            else:
                prop[r, k] = int(out[r, j + 1 + k % period])
        use_draft[r] = ud
        start[r] = st
    return prop, use_draft, start


def accept(tokens, nxt, out, tok, last, done, draft_next, start, use_draft, limit: int, eos: int) -> None:
    """In place on rows 0..B-1: a running row keeps argmax 0..n at positions last+1+j, n = its leading proposed tokens
    equal to the argmax before them, cut at the first EOS / position >= limit among those."""
    b, width = tokens.shape
    cap = out.shape[1]
    for r in range(b):
        if done[r]:
            continue
        p = int(last[r]) + 1
        g = [int(x) for x in nxt[r]]
        fed = [int(tokens[r, j + 1]) if j + 1 < width else -2 for j in range(width)]
        kept = width - 1
        for j in range(width):
            if fed[j] != g[j]:
                kept = min(j, width - 1)
                break
        n = kept
        ended = False
        for j in range(kept + 1):
            if g[j] == eos or p + j >= limit:
                n, ended = j, True
                break
        for j in range(n + 1):
            out[r, min(p + j, cap - 1)] = g[j]
        tok[r] = g[n]
        last[r] = p + n
        done[r] = ended
        base = int(start[r]) if use_draft[r] else int(draft_next[r])
        draft_next[r] = base + n + 1
