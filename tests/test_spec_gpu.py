"""Speculative decoding's control kernels (propose / accept) against the reference's golden vectors and the
oracle, bit-exact. The reference checks its Triton propose against a PyTorch statement of the rule
(tests/test_spec.py:206-228); these restate that check for the CUDA kernels, plus accept, which the reference
covers only through token equality of whole decodes (also run here, tests/test_dropin_gpu.py)."""

import numpy as np
import pytest
import torch

from conftest import GOLDEN
DEVICE = "cuda"
from oracle import spec as ospec

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

NGRAM, BEHIND, AHEAD, REACH, SELF_WINDOW, SELF_MIN, DRAFT_CAPACITY = 8, 64, 160, ((1, 1), (4, 2), (12, 4), (40, 6)), \
    256, 3, 1024


def K():
    from omniasr_b200 import kernels

    return kernels


def run_propose(out, draft, dlen, last, first, nxt, k, **kw):
    d = torch.device(DEVICE)
    t = lambda a, dt: torch.as_tensor(a, dtype=dt, device=d)  # noqa: E731
    start = torch.full((len(last),), -7, dtype=torch.int64, device=d)
    args = dict(ngram=NGRAM, behind=BEHIND, ahead=AHEAD, reach=REACH, self_window=SELF_WINDOW, self_min=SELF_MIN)
    args.update(kw)
    prop, ud = K().propose(t(out, torch.int32), t(draft, torch.int32), t(dlen, torch.int64), t(last, torch.int64),
                           t(first, torch.int64), t(nxt, torch.int64), start, k, args["ngram"], args["behind"],
                           args["ahead"], args["reach"], args["self_window"], args["self_min"])
    torch.cuda.synchronize()
    return prop.cpu().numpy(), ud.cpu().numpy(), start.cpu().numpy()


def test_propose_matches_reference_golden():
    d = np.load(GOLDEN / "propose.npz")
    reach = tuple(tuple(int(x) for x in r) for r in d["reach"])
    for t in range(len(d["k"])):
        k = int(d["k"][t])
        prop, ud, start = run_propose(d["out"][t], d["draft"][t], d["draft_len"][t], d["last"][t], d["first"][t],
                                      d["nxt"][t], k, ngram=int(d["ngram"]), behind=int(d["behind"]),
                                      ahead=int(d["ahead"]), reach=reach, self_window=int(d["self_window"]),
                                      self_min=int(d["self_min"]))
        assert np.array_equal(ud, d["use_draft"][t]), t
        assert np.array_equal(start, d["start"][t]), t
        assert np.array_equal(prop, d["prop"][t][:, :k]), t
    assert K().read_status(torch.device(DEVICE)) == 0


def draw(rng, b=8, cap=1024, vocab=5):
    out = rng.integers(3, vocab, (b, cap)).astype(np.int32)
    first = rng.integers(0, 300, b)
    last = first + rng.integers(0, cap - 300, b)
    last[0] = first[0]
    out[np.arange(cap)[None, :] < first[:, None]] = 1
    draft = rng.integers(3, vocab, (b, DRAFT_CAPACITY)).astype(np.int32)
    dlen = rng.integers(0, DRAFT_CAPACITY + 1, b)
    dlen[1] = 0
    draft[np.arange(DRAFT_CAPACITY)[None, :] >= dlen[:, None]] = -1
    nxt = (rng.random(b) * (dlen + 8)).astype(np.int64)
    # Some rows repeat their own recent tokens (prompt lookup wins), some copy the draft (the draft wins).
    for r in range(2, b, 3):
        n = int(last[r] - first[r])
        if n > 40:
            out[r, last[r] - 20:last[r] + 1] = out[r, last[r] - 33:last[r] - 12]
    for r in range(4, b, 3):
        if dlen[r] > 50 and last[r] - first[r] > 10:
            a = int(min(nxt[r], dlen[r] - 1))
            n = min(9, a, int(last[r] - first[r]))
            draft[r, a - n:a] = out[r, last[r] - n + 1:last[r] + 1]
    return out, draft, dlen, last, first, nxt


@pytest.mark.parametrize("k", [1, 4, 7])
def test_propose_matches_oracle_random(k):
    rng = np.random.default_rng(70 + k)
    for trial in range(6):
        out, draft, dlen, last, first, nxt = draw(rng, vocab=4 + trial % 4)
        prop, ud, start = run_propose(out, draft, dlen, last, first, nxt, k)
        want = ospec.propose(out, draft, dlen, last, first, nxt, k, NGRAM, BEHIND, AHEAD, REACH, SELF_WINDOW,
                             SELF_MIN)
        assert np.array_equal(ud, want[1]), trial
        assert np.array_equal(start, want[2]), trial
        assert np.array_equal(prop, want[0]), trial


def test_propose_other_window_sizes():
    """Non-default search sizes (own window not a power of two: the next power of two is searched, as the
    reference's launch does)."""
    rng = np.random.default_rng(5)
    out, draft, dlen, last, first, nxt = draw(rng, vocab=4)
    kw = dict(ngram=5, behind=17, ahead=40, reach=((0, 1), (3, 2), (9, 3), (20, 4)), self_window=100, self_min=2)
    prop, ud, start = run_propose(out, draft, dlen, last, first, nxt, 3, **kw)
    want = ospec.propose(out, draft, dlen, last, first, nxt, 3, kw["ngram"], kw["behind"], kw["ahead"], kw["reach"],
                         kw["self_window"], kw["self_min"])
    assert np.array_equal(prop, want[0]) and np.array_equal(ud, want[1]) and np.array_equal(start, want[2])


def test_propose_out_of_range_row_is_flagged():
    rng = np.random.default_rng(6)
    out, draft, dlen, last, first, nxt = draw(rng, b=3, cap=512)
    last[2] = 600  # past the token buffer
    K().read_status(torch.device(DEVICE))
    prop, ud, start = run_propose(out, draft, dlen, last, first, nxt, 2)
    assert K().read_status(torch.device(DEVICE)) & 1
    assert ud[2] and start[2] == nxt[2] and (prop[2] == 0).all()
    want = ospec.propose(out[:2], draft[:2], dlen[:2], last[:2], first[:2], nxt[:2], 2, NGRAM, BEHIND, AHEAD, REACH,
                         SELF_WINDOW, SELF_MIN)
    assert np.array_equal(prop[:2], want[0])


@pytest.mark.parametrize("width", [1, 5, 9])
def test_accept_matches_oracle(width):
    rng = np.random.default_rng(80 + width)
    b, cap, eos, limit = 64, 300, 2, 260
    tokens = rng.integers(3, 6, (b, width)).astype(np.int64)
    nxt = rng.integers(3, 6, (b, width)).astype(np.int64)
    for r in range(b):  # leading runs of matches of every length
        n = r % (width + 1)
        nxt[r, :max(0, n - 1)] = tokens[r, 1:n]
    nxt[5::11, min(1, width - 1)] = eos
    last = rng.integers(200, 270, b).astype(np.int64)  # some past the limit
    out = rng.integers(3, 9, (b, cap)).astype(np.int32)
    tok = rng.integers(3, 9, b).astype(np.int64)
    done = rng.random(b) < 0.15
    draft_next = rng.integers(0, 50, b).astype(np.int64)
    start = rng.integers(0, 50, b).astype(np.int64)
    use_draft = rng.random(b) < 0.5
    d = torch.device(DEVICE)
    tt = lambda a: torch.as_tensor(a.copy(), device=d)  # noqa: E731
    g = [tt(x) for x in (out, tok, last, done, draft_next)]
    K().accept(tt(tokens), tt(nxt), g[0], g[1], g[2], g[3], g[4], tt(start), tt(use_draft), limit, eos)
    torch.cuda.synchronize()
    w = [x.copy() for x in (out, tok, last, done, draft_next)]
    ospec.accept(tokens, nxt, w[0], w[1], w[2], w[3], w[4], start, use_draft, limit, eos)
    for got, want, name in zip(g, w, ("out", "tok", "last", "done", "draft_next")):
        assert np.array_equal(got.cpu().numpy(), want), name
    assert K().read_status(d) == 0


def test_accept_matches_reference_golden(golden):
    """Against the reference's own Triton _accept (kernels.py:271-291), recorded on a GPU by
    tests/golden/make_accept_golden.py: every state field bit-exact, widths 1, 2, 5 and 9."""
    d = golden("accept")
    dev = torch.device(DEVICE)
    tt = lambda a: torch.as_tensor(a.copy(), device=dev)  # noqa: E731
    for width in d["widths"]:
        p = f"w{int(width)}_"
        g = [tt(d[p + k]) for k in ("out", "tok", "last", "done", "draft_next")]
        K().accept(tt(d[p + "tokens"]), tt(d[p + "nxt"]), *g, tt(d[p + "start"]), tt(d[p + "use_draft"]),
                   int(d["limit"]), int(d["eos"]))
        torch.cuda.synchronize()
        for got, k in zip(g, ("out", "tok", "last", "done", "draft_next")):
            assert np.array_equal(got.cpu().numpy(), d[p + k + "_after"]), f"width {int(width)}: {k}"
    assert K().read_status(dev) == 0
