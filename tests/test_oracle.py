"""The CPU oracle against the golden vectors produced by the reference's own code (tests/golden/make_golden.py)."""

import numpy as np
import pytest
import torch

import inputs as gi
from conftest import GOLDEN
from oracle import attention, bf16, gather, rope, splits


def test_bf16_conversion_matches_torch():
    rng = np.random.default_rng(0)
    x = np.concatenate([rng.standard_normal(100000, dtype=np.float32) * 10.0 ** rng.integers(-30, 30, 100000),
                        np.array([0.0, -0.0, np.inf, -np.inf, 1e-45, 3.3895314e38, 65504.0], dtype=np.float32)])
    x = x.astype(np.float32)
    want = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)
    assert np.array_equal(bf16.from_float32(x), want)
    ties = (np.arange(1000, dtype=np.uint32) << 16 | 0x8000).view(np.float32)  # exact halfway cases
    want = torch.from_numpy(ties).to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)
    assert np.array_equal(bf16.from_float32(ties), want)
    nan = np.array([np.nan], dtype=np.float32)
    assert np.isnan(bf16.to_float32(bf16.from_float32(nan)))[0]


@pytest.mark.parametrize("name", ["rope_bf16_h4_d128", "rope_f32_h4_d128", "rope_bf16_h2_d512", "rope_f32_h2_d16"])
def test_rope_oracle_bit_exact(golden, name):
    g = golden(name)
    is_bf16 = bool(g["is_bf16"])
    h, d = int(g["heads"]), g["qkv"].shape[1] // (3 * int(g["heads"]))
    dt = np.uint16 if is_bf16 else np.float32
    for slots, cpos in ((None, None), (g["slots"], None), (g["slots"], g["cache_pos"])):
        kc = np.zeros((int(g["rows"]), h, int(g["cache_len"]), d), dtype=dt)
        vc = np.zeros_like(kc)
        q = rope.rope_kv(g["qkv"], g["cs"], g["pos"], kc, vc, h, slots, cpos, is_bf16)
        assert np.array_equal(q.view(np.uint32 if not is_bf16 else np.uint16),
                              g["q"].view(np.uint32 if not is_bf16 else np.uint16))
        rows = np.arange(len(g["pos"])) if slots is None else slots
        at = g["pos"] if cpos is None else cpos
        assert np.array_equal(kc[rows, :, at], g["k"])
        assert np.array_equal(vc[rows, :, at], g["v"])


def test_gather_oracle(golden):
    g = golden("gather")
    assert np.array_equal(gather.reorder_gather(g["ptr"], g["parent"]), g["ptr_out"])
    assert np.array_equal(gather.reorder_gather(g["hist"], g["parent"]), g["hist_out"])
    assert np.array_equal(gather.reorder_gather(g["kv"], g["parent"]), g["kv_out"])
    with pytest.raises(IndexError):
        gather.reorder_gather(g["ptr"], np.array([0, 6]))


def test_splits_oracle(golden):
    for rows, heads, keys, block, programs, s, c in golden("splits")["cases"]:
        assert splits.splits_for(int(rows), int(heads), int(keys), int(block), int(programs)) == (s, c)


def _t(a, is_bf16):
    return torch.from_numpy(gi.values(a, is_bf16))


@pytest.mark.parametrize("is_bf16", [True, False])
def test_decode_oracle(golden, is_bf16):
    g = golden("decode_bf16" if is_bf16 else "decode_f32")
    q, k, v, lengths = gi.decode_inputs(is_bf16)
    assert gi.digest(q, k, v, lengths) == str(g["digest"])
    out = attention.decode_attention(_t(q, is_bf16), _t(k, is_bf16), _t(v, is_bf16), torch.from_numpy(lengths),
                                     float(g["scale"]))
    np.testing.assert_allclose(out.numpy(), g["out"], atol=1e-12, rtol=0)


@pytest.mark.parametrize("is_bf16", [True, False])
def test_draft_oracle(golden, is_bf16):
    g = golden("draft_bf16" if is_bf16 else "draft_f32")
    q, k, v, lengths = gi.draft_inputs(is_bf16)
    assert gi.digest(q, k, v, lengths) == str(g["digest"])
    out = attention.draft_attention(_t(q, is_bf16), _t(k, is_bf16), _t(v, is_bf16), torch.from_numpy(lengths),
                                    gi.DRAFT["t"], float(g["scale"]))
    np.testing.assert_allclose(out.numpy(), g["out"], atol=1e-12, rtol=0)


@pytest.mark.parametrize("is_bf16", [True, False])
def test_beam_oracle(golden, is_bf16):
    g = golden("beam_bf16" if is_bf16 else "beam_f32")
    q, kc, vc, ctx_len, kg, vg, ptr, gen_len = gi.beam_inputs(is_bf16)
    assert gi.digest(q, kc, vc, ctx_len, kg, vg, ptr, gen_len) == str(g["digest"])
    out = attention.beam_attention(_t(q, is_bf16), _t(kc, is_bf16), _t(vc, is_bf16), torch.from_numpy(ctx_len),
                                   _t(kg, is_bf16), _t(vg, is_bf16), torch.from_numpy(ptr),
                                   torch.from_numpy(gen_len), gi.BEAM["beams"], float(g["scale"]))
    # The reference's branch computes its scores in float32 (beam.py:230 `.float()`), the oracle in float64.
    np.testing.assert_allclose(out.numpy(), g["out"], atol=2e-6, rtol=0)
    assert np.all(g["out"][-gi.BEAM["beams"]:] == 0)  # the finished input: no keys, zeros


def test_oracle_catches_a_planted_error(golden):
    """A wrong oracle (one key too many per row) must disagree with the reference's vectors."""
    g = golden("decode_f32")
    q, k, v, lengths = gi.decode_inputs(False)
    wrong = attention.decode_attention(_t(q, False), _t(k, False), _t(v, False), torch.from_numpy(lengths) + 1,
                                       float(g["scale"]))
    assert np.abs(wrong.numpy() - g["out"]).max() > 1e-3


def test_propose_oracle_matches_reference_golden():
    """The speculative proposal (oracle.spec.propose) against the reference's own PyTorch statement of it
    (tests/test_spec.py:43-92 of the reference), twelve trials of 8 rows with few symbols."""
    from oracle import spec as ospec

    d = np.load(GOLDEN / "propose.npz")
    reach = [tuple(int(x) for x in r) for r in d["reach"]]
    for t in range(len(d["k"])):
        k = int(d["k"][t])
        prop, use_draft, start = ospec.propose(d["out"][t], d["draft"][t], d["draft_len"][t], d["last"][t],
                                               d["first"][t], d["nxt"][t], k, int(d["ngram"]), int(d["behind"]),
                                               int(d["ahead"]), reach, int(d["self_window"]), int(d["self_min"]))
        assert np.array_equal(use_draft, d["use_draft"][t]), t
        assert np.array_equal(start, d["start"][t]), t
        assert np.array_equal(prop, d["prop"][t][:, :k]), t


def test_accept_oracle_rules():
    """oracle.spec.accept on hand-made rows: leading matches kept, EOS and the length limit end a row inside the
    step, finished rows untouched (the reference's _accept, kernels.py:264-291)."""
    from oracle import spec as ospec

    eos, limit = 2, 100
    tokens = np.array([[7, 5, 6, 9], [7, 5, 6, 9], [7, 5, 6, 9], [7, 5, 6, 9], [7, 5, 6, 9]], dtype=np.int64)
    nxt = np.array([[5, 6, 8, 4], [5, 2, 9, 4], [3, 6, 9, 4], [5, 6, 9, 4], [5, 6, 9, 4]], dtype=np.int64)
    out = np.full((5, 128), 1, dtype=np.int32)
    tok = np.zeros(5, dtype=np.int64)
    last = np.array([10, 10, 10, 97, 10], dtype=np.int64)
    done = np.array([False, False, False, False, True])
    draft_next = np.array([20, 20, 20, 20, 20], dtype=np.int64)
    start = np.array([30, 30, 30, 30, 30], dtype=np.int64)
    use_draft = np.array([True, False, True, True, True])
    ospec.accept(tokens, nxt, out, tok, last, done, draft_next, start, use_draft, limit, eos)
    # row 0: 5, 6 match the fed tokens, 8 does not -> argmax 0..2 kept
    assert list(out[0, 11:14]) == [5, 6, 8] and last[0] == 13 and tok[0] == 8 and not done[0]
    assert draft_next[0] == 30 + 3
    # row 1: EOS at argmax 1 (within the kept run) ends the row there
    assert list(out[1, 11:13]) == [5, 2] and last[1] == 12 and tok[1] == 2 and done[1] and draft_next[1] == 22
    # row 2: first argmax differs from the fed token: one token
    assert out[2, 11] == 3 and out[2, 12] == 1 and last[2] == 11 and draft_next[2] == 31
    # row 3: positions 98, 99 kept, 100 reaches the limit and ends the row
    assert list(out[3, 98:101]) == [5, 6, 9] and last[3] == 100 and done[3]
    # row 4: finished, untouched
    assert last[4] == 10 and (out[4] == 1).all() and draft_next[4] == 20


@pytest.mark.parametrize("name,is_bf16,case", [("prefill_bf16", True, gi.PREFILL), ("prefill_f32", False, gi.PREFILL),
                                               ("prefill_bf16_d512", True, gi.PREFILL_D512)])
def test_prefill_oracle(golden, name, is_bf16, case):
    """The causal prefill (oracle.attention.prefill_attention) against the reference's prefill call, SDPA with
    is_causal=True as decode.py:171 makes it (float64, stored as float32)."""
    g = golden(name)
    q, k, v = gi.prefill_inputs(is_bf16, case)
    assert gi.digest(q, k, v) == str(g["digest"])
    out = attention.prefill_attention(_t(q, is_bf16), _t(k, is_bf16), _t(v, is_bf16))
    np.testing.assert_allclose(out.numpy(), g["out"], atol=2e-6, rtol=1e-6)
    wrong = attention.prefill_attention(_t(q, is_bf16), _t(k, is_bf16), _t(v, is_bf16).roll(1, dims=2))
    assert np.abs(wrong.numpy() - g["out"]).max() > 1e-2  # a planted error (values shifted by one key) shows


def test_accept_oracle_matches_reference_golden():
    """The acceptance rule (oracle.spec.accept) against the reference's own Triton kernel (_accept,
    kernels.py:271-291), whose outputs tests/golden/make_accept_golden.py recorded on a GPU."""
    from oracle import spec as ospec

    path = GOLDEN / "accept.npz"
    if not path.exists():
        pytest.fail("tests/golden/accept.npz is missing: run tests/golden/make_accept_golden.py on a GPU")
    d = np.load(path)
    for width in d["widths"]:
        p = f"w{int(width)}_"
        state = [d[p + k].copy() for k in ("out", "tok", "last", "done", "draft_next")]
        ospec.accept(d[p + "tokens"], d[p + "nxt"], *state, d[p + "start"], d[p + "use_draft"], int(d["limit"]),
                     int(d["eos"]))
        for got, k in zip(state, ("out", "tok", "last", "done", "draft_next")):
            assert np.array_equal(got, d[p + k + "_after"]), f"width {int(width)}: {k}"
        assert not np.array_equal(d[p + "last"], d[p + "last_after"])  # the step advanced some rows


BEAM_FIELDS = ("score", "ended", "count", "tok", "hist", "ptr", "k_step", "ctx", "gdone")


def _beam_record(z, i):
    beams, ln = (int(v) for v in z[f"{i}_meta"])
    state = {k: z[f"{i}_in_{k}"].copy() for k in BEAM_FIELDS}
    want = {k: z[f"{i}_out_{k}"] for k in BEAM_FIELDS}
    return z[f"{i}_logp"], state, want, beams, bool(ln)


def test_beam_select_oracle_matches_reference_golden():
    """The selection tail of the reference's BeamDecoder.step_beam (beam.py:161-187), recorded step by step from
    its own PyTorch path (tests/golden/make_beam_golden.py): the numpy restatement gives every state field exactly."""
    from oracle import beam

    z = np.load(GOLDEN / "beam_select.npz")
    n = int(z["n"])
    assert n >= 90
    seen_ended = seen_done = seen_norm = 0
    for i in range(n):
        logp, st, want, beams, ln = _beam_record(z, i)
        seen_ended += bool(st["ended"].any())
        seen_done += bool(st["gdone"].any())
        seen_norm += ln
        beam.beam_select(logp, **st, beams=beams, length_norm=ln, eos=2, pad=1, limit=8188)
        for k in BEAM_FIELDS:
            assert np.array_equal(st[k], want[k]), (i, k)
    assert seen_ended and seen_done and seen_norm  # the golden covers ended rows, done groups, length_norm


def test_beam_select_oracle_tie_order():
    """Equal values in the order torch.topk(sorted=True) returns them on a CUDA tensor, which is how the reference's
    beam search selects (beam.py:171): recorded with torch on a GPU (tests/golden/make_topk_golden.py)."""
    from oracle import beam

    z = np.load(GOLDEN / "topk_ties.npz")
    for k in range(1, 33):
        assert np.array_equal(beam.topk_order(np.zeros(40, np.float32), k), z[f"eq_k{k}"]), k
    for i in range(int(z["n"])):
        codes = z[f"case{i}_x"]
        x = np.where(codes < 0, -np.inf, codes).astype(np.float32)
        want = z[f"case{i}_i"]
        assert np.array_equal(beam.topk_order(x, len(want)), want), i
