"""Beam search's selection step (``kernels.beam_select``, csrc/beam.cu) on the GPU, bit-exact.

* Against the golden steps recorded from the reference's own BeamDecoder (tests/golden/make_beam_golden.py): every
  state field after the step, exactly.
* At BASELINE config 3's shape (8 inputs x 5 beams, vocabulary 10288, bf16 log-probabilities, the history and
  pointer rows of a long search) against the numpy oracle, with and without length normalisation, ended rows and
  finished groups; 1, 2, 7 and 16 beams; fp32 log-probabilities; ties planted at and inside the selection (the order
  torch.topk gives on a CUDA tensor: value descending, then index ascending -- checked against torch itself).
* A history position outside its row sets status bit 1 instead of writing.
"""

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import beam as obeam

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

FIELDS = ("score", "ended", "count", "tok", "hist", "ptr", "k_step", "ctx", "gdone")
EOS, PAD, LIMIT = 2, 1, 8188


@pytest.fixture(scope="module")
def K():
    from omniasr_b200 import kernels

    kernels.read_status()
    return kernels


def _run_kernel(K, logp: np.ndarray, st: dict, beams: int, ln: bool, logp_dtype=torch.float32) -> dict:
    dev = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in st.items()}
    lp = torch.from_numpy(logp).to(logp_dtype).cuda()
    K.beam_select(lp, dev["score"], dev["ended"], dev["count"], dev["tok"], dev["hist"], dev["ptr"], dev["k_step"],
                  dev["ctx"], dev["gdone"], beams, ln, EOS, PAD, LIMIT)
    return {k: v.cpu().numpy() for k, v in dev.items()}


def _oracle(logp: np.ndarray, st: dict, beams: int, ln: bool) -> dict:
    o = {k: v.copy() for k, v in st.items()}
    obeam.beam_select(logp.astype(np.float32), **o, beams=beams, length_norm=ln, eos=EOS, pad=PAD, limit=LIMIT)
    return o


def _same(got: dict, want: dict, what: str):
    for k in FIELDS:
        assert np.array_equal(got[k], want[k]), f"{what}: {k} differs"


def test_matches_reference_golden_steps(K):
    z = np.load(GOLDEN / "beam_select.npz")
    for i in range(int(z["n"])):
        beams, ln = (int(v) for v in z[f"{i}_meta"])
        st = {k: z[f"{i}_in_{k}"] for k in FIELDS}
        got = _run_kernel(K, z[f"{i}_logp"], st, beams, bool(ln))
        _same(got, {k: z[f"{i}_out_{k}"] for k in FIELDS}, f"golden step {i}")
    assert K.read_status() == 0


def _state(groups: int, beams: int, vocab: int, width: int, seed: int, ties: bool = False):
    """A search in progress: log-softmax rows of random logits (bf16-representable), scores of earlier steps, some
    ended rows, one finished group, token histories and pointers."""
    g = torch.Generator().manual_seed(seed)
    r = groups * beams
    logits = torch.randn(r, vocab, generator=g) * 3
    logp = torch.log_softmax(logits, -1).to(torch.bfloat16).float()
    if ties:  # copies of each row's best values: equal candidates at and inside the selection
        for b in range(r):
            top = logp[b].topk(beams + 1).values
            idx = torch.randperm(vocab, generator=g)[: 2 * beams]
            logp[b, idx[:beams]] = top[0]
            logp[b, idx[beams:]] = top[beams - 1]
    k = torch.randint(1, width - 2, (groups,), generator=g)
    st = {
        "score": (-torch.rand(r, generator=g) * 20).float().numpy(),
        "ended": (torch.rand(r, generator=g) < 0.2).numpy(),
        "count": torch.randint(0, 50, (r,), generator=g).numpy(),
        "tok": torch.randint(3, vocab, (r,), generator=g).numpy(),
        "hist": torch.randint(0, vocab, (r, width + 1), generator=g).to(torch.int32).numpy(),
        "ptr": (torch.arange(r)[:, None] // beams * beams + torch.randint(0, beams, (r, width), generator=g))
        .to(torch.int32).numpy(),
        "k_step": k.numpy(),
        "ctx": torch.randint(300, 1801, (groups,), generator=g).numpy(),
        "gdone": np.zeros(groups, dtype=bool),
    }
    if ties:  # equal scores within a group: equal candidates across beams too
        st["score"][:] = st["score"][(np.arange(r) // beams) * beams]
    st["gdone"][groups // 2] = True
    st["count"][0] = 0  # group 0: row 0 has counted nothing (length normalisation off for it)
    st["ended"][beams * (groups - 1): beams * groups] = True  # a group whose rows have all ended but is not done
    st["ended"][beams * (groups - 1)] = False
    return logp.numpy(), st


@pytest.mark.parametrize("length_norm", [False, True])
def test_config3_shape_bf16(K, length_norm):
    logp, st = _state(8, 5, 10288, 8192, seed=1 + length_norm)
    got = _run_kernel(K, logp, st, 5, length_norm, torch.bfloat16)
    _same(got, _oracle(logp, st, 5, length_norm), f"config 3 length_norm={length_norm}")
    assert K.read_status() == 0


@pytest.mark.parametrize("beams,vocab", [(1, 10288), (2, 517), (7, 10288), (16, 3001)])
def test_other_beam_counts_fp32(K, beams, vocab):
    logp, st = _state(5, beams, vocab, 300, seed=10 + beams)
    for ln in (False, True):
        got = _run_kernel(K, logp, st, beams, ln, torch.float32)
        _same(got, _oracle(logp, st, beams, ln), f"beams {beams} vocab {vocab} length_norm={ln}")
    assert K.read_status() == 0


def test_ties_follow_cuda_topk(K):
    """Planted ties: the kernel, the oracle and torch.topk on the GPU choose the same candidates in the same order."""
    beams, vocab, groups = 5, 10288, 8
    logp, st = _state(groups, beams, vocab, 256, seed=33, ties=True)
    for ln in (False, True):
        cand = obeam.candidates(logp, st["score"], st["ended"], st["count"], beams, ln, EOS)
        _, pick = torch.from_numpy(cand).cuda().view(groups, beams * vocab).topk(beams, dim=-1, sorted=True)
        pick = pick.cpu().numpy()
        for g in range(groups):
            assert np.array_equal(pick[g], obeam.topk_order(cand.reshape(groups, -1)[g], beams)), (ln, g)
        got = _run_kernel(K, logp, st, beams, ln, torch.bfloat16)
        _same(got, _oracle(logp, st, beams, ln), f"ties length_norm={ln}")
    assert K.read_status() == 0


def test_history_position_outside_row_sets_status(K):
    """The reference's scatter would fail on the device; the kernel skips that write and reports bit 1."""
    logp, st = _state(2, 3, 100, 40, seed=5)
    st["gdone"][:] = False
    st["k_step"][1] = 41  # the history rows have 41 columns: position 41 is outside
    got = _run_kernel(K, logp, st, 3, False)
    assert K.read_status() == 1
    _same(got, _oracle(logp, st, 3, False), "position outside the history")
