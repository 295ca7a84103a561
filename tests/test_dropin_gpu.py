"""The reference's own decoders running on these kernels (drop-in), against the reference's own PyTorch paths.

The reference package (Wataru-Nakata/omniasr-trt, pure Python) is imported from ``baseline/_ref`` where it is
installed next to this repository; ``omniasr_b200.dropin.install()`` swaps its ``omniasr_trt.kernels``. These
restate the reference's CUDA integration tests (tests/test_kernels.py:58-95, :129-150; tests/test_spec.py:111-198)
with the same small random model (tests/test_decode.py:17-28): token sequences must be identical to the unfused
PyTorch step, to the greedy search and to the reference-order loops, and LLMTranscriber.transcribe must give the
reference-order transcripts.
"""

import sys

import pytest
import torch

from conftest import ROOT

REF = ROOT / "baseline" / "_ref"
pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU"),
]


@pytest.fixture(scope="module")
def ref():
    # The reference package is the host these tests drive; build() places it in baseline/_ref. Missing, the tests
    # fail: a drop-in check that silently skips proves nothing.
    if not (REF / "omniasr_trt" / "decode.py").exists():
        pytest.fail(f"the reference package is missing from {REF} (run __graft_entry__.build() where the reference "
                    "checkout is present)")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from omniasr_b200 import dropin
    from omniasr_b200 import kernels as ours

    k = dropin.install()
    from omniasr_trt import beam, decode, llm, modeling, spec

    assert decode.kernels is k and spec.kernels is k and beam.kernels is k
    assert k.rope_kv is ours.rope_kv and k.decode_attention is ours.decode_attention
    assert k.propose is ours.propose and k.accept is ours.accept  # no reference Triton kernel left on the path
    assert isinstance(decode.F, dropin._Functional)  # the prefill's causal SDPA runs prefill_attention
    return {"decode": decode, "spec": spec, "beam": beam, "llm": llm, "modeling": modeling, "kernels": k}


class FakeTokenizer:
    def decode(self, ids):
        return " ".join(map(str, ids))


def small_model(modeling, seed=0, vocab=12):
    """The reference tests' tiny random model (tests/test_decode.py:17-28), fp32 on the GPU."""
    torch.manual_seed(seed)
    enc = modeling.EncoderConfig(model_dim=16, num_layers=2, num_heads=2, ffn_dim=32, feature_dim=8,
                                 conv_layers=((8, 10, 5), (8, 3, 2), (8, 2, 2)), pos_kernel=4, pos_groups=2)
    dec = modeling.DecoderConfig(model_dim=32, num_layers=2, num_heads=2, ffn_dim=24, vocab_size=vocab, num_langs=5,
                                 max_seq_len=8192)
    m = modeling.LLMModel(enc, dec).double().eval()
    with torch.no_grad():
        for p in m.parameters():
            p.normal_(0, 0.5)
        m.final_proj.weight.mul_(4)
    m = m.float().cuda()
    m.rope = modeling.rope_table(m.dec_cfg, "cuda")
    return m


def test_fused_greedy_decoder_matches_torch_path(ref):
    """Fused step (rope_kv + decode_attention, CUDA graphs) against the unfused PyTorch step; both prefill through
    prefill_attention, which the reference-order loops of the other tests pin against PyTorch."""
    m = small_model(ref["modeling"], seed=2)
    torch.manual_seed(3)
    ctxs = [torch.randn(n, 32, device="cuda") for n in (5, 33, 17, 60)]
    dec = ref["decode"].GreedyDecoder
    a = dec(m, max_batch=4, sync_every=8, fused=False, graphs=False, reserve=64).generate(ctxs)
    fast = dec(m, max_batch=4, sync_every=8, fused=True, graphs=True, reserve=64)
    assert fast.fused
    assert fast.generate(ctxs) == a


def test_fused_streams_across_calls(ref):
    m = small_model(ref["modeling"], seed=7)
    t = ref["llm"].LLMTranscriber(m, FakeTokenizer(), max_batch=3)
    dec = ref["decode"].GreedyDecoder(m, max_batch=3, sync_every=4, fused=True, graphs=True, reserve=8)
    torch.manual_seed(8)
    for n, lengths in ((7, (250, 40, 5, 251, 90, 12, 248)), (2, (30, 8)), (5, (60, 252, 9, 33, 100)), (1, (17,))):
        ctxs = [torch.randn(k, 32, device="cuda") for k in lengths[:n]]
        assert dec.generate(ctxs) == [t.greedy_reference(c) for c in ctxs], (n, lengths)
        torch.cuda.synchronize()


@pytest.mark.parametrize("beams,length_norm", [(3, False), (5, True)])
def test_fused_beam_decoder(ref, beams, length_norm):
    m = small_model(ref["modeling"], seed=16)
    t = ref["llm"].LLMTranscriber(m, FakeTokenizer())
    dec = ref["beam"].BeamDecoder(m, beams=beams, length_norm=length_norm, max_batch=3, sync_every=4, fused=True,
                                  graphs=True, reserve=8)
    torch.manual_seed(17)
    for lengths in ((250, 40, 5, 251, 90), (30, 8), (60, 252, 9, 33)):
        ctxs = [torch.randn(k, 32, device="cuda") for k in lengths]
        assert dec.generate(ctxs) == [t.beam_reference(c, beams, length_norm) for c in ctxs], lengths
        torch.cuda.synchronize()


def test_speculative_decoder_same_tokens_as_greedy(ref):
    """Drafted steps (draft_attention for 1 + 4 queries per row) give the greedy search's tokens."""
    m = small_model(ref["modeling"], seed=21)
    t = ref["llm"].LLMTranscriber(m, FakeTokenizer())
    torch.manual_seed(22)
    ctxs = [torch.randn(n, 32, device="cuda") for n in (40, 7, 251, 90, 13, 60)]
    want = [t.greedy_reference(c) for c in ctxs]
    dec = ref["spec"].SpecDecoder(m, draft_tokens=4, max_batch=4, sync_every=3, reserve=8)
    dec.drafts = lambda j: (want[j] + [5, 6, 7], 0)  # perfect drafts: several tokens per step
    assert dec.generate(ctxs) == want
    assert dec.stats["tokens"] / dec.stats["rows_steps"] > 1.5


# --- speculative decoding on these kernels (propose / accept, RoPE + append, verify attention): whatever the drafts,
# the tokens are the greedy search's. The scenarios (model seeds, context lengths, random draws) are those of the
# reference's own tests/test_spec.py:111-198, which pin the same behaviour on its Triton kernels.

def _corrupt(tokens, rng, vocab=12):
    """A draft that drifts from the tokens: some replaced, some dropped, some doubled with a stray token, and five
    random tokens at the end."""
    out = []
    for tok in tokens:
        u = rng.random()
        if u < 0.1:
            out.append(int(rng.integers(3, vocab)))
        elif u < 0.15:
            pass
        elif u < 0.2:
            out.extend([tok, int(rng.integers(3, vocab))])
        else:
            out.append(tok)
    return out + [int(x) for x in rng.integers(3, vocab, 5)]


def _spec_run(dec, ctxs, drafts):
    dec.drafts = lambda j: drafts[j]
    return dec.generate(ctxs)


@pytest.mark.parametrize("draft_tokens", [1, 4, 8])
def test_speculative_decoder_any_draft(ref, draft_tokens):
    import numpy as np

    m = small_model(ref["modeling"], seed=21)
    t = ref["llm"].LLMTranscriber(m, FakeTokenizer())
    torch.manual_seed(22)
    ctxs = [torch.randn(n, 32, device="cuda") for n in (40, 7, 251, 90, 13, 60)]
    want = [t.greedy_reference(c) for c in ctxs]
    assert min(len(w) for w in want) >= 3
    rng = np.random.default_rng(0)
    dec = ref["spec"].SpecDecoder(m, draft_tokens=draft_tokens, max_batch=4, sync_every=3, reserve=8)
    assert _spec_run(dec, ctxs, [(w + [5, 6, 7], 0) for w in want]) == want  # right, and running on past EOS
    per_step = dec.stats["tokens"] / dec.stats["rows_steps"]
    assert _spec_run(dec, ctxs, [(_corrupt(w, rng), 0) for w in want]) == want
    assert _spec_run(dec, ctxs, [(_corrupt(w[3:], rng), 2) for w in want]) == want  # the draft starts later
    others = [[int(x) for x in rng.integers(3, 12, 30)] for _ in ctxs[2:]]
    assert _spec_run(dec, ctxs, [None, ([], 0)] + [(o, 0) for o in others]) == want  # none, empty, unrelated
    if draft_tokens > 1:
        assert per_step > 1.5  # right drafts: several tokens per step


def test_speculative_decoder_eos_and_limit_inside_a_step(ref, monkeypatch):
    """Rows that reach EOS or the position limit in the middle of a drafted step stop there, as the greedy search."""
    m = small_model(ref["modeling"], seed=23)
    with torch.no_grad():
        m.final_proj.weight[ref["llm"].EOS] *= 0.3  # long generations
    monkeypatch.setattr(ref["decode"], "LIMIT", 70)
    monkeypatch.setattr(ref["spec"], "LIMIT", 70)
    torch.manual_seed(24)
    ctxs = [torch.randn(n, 32, device="cuda") for n in (5, 30, 64, 69, 12)]
    want = ref["decode"].GreedyDecoder(m, max_batch=3, sync_every=4, reserve=8).generate(ctxs)
    dec = ref["spec"].SpecDecoder(m, draft_tokens=6, max_batch=3, sync_every=4, reserve=8)
    assert _spec_run(dec, ctxs, [(w + [4] * 20, 0) for w in want]) == want


def test_speculative_decoder_repetition_stop(ref):
    """Without EOS a row ends by the repetition stop, and the cache grows meanwhile."""
    import numpy as np

    m = small_model(ref["modeling"], seed=15)
    with torch.no_grad():
        m.final_proj.weight[ref["llm"].EOS] = 0.0
    t = ref["llm"].LLMTranscriber(m, FakeTokenizer())
    torch.manual_seed(25)
    ctxs = [torch.randn(n, 32, device="cuda") for n in (5, 60, 140, 151)]
    want = [t.greedy_reference(c) for c in ctxs]
    rng = np.random.default_rng(3)
    dec = ref["spec"].SpecDecoder(m, draft_tokens=4, max_batch=3, sync_every=5, reserve=8)
    dec.context_floor = 0
    assert _spec_run(dec, ctxs, [(_corrupt(w, rng), 0) for w in want]) == want
    assert dec.stats["grows"] >= 1


def test_speculative_decoder_own_tokens(ref):
    """No draft: the proposals come from the row's own repeating tokens (several tokens per step)."""
    m = small_model(ref["modeling"], seed=15)
    with torch.no_grad():
        m.final_proj.weight[ref["llm"].EOS] = 0.0
    t = ref["llm"].LLMTranscriber(m, FakeTokenizer())
    torch.manual_seed(26)
    ctxs = [torch.randn(n, 32, device="cuda") for n in (5, 60, 99)]
    want = [t.greedy_reference(c) for c in ctxs]
    dec = ref["spec"].SpecDecoder(m, draft_tokens=4, max_batch=3, sync_every=5, reserve=8)
    assert _spec_run(dec, ctxs, [None] * len(ctxs)) == want
    assert dec.stats["tokens"] / dec.stats["rows_steps"] > 1.5


def test_transcriber_on_these_kernels(ref):
    """LLMTranscriber.transcribe end to end (segmentation, context building, prefill, decoding) with frame drafts,
    partial drafts, own tokens and one token per step gives the reference-order transcripts."""
    import numpy as np

    llm = ref["llm"]
    m = small_model(ref["modeling"], seed=3)
    t = llm.LLMTranscriber(m, FakeTokenizer(), max_batch=3)
    rng = np.random.default_rng(0)
    old = llm.SEGMENT
    llm.SEGMENT = 2000
    try:
        waves = [rng.standard_normal(n).astype(np.float32) for n in (5000, 2000, 900)]
        langs = ["aae_Latn", None, "AAL_latn"]
        want = t.transcribe(waves, langs, mode="reference")
        frames = [rng.integers(0, 12, n // 320) for n in (5000, 2000, 900)]
        assert t.transcribe(waves, langs, drafts=frames) == want
        assert t.transcribe(waves, langs, drafts=[None, frames[1], None]) == want
        assert t.transcribe(waves, langs) == want
        t.draft_tokens = 0  # one token per step
        assert t.transcribe(waves, langs) == want
    finally:
        llm.SEGMENT = old


def test_public_api_on_these_kernels(ref):
    """The reference's public surface on these kernels: OmniASRLLM.transcribe and compat.Pipeline.transcribe (the
    omnilingual-asr look-alike: dict inputs, 16 kHz, greedy or beam search by its config) give the reference-order
    transcripts."""
    import numpy as np

    llm = ref["llm"]
    import omniasr_trt
    from omniasr_trt import compat

    m = small_model(ref["modeling"], seed=40)
    t = llm.LLMTranscriber(m, FakeTokenizer(), max_batch=2)
    rng = np.random.default_rng(41)
    old = llm.SEGMENT
    llm.SEGMENT = 2000
    try:
        waves = [rng.standard_normal(n).astype(np.float32) for n in (4100, 900, 2600)]
        langs = [None, "aae_Latn", None]
        greedy = t.transcribe(waves, langs, mode="reference")
        beam3 = t.transcribe(waves, langs, mode="reference", beams=3)
        model = omniasr_trt.OmniASRLLM(t)
        assert model.transcribe(waves, langs) == greedy
        inputs = [{"waveform": w, "sample_rate": 16000} for w in waves]
        assert compat.Pipeline(model).transcribe(inputs, lang=langs) == greedy
        assert compat.Pipeline(model, {"nbest": 3}).transcribe(inputs, lang=langs) == beam3
    finally:
        llm.SEGMENT = old


def sharded_gpu_factory(rank, device):
    """A launcher worker: the drop-in installed in its own process, the reference's SpecDecoder on ``device``."""
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from omniasr_b200 import dropin

    dropin.install()
    from omniasr_trt import modeling, spec

    m = small_model(modeling, seed=21)
    dec = spec.SpecDecoder(m, draft_tokens=4, max_batch=4, sync_every=3, reserve=8)
    return lambda shard: dec.generate([c.to(device) for c in shard])


def test_sharded_launcher_on_the_gpus(ref):
    """omniasr_b200.launch.run_sharded over every visible GPU (one worker process each, these kernels dropped in)
    gives the reference-order greedy tokens, in request order."""
    from omniasr_b200 import launch

    m = small_model(ref["modeling"], seed=21)
    t = ref["llm"].LLMTranscriber(m, FakeTokenizer())
    torch.manual_seed(22)
    ctxs = [torch.randn(n, 32) for n in (40, 7, 251, 90, 13, 60)]
    want = [t.greedy_reference(c.cuda()) for c in ctxs]
    world = min(launch.visible_gpus(), len(ctxs))
    got = launch.run_sharded(sharded_gpu_factory, ctxs, world, device_type="cuda",
                             backend="nccl" if world > 1 else None, timeout_s=600)
    assert got == want
