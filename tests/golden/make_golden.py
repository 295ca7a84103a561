"""Golden vectors of the decoder-attention path, produced by running the reference's own code on the CPU.

    python tests/golden/make_golden.py --reference <checkout of Wataru-Nakata/omniasr-trt>/src

Needs the reference package importable (pure Python + torch); writes ``tests/golden/*.npz``. The tests only read
those files, so they run where the reference is absent. Which reference code produced each file:

* ``rope_*.npz``     -- ``modeling.rope_table`` and ``modeling.apply_rope`` (modeling.py:293-306), the check of the
                        reference's own kernel test (tests/test_kernels.py:24-38), incl. scattered ``slots`` and
                        beam-style ``cache_pos``;
* ``gather.npz``     -- ``Tensor.index_select(0, parent)`` (llm.py:237-238) and ``ptr[parent]`` (beam.py:175-176);
* ``splits.npz``     -- ``kernels.splits_for`` (kernels.py:393-400);
* ``decode_*.npz``   -- ``F.scaled_dot_product_attention`` per row, the reference-order q_len-1 attention
                        (modeling.py:396-397), float64; rows of length 0 are zeros (kernels.py:8-9);
* ``draft_*.npz``    -- the ``tril(past)`` mask + SDPA of ``LLMModel.decoder_forward`` (modeling.py:400-403), float64;
* ``beam_*.npz``     -- ``BeamDecoder.attention`` on its PyTorch branch (beam.py:215-233), float64 model;
* ``prefill_*.npz``  -- the prefill's ``F.scaled_dot_product_attention(q, k, v, is_causal=True)`` exactly as
                        ``GreedyDecoder.prefill_into`` calls it (decode.py:171; reference-order form
                        modeling.py:398-399), float64 (stored as float32), at head_dim 128 (crossing a 128-position tile) and 512 (the
                        shipped model's heads);
* ``accept.npz``     -- not made here: the acceptance rule exists only as the reference's Triton kernel, so
                        ``make_accept_golden.py`` runs it on a GPU;
* ``propose.npz``    -- ``reference_propose``, the PyTorch statement of the speculative proposal that the
                        reference's own kernel test checks its Triton kernel against (tests/test_spec.py:43-92,
                        :206-228), on inputs drawn like that test's (few symbols: many partial matches and ties).
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np
import torch
import torch.nn.functional as F

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))  # the repo root: oracle.bf16 for the bf16 bit patterns
sys.path.insert(0, str(HERE))

import inputs as gi  # noqa: E402

from oracle import bf16  # noqa: E402


def tensor(a: np.ndarray, is_bf16: bool) -> torch.Tensor:
    """Raw numpy (uint16 bf16 bits / float32) -> torch tensor of the same values and dtype."""
    if is_bf16:
        return torch.from_numpy(a.astype(np.int16)).view(torch.bfloat16)
    return torch.from_numpy(a)


def bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.contiguous().view(torch.int16).numpy().astype(np.uint16)
    return t.contiguous().numpy()


def rope_case(name: str, h: int, d: int, positions: int, is_bf16: bool, seed: int):
    from omniasr_trt.modeling import DecoderConfig, apply_rope, rope_table

    rng = np.random.default_rng(seed)
    n, rows, s = 6, 8, positions
    cs = rope_table(DecoderConfig(model_dim=h * d, num_heads=h, max_seq_len=positions))  # [P, D/2, 2] fp32
    qkv = gi.normal(rng, (n, 3 * h * d), is_bf16)
    pos = np.array([0, 7, positions - 1, positions // 2, 31 % positions, 3], dtype=np.int64)
    slots = np.array([6, 0, 3, 5, 1, 7], dtype=np.int64)
    cache_pos = np.array([2, 0, 5, 1, 4, 3], dtype=np.int64)  # beam search: generated positions
    t = tensor(qkv, is_bf16).view(n, 3, h, d)
    rq, rk, rv = t.unbind(1)
    c = cs[torch.from_numpy(pos)][:, None]
    q = apply_rope(rq, c)
    k = apply_rope(rk, c)
    np.savez_compressed(HERE / f"{name}.npz", qkv=qkv, cs=cs.numpy(), pos=pos, slots=slots, cache_pos=cache_pos,
                        q=bits(q), k=bits(k), v=bits(rv), heads=h, rows=rows, cache_len=s, is_bf16=is_bf16)


def gather_case():
    rng = np.random.default_rng(21)
    ptr = rng.integers(0, 40, (6, 40)).astype(np.int32)  # beam pointers [R, G]
    hist = rng.integers(0, 12, (6, 41)).astype(np.int32)  # token history [R, G + 1]
    kv = bf16.from_float32(rng.standard_normal((6, 2, 16, 8), dtype=np.float32))  # a layer's K cache [R, H, S, D]
    parent = np.array([2, 2, 0, 5, 3, 3], dtype=np.int64)
    t_ptr, t_hist, t_kv = torch.from_numpy(ptr), torch.from_numpy(hist), tensor(kv, True)
    p = torch.from_numpy(parent)
    np.savez_compressed(HERE / "gather.npz", ptr=ptr, hist=hist, kv=kv, parent=parent, ptr_out=t_ptr[p].numpy(),
                        hist_out=t_hist[p].numpy(), kv_out=bits(t_kv.index_select(0, p)))


def splits_case():
    from omniasr_trt import kernels

    cases = []
    for rows in (1, 3, 8, 16, 40):
        for heads in (8, 32):
            for keys in (0, 64, 256, 1024, 2048, 4096, 8192):
                for block, programs in ((64, 264), (32, 264), (16, 528)):
                    cases.append((rows, heads, keys, block, programs, *kernels.splits_for(rows, heads, keys, block,
                                                                                           programs)))
    np.savez_compressed(HERE / "splits.npz", cases=np.array(cases, dtype=np.int64))


def decode_case(is_bf16: bool):
    c = gi.DECODE
    q, k, v, lengths = gi.decode_inputs(is_bf16)
    qd, kd, vd = (torch.from_numpy(gi.values(a, is_bf16)) for a in (q, k, v))
    scale = c["d"] ** -0.5
    out = torch.zeros(c["b"], c["h"], c["d"], dtype=torch.float64)
    for r in range(c["b"]):
        n = int(lengths[r])
        if n == 0:
            continue  # a finished row reads nothing and gets zeros
        o = F.scaled_dot_product_attention(qd[r : r + 1, :, None], kd[r : r + 1, :, :n], vd[r : r + 1, :, :n],
                                           scale=scale)
        out[r] = o[0, :, 0]
    tag = "bf16" if is_bf16 else "f32"
    np.savez_compressed(HERE / f"decode_{tag}.npz", out=out.numpy(), digest=gi.digest(q, k, v, lengths),
                        scale=scale)


def draft_case(is_bf16: bool):
    c = gi.DRAFT
    q, k, v, lengths = gi.draft_inputs(is_bf16)
    qd, kd, vd = (torch.from_numpy(gi.values(a, is_bf16)) for a in (q, k, v))
    t, h, d = c["t"], c["h"], c["d"]
    scale = d**-0.5
    out = torch.zeros(c["b"] * t, h, d, dtype=torch.float64)
    for r in range(c["b"]):
        past = int(lengths[r]) - 1  # keys before the block's first query (which sees its own key too)
        total = past + t
        qq = qd[r * t : (r + 1) * t].transpose(0, 1)[None]  # [1, H, T, D]
        mask = torch.ones(t, total, dtype=torch.bool).tril(past)  # modeling.py:402
        o = F.scaled_dot_product_attention(qq, kd[r : r + 1, :, :total], vd[r : r + 1, :, :total], attn_mask=mask,
                                           scale=scale)
        out[r * t : (r + 1) * t] = o[0].transpose(0, 1)
    tag = "bf16" if is_bf16 else "f32"
    np.savez_compressed(HERE / f"draft_{tag}.npz", out=out.numpy(), digest=gi.digest(q, k, v, lengths), scale=scale)


def beam_case(is_bf16: bool):
    from omniasr_trt.beam import BeamDecoder
    from omniasr_trt.modeling import DecoderConfig, EncoderConfig, LLMModel

    c = gi.BEAM
    q, kc, vc, ctx_len, kg, vg, ptr, gen_len = gi.beam_inputs(is_bf16)
    h, d = c["h"], c["d"]
    enc = EncoderConfig(model_dim=16, num_layers=1, num_heads=2, ffn_dim=16, feature_dim=8,
                        conv_layers=((8, 10, 5),), pos_kernel=4, pos_groups=2)
    dec_cfg = DecoderConfig(model_dim=h * d, num_layers=1, num_heads=h, ffn_dim=16, vocab_size=12, num_langs=2,
                            max_seq_len=64)
    torch.manual_seed(0)
    model = LLMModel(enc, dec_cfg).double().eval()
    dec = BeamDecoder(model, beams=c["beams"], max_batch=c["groups"], graphs=False, fused=False)
    assert not dec.fused
    to = lambda a: torch.from_numpy(gi.values(a, is_bf16))  # noqa: E731
    dec.kc, dec.vc = to(kc)[None], to(vc)[None]
    dec.kg, dec.vg = to(kg)[None], to(vg)[None]
    dec.ptr = torch.from_numpy(ptr)
    with torch.inference_mode():
        out = dec.attention(0, to(q), torch.from_numpy(ctx_len), torch.from_numpy(gen_len), c["groups"],
                            c["ctx_keys"], c["g"])
    tag = "bf16" if is_bf16 else "f32"
    np.savez_compressed(HERE / f"beam_{tag}.npz", out=out.numpy(), scale=d**-0.5,
                        digest=gi.digest(q, kc, vc, ctx_len, kg, vg, ptr, gen_len))


def prefill_case(name: str, is_bf16: bool, c: dict):
    from omniasr_trt import decode

    q, k, v = gi.prefill_inputs(is_bf16, c)
    qd, kd, vd = (torch.from_numpy(gi.values(a, is_bf16)) for a in (q, k, v))
    out = decode.F.scaled_dot_product_attention(qd, kd, vd, is_causal=True)  # decode.py:171, torch's SDPA
    np.savez_compressed(HERE / f"{name}.npz", out=out.numpy().astype(np.float32), digest=gi.digest(q, k, v),
                        scale=c["d"] ** -0.5)


def propose_case(ref_src: str):
    """Twelve trials of 8 rows (proposal lengths 1, 4 and 7), the reference's constants (spec.py:33-39)."""
    from types import SimpleNamespace

    tests_dir = str(Path(ref_src).resolve().parent / "tests")
    if tests_dir not in sys.path:
        sys.path.insert(0, tests_dir)
    import test_spec as ts  # the reference's test module: its reference_propose
    from omniasr_trt import spec

    rng = np.random.default_rng(40)
    b, cap, dcap = 8, 2048, spec.DRAFT_CAPACITY
    fields = {k: [] for k in ("k", "out", "draft", "draft_len", "last", "first", "nxt", "prop", "use_draft", "start")}
    for trial in range(12):
        k = (1, 4, 7)[trial % 3]
        vocab = 4 + trial % 5
        out = rng.integers(3, vocab, (b, cap)).astype(np.int32)
        first = rng.integers(0, 600, b)
        last = first + rng.integers(0, 1400, b)
        last[0] = first[0]
        out[np.arange(cap)[None, :] < first[:, None]] = 1  # PAD before the segment
        draft = rng.integers(3, vocab, (b, dcap)).astype(np.int32)
        dlen = rng.integers(0, dcap + 1, b)
        dlen[1] = 0
        draft[np.arange(dcap)[None, :] >= dlen[:, None]] = -1
        nxt = (rng.random(b) * (dlen + 8)).astype(np.int64)
        st = SimpleNamespace(device=torch.device("cpu"), draft_tokens=k, out=torch.from_numpy(out),
                             draft=torch.from_numpy(draft), draft_len=torch.from_numpy(dlen),
                             last=torch.from_numpy(last), first=torch.from_numpy(first), next=torch.from_numpy(nxt))
        prop, use_draft, start = ts.reference_propose(st, b)
        pad = np.zeros((b, 7), dtype=np.int64)
        pad[:, :k] = prop.numpy()
        for name, v in (("k", k), ("out", out), ("draft", draft), ("draft_len", dlen), ("last", last),
                        ("first", first), ("nxt", nxt), ("prop", pad), ("use_draft", use_draft.numpy()),
                        ("start", start.numpy())):
            fields[name].append(v)
    consts = dict(ngram=spec.NGRAM, behind=spec.BEHIND, ahead=spec.AHEAD, reach=np.array(spec.REACH),
                  self_window=spec.SELF_WINDOW, self_min=spec.SELF_MIN)
    np.savez_compressed(HERE / "propose.npz", **{k: np.stack(v) for k, v in fields.items()}, **consts)


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--reference", default="/root/reference/src", help="the reference's src/ directory")
    args = p.parse_args()
    sys.path.insert(0, args.reference)
    rope_case("rope_bf16_h4_d128", 4, 128, 64, True, 1)
    rope_case("rope_f32_h4_d128", 4, 128, 64, False, 2)
    rope_case("rope_bf16_h2_d512", 2, 512, 32, True, 3)
    rope_case("rope_f32_h2_d16", 2, 16, 40, False, 4)
    gather_case()
    splits_case()
    for is_bf16 in (True, False):
        decode_case(is_bf16)
        draft_case(is_bf16)
        beam_case(is_bf16)
    prefill_case("prefill_bf16", True, gi.PREFILL)
    prefill_case("prefill_f32", False, gi.PREFILL)
    prefill_case("prefill_bf16_d512", True, gi.PREFILL_D512)
    propose_case(args.reference)
    for f in sorted(HERE.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    main()
