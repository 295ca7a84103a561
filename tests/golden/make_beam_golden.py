"""Golden vectors of beam search's selection step, produced by the reference's own BeamDecoder.

    python tests/golden/make_beam_golden.py --out tests/golden/beam_select.npz

The reference states the selection only inline, as the tail of ``BeamDecoder.step_beam`` (omniasr_trt/beam.py:
161-187: candidates, per-group ``topk``, parents, the pointer / history reorder and the state updates). This script
runs the reference's BeamDecoder unmodified (its PyTorch path, ``fused=False``, on the CPU) on the small random model
of the reference's own tests (tests/test_decode.py:17-28, float32) with and without length normalisation, and records
at every step the state right before the tail (captured when the step calls ``F.log_softmax``: the log-probabilities,
score, ended, count, tok, hist, ptr, k_step, ctx, gdone) and the state right after the step. ``tests/test_oracle.py``
pins the numpy restatement (``oracle/beam.py``) to these vectors and ``tests/test_beam_select_gpu.py`` the CUDA kernel.

torch.topk on the CPU orders equal values in no fixed way, so steps whose selection has a tie at the boundary or
inside the chosen candidates are left out (the script counts them).
"""

from __future__ import annotations

import argparse
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
KEEP = 96
FIELDS = ("score", "ended", "count", "tok", "hist", "ptr", "k_step", "ctx", "gdone")


def small_model(modeling, torch, seed: int, vocab: int = 12):
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
    return m.float()


def main():
    p = argparse.ArgumentParser()
    p.add_argument("--out", default=str(HERE / "beam_select.npz"))
    p.add_argument("--reference", default=str(ROOT / "baseline" / "_ref"), help="directory holding omniasr_trt")
    args = p.parse_args()
    sys.path.insert(0, args.reference)
    import torch
    import torch.nn.functional as tF
    from omniasr_trt import beam, modeling

    records = []
    skipped = 0

    class Recorder:
        """``torch.nn.functional`` as beam.py sees it; log_softmax also snapshots the decoder's state."""

        def __init__(self):
            self.dec = None
            self.pending = None

        def __getattr__(self, name):
            return getattr(tF, name)

        def log_softmax(self, x, dim=-1, **kw):
            out = tF.log_softmax(x, dim=dim, **kw)
            d = self.dec
            r = out.size(0)
            s = r // d.beams
            before = {"score": d.score[:r], "ended": d.ended[:r], "count": d.count[:r], "tok": d.tok[:r],
                      "hist": d.hist[:r], "ptr": d.ptr[:r], "k_step": d.k_step[:s], "ctx": d.ctx[:s],
                      "gdone": d.gdone[:s]}
            self.pending = (out.detach().clone(), {k: v.clone() for k, v in before.items()}, r, s)
            return out

    rec = Recorder()
    beam.F = rec
    step = beam.BeamDecoder.step_beam

    def recorded_step(self, s, ckeys, gkeys):
        nonlocal skipped
        step(self, s, ckeys, gkeys)
        logp, before, r, s2 = rec.pending
        after = {"score": self.score[:r], "ended": self.ended[:r], "count": self.count[:r], "tok": self.tok[:r],
                 "hist": self.hist[:r], "ptr": self.ptr[:r], "k_step": self.k_step[:s2], "ctx": self.ctx[:s2],
                 "gdone": self.gdone[:s2]}
        # ties at or inside the selection make the CPU's topk order arbitrary: leave those steps out
        from oracle.beam import candidates
        cand = candidates(logp.numpy(), before["score"].numpy(), before["ended"].numpy(), before["count"].numpy(),
                          self.beams, self.length_norm, 2)
        flat = cand.reshape(s2, -1)
        for g in range(s2):
            if bool(before["gdone"][g]):
                continue
            kth = np.sort(flat[g])[::-1][: self.beams + 1]
            if len(np.unique(kth)) < len(kth):
                skipped += 1
                return
        records.append((logp.numpy(), {k: v.numpy() for k, v in before.items()},
                        {k: v.clone().numpy() for k, v in after.items()}, self.beams, int(self.length_norm)))

    beam.BeamDecoder.step_beam = recorded_step
    sys.path.insert(0, str(ROOT))
    for case, (beams, length_norm, seed) in enumerate(((3, False, 16), (5, True, 21), (4, True, 5))):
        m = small_model(modeling, torch, seed)
        m.rope = modeling.rope_table(m.dec_cfg, "cpu")
        dec = beam.BeamDecoder(m, beams=beams, length_norm=length_norm, max_batch=3, sync_every=4, fused=False,
                               graphs=False, reserve=8)
        rec.dec = dec
        g = torch.Generator().manual_seed(100 + case)
        for lengths in ((25, 40, 5), (30, 8), (60, 12, 9)):
            ctxs = [torch.randn(k, 32, generator=g) for k in lengths]
            dec.generate(ctxs)
    beam.BeamDecoder.step_beam = step
    beam.F = tF

    stride = max(1, len(records) // KEEP)  # an even sample of the steps, to keep the file small
    kept = records[::stride][:KEEP]
    out = {"n": np.array(len(kept))}
    for i, (logp, before, after, beams, ln) in enumerate(kept):
        out[f"{i}_logp"] = logp
        out[f"{i}_meta"] = np.array([beams, ln])
        for k in FIELDS:
            out[f"{i}_in_{k}"] = before[k]
            out[f"{i}_out_{k}"] = after[k]
    np.savez_compressed(args.out, **out)
    print(f"{len(records)} steps recorded, {skipped} left out for ties, {len(kept)} kept; -> {args.out}")


if __name__ == "__main__":
    main()
