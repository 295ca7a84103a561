"""head_dim 512, the shipped model's geometry (8 heads x 512, the reference's modeling.py:30-35), on the tensor cores.

The BASELINE configs 1-3 at 8 x 512 instead of 32 x 128 (the same bytes per token), full size: a key tile is four
128-dim chunks streaming through the pass's ring, S^T accumulates over them and O^T has one accumulator per chunk;
units are split across many CTAs and merged in the pass (decode, draft) or in the combine (beam). Cache rows past each
row's keys hold NaN, so a V row the pass fails to zero would show. Against the float64 oracle: bf16 max-abs <= 2e-2,
mean-abs <= 2e-3.
"""

import pytest
import torch

from gpu_util import check_attention, randn
from oracle import attention as oatt

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

H, D = 8, 512


@pytest.fixture(scope="module")
def K():
    from omniasr_b200 import kernels

    kernels.read_status()
    return kernels


def _nan_tail(c: torch.Tensor, lengths) -> torch.Tensor:
    for r, n in enumerate(lengths):
        c[r, :, int(n):] = float("nan")
    return c


@pytest.mark.parametrize("tokens", [1, 5, 9])
def test_draft_d512_config2_shape(K, tokens):
    """Config 2 at 8 x 512: 8 rows, lengths U[200, 2000], capacity 4096 (T = 1 is the decode of config 1's form)."""
    b, cap = 8, 4096
    lengths = torch.randint(200, 2001, (b,), generator=torch.Generator().manual_seed(0))
    keys = int((lengths.max() + tokens + 255) // 256 * 256)
    kc = _nan_tail(randn((b, H, cap, D), torch.bfloat16, 500), lengths + tokens - 1)
    vc = _nan_tail(randn((b, H, cap, D), torch.bfloat16, 501), lengths + tokens - 1)
    q = randn((b * tokens, H, D), torch.bfloat16, 502)
    if tokens == 1:
        out = K.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), keys, D**-0.5)
    else:
        out = K.draft_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), tokens, keys, D**-0.5)
    assert not torch.isnan(out).any()
    kz, vz = kc.nan_to_num(0.0), vc.nan_to_num(0.0)
    want = oatt.draft_attention(q, kz, vz, lengths, tokens, D**-0.5)
    check_attention(out, want, torch.bfloat16, what=f"8x512 T={tokens}")
    assert K.read_status() == 0


def test_decode_d512_config1_shape(K):
    """Config 1 at 8 x 512: 8 rows of 1024 keys, every unit split across CTAs and merged in the pass."""
    b, L = 8, 1024
    kc = randn((b, H, L, D), torch.bfloat16, 510)
    vc = randn((b, H, L, D), torch.bfloat16, 511)
    q = randn((b, H, D), torch.bfloat16, 512)
    lengths = torch.full((b,), L)
    out = K.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), L, D**-0.5)
    check_attention(out, oatt.decode_attention(q, kc, vc, lengths, D**-0.5), torch.bfloat16, what="8x512 config 1")
    assert K.read_status() == 0


@pytest.mark.parametrize("beams", [3, 5])
def test_beam_d512_config3_shape(K, beams):
    """Config 3 at 8 x 512: 8 inputs, context U[300, 1800] shared by the beams, 32 generated keys per row through the
    pointers; the combine attends the generated keys and merges the pass's segments."""
    s, cap, gcap = 8, 2048, 32
    r = s * beams
    g = torch.Generator().manual_seed(520 + beams)
    ctx_len = torch.randint(300, 1801, (s,), generator=g)
    gen_len = torch.randint(0, gcap + 1, (r,), generator=g)
    kc = _nan_tail(randn((s, H, cap, D), torch.bfloat16, 521), ctx_len)
    vc = _nan_tail(randn((s, H, cap, D), torch.bfloat16, 522), ctx_len)
    kg = randn((r, H, gcap, D), torch.bfloat16, 523)
    vg = randn((r, H, gcap, D), torch.bfloat16, 524)
    q = randn((r, H, D), torch.bfloat16, 525)
    ptr = (torch.arange(r)[:, None] // beams * beams + torch.randint(0, beams, (r, gcap), generator=g)).to(torch.int32)
    ctx_keys = int((ctx_len.max() + 255) // 256 * 256)
    out = K.beam_attention(q.cuda(), kc.cuda(), vc.cuda(), ctx_len.cuda(), kg.cuda(), vg.cuda(), ptr.cuda(),
                           gen_len.cuda(), beams, ctx_keys, D**-0.5)
    assert not torch.isnan(out).any()
    want = oatt.beam_attention(q, kc.nan_to_num(0.0), vc.nan_to_num(0.0), ctx_len, kg, vg, ptr, gen_len, beams,
                               D**-0.5)
    check_attention(out, want, torch.bfloat16, what=f"8x512 beam {beams}")
    assert K.read_status() == 0


@pytest.mark.parametrize("path", ["wide", "grouped"])
@pytest.mark.parametrize("b,w", [(2, 70), (3, 129), (8, 1500)])
def test_prefill_d512(K, b, w, path):
    """The causal prefill at 8 x 512: the two-pass tensor-core prefill kernel (prefill_attention) and the decode pass
    in groups of 16 query positions (prefill_attention_grouped); ragged last tiles and groups, cache views longer
    than the width. Checked on every (row, head) at sampled positions; config 4's 8 x 1500 among the shapes."""
    cap = w + 37
    q = randn((b * w, H, D), torch.bfloat16, 530 + w).cuda().view(b, w, H, D).transpose(1, 2)
    kc = randn((b + 1, H, cap, D), torch.bfloat16, 531 + w).cuda()
    vc = randn((b + 1, H, cap, D), torch.bfloat16, 532 + w).cuda()
    k, v = kc[:b, :, :w], vc[:b, :, :w]
    out = (K.prefill_attention if path == "wide" else K.prefill_attention_grouped)(q, k, v)
    assert out.shape == (b, H, w, D)
    g = torch.Generator().manual_seed(533)
    pos = torch.cat([torch.tensor([0, 15, 16, w - 1]), torch.randint(0, w, (28,), generator=g)]).clamp(max=w - 1).unique()
    qc, kcc, vcc, oc = q.cpu(), k.cpu(), v.cpu(), out.cpu()
    for hh in range(H):
        want = oatt.prefill_attention_rows(qc[:, hh:hh + 1], kcc[:, hh:hh + 1], vcc[:, hh:hh + 1], pos)
        check_attention(oc[:, hh:hh + 1, pos], want, torch.bfloat16, what=f"prefill 8x512 {path} b={b} w={w} h{hh}")
    assert K.read_status() == 0
