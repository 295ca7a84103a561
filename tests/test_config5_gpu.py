"""BASELINE config 5 at full size: 64 rows, 32 x 128 heads, cached lengths 512 / 2048 / 8192, q_len 1 and 5.

Each case runs the decoder's order of calls on one layer: ``rope_kv`` appends the step's new keys at positions
L .. L+T-1 (so RoPE positions reach 8196 and need a table of more than 8192 rows), then decode (T = 1) or draft
verification (T = 5) attends over the L + 1 + i keys query i sees. The append is checked bit-exact against the oracle
for every row, head and new token; the attention against the float64 oracle on 12 sampled (row, head) pairs per case,
read back from the full-size device tensors (the whole 8.6 GB case is too large for the CPU oracle).
"""

import numpy as np
import pytest
import torch

from gpu_util import check_attention, raw
from oracle import attention as oatt
from oracle import rope as orope

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]

ROWS, H, D = 64, 32, 128
TABLE = 8200  # RoPE positions: the longest case writes at 8192 .. 8196


@pytest.fixture(scope="module")
def K():
    from omniasr_b200 import kernels

    kernels.read_status()
    return kernels


@pytest.mark.parametrize("tokens", [1, 5])
@pytest.mark.parametrize("length", [512, 2048, 8192])
def test_config5_append_and_attention(K, length, tokens):
    dev = torch.device("cuda")
    cap = length + 8
    g = torch.Generator(device=dev).manual_seed(500 + length + tokens)
    kc = torch.randn(ROWS, H, cap, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    vc = torch.randn(ROWS, H, cap, D, generator=g, device=dev, dtype=torch.float32).to(torch.bfloat16)
    gc = torch.Generator().manual_seed(600 + length + tokens)
    qkv = torch.randn(ROWS * tokens, 3 * H * D, generator=gc).to(torch.bfloat16)
    cs = orope.rope_table(D, TABLE)
    pos = (torch.full((ROWS, 1), length) + torch.arange(tokens)).reshape(-1)  # L .. L+T-1 per row
    slots = torch.arange(ROWS).repeat_interleave(tokens)

    q = K.rope_kv(qkv.to(dev), cs.to(dev), pos.to(dev), kc, vc, H, slots.to(dev))
    # Bit-exact append: the oracle writes the same tokens into a [rows, H, T, D] block.
    kn = np.zeros((ROWS, H, tokens, D), dtype=np.uint16)
    vn = np.zeros_like(kn)
    block_pos = np.tile(np.arange(tokens), ROWS)
    qn = orope.rope_kv(raw(qkv), cs.numpy(), pos.numpy(), kn, vn, H, slots.numpy(), block_pos, True)
    assert np.array_equal(raw(q), qn), "rope_kv q"
    assert np.array_equal(raw(kc[:, :, length:length + tokens]), kn), "appended k"
    assert np.array_equal(raw(vc[:, :, length:length + tokens]), vn), "appended v"

    lengths = torch.full((ROWS,), length + 1, device=dev)  # the first new token sees its own key (decode.py:193)
    scale = D**-0.5
    if tokens == 1:
        out = K.decode_attention(q, kc, vc, lengths, cap, scale)
    else:
        out = K.draft_attention(q, kc, vc, lengths, tokens, cap, scale)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    pick = torch.Generator().manual_seed(700 + length)
    rows = torch.randint(0, ROWS, (12,), generator=pick).tolist()
    heads = torch.randint(0, H, (12,), generator=pick).tolist()
    rows[0], heads[0] = ROWS - 1, H - 1
    for r, h in zip(rows, heads):
        keys = length + tokens
        kr = kc[r:r + 1, h:h + 1, :keys].cpu()
        vr = vc[r:r + 1, h:h + 1, :keys].cpu()
        qr = q[r * tokens:(r + 1) * tokens, h:h + 1].cpu()
        want = oatt.draft_attention(qr, kr, vr, torch.tensor([length + 1]), tokens, scale)
        check_attention(out[r * tokens:(r + 1) * tokens, h:h + 1], want, torch.bfloat16,
                        what=f"L={length} T={tokens} row {r} head {h}")
    assert K.read_status() == 0
