"""The QKV product with RoPE and the KV-cache append in its epilogue (kernels.decode_gemm_rope): the decoder step's
``qkv = norm(h) @ qkv_w.t()`` followed by ``kernels.rope_kv`` (the reference's decode.py:201-203, spec.py:100-101)
in one kernel.

* Bit-exact with this library's own two-step path on the same inputs -- decode_gemm (store) into a qkv buffer, then
  rope_kv -- q, the k cache and the v cache alike: the product is the same kernel's, rounded to bf16 the same way, and
  the rotation the same non-contracting fp32 arithmetic.
* Against the numpy RoPE oracle applied to the float32 product rounded to bf16: q and the appended rows within the
  GEMM's bf16 tolerance (the products are summed in another order).
* Config 2's 8 rows x 5 tokens at 32 x 128 with cache rows and positions given, the 8 x 512 geometry, one row, and a
  position outside the cos/sin table (status bit 1, q zero, no k written).
"""

import numpy as np
import pytest
import torch

from oracle import rope as orope

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


@pytest.fixture(scope="module")
def K():
    from omniasr_b200 import kernels

    kernels.read_status()
    return kernels


def _case(rows, heads, dim, k, cap, seed, tokens=1):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, k, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(3 * heads * dim, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    cs = orope.rope_table(dim, cap + 8).contiguous().cuda()
    b = rows // tokens
    base = torch.randint(0, cap - tokens, (b,), generator=torch.Generator().manual_seed(seed))
    pos = (base[:, None] + torch.arange(tokens)[None]).reshape(-1).cuda()
    slots = (torch.arange(b)[:, None].expand(b, tokens).reshape(-1) + 1).cuda()  # row 0 of the cache left alone
    kc = torch.randn(b + 2, heads, cap, dim, generator=g, device="cuda").to(torch.bfloat16)
    vc = torch.randn(b + 2, heads, cap, dim, generator=g, device="cuda").to(torch.bfloat16)
    return x, w, cs, pos, slots, kc, vc


@pytest.mark.parametrize("rows,heads,dim,k,tokens", [(40, 32, 128, 4096, 5), (8, 8, 512, 4096, 1), (1, 32, 128, 4096, 1),
                                                     (64, 4, 128, 320, 4)])
def test_matches_two_step_path_bit_exact(K, rows, heads, dim, k, tokens):
    x, w, cs, pos, slots, kc, vc = _case(rows, heads, dim, k, 300, rows + dim, tokens)
    kc1, vc1, kc2, vc2 = kc.clone(), vc.clone(), kc.clone(), vc.clone()
    qkv = K.decode_gemm(x, w)
    q1 = K.rope_kv(qkv, cs, pos, kc1, vc1, heads, slots=slots)
    q2 = K.decode_gemm_rope(x, w, cs, pos, kc2, vc2, heads, slots=slots)
    torch.cuda.synchronize()
    assert torch.equal(q1.view(torch.int16), q2.view(torch.int16))
    assert torch.equal(kc1.view(torch.int16), kc2.view(torch.int16))
    assert torch.equal(vc1.view(torch.int16), vc2.view(torch.int16))
    assert K.read_status() == 0


def test_against_oracle_rope_of_fp32_product(K):
    rows, heads, dim, k, tokens = 40, 32, 128, 4096, 5
    x, w, cs, pos, slots, kc, vc = _case(rows, heads, dim, k, 300, 99, tokens)
    kc_o = kc.view(torch.int16).cpu().numpy().view(np.uint16).copy()
    vc_o = vc.view(torch.int16).cpu().numpy().view(np.uint16).copy()
    q = K.decode_gemm_rope(x, w, cs, pos, kc, vc, heads, slots=slots, cache_pos=pos)
    torch.cuda.synchronize()
    qkv = (x.float() @ w.float().t()).to(torch.bfloat16).cpu()
    q_o = orope.rope_kv(qkv.view(torch.int16).numpy().view(np.uint16), cs.cpu().numpy(), pos.cpu().numpy(), kc_o, vc_o,
                        heads, slots.cpu().numpy(), pos.cpu().numpy())
    as_f = lambda u: torch.from_numpy((u.astype(np.uint32) << 16).view(np.float32))  # noqa: E731
    torch.testing.assert_close(q.float().cpu().reshape(rows, -1), as_f(q_o).reshape(rows, -1), rtol=1e-2, atol=2e-2)
    torch.testing.assert_close(kc.float().cpu(), as_f(kc_o).reshape(kc.shape), rtol=1e-2, atol=2e-2)
    torch.testing.assert_close(vc.float().cpu(), as_f(vc_o).reshape(vc.shape), rtol=1e-2, atol=2e-2)
    assert K.read_status() == 0


def test_position_outside_the_table(K):
    """Token 2's position has no cos/sin row (its cache position is given, inside the cache): as rope_kv, a zero q,
    no k written, v written, status bit 1 -- bit for bit the two-step path's result."""
    rows, heads, dim, k = 4, 4, 128, 256
    x, w, cs, pos, slots, kc, vc = _case(rows, heads, dim, k, 64, 5)
    cache_pos = pos.clone()
    pos[2] = cs.size(0)
    kc1, vc1, kc2, vc2 = kc.clone(), vc.clone(), kc.clone(), vc.clone()
    q1 = K.rope_kv(K.decode_gemm(x, w), cs, pos, kc1, vc1, heads, slots=slots, cache_pos=cache_pos)
    assert K.read_status() == 1
    q2 = K.decode_gemm_rope(x, w, cs, pos, kc2, vc2, heads, slots=slots, cache_pos=cache_pos)
    torch.cuda.synchronize()
    assert K.read_status() == 1
    assert not q2[2].view(torch.int16).any()
    assert torch.equal(kc2[slots[2]], kc[slots[2]])
    assert torch.equal(q1.view(torch.int16), q2.view(torch.int16))
    assert torch.equal(kc1.view(torch.int16), kc2.view(torch.int16))
    assert torch.equal(vc1.view(torch.int16), vc2.view(torch.int16))
