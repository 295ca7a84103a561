"""Decode-time weight GEMMs (kernels.decode_gemm) against a float32 PyTorch reference of the same op: the decoder
step's ``norm(h) @ qkv_w.t()``, ``torch.addmm(h, o, out_w.t())`` and ``inner * F.silu(gate)`` of
``(norm(h) @ gi_w.t()).chunk(2, -1)`` (the reference's decode.py:201-205, spec.py:100-107), bf16 in and out."""

import pytest
import torch
import torch.nn.functional as F

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


def K():
    from omniasr_b200 import kernels

    return kernels


def data(rows, n, k, seed, wrows=None):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, k, generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn(wrows or n, k, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    return x, w


def close(got, want):
    # bf16 output (relative rounding 2^-9) after an fp32 sum in another order
    torch.testing.assert_close(got.float(), want, rtol=1e-2, atol=2e-2)


@pytest.mark.parametrize("rows", [1, 8, 40, 64])
@pytest.mark.parametrize("n,k", [(12288, 4096), (4096, 11008), (1000, 320), (130, 64)])
def test_store(rows, n, k):
    x, w = data(rows, n, k, rows * 7 + n)
    y = K().decode_gemm(x, w)
    torch.cuda.synchronize()
    close(y, x.float() @ w.float().t())
    assert K().read_status() == 0


@pytest.mark.parametrize("rows", [5, 40])
@pytest.mark.parametrize("n,k", [(4096, 4096), (4096, 11008), (200, 192)])
def test_residual(rows, n, k):
    x, w = data(rows, n, k, rows + n + 1)
    h = torch.randn(rows, n, device="cuda").to(torch.bfloat16)
    y = K().decode_gemm(x, w, "residual", residual=h)
    torch.cuda.synchronize()
    close(y, h.float() + x.float() @ w.float().t())
    # the reference's own bf16 call, for scale
    close(y, torch.addmm(h, x, w.t()).float())


@pytest.mark.parametrize("rows", [8, 40])
@pytest.mark.parametrize("f,k", [(11008, 4096), (2048, 4096), (100, 256)])
def test_swiglu(rows, f, k):
    x, w = data(rows, f, k, rows + f + 2, wrows=2 * f)
    y = K().decode_gemm(x, w, "swiglu")
    torch.cuda.synchronize()
    acc = x.float() @ w.float().t()
    g, u = acc[:, :f].to(torch.bfloat16).float(), acc[:, f:].to(torch.bfloat16).float()
    s = F.silu(g).to(torch.bfloat16).float()
    close(y, u * s)
    gate, inner = (x @ w.t()).chunk(2, -1)
    close(y, (inner * F.silu(gate)).float())


def test_bad_arguments_refused():
    x, w = data(65, 128, 64, 1)
    with pytest.raises(ValueError):
        K().decode_gemm(x, w)  # more than 64 token rows


def test_shapes_in_turn_share_one_workspace():
    """Calls of different shapes on one stream share the persistent workspace (its tile counters must come back to
    zero after every call): wide, narrow, SwiGLU and residual calls interleaved, each checked."""
    for rows, n, k, mode in [(40, 12288, 4096, "store"), (8, 11008, 4096, "swiglu"), (40, 4096, 4096, "residual"),
                             (3, 300, 128, "store"), (40, 11008, 4096, "swiglu"), (16, 4096, 11008, "residual")]:
        x, w = data(rows, n, k, rows + n, wrows=2 * n if mode == "swiglu" else None)
        h = torch.randn(rows, n, device="cuda").to(torch.bfloat16)
        y = K().decode_gemm(x, w, mode, residual=h if mode == "residual" else None)
        acc = x.float() @ w.float().t()
        if mode == "swiglu":
            g, u = acc[:, :n].to(torch.bfloat16).float(), acc[:, n:].to(torch.bfloat16).float()
            want = u * F.silu(g).to(torch.bfloat16).float()
        else:
            want = acc + (h.float() if mode == "residual" else 0)
        close(y, want)


@pytest.mark.parametrize("rows,n,k,mode", [(40, 12288, 4096, "store"), (40, 4096, 4096, "residual"),
                                           (40, 4096, 11008, "residual"), (40, 11008, 4096, "swiglu"),
                                           (40, 2048, 4096, "swiglu"), (1, 4096, 4096, "store"),
                                           (8, 10288, 4096, "store")])
def test_repeated_calls_give_the_same_bits(rows, n, k, mode):
    """Tiles split between CTAs are summed in one fixed order whichever CTA finishes them (stream-K) and in rank
    order within a tile's cluster (the 4096-wide and 2048-wide shapes), so repeated calls on the same inputs give
    identical bits."""
    x, w = data(rows, n, k, 3 * rows + n, wrows=2 * n if mode == "swiglu" else None)
    h = torch.randn(rows, n, device="cuda").to(torch.bfloat16) if mode == "residual" else None
    first = K().decode_gemm(x, w, mode, residual=h).clone()
    for _ in range(20):
        again = K().decode_gemm(x, w, mode, residual=h)
        assert torch.equal(first.view(torch.int16), again.view(torch.int16))
    assert K().read_status() == 0


def test_drop_in_weight_views_route_here():
    """``dropin.install(gemm=True)``'s weight views: ``x @ w.t()`` and ``torch.addmm(h, x, w.t())`` with at most 64
    bf16 rows are this GEMM (bit for bit the direct call); more rows are torch's own product."""
    from omniasr_b200 import dropin

    cls = dropin._weight_class()
    x, w = data(40, 4096, 4096, 7)
    h = torch.randn(40, 4096, device="cuda").to(torch.bfloat16)
    v = w.as_subclass(cls)
    assert torch.equal((x @ v.t()).view(torch.int16), K().decode_gemm(x, w).view(torch.int16))
    assert torch.equal(torch.addmm(h, x, v.t()).view(torch.int16),
                       K().decode_gemm(x, w, "residual", residual=h).view(torch.int16))
    big = torch.randn(100, 4096, device="cuda").to(torch.bfloat16)
    assert torch.equal(big @ v.t(), big @ w.t())
    assert K().read_status() == 0
