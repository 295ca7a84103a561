"""The CUDA kernels (through the C ABI) against the golden vectors and the CPU oracle.

Bit-exact: RoPE + KV append and the reorder gather. Attention: bf16 max-abs <= 2e-2 and mean-abs <= 2e-3 against a
float64 reference; fp32 within the reference's own test tolerances (2e-5 decode, 1e-4 draft / beam). The cases of
the reference's CUDA tests (tests/test_kernels.py, tests/test_spec.py: H=8, D=512, fp32 and bf16) are restated here
against the oracle, plus the graded shapes (H=32, D=128) and the edge cases (length 0 and 1, tile and split
boundaries, cache capacity, strided cache views, CUDA-graph capture, out-of-range indices).
"""

import numpy as np
import pytest
import torch

import inputs as gi
from gpu_util import check_attention, dev, randn, raw
from oracle import attention as oatt
from oracle import gather as ogather
from oracle import rope as orope

pytestmark = [pytest.mark.gpu, pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a GPU")]


@pytest.fixture(scope="module")
def K():
    from omniasr_b200 import kernels

    assert kernels.available(torch.device("cuda")), "not a B200 (compute capability 10.0)"
    kernels.read_status()
    return kernels


@pytest.fixture(autouse=True)
def clean_status(K):
    """Every test leaves the status word clean unless it expects an error bit."""
    K.read_status()
    yield


# --------------------------------------------------------------------------------------------------- RoPE + append


@pytest.mark.parametrize("name", ["rope_bf16_h4_d128", "rope_f32_h4_d128", "rope_bf16_h2_d512", "rope_f32_h2_d16"])
def test_rope_kv_golden_bit_exact(K, golden, name):
    g = golden(name)
    is_bf16 = bool(g["is_bf16"])
    h = int(g["heads"])
    d = g["qkv"].shape[1] // (3 * h)
    dt = torch.bfloat16 if is_bf16 else torch.float32
    qkv, cs, pos = dev(g["qkv"], is_bf16), torch.from_numpy(g["cs"]).cuda(), torch.from_numpy(g["pos"]).cuda()
    for slots, cpos in ((None, None), (g["slots"], None), (g["slots"], g["cache_pos"])):
        kc = torch.zeros(int(g["rows"]), h, int(g["cache_len"]), d, dtype=dt, device="cuda")
        vc = torch.zeros_like(kc)
        ts = None if slots is None else torch.from_numpy(slots).cuda()
        tc = None if cpos is None else torch.from_numpy(cpos).cuda()
        q = K.rope_kv(qkv, cs, pos, kc, vc, h, ts, tc)
        assert np.array_equal(raw(q), g["q"])
        rows = np.arange(len(g["pos"])) if slots is None else slots
        at = g["pos"] if cpos is None else cpos
        assert np.array_equal(raw(kc)[rows, :, at], g["k"])
        assert np.array_equal(raw(vc)[rows, :, at], g["v"])
        written = np.zeros(kc.shape[:3], dtype=bool)
        written[rows, :, at] = True
        assert not raw(kc)[~written].any()  # nothing else touched
    assert K.read_status() == 0


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("h,d,n", [(32, 128, 40), (8, 512, 5), (2, 16, 7)])
def test_rope_kv_matches_oracle(K, dtype, h, d, n):
    """Graded shape (spec-4 batch 8: 40 tokens x 32 heads x 128) and the reference test's (8 x 512)."""
    is_bf16 = dtype == torch.bfloat16
    positions, rows, s = 4200, n + 3, 4200
    cs = orope.rope_table(d, positions)
    g = torch.Generator().manual_seed(5)
    qkv = randn((n, 3 * h * d), dtype, 100 + n)
    pos = torch.randperm(positions, generator=g)[:n]
    slots = torch.randperm(rows, generator=g)[:n]
    kc = torch.zeros(rows, h, s, d, dtype=dtype, device="cuda")
    vc = torch.zeros_like(kc)
    q = K.rope_kv(qkv.cuda(), cs.cuda(), pos.cuda(), kc, vc, h, slots.cuda())
    kn = np.zeros((rows, h, s, d), dtype=np.uint16 if is_bf16 else np.float32)
    vn = np.zeros_like(kn)
    qn = orope.rope_kv(raw(qkv), cs.numpy(), pos.numpy(), kn, vn, h, slots.numpy(), None, is_bf16)
    assert np.array_equal(raw(q), qn)
    sl, ps = slots.numpy(), pos.numpy()
    assert np.array_equal(raw(kc[slots.cuda(), :, pos.cuda()]), kn[sl, :, ps])
    assert np.array_equal(raw(vc[slots.cuda(), :, pos.cuda()]), vn[sl, :, ps])


def test_rope_kv_into_layer_slice_of_5d_cache(K):
    """The decoders pass ``self.k[i]``, a slice of [L, B, H, S, D]: strided rows, bit-exact writes."""
    L, b, h, s, d = 3, 4, 32, 512, 128
    k5 = torch.zeros(L, b, h, s, d, dtype=torch.bfloat16, device="cuda")
    v5 = torch.zeros_like(k5)
    cs = orope.rope_table(d, s)
    qkv = randn((b, 3 * h * d), torch.bfloat16, 7)
    pos = torch.tensor([0, 511, 256, 17])
    K.rope_kv(qkv.cuda(), cs.cuda(), pos.cuda(), k5[1], v5[1], h)
    kn = np.zeros((b, h, s, d), dtype=np.uint16)
    vn = np.zeros_like(kn)
    orope.rope_kv(raw(qkv), cs.numpy(), pos.numpy(), kn, vn, h, None, None, True)
    assert np.array_equal(raw(k5[1]), kn) and np.array_equal(raw(v5[1]), vn)
    assert not k5[0].any() and not k5[2].any()


def test_rope_kv_out_of_range_index_is_flagged_not_written(K):
    h, d, s = 2, 128, 64
    cs = orope.rope_table(d, 64)
    qkv = randn((3, 3 * h * d), torch.bfloat16, 9).cuda()
    kc = torch.zeros(4, h, s, d, dtype=torch.bfloat16, device="cuda")
    vc = torch.zeros_like(kc)
    pos = torch.tensor([1, 64, 2], device="cuda")  # 64: beyond the table and the cache
    q = K.rope_kv(qkv, cs.cuda(), pos, kc, vc, h, torch.tensor([0, 1, 9], device="cuda"))  # slot 9: no such row
    assert K.read_status() & 1
    assert kc[0, :, 1].any() and not kc[1].any() and not vc[1].any()
    assert not q[1].any()


# ------------------------------------------------------------------------------------------------------- decode


@pytest.mark.parametrize("is_bf16", [True, False])
def test_decode_attention_golden(K, golden, is_bf16):
    g = golden("decode_bf16" if is_bf16 else "decode_f32")
    q, k, v, lengths = gi.decode_inputs(is_bf16)
    c = gi.DECODE
    out = K.decode_attention(dev(q, is_bf16), dev(k, is_bf16), dev(v, is_bf16), torch.from_numpy(lengths).cuda(),
                             c["keys"], float(g["scale"]))
    dtype = torch.bfloat16 if is_bf16 else torch.float32
    check_attention(out, torch.from_numpy(g["out"]), dtype, 2e-5, "decode golden")
    assert not out[2].any()  # length 0: zeros
    assert K.read_status() == 0


@pytest.mark.parametrize("b,keys", [(1, 256), (3, 1024), (8, 2048), (16, 512)])
def test_decode_attention_reference_cases(K, b, keys):
    """tests/test_kernels.py:41-55 of the reference: fp32, H=8, D=512, capacity 2048, random lengths."""
    h, d, cap = 8, 512, 2048
    g = torch.Generator().manual_seed(1)
    kc = randn((b + 1, h, cap, d), torch.float32, 2)
    vc = randn((b + 1, h, cap, d), torch.float32, 3)
    q = randn((b, h, d), torch.float32, 4)
    lengths = torch.randint(1, keys + 1, (b,), generator=g)
    lengths[0] = keys
    out = K.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), keys, d**-0.5)
    want = oatt.decode_attention(q, kc, vc, lengths, d**-0.5)
    check_attention(out, want, torch.float32, 2e-5, f"decode b={b} keys={keys}")


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
@pytest.mark.parametrize("d", [16, 64, 128, 256, 512])
def test_decode_attention_edge_lengths(K, dtype, d):
    """Lengths 0, 1, around a 32-key tile and a 128-key split, and the full capacity (cache rows strided)."""
    h, cap = 4, 1030
    lengths = torch.tensor([0, 1, 31, 32, 33, 127, 128, 129, 1029, 1030])
    b = lengths.numel()
    full_k = randn((2, b + 1, h, cap, d), dtype, 10 + d)  # a layer slice of a [L, B, H, S, D] cache
    full_v = randn((2, b + 1, h, cap, d), dtype, 11 + d)
    q = randn((b, h, d), dtype, 12 + d)
    kc, vc = full_k.cuda()[1], full_v.cuda()[1]
    out = K.decode_attention(q.cuda(), kc, vc, lengths.cuda(), cap, d**-0.5)
    want = oatt.decode_attention(q, full_k[1], full_v[1], lengths, d**-0.5)
    check_attention(out, want, dtype, 2e-5, f"decode edges d={d}")
    assert not out[0].any()
    assert K.read_status() == 0


def test_decode_attention_graded_shape_full_size(K):
    """B=8, q_len 1, 32 x 128, 1024 keys, bf16 N(0,1) seed 0, scale 1/sqrt(128)."""
    b, h, d, s = 8, 32, 128, 1024
    q = randn((b, h, d), torch.bfloat16, 0)
    kc = randn((b, h, s, d), torch.bfloat16, 1)
    vc = randn((b, h, s, d), torch.bfloat16, 2)
    lengths = torch.full((b,), s)
    out = K.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), s, d**-0.5)
    want = oatt.decode_attention(q, kc, vc, lengths, d**-0.5)
    mx, mean = check_attention(out, want, torch.bfloat16, what="config 1")
    assert mean < 1e-3


def test_decode_attention_in_a_cuda_graph(K):
    b, h, d, s = 4, 8, 128, 512
    q = randn((b, h, d), torch.bfloat16, 20).cuda()
    kc = randn((b, h, s, d), torch.bfloat16, 21).cuda()
    vc = randn((b, h, s, d), torch.bfloat16, 22).cuda()
    lengths = torch.tensor([512, 300, 1, 0], device="cuda")
    eager = K.decode_attention(q, kc, vc, lengths, s, d**-0.5)
    stream = torch.cuda.Stream()
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        K.decode_attention(q, kc, vc, lengths, s, d**-0.5)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            out = K.decode_attention(q, kc, vc, lengths, s, d**-0.5)
    torch.cuda.current_stream().wait_stream(stream)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    lengths.copy_(torch.tensor([5, 6, 7, 8]))  # lengths are read on the device at replay
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, K.decode_attention(q, kc, vc, lengths, s, d**-0.5))


def test_decode_attention_length_beyond_cache_is_flagged(K):
    b, h, d, s = 2, 2, 128, 256
    q = randn((b, h, d), torch.float32, 30).cuda()
    kc = randn((b, h, s, d), torch.float32, 31).cuda()
    vc = randn((b, h, s, d), torch.float32, 32).cuda()
    out = K.decode_attention(q, kc, vc, torch.tensor([300, 10], device="cuda"), s, d**-0.5)
    assert K.read_status() & 1
    want = oatt.decode_attention(q.cpu(), kc.cpu(), vc.cpu(), torch.tensor([256, 10]), d**-0.5)
    check_attention(out, want, torch.float32, 2e-5, "clamped")  # clamped to the cache


def test_decode_attention_argument_errors(K):
    q = torch.zeros(2, 2, 128, dtype=torch.bfloat16, device="cuda")
    kc = torch.zeros(2, 2, 64, 128, dtype=torch.bfloat16, device="cuda")
    lengths = torch.zeros(2, dtype=torch.long, device="cuda")
    with pytest.raises(ValueError, match="keys"):
        K.decode_attention(q, kc, kc, lengths, 65, 0.1)
    with pytest.raises(ValueError, match="head_dim"):
        K.decode_attention(q[..., :96].contiguous(), kc[..., :96].contiguous(), kc[..., :96].contiguous(), lengths,
                           64, 0.1)
    with pytest.raises(ValueError, match="rows"):
        K.decode_attention(torch.zeros(3, 2, 128, dtype=torch.bfloat16, device="cuda"), kc, kc,
                           torch.zeros(3, dtype=torch.long, device="cuda"), 64, 0.1)
    with pytest.raises(ValueError, match="dtype"):
        K.decode_attention(q.half(), kc.half(), kc.half(), lengths, 64, 0.1)


# -------------------------------------------------------------------------------------------------------- draft


@pytest.mark.parametrize("is_bf16", [True, False])
def test_draft_attention_golden(K, golden, is_bf16):
    g = golden("draft_bf16" if is_bf16 else "draft_f32")
    q, k, v, lengths = gi.draft_inputs(is_bf16)
    c = gi.DRAFT
    out = K.draft_attention(dev(q, is_bf16), dev(k, is_bf16), dev(v, is_bf16), torch.from_numpy(lengths).cuda(),
                            c["t"], c["keys"], float(g["scale"]))
    check_attention(out, torch.from_numpy(g["out"]), torch.bfloat16 if is_bf16 else torch.float32, 1e-4, "draft")
    assert K.read_status() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("tokens", [1, 3, 5, 9])
def test_draft_attention_reference_cases(K, dtype, tokens):
    """tests/test_spec.py:91-108 of the reference: H=8, D=512, capacity 700, keys 640, lengths 600/257/1/0."""
    b, h, d, cap = 4, 8, 512, 700
    kc = randn((b + 1, h, cap, d), dtype, 40)
    vc = randn((b + 1, h, cap, d), dtype, 41)
    q = randn((b * tokens, h, d), dtype, 42)
    lengths = torch.tensor([600, 257, 1, 0])
    out = K.draft_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), tokens, 640, d**-0.5)
    want = oatt.draft_attention(q, kc, vc, lengths, tokens, d**-0.5)
    rows = 3 * tokens  # the finished row (length 0) is not checked, as in the reference
    check_attention(out[:rows], want[:rows], dtype, 1e-4, f"draft T={tokens}")


def test_draft_attention_graded_shape_full_size(K):
    """BASELINE config 2 attention: B=8, T=5, 32 x 128, lengths U[200, 2000], capacity 4096."""
    b, t, h, d, cap = 8, 5, 32, 128, 4096
    g = torch.Generator().manual_seed(0)
    lengths = torch.randint(200, 2001, (b,), generator=g)
    kc = randn((b, h, cap, d), torch.bfloat16, 50)
    vc = randn((b, h, cap, d), torch.bfloat16, 51)
    q = randn((b * t, h, d), torch.bfloat16, 52)
    keys = int((lengths.max() + t + 255) // 256 * 256)
    out = K.draft_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), t, keys, d**-0.5)
    want = oatt.draft_attention(q, kc, vc, lengths, t, d**-0.5)
    check_attention(out, want, torch.bfloat16, what="config 2")


# --------------------------------------------------------------------------------------------------------- beam


@pytest.mark.parametrize("is_bf16", [True, False])
def test_beam_attention_golden(K, golden, is_bf16):
    g = golden("beam_bf16" if is_bf16 else "beam_f32")
    q, kc, vc, ctx_len, kg, vg, ptr, gen_len = gi.beam_inputs(is_bf16)
    c = gi.BEAM
    out = K.beam_attention(dev(q, is_bf16), dev(kc, is_bf16), dev(vc, is_bf16), torch.from_numpy(ctx_len).cuda(),
                           dev(kg, is_bf16), dev(vg, is_bf16), torch.from_numpy(ptr).cuda(),
                           torch.from_numpy(gen_len).cuda(), c["beams"], c["ctx_keys"], float(g["scale"]))
    check_attention(out, torch.from_numpy(g["out"]), torch.bfloat16 if is_bf16 else torch.float32, 1e-4, "beam")
    assert not out[-c["beams"]:].any()
    assert K.read_status() == 0


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("beams", [1, 3, 5])
def test_beam_attention_reference_cases(K, dtype, beams):
    """tests/test_kernels.py:98-126 of the reference: S=4, H=8, D=512, ctx cap 600, gen cap 300, ctx_keys 640."""
    s, h, d, cap, gcap = 4, 8, 512, 600, 300
    r = s * beams
    g = torch.Generator().manual_seed(9)
    kc = randn((s + 1, h, cap, d), dtype, 60)
    vc = randn((s + 1, h, cap, d), dtype, 61)
    kg = randn((r + 2, h, gcap, d), dtype, 62)
    vg = randn((r + 2, h, gcap, d), dtype, 63)
    q = randn((r, h, d), dtype, 64)
    ctx_len = torch.tensor([600, 333, 1, 0])
    gen_len = torch.randint(0, gcap, (r,), generator=g)
    gen_len[-beams:] = 0
    ptr = torch.randint(0, r, (r, gcap), generator=g, dtype=torch.int32)
    out = K.beam_attention(q.cuda(), kc.cuda(), vc.cuda(), ctx_len.cuda(), kg.cuda(), vg.cuda(), ptr.cuda(),
                           gen_len.cuda(), beams, 600, d**-0.5)
    want = oatt.beam_attention(q, kc, vc, ctx_len, kg, vg, ptr, gen_len, beams, d**-0.5)
    check_attention(out, want, dtype, 1e-4, f"beam {beams}")
    assert not out[-beams:].any()


def test_beam_attention_graded_shape(K):
    """8 inputs x 5 beams, 32 x 128, context lengths U[300, 1800] shared per input."""
    s, n, h, d, gcap = 8, 5, 32, 128, 64
    r = s * n
    g = torch.Generator().manual_seed(0)
    ctx_len = torch.randint(300, 1801, (s,), generator=g)
    cap = 2048
    kc = randn((s, h, cap, d), torch.bfloat16, 70)
    vc = randn((s, h, cap, d), torch.bfloat16, 71)
    kg = randn((r, h, gcap, d), torch.bfloat16, 72)
    vg = randn((r, h, gcap, d), torch.bfloat16, 73)
    q = randn((r, h, d), torch.bfloat16, 74)
    gen_len = torch.randint(0, gcap + 1, (r,), generator=g)
    ptr = (torch.arange(r)[:, None] // n * n + torch.randint(0, n, (r, gcap), generator=g)).to(torch.int32)
    out = K.beam_attention(q.cuda(), kc.cuda(), vc.cuda(), ctx_len.cuda(), kg.cuda(), vg.cuda(), ptr.cuda(),
                           gen_len.cuda(), n, cap, d**-0.5)
    want = oatt.beam_attention(q, kc, vc, ctx_len, kg, vg, ptr, gen_len, n, d**-0.5)
    check_attention(out, want, torch.bfloat16, what="config 3")


@pytest.mark.parametrize("s,n,gcap", [(64, 4, 40), (3, 9, 17)])
def test_beam_attention_many_items_and_empty_rows(K, s, n, gcap):
    """The beam combine's warps each take many (row, head) items (64 inputs x 4 beams x 32 heads), or nine beams per
    input (the 16-query pass); an input without context and rows without generated keys (one row with neither:
    zeros)."""
    h, d, cap = 32, 128, 1100
    r = s * n
    g = torch.Generator().manual_seed(180 + n)
    ctx_len = torch.randint(1, cap + 1, (s,), generator=g)
    ctx_len[1] = 0
    gen_len = torch.randint(0, gcap + 1, (r,), generator=g)
    gen_len[n] = 0  # input 1's first beam: no context, no generated keys
    gen_len[0] = 0
    kc = randn((s, h, cap, d), torch.bfloat16, 181)
    vc = randn((s, h, cap, d), torch.bfloat16, 182)
    kg = randn((r, h, gcap, d), torch.bfloat16, 183)
    vg = randn((r, h, gcap, d), torch.bfloat16, 184)
    q = randn((r, h, d), torch.bfloat16, 185)
    ptr = (torch.arange(r)[:, None] // n * n + torch.randint(0, n, (r, gcap), generator=g)).to(torch.int32)
    out = K.beam_attention(q.cuda(), kc.cuda(), vc.cuda(), ctx_len.cuda(), kg.cuda(), vg.cuda(), ptr.cuda(),
                           gen_len.cuda(), n, cap, d**-0.5)
    want = oatt.beam_attention(q, kc, vc, ctx_len, kg, vg, ptr, gen_len, n, d**-0.5)
    check_attention(out, want, torch.bfloat16, what=f"beam s={s} n={n}")
    assert not out[n].any()
    assert K.read_status() == 0


def test_beam_pointer_out_of_range_is_flagged(K):
    s, n, h, d, cap, gcap = 1, 2, 1, 128, 64, 8
    kc = torch.zeros(s, h, cap, d, device="cuda")
    kg = torch.zeros(s * n, h, gcap, d, device="cuda")
    q = torch.zeros(s * n, h, d, device="cuda")
    ptr = torch.full((s * n, gcap), 7, dtype=torch.int32, device="cuda")  # rows 7: no such row
    K.beam_attention(q, kc, kc, torch.tensor([3], device="cuda"), kg, kg, ptr, torch.tensor([4, 4], device="cuda"),
                     n, cap, 0.1)
    assert K.read_status() & 1


# ------------------------------------------------------------------------------------------------------- gather


def test_reorder_gather_golden(K, golden):
    g = golden("gather")
    parent = torch.from_numpy(g["parent"]).cuda()
    for key, is_bf16 in (("ptr", False), ("hist", False), ("kv", True)):
        src = dev(g[key], is_bf16) if is_bf16 else torch.from_numpy(g[key]).cuda()
        out = K.reorder_gather(src, parent)
        assert np.array_equal(raw(out), g[f"{key}_out"]), key
        out32 = K.reorder_gather(src, parent.to(torch.int32))
        assert np.array_equal(raw(out32), g[f"{key}_out"]), key
    assert K.read_status() == 0


@pytest.mark.parametrize("shape,dtype", [((40, 32, 1800, 128), torch.bfloat16), ((40, 513), torch.int32),
                                         ((40, 8193), torch.int32), ((13, 3, 7), torch.uint8)])
def test_reorder_gather_matches_oracle(K, shape, dtype):
    """Config 3's reorder (40 beam rows of a layer's [H, S, D] cache) and odd-length int32 / byte rows."""
    g = torch.Generator().manual_seed(80)
    if dtype.is_floating_point:
        src = randn(shape, dtype, 81)
    else:
        src = torch.randint(0, 100, shape, generator=g).to(dtype)
    if shape[0] % 5 == 0:  # beam rows: input g's beams follow parents among g's 5 rows
        picks = torch.randint(0, 5, (shape[0] // 5, 5), generator=g).numpy()
        parent = ogather.beam_parents(shape[0] // 5, 5, picks)
    else:
        parent = torch.randint(0, shape[0], (shape[0] + 4,), generator=g).numpy()
    out = K.reorder_gather(src.cuda(), torch.from_numpy(parent).cuda())
    assert np.array_equal(raw(out), ogather.reorder_gather(raw(src), parent))


def test_reorder_gather_rejects_overlap_and_flags_bad_parent(K):
    src = torch.arange(64, dtype=torch.int32, device="cuda").view(8, 8)
    with pytest.raises(ValueError, match="overlap"):
        K.reorder_gather(src, torch.tensor([1, 0], device="cuda"), out=src)
    out = K.reorder_gather(src, torch.tensor([1, 8, 0], device="cuda"))
    assert K.read_status() & 1
    assert torch.equal(out[0], src[1]) and torch.equal(out[2], src[0])


@pytest.mark.parametrize("tokens", [1, 2, 3, 4, 6, 8, 9, 16])
def test_draft_attention_every_query_count_d128(K, tokens):
    """bf16 head_dim 128 runs on the tensor cores for 1..16 queries per row: every compile-time width, ragged lengths
    (units cut between CTAs and partial last tiles), finished rows (length 0)."""
    b, h, d, cap = 6, 16, 128, 3000
    g = torch.Generator().manual_seed(100 + tokens)
    lengths = torch.randint(1, 2800 - tokens, (b,), generator=g)
    lengths[1] = 0
    lengths[2] = 128 - tokens + 1  # the last query ends exactly on a tile boundary
    kc = randn((b, h, cap, d), torch.bfloat16, 110)
    vc = randn((b, h, cap, d), torch.bfloat16, 111)
    q = randn((b * tokens, h, d), torch.bfloat16, 112)
    keys = int((lengths.max() + tokens + 255) // 256 * 256)
    out = K.draft_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), tokens, min(keys, cap), d**-0.5)
    want = oatt.draft_attention(q, kc, vc, lengths, tokens, d**-0.5)
    check_attention(out, want, torch.bfloat16, what=f"draft T={tokens}")
    assert K.read_status() == 0


def test_tc_attention_uninitialised_cache_tail_is_ignored(K):
    """Keys past a row's length may hold anything (NaN here): they must not reach the output."""
    b, h, d, cap = 3, 4, 128, 700
    kc = randn((b, h, cap, d), torch.bfloat16, 120)
    vc = randn((b, h, cap, d), torch.bfloat16, 121)
    lengths = torch.tensor([300, 129, 1])
    for r in range(b):
        kc[r, :, int(lengths[r]):] = float("nan")
        vc[r, :, int(lengths[r]):] = float("nan")
    q = randn((b, h, d), torch.bfloat16, 122)
    out = K.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), cap, d**-0.5)
    assert not torch.isnan(out).any()
    kz, vz = kc.nan_to_num(0.0), vc.nan_to_num(0.0)
    check_attention(out, oatt.decode_attention(q, kz, vz, lengths, d**-0.5), torch.bfloat16, what="nan tail")


# In-pass merge: the last CTA to finish a (row, head) unit merges the unit's segments through the unit counters at the
# head of the decode / draft workspace (no combine kernel); those counters must be zero again after every call.

def _counters_zero(K):
    ws = K._ATTN_WS[(torch.cuda.current_device(), torch.cuda.current_stream().cuda_stream)]
    torch.cuda.synchronize()
    return not ws[:65536].any()


@pytest.mark.parametrize("tokens", [1, 5])
def test_tc_merge_of_many_segments(K, tokens):
    """One row and one head over 4000 keys: each of the 148 CTAs gets about one tile, so the unit has ~32 segments
    and the last CTA to finish merges all of them."""
    d, cap = 128, 4096
    lengths = torch.tensor([4000 - tokens])
    kc = randn((1, 1, cap, d), torch.bfloat16, 130)
    vc = randn((1, 1, cap, d), torch.bfloat16, 131)
    q = randn((tokens, 1, d), torch.bfloat16, 132)
    if tokens == 1:
        out = K.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), cap, d**-0.5)
        want = oatt.decode_attention(q, kc, vc, lengths, d**-0.5)
    else:
        out = K.draft_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), tokens, cap, d**-0.5)
        want = oatt.draft_attention(q, kc, vc, lengths, tokens, d**-0.5)
    check_attention(out, want, torch.bfloat16, what=f"many segments T={tokens}")
    assert _counters_zero(K)
    assert K.read_status() == 0


def test_tc_merge_shapes_in_turn_share_one_workspace(K):
    """Calls of different shapes in a row reuse the stream's workspace: every result is right and the counters are
    zero after each."""
    d, cap = 128, 2048
    kc = randn((8, 32, cap, d), torch.bfloat16, 140).cuda()
    vc = randn((8, 32, cap, d), torch.bfloat16, 141).cuda()
    g = torch.Generator().manual_seed(142)
    for i, (b, h, tokens) in enumerate(((8, 32, 5), (3, 7, 1), (8, 32, 1), (5, 32, 9), (8, 32, 5))):
        lengths = torch.randint(0, cap - tokens, (b,), generator=g)
        q = randn((b * tokens, h, d), torch.bfloat16, 150 + i)
        if tokens == 1:
            out = K.decode_attention(q.cuda(), kc[:, :h], vc[:, :h], lengths.cuda(), cap, d**-0.5)
            want = oatt.decode_attention(q, kc[:, :h].cpu(), vc[:, :h].cpu(), lengths, d**-0.5)
        else:
            out = K.draft_attention(q.cuda(), kc[:, :h], vc[:, :h], lengths.cuda(), tokens, cap, d**-0.5)
            want = oatt.draft_attention(q, kc[:, :h].cpu(), vc[:, :h].cpu(), lengths, tokens, d**-0.5)
        check_attention(out, want, torch.bfloat16, what=f"call {i}: b={b} h={h} T={tokens}")
        assert _counters_zero(K), f"counters left non-zero after call {i}"
    assert K.read_status() == 0


def test_tc_merge_writes_every_output_row_through_the_c_abi(K):
    """Through the C ABI with an output pre-filled with NaN and a freshly zeroed workspace: rows of length 0 get
    zeros (the pass writes them; no combine runs), every other row its attention."""
    import ctypes

    from omniasr_b200 import _lib

    lib = _lib.load()
    b, h, d, cap = 6, 16, 128, 1500
    lengths = torch.tensor([0, 1400, 0, 7, 129, 1500])
    kc = randn((b, h, cap, d), torch.bfloat16, 160)
    vc = randn((b, h, cap, d), torch.bfloat16, 161)
    q = randn((b, h, d), torch.bfloat16, 162)
    qd, kd, vd, ld = q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda()
    out = torch.full((b, h, d), float("nan"), dtype=torch.bfloat16, device="cuda")
    nbytes = lib.omniasr_attention_workspace(_lib.DECODE, _lib.BF16, b, 1, h, d, cap, 0)
    ws = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    vp = ctypes.c_void_p
    code = lib.omniasr_decode_attention(vp(qd.data_ptr()), vp(kd.data_ptr()), vp(vd.data_ptr()), b, cap,
                                        kd.stride(0), kd.stride(1), kd.stride(2), vp(ld.data_ptr()),
                                        vp(out.data_ptr()), b, h, d, cap, d**-0.5, _lib.BF16, vp(ws.data_ptr()),
                                        ws.numel(), vp(status.data_ptr()),
                                        vp(torch.cuda.current_stream().cuda_stream))
    assert code == 0, lib.omniasr_last_error()
    torch.cuda.synchronize()
    assert not torch.isnan(out).any()
    assert not out[0].any() and not out[2].any()
    check_attention(out, oatt.decode_attention(q, kc, vc, lengths, d**-0.5), torch.bfloat16, what="c abi")
    assert not ws[:65536].any() and int(status.item()) == 0


@pytest.mark.parametrize("tokens", [1, 3])
def test_tc_merge_with_more_rows_than_the_shared_length_table(K, tokens):
    """300 rows x 32 heads: more rows than the pass keeps in shared memory (256; the schedule then walks the lengths
    in global memory) but within the unit counters, so split units are still merged inside the pass."""
    b, h, d, cap = 300, 32, 128, 384
    lengths = torch.randint(0, cap - tokens + 1, (b,), generator=torch.Generator().manual_seed(175 + tokens))
    kc = randn((b, h, cap, d), torch.bfloat16, 176)
    vc = randn((b, h, cap, d), torch.bfloat16, 177)
    q = randn((b * tokens, h, d), torch.bfloat16, 178)
    if tokens == 1:
        out = K.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), cap, d**-0.5)
        want = oatt.decode_attention(q, kc, vc, lengths, d**-0.5)
    else:
        out = K.draft_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), tokens, cap, d**-0.5)
        want = oatt.draft_attention(q, kc, vc, lengths, tokens, d**-0.5)
    check_attention(out, want, torch.bfloat16, what=f"300 rows T={tokens}")
    assert _counters_zero(K)
    assert K.read_status() == 0


def test_tc_shape_past_the_counters_uses_the_combine(K):
    """More (row, head) units than the workspace has counters for (520 x 32 > 16384): the split units are merged by
    the combine kernel instead, with the same results."""
    b, h, d, cap = 520, 32, 128, 128
    lengths = torch.randint(0, cap + 1, (b,), generator=torch.Generator().manual_seed(170))
    kc = randn((b, h, cap, d), torch.bfloat16, 171)
    vc = randn((b, h, cap, d), torch.bfloat16, 172)
    q = randn((b, h, d), torch.bfloat16, 173)
    out = K.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), lengths.cuda(), cap, d**-0.5)
    check_attention(out, oatt.decode_attention(q, kc, vc, lengths, d**-0.5), torch.bfloat16, what="combine path")
    assert K.read_status() == 0


# ------------------------------------------------------------------------------------------------------ prefill


def _prefill_inputs(b, h, w, d, dtype, seed):
    """q as the decoder makes it (rope_kv's [B*W, H, D] seen as [B, H, W, D]), k / v as cache views [B, H, W, D]."""
    q = randn((b * w, h, d), dtype, seed).cuda().view(b, w, h, d).transpose(1, 2)
    cap = w + 37
    kc = randn((b + 1, h, cap, d), dtype, seed + 1).cuda()
    vc = randn((b + 1, h, cap, d), dtype, seed + 2).cuda()
    return q, kc[:b, :, :w], vc[:b, :, :w]


@pytest.mark.parametrize("b,h,w", [(1, 2, 1), (2, 2, 100), (3, 2, 128), (2, 3, 129), (1, 4, 257), (2, 2, 640)])
def test_prefill_attention_matches_oracle(K, b, h, w):
    """bf16 head_dim 128 on the tensor cores: every query-tile / key-tile edge (1, 128, 129, 257), strided cache
    views, the decoder's transposed q; output [B, H, W, D] (a view of [B, W, H, D])."""
    d = 128
    q, k, v = _prefill_inputs(b, h, w, d, torch.bfloat16, 200 + w)
    out = K.prefill_attention(q, k, v)
    assert out.shape == (b, h, w, d) and out.transpose(1, 2).is_contiguous()
    want = oatt.prefill_attention(q.cpu(), k.cpu(), v.cpu())
    check_attention(out, want, torch.bfloat16, what=f"prefill b={b} h={h} w={w}")
    assert K.read_status() == 0


@pytest.mark.parametrize("dtype,d,w", [(torch.float32, 16, 60), (torch.float32, 128, 130), (torch.bfloat16, 64, 90)])
def test_prefill_attention_other_dtypes(K, dtype, d, w):
    """fp32 (the reference's fp32 tests) and other head dims run as a W-query draft on the CUDA cores."""
    q, k, v = _prefill_inputs(2, 2, w, d, dtype, 250 + w)
    out = K.prefill_attention(q, k, v)
    want = oatt.prefill_attention(q.cpu(), k.cpu(), v.cpu())
    check_attention(out, want, dtype, 1e-4, f"prefill {dtype} d={d}")


def test_prefill_attention_config4_shape(K):
    """BASELINE config 4's prefill: 8 contexts x 1500 positions, 32 x 128 heads. Every (row, head) pair is checked
    on 40 query positions: the tile edges (0, 127, 128, 1279, 1280, 1499) and 34 drawn per pair."""
    b, h, w, d = 8, 32, 1500, 128
    q, k, v = _prefill_inputs(b, h, w, d, torch.bfloat16, 7)
    out = K.prefill_attention(q, k, v)
    g = torch.Generator().manual_seed(8)
    qc, kc, vc, oc = q.cpu(), k.cpu(), v.cpu(), out.cpu()
    edges = torch.tensor([0, 127, 128, 1279, 1280, 1499])
    for hh in range(h):
        pos = torch.cat([edges, torch.randint(0, w, (34,), generator=g)]).unique()
        want = oatt.prefill_attention_rows(qc[:, hh:hh + 1], kc[:, hh:hh + 1], vc[:, hh:hh + 1], pos)
        check_attention(oc[:, hh:hh + 1, pos], want, torch.bfloat16, what=f"config 4 head {hh}")
    assert K.read_status() == 0


@pytest.mark.parametrize("name,is_bf16,case", [("prefill_bf16", True, gi.PREFILL), ("prefill_f32", False, gi.PREFILL),
                                               ("prefill_bf16_d512", True, gi.PREFILL_D512)])
def test_prefill_attention_golden(K, golden, name, is_bf16, case):
    """Against the reference's own prefill call (SDPA is_causal, decode.py:171) on the golden inputs; bf16 head_dim
    128 on the tensor cores, fp32 and head_dim 512 on the drafted-verify path."""
    g = golden(name)
    q, k, v = (dev(a, is_bf16) for a in gi.prefill_inputs(is_bf16, case))
    out = K.prefill_attention(q, k, v)
    check_attention(out, torch.from_numpy(g["out"]), q.dtype, 1e-4, name)
    assert K.read_status() == 0
