"""The drop-in's opt-in routing of the decoders' weight products (``dropin.install(gemm=True)``): the reference's
``decode.fuse_projections`` (decode.py:34-54) is wrapped so that the tuples the decoders keep hold weight views whose
``x @ w.t()`` and ``torch.addmm(h, x, w.t())`` (decode.py:201-205) run ``kernels.decode_gemm`` for at most 64 bf16
CUDA token rows. On the CPU -- and for every other shape or dtype -- the views are torch's own operations: checked
here without a GPU, with the reference package as the host."""

import sys

import pytest
import torch

from conftest import ROOT

REF = ROOT / "baseline" / "_ref"


@pytest.fixture(scope="module")
def dropin():
    if not (REF / "omniasr_trt" / "decode.py").exists():
        pytest.fail(f"the reference package is missing from {REF} (run __graft_entry__.build() where the reference "
                    "checkout is present)")
    if str(REF) not in sys.path:
        sys.path.insert(0, str(REF))
    from omniasr_b200 import dropin as d

    yield d
    d.install()  # leave the reference's own fuse_projections in place for the other tests


def test_install_switches_the_projection_routing(dropin):
    dropin.install(gemm=True)
    from omniasr_trt import decode

    assert decode.fuse_projections.reference is not None
    dropin.install(gemm=True)  # idempotent
    assert decode.fuse_projections.reference.__name__ == "fuse_projections"
    assert getattr(decode.fuse_projections.reference, "reference", None) is None
    dropin.install()
    assert getattr(decode.fuse_projections, "reference", None) is None


def test_views_are_torch_operations_off_the_gpu(dropin):
    cls = dropin._weight_class()
    g = torch.Generator().manual_seed(0)
    w = torch.randn(256, 128, generator=g).to(torch.bfloat16)
    v = w.as_subclass(cls)
    x = torch.randn(4, 128, generator=g).to(torch.bfloat16)
    h = torch.randn(4, 256, generator=g).to(torch.bfloat16)
    y = x @ v.t()
    assert type(y) is torch.Tensor and torch.equal(y, x @ w.t())
    z = torch.addmm(h, x, v.t())
    assert type(z) is torch.Tensor and torch.equal(z, torch.addmm(h, x, w.t()))
    assert torch.equal(torch.matmul(x, v.t()), x @ w.t())
    s = v[:8] * 2 + 1  # any other use: a plain tensor, torch's result
    assert type(s) is torch.Tensor and torch.equal(s, w[:8] * 2 + 1)
    assert v.shape == w.shape and v.dtype == w.dtype


def test_routed_projections_wrap_every_weight(dropin):
    calls = []

    def fuse(model):
        calls.append(model)
        return [(torch.zeros(6, 4), torch.zeros(2, 2), torch.zeros(8, 4), torch.zeros(4, 4))]

    routed = dropin._routed_projections(fuse)
    layers = routed("m")
    assert calls == ["m"] and routed.reference is fuse
    cls = dropin._weight_class()
    assert all(isinstance(w, cls) for w in layers[0])
