"""The decoder layer's glue kernels against the reference's eager ops (needs a B200).

``pkv_add_rms_norm`` replaces ``x = x + block(x)`` followed by the reference's ``RMSNorm``
(engine/model.py:162-166, 278-280); ``pkv_silu_mul`` the MLP's ``F.silu(gate) * up``
(engine/model.py:262-264). The residual add and ``silu * up`` must be bit-identical to
torch's eager result; the norm rounds where the reference rounds, but sums the squares in
its own float32 order, so where the float32 value lands next to a rounding boundary the
normalised value may round one unit the other way, which the weight multiply carries into
at most two units of the output (and the test requires that of at most 1% of elements).
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    return torch.device("cuda", 0)


def reference_rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """engine/model.py:162-166, op for op."""
    x32 = x.float()
    x32 = x32 * torch.rsqrt(x32.pow(2).mean(-1, keepdim=True) + eps)
    return weight * x32.to(x.dtype)


def ulp_diff(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """|a - b| in units of the dtype's spacing at b (float32 math on the rounded values)."""
    eps = torch.finfo(b.dtype).eps
    tiny = torch.finfo(b.dtype).tiny
    scale = torch.clamp(b.float().abs(), min=tiny) * eps
    return (a.float() - b.float()).abs() / scale


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,hidden", [(1, 896), (7, 896), (190, 896), (4096, 896), (64, 3584), (5, 8192),
                                         (3, 100), (9, 4104)])
@pytest.mark.parametrize("with_residual", [False, True])
def test_add_rms_norm_matches_the_reference(dev, dtype, rows, hidden, with_residual):
    from mini_inference_b200 import ops

    g = torch.Generator(device=dev).manual_seed(rows * 7 + hidden)
    x = torch.randn(rows, hidden, generator=g, device=dev).to(dtype)
    w = (1 + 0.1 * torch.randn(hidden, generator=g, device=dev)).to(dtype)
    eps = 1e-6
    if with_residual:
        h0 = (3 * torch.randn(rows, hidden, generator=g, device=dev)).to(dtype)
        h = h0.clone()
        got = ops.add_rms_norm(x, w, eps, residual=h)
        want_h = h0 + x
        assert torch.equal(h, want_h)  # the residual add, bit for bit
        want = reference_rms_norm(want_h, w, eps)
    else:
        got = ops.add_rms_norm(x, w, eps)
        want = reference_rms_norm(x, w, eps)
    torch.cuda.synchronize()
    d = ulp_diff(got, want)
    assert d.max().item() <= 2.0 + 1e-6, d.max().item()
    assert (got != want).float().mean().item() <= 0.01


def test_add_rms_norm_in_the_model_layout(dev):
    """[B, T, H] activations, output written over the input, a 1-row decode batch."""
    from mini_inference_b200 import ops

    g = torch.Generator(device=dev).manual_seed(3)
    for shape in ((4, 33, 896), (1, 1, 896)):
        x = torch.randn(*shape, generator=g, device=dev).half()
        w = torch.randn(shape[-1], generator=g, device=dev).half()
        want = reference_rms_norm(x, w, 1e-6)
        got = ops.add_rms_norm(x, w, 1e-6, out=x)  # in place
        assert got.data_ptr() == x.data_ptr() and got.shape == shape
        assert ulp_diff(got, want).max().item() <= 2.0 + 1e-6


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("rows,inter", [(1, 4864), (190, 4864), (64, 18944), (2048, 4864), (3, 36)])
def test_silu_mul_is_bit_identical_to_torch(dev, dtype, rows, inter):
    from mini_inference_b200 import ops

    g = torch.Generator(device=dev).manual_seed(rows + inter)
    gate_up = (4 * torch.randn(rows, 2 * inter, generator=g, device=dev)).to(dtype)
    gate, up = gate_up.chunk(2, dim=-1)
    want = F.silu(gate) * up
    got = ops.silu_mul(gate_up)
    assert torch.equal(got, want), (got.float() - want.float()).abs().max().item()


def test_silu_mul_edge_values(dev):
    from mini_inference_b200 import ops

    v = torch.tensor([0.0, -0.0, 1e-4, -1e-4, 20.0, -20.0, 88.0, -88.0, 65504.0, -65504.0, float("inf"),
                      -float("inf"), 11.0, -11.0, 3.0, -3.0], device=dev).half()
    gate_up = torch.cat([v, torch.full_like(v, 1.5)]).view(1, -1)
    want = F.silu(v) * 1.5
    got = ops.silu_mul(gate_up)[0]
    assert torch.equal(got.isnan(), want.isnan())
    assert torch.equal(got[~want.isnan()], want[~want.isnan()])


def test_layer_ops_reject_bad_arguments(dev):
    from mini_inference_b200 import ops

    x = torch.randn(4, 64, device=dev).half()
    with pytest.raises(ValueError):
        ops.add_rms_norm(x, torch.ones(32, device=dev).half(), 1e-6)
    with pytest.raises(ValueError):
        ops.add_rms_norm(x, torch.ones(64, device=dev), 1e-6)  # weight dtype
    with pytest.raises(ValueError):
        ops.silu_mul(torch.randn(4, 7, device=dev).half())
    with pytest.raises(ValueError):
        ops.add_rms_norm(x.t(), torch.ones(4, device=dev).half(), 1e-6)  # strided last dim


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("splits,rows", [(1, 5), (4, 190), (8, 64)])
def test_add_rms_norm_of_split_k_partials(dev, dtype, splits, rows):
    """x given as float32 split-K partials: summed slice by slice in order and rounded to the
    dtype (where F.linear rounds), then the same residual add and norm, bit for bit."""
    from mini_inference_b200 import ops

    g = torch.Generator(device=dev).manual_seed(splits * 100 + rows)
    parts = torch.randn(splits, rows, 896, generator=g, device=dev)
    w = (1 + 0.1 * torch.randn(896, generator=g, device=dev)).to(dtype)
    h0 = torch.randn(rows, 896, generator=g, device=dev).to(dtype)
    acc = parts[0].clone()
    for s in range(1, splits):
        acc += parts[s]
    x = acc.to(dtype)
    h_want, h_got = h0.clone(), h0.clone()
    want = ops.add_rms_norm(x, w, 1e-6, residual=h_want)
    got = ops.add_rms_norm(parts, w, 1e-6, residual=h_got)
    assert torch.equal(h_got, h_want)
    assert torch.equal(got, want)


def test_split_k_projection_matches_one_gemm(dev):
    """The model's split-K down_proj (a batched cuBLAS GEMM with float32 partials) against the
    single GEMM the reference runs: the same float32 dot products in another order."""
    from mini_inference_b200.model import _linear_split_k, _split_k

    g = torch.Generator(device=dev).manual_seed(5)
    act = torch.randn(190, 4864, generator=g, device=dev).half()
    wd = (0.02 * torch.randn(896, 4864, generator=g, device=dev)).half()
    s = _split_k(190, wd)
    assert s == 4 and _split_k(64, wd) == 8 and _split_k(4096, wd) == 0
    parts = _linear_split_k(act, wd, s)
    ref = act.double() @ wd.double().t()
    assert (parts.double().sum(0) - ref).abs().max().item() < 1e-3
