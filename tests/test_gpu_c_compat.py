"""GPU parity of ``genie_tk._C`` (the reference's native module, kernels/bindings.cpp:69-101)
on the B200 kernels: each function against its definition evaluated in fp32, and the
reference's own CUDA call path of the multiplicative update (triangle_mul.py:134-169,
with ``_C.triangle_mul_*`` from this package) against the fused module."""

import pytest
import torch
import torch.nn.functional as F

from gpu_util import assert_parity, assert_status_clean, require_gpu, to_dev
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.detach().float(), b.detach().float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("B,N,C", [(1, 64, 128), (2, 77, 32), (1, 130, 8)])
def test_triangle_mul_matches_einsum(outgoing, B, N, C):
    dev = require_gpu()
    from genie_tk import _C
    gen = torch.Generator().manual_seed(N + C + int(outgoing))
    a = torch.randn(B, N, N, C, generator=gen).to(dev, torch.bfloat16)
    b = torch.randn(B, N, N, C, generator=gen).to(dev, torch.bfloat16)
    mask = torch.ones(B, N, N, device=dev)
    fn = _C.triangle_mul_outgoing if outgoing else _C.triangle_mul_incoming
    x = fn(a, b, mask)
    eq = "bikc,bjkc->bijc" if outgoing else "bkic,bkjc->bijc"
    ref = torch.einsum(eq, a.float(), b.float())
    torch.cuda.synchronize()
    assert x.dtype == torch.bfloat16 and x.shape == ref.shape
    assert _rel(x, ref) < 6e-3
    assert_status_clean(dev)


def _attention_reference(q, k, v, bias, mask, scale):
    """The definition in fp32: starting-node attention over keys k of each row i."""
    s = torch.einsum("bhijd,bhikd->bhijk", q.float(), k.float()) * scale
    s = s + bias.float()[:, :, None] + (1e9 * (mask.float() - 1.0))[:, None, :, None, :]
    return torch.einsum("bhijk,bhikd->bhijd", torch.softmax(s, dim=-1), v.float())


@pytest.mark.parametrize("starting", [True, False])
@pytest.mark.parametrize("B,N,H,D", [(1, 40, 4, 32), (2, 100, 4, 32), (1, 257, 4, 32), (2, 45, 4, 8),
                                     (1, 70, 2, 16), (1, 33, 3, 64)])
def test_triangle_attention_matches_definition(starting, B, N, H, D):
    """The reference kernel's shape (4 heads of 32) on the tuned core, any other on the
    tensor-core core of the training path (the reference module's default head_dim 8 among them)."""
    dev = require_gpu()
    from genie_tk import _C
    gen = torch.Generator().manual_seed(3 * N + B + int(starting) + D)
    q, k, v = (torch.randn(B, H, N, N, D, generator=gen).to(dev, torch.bfloat16) for _ in range(3))
    bias = torch.randn(B, H, N, N, generator=gen).to(dev)
    mask = (torch.rand(B, N, N, generator=gen) > 0.15).float().to(dev)
    mask[:, -2:, :] = 0  # fully masked rows
    scale = D ** -0.5
    fn = _C.triangle_attention_starting if starting else _C.triangle_attention_ending
    o = fn(q, k, v, bias, mask, scale)
    if starting:
        ref = _attention_reference(q, k, v, bias, mask, scale)
    else:
        sw = lambda t: t.transpose(2, 3)  # noqa: E731
        ref = sw(_attention_reference(sw(q), sw(k), sw(v), bias, mask.transpose(1, 2), scale))
    torch.cuda.synchronize()
    assert o.dtype == torch.bfloat16 and o.shape == ref.shape
    assert_parity(o, ref, what=f"attention start={starting} N={N}")
    assert_status_clean(dev)


@pytest.mark.parametrize("shape", [(5, 128), (3, 7, 130), (2, 1), (4, 4096)])
def test_layernorm_and_fused_linear_match_torch(shape):
    dev = require_gpu()
    from genie_tk import _C
    gen = torch.Generator().manual_seed(sum(shape))
    x = (3.0 * torch.randn(*shape, generator=gen) + 1.5).to(dev)
    D = shape[-1]
    g = (1 + 0.1 * torch.randn(D, generator=gen)).to(dev)
    b = (0.1 * torch.randn(D, generator=gen)).to(dev)
    y = _C.layernorm(x, g, b)
    ref = F.layer_norm(x, (D,), g, b, 1e-5)
    assert float((y - ref).abs().max()) <= 1e-5 * max(1.0, float(ref.abs().max()))
    w = (torch.randn(D, 24, generator=gen) / D ** 0.5).to(dev)
    bb = torch.randn(24, generator=gen).to(dev)
    out = _C.fused_layernorm_linear(x, g, b, w, bb)
    ref2 = ref @ w + bb
    assert out.shape == ref2.shape and float((out - ref2).abs().max()) <= 1e-4
    assert torch.allclose(_C.fused_layernorm_linear(x, g, b, w), ref @ w, rtol=0, atol=1e-4)
    # in place through the C ABI: out may alias x
    from genie_tk import ops
    xx = x.clone()
    ops.layernorm(xx, g, b, out=xx)
    assert torch.equal(xx, y)


@pytest.mark.parametrize("outgoing", [True, False])
def test_reference_cuda_call_path_runs_on_this_library(outgoing):
    """TriangleMultiplicativeUpdate._forward_cuda (triangle_mul.py:134-169) written out with
    this package's ``_C``: the same result as the fused module and the oracle."""
    dev = require_gpu()
    import genie_tk
    from genie_tk import _C
    gen = torch.Generator().manual_seed(12 + int(outgoing))
    B, N = 1, 96
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = torch.ones(B, N, N)
    mask[:, -5:, :] = 0
    mask = mask.to(dev)
    p = to_dev(O.make_trimul_params(128, 128, gen, gate_bias=1.0), dev)
    m = mask.unsqueeze(-1)
    zn = F.layer_norm(z, (128,), p["layer_norm_in.weight"], p["layer_norm_in.bias"], 1e-5)
    lin = lambda x, n: F.linear(x, p[n + ".weight"], p[n + ".bias"])  # noqa: E731
    a = (lin(zn, "linear_a_p") * torch.sigmoid(lin(zn, "linear_a_g")) * m).contiguous().to(torch.bfloat16)
    b = (lin(zn, "linear_b_p") * torch.sigmoid(lin(zn, "linear_b_g")) * m).contiguous().to(torch.bfloat16)
    fn = _C.triangle_mul_outgoing if outgoing else _C.triangle_mul_incoming
    x = fn(a, b, mask.float()).to(z.dtype)
    x = F.layer_norm(x, (128,), p["layer_norm_out.weight"], p["layer_norm_out.bias"], 1e-5)
    via_c = lin(x, "linear_z") * torch.sigmoid(lin(zn, "linear_g"))
    cls = genie_tk.TriangleMultiplicationOutgoing if outgoing else genie_tk.TriangleMultiplicationIncoming
    mod = cls(128, 128).to(dev)
    mod.load_state_dict(p)
    with torch.no_grad():
        fused = mod(z, mask)
    ref = O.trimul_forward(z, mask, p, outgoing)
    assert_parity(via_c, ref, what="reference _forward_cuda on _C")
    assert_parity(fused, via_c, what="fused module vs _C path")
    assert_status_clean(dev)
