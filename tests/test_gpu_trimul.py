"""GPU parity of the triangle multiplicative update (C ABI through genie_tk.ops / modules)."""

import pytest
import torch

from golden_util import load_case
from gpu_util import assert_parity, assert_status_clean, require_gpu, to_dev
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


def _planes(B, R, C, cols, device, gen):
    from genie_tk import ops
    ld = ops.plane_pitch(cols)
    t = torch.zeros(B, R, C, ld, dtype=torch.float16, device=device)
    t[..., :cols] = torch.randn(B, R, C, cols, generator=gen, device="cpu").to(device, torch.float16)
    return t


@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("B,C,M,Nj,K", [(1, 2, 16, 16, 16), (2, 3, 100, 72, 40), (1, 2, 256, 256, 256),
                                        (1, 1, 384, 520, 130), (1, 2, 129, 257, 1000)])
def test_contract_matches_fp32_matmul(outgoing, B, C, M, Nj, K):
    dev = require_gpu()
    from genie_tk import ops
    gen = torch.Generator().manual_seed(M * 7 + Nj + K)
    if outgoing:
        a = _planes(B, M, C, K, dev, gen)
        b = _planes(B, Nj, C, K, dev, gen)
        ref = torch.einsum("bick,bjck->bicj", a[..., :K].float(), b[..., :K].float())
    else:
        a = _planes(B, K, C, M, dev, gen)
        b = _planes(B, K, C, Nj, dev, gen)
        ref = torch.einsum("bkci,bkcj->bicj", a[..., :M].float(), b[..., :Nj].float())
    scale = 0.5
    x = ops.trimul_contract(a, b, outgoing, M, Nj, K, out_scale=scale)
    torch.cuda.synchronize()
    got = x[..., :Nj].float() / scale
    # fp16 output rounding only: relative 2^-11 of the magnitude
    tol = 2e-3 * ref.abs().clamp_min(1.0)
    assert ((got - ref).abs() <= tol).all(), float((got - ref).abs().max())
    assert_status_clean(dev)


def test_project_stage_matches_oracle():
    dev = require_gpu()
    from genie_tk import ops
    op, dims, z, mask, params, out = load_case("trimul_in_c128")
    p = to_dev(params, dev)
    packed = ops.pack_trimul(p, dev)
    zd, md = z.to(dev), mask.to(dev)
    a, b = ops.trimul_project(zd, md, packed)
    torch.cuda.synchronize()
    zn = O.layer_norm(zd, p["layer_norm_in.weight"], p["layer_norm_in.bias"])
    m = md.unsqueeze(-1)
    a_ref = O.linear(zn, p, "linear_a_p") * torch.sigmoid(O.linear(zn, p, "linear_a_g")) * m
    b_ref = O.linear(zn, p, "linear_b_p") * torch.sigmoid(O.linear(zn, p, "linear_b_g")) * m
    N = z.shape[1]
    assert_parity(a[..., :N], a_ref.permute(0, 1, 3, 2), max_abs=3e-2, mean_abs=3e-3, what="a planes")
    assert_parity(b[..., :N], b_ref.permute(0, 1, 3, 2), max_abs=3e-2, mean_abs=3e-3, what="b planes")
    assert_status_clean(dev)


@pytest.mark.parametrize("name", ["trimul_out_c128", "trimul_in_c128"])
def test_module_matches_reference_golden(name):
    dev = require_gpu()
    import genie_tk
    op, dims, z, mask, params, out = load_case(name)
    cls = genie_tk.TriangleMultiplicationOutgoing if op == "trimul_out" else genie_tk.TriangleMultiplicationIncoming
    mod = cls(dims["c_z"], dims["c_hidden"]).to(dev)
    mod.load_state_dict(params)
    got = mod(z.to(dev), mask.to(dev))
    torch.cuda.synchronize()
    assert_parity(got, out, what=name)
    assert_status_clean(dev)


@pytest.mark.parametrize("cfg,N,B,outgoing", [(1, 128, 1, True), (2, 384, 2, False), (2, 200, 2, True),
                                              (1, 77, 1, False)])
def test_config_matches_oracle(cfg, N, B, outgoing):
    dev = require_gpu()
    import genie_tk
    z, mask, params = O.config_inputs(cfg, N=N, B=B)
    cls = genie_tk.TriangleMultiplicationOutgoing if outgoing else genie_tk.TriangleMultiplicationIncoming
    mod = cls(128, 128).to(dev)
    mod.load_state_dict(params)
    zd, md = z.to(dev), mask.to(dev)
    got = mod(zd, md)
    ref = O.trimul_forward(zd, md, to_dev(params, dev), outgoing=outgoing)
    assert_parity(got, ref, what=f"cfg{cfg} N={N}")
    # fused residual, in place (a graph-less kernel call: inference mode)
    z2 = zd.clone()
    with torch.no_grad():
        mod(z2, md, out=z2, add_residual=True)
    assert_parity(z2, zd + ref, what="residual in place")
    assert_status_clean(dev)


@pytest.mark.parametrize("c,N,B,outgoing", [(64, 150, 2, True), (64, 150, 1, False), (1, 40, 1, True),
                                            (17, 77, 1, False), (127, 130, 1, True)])
def test_narrower_hidden_runs_on_the_tuned_kernels(c, N, B, outgoing):
    """c_z = 128 with c_hidden = c < 128 (the c_hidden_mul = 64 of examples/basic_usage.py:140):
    the packed projections are zero past c, so the padded a / b / x channels are exactly zero,
    W_z has zero columns there and LN_out's statistics cover the c real channels."""
    dev = require_gpu()
    import genie_tk
    from genie_tk import _lib
    lib = _lib.load()
    assert lib.gtk_trimul_packed_bytes(128, c) == lib.gtk_trimul_packed_bytes(128, 128)
    gen = torch.Generator().manual_seed(300 + c + N)
    z = torch.randn(B, N, N, 128, generator=gen)
    mask = (torch.rand(B, N, N, generator=gen) > 0.2).float()
    params = O.make_trimul_params(128, c, gen, ln_random=True, bias_random=True)
    cls = genie_tk.TriangleMultiplicationOutgoing if outgoing else genie_tk.TriangleMultiplicationIncoming
    mod = cls(128, c).to(dev)
    mod.load_state_dict(to_dev(params, dev))
    zd, md = z.to(dev), mask.to(dev)
    with torch.no_grad():
        got = mod(zd, md)
        z2 = zd.clone()
        mod(z2, md, out=z2, add_residual=True)
    ref = O.trimul_forward(zd, md, to_dev(params, dev), outgoing=outgoing)
    torch.cuda.synchronize()
    assert_parity(got, ref, what=f"trimul c_hidden={c} N={N}")
    assert_parity(z2, zd + ref, what="residual in place")
    assert_status_clean(dev)


@pytest.mark.parametrize("outgoing", [True, False])
def test_narrower_hidden_with_dropout(outgoing):
    """The tuned kernels' dropout instantiation (K2e<1>) at c_hidden = 64: the keep bits act on
    the 128 output channels, the zero-padded hidden channels only on LN_out's statistics."""
    dev = require_gpu()
    import numpy as np
    from genie_tk import ops
    from oracle import dropout_oracle as D
    B, N, c = 2, 96, 64
    gen = torch.Generator().manual_seed(17 + int(outgoing))
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = (torch.rand(B, N, N, generator=gen) > 0.2).float().to(dev)
    params = to_dev(O.make_trimul_params(128, c, gen, ln_random=True, bias_random=True), dev)
    packed = ops.pack_trimul(params, dev)
    drop = ops.dropout_mask_philox(B, N, 0.25, seed=3, offset=1, shared_across_rows=True, device=dev)
    out = torch.empty_like(z)
    ops.trimul_forward(z, mask, packed, outgoing, out=out, add_residual=True, dropout=drop)
    torch.cuda.synchronize()
    assert_status_clean(dev)
    bits = drop.keep_bits.cpu().numpy().view(np.uint32).reshape(-1, 4)
    mult = D.multipliers_from_bits(bits, drop.scale, B, N, True).to(dev)
    ref = z + O.trimul_forward(z, mask, params, outgoing=outgoing) * mult
    assert_parity(out, ref, what=f"trimul c_hidden={c} dropout outgoing={outgoing}")
