"""GPU parity at the shapes other than the benchmark's 128-channel one: those the tuned
kernels take with zero-padded weights and those the general-shape kernels run (the
reference's defaults c_hidden_tri_att = 32 with 4 heads, head_dim 8 --
src/genie_tk/pair_transform.py:113-119; the c_hidden_mul = 64 and c_hidden_tri_att = 16 of
examples/basic_usage.py:140-142; the c_z = 64 / 32 widths of tests/test_triangle_mul.py:37 and
tests/test_triangle_attention.py:36,74,127-137), through the same C ABI entry points
(gtk_trimul_forward, gtk_triatt_forward, gtk_transition_forward).

Checked against golden outputs of the reference's own modules (tests/golden/gen_*.npz) and
against the fp32 oracle at larger, ragged sizes, with masks, in-place residuals, channel
dropout and gradients, at the stated bar (max-abs <= 2e-2, mean-abs <= 2e-3).
"""

import numpy as np
import pytest
import torch

from golden_util import GENERAL_CASES, LAYER_CASES, load_case, load_layer, load_transition, oracle_layer
from gpu_util import assert_parity, assert_status_clean, require_gpu, to_dev
from oracle import dropout_oracle as D
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


def _module(op, c_z, c, H, dev):
    import genie_tk
    if op == "trimul_out":
        return genie_tk.TriangleMultiplicationOutgoing(c_z, c).to(dev)
    if op == "trimul_in":
        return genie_tk.TriangleMultiplicationIncoming(c_z, c).to(dev)
    if op == "triatt_start":
        return genie_tk.TriangleAttentionStartingNode(c_z, c, H).to(dev)
    return genie_tk.TriangleAttentionEndingNode(c_z, c, H).to(dev)


def _oracle(op, z, mask, p, H):
    if op.startswith("trimul"):
        return O.trimul_forward(z, mask, p, outgoing=op == "trimul_out")
    return O.triatt_forward(z, mask, p, starting=op == "triatt_start", no_heads=H)


@pytest.mark.parametrize("name", GENERAL_CASES)
def test_module_matches_reference_golden(name):
    dev = require_gpu()
    op, dims, z, mask, params, out = load_case(name)
    mod = _module(op, dims["c_z"], dims["c_hidden"], dims["heads"], dev)
    mod.load_state_dict(to_dev(params, dev))
    got = mod(z.to(dev), mask.to(dev))
    torch.cuda.synchronize()
    assert got.shape == out.shape
    assert_parity(got, out, what=name)
    assert_status_clean(dev)


@pytest.mark.parametrize("op,c_z,c,H", [("trimul_out", 64, 32, 0), ("trimul_in", 128, 64, 0),
                                        ("trimul_out", 96, 48, 0), ("triatt_start", 128, 32, 4),
                                        ("triatt_end", 128, 32, 4), ("triatt_start", 64, 16, 4),
                                        ("triatt_end", 48, 36, 3), ("triatt_start", 128, 128, 2)])
@pytest.mark.parametrize("N,B", [(1, 1), (37, 2), (130, 1)])
def test_general_shapes_match_oracle(op, c_z, c, H, N, B):
    """Ragged N (one element, a partial 32-key tile, more than one 128-query block), B = 2,
    a mask with padded rows and columns, and head dims 4 ... 64."""
    dev = require_gpu()
    gen = torch.Generator().manual_seed(N * 13 + B + c_z + c)
    z = torch.randn(B, N, N, c_z, generator=gen)
    mask = torch.ones(B, N, N)
    if N > 4:
        mask[-1, -3:, :] = 0
        mask[-1, :, -2:] = 0
    params = (O.make_trimul_params(c_z, c, gen, ln_random=True, bias_random=True) if op.startswith("trimul")
              else O.make_triatt_params(c_z, c, H, gen, ln_random=True, bias_random=True))
    p = to_dev(params, dev)
    zd, md = z.to(dev), mask.to(dev)
    mod = _module(op, c_z, c, H, dev)
    mod.load_state_dict(p)
    with torch.no_grad():
        got = mod(zd, md)
    ref = _oracle(op, zd, md, p, H)
    torch.cuda.synchronize()
    assert_parity(got, ref, what=f"{op} c_z={c_z} c={c} H={H} N={N}")
    # in place, with the residual fused: out = z + update
    zz = zd.clone()
    with torch.no_grad():
        mod(zz, md, out=zz, add_residual=True)
    torch.cuda.synchronize()
    assert_parity(zz, zd + ref, what=f"{op} in place")
    assert_status_clean(dev)


@pytest.mark.parametrize("kind", ["trimul_out", "trimul_in", "triatt_start", "triatt_end"])
@pytest.mark.parametrize("rowwise", [True, False])
def test_general_shapes_with_dropout(kind, rowwise):
    dev = require_gpu()
    from genie_tk import ops
    B, N, c_z = 2, 45, 64
    gen = torch.Generator().manual_seed(91 + int(rowwise))
    z = torch.randn(B, N, N, c_z, generator=gen).to(dev)
    mask = torch.ones(B, N, N, device=dev)
    params = to_dev(O.make_trimul_params(c_z, 32, gen, gate_bias=1.0) if kind.startswith("trimul")
                    else O.make_triatt_params(c_z, 32, 4, gen, gate_bias=1.0), dev)
    if kind.startswith("trimul"):
        packed = ops.pack_trimul(params, dev)
    else:
        packed = ops.pack_triatt(params, dev, 4)
    drop = ops.dropout_mask_philox(B, N, 0.25, seed=7, offset=int(rowwise), shared_across_rows=rowwise, device=dev)
    out = torch.empty_like(z)
    if kind.startswith("trimul"):
        ops.trimul_forward(z, mask, packed, kind == "trimul_out", out=out, add_residual=True, dropout=drop)
    else:
        ops.triatt_forward(z, mask, packed, kind == "triatt_start", out=out, add_residual=True, dropout=drop)
    torch.cuda.synchronize()
    assert_status_clean(dev)
    bits = drop.keep_bits.cpu().numpy().view(np.uint32).reshape(-1, 4)
    mult = D.multipliers_from_bits(bits, drop.scale, B, N, rowwise)[..., :c_z].to(dev)
    ref = z + _oracle(kind, z, mask, params, 4) * mult
    assert_parity(out, ref, what=f"{kind} dropout rowwise={rowwise}")
    dropped = (mult == 0).expand_as(out)
    assert torch.equal(out[dropped], z[dropped])


def test_transition_c64_matches_reference_golden():
    dev = require_gpu()
    import genie_tk
    z, mask, params, out = load_transition("gen_transition_c64")
    mod = genie_tk.pair_transform.PairTransition(64, 4).to(dev)
    mod.load_state_dict(to_dev(params, dev))
    zd, md = z.to(dev), mask.to(dev)
    got = mod(zd, md)
    torch.cuda.synchronize()
    assert_parity(got, out, what="transition c_p=64")
    zz = zd.clone()
    mod.residual_masked_(zz, md)
    torch.cuda.synchronize()
    assert_parity(zz, (zd + out.to(dev)) * md.unsqueeze(-1), what="transition residual + mask")
    assert_status_clean(dev)


@pytest.mark.parametrize("name", LAYER_CASES)
def test_pair_transform_layer_matches_reference_golden(name):
    """A whole PairTransformLayer (eval mode) built with the reference's default keyword
    arguments, or with the shapes of the reference's own layer test."""
    dev = require_gpu()
    import genie_tk
    dims, z, mask, blocks, out = load_layer(name)
    layer = genie_tk.PairTransformLayer(c_p=dims["c_p"], c_hidden_mul=dims["c_mul"], c_hidden_tri_att=dims["c_att"],
                                        n_head_tri=dims["heads"]).to(dev).eval()
    sd = {f"{b}.{k}": v for b, p in blocks.items() for k, v in p.items()}
    layer.load_state_dict(to_dev(sd, dev))
    with torch.no_grad():
        got, gm = layer((z.to(dev), mask.to(dev)))
    torch.cuda.synchronize()
    assert_parity(got, out, what=name)
    assert_status_clean(dev)


def test_pair_transform_net_with_default_arguments():
    """PairTransformNet(128, n_layers) with every other argument at the reference's default
    (c_hidden_tri_att = 32, 4 heads: head_dim 8) against the oracle, two layers, N = 96."""
    dev = require_gpu()
    import genie_tk
    gen = torch.Generator().manual_seed(17)
    net = genie_tk.PairTransformNet(128, 2).to(dev).eval()
    blocks = []
    with torch.no_grad():
        for layer in net.layers:
            b = {"tri_mul_out": O.make_trimul_params(128, 128, gen, ln_random=True, bias_random=True),
                 "tri_mul_in": O.make_trimul_params(128, 128, gen, ln_random=True, bias_random=True),
                 "tri_att_start": O.make_triatt_params(128, 32, 4, gen, ln_random=True, bias_random=True),
                 "tri_att_end": O.make_triatt_params(128, 32, 4, gen, ln_random=True, bias_random=True),
                 "pair_transition": O.make_transition_params(128, 4, gen)}
            layer.load_state_dict(to_dev({f"{k}.{n}": v for k, p in b.items() for n, v in p.items()}, dev))
            blocks.append(to_dev_blocks(b, dev))
    N = 96
    z = torch.randn(1, N, N, 128, generator=gen).to(dev)
    mask = torch.ones(1, N, N, device=dev)
    mask[0, -5:, :] = 0
    mask[0, :, -5:] = 0
    with torch.no_grad():
        got = net(z, mask)
    ref = z
    for b in blocks:
        ref = oracle_layer(ref, mask, b, heads=4, chunk_rows=32)
    torch.cuda.synchronize()
    assert_parity(got, ref, what="PairTransformNet(128, 2) defaults")
    assert_status_clean(dev)


def to_dev_blocks(b, dev):
    return {k: to_dev(p, dev) for k, p in b.items()}


def _rel(a, b):
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


@pytest.mark.parametrize("op,c_z,c,H", [("trimul_out", 64, 32, 0), ("triatt_end", 64, 32, 4),
                                        ("triatt_start", 128, 32, 4)])
def test_general_shape_gradients_match_oracle(op, c_z, c, H):
    """Training through a general-shape block: the forward on the kernels, the backward
    through the library's recomputation, against the oracle's fp32 autograd."""
    dev = require_gpu()
    gen = torch.Generator().manual_seed(c_z + c + H)
    B, N = 1, 40
    z = torch.randn(B, N, N, c_z, generator=gen).to(dev)
    mask = torch.ones(B, N, N, device=dev)
    mask[0, -4:, :] = 0
    w = torch.randn(B, N, N, c_z, generator=gen).to(dev)
    params = to_dev(O.make_trimul_params(c_z, c, gen, gate_bias=1.0) if op.startswith("trimul")
                    else O.make_triatt_params(c_z, c, H, gen, gate_bias=1.0), dev)
    mod = _module(op, c_z, c, H, dev)
    mod.load_state_dict(params)
    zz = z.clone().requires_grad_(True)
    out = mod(zz, mask)
    (out * w).sum().backward()
    pz = z.clone().requires_grad_(True)
    pp = {k: v.clone().requires_grad_(True) for k, v in params.items()}
    ref = _oracle(op, pz, mask, pp, H)
    grads = torch.autograd.grad((ref * w).sum(), [pz] + list(pp.values()))
    torch.cuda.synchronize()
    assert_status_clean(dev)
    assert_parity(out.detach(), ref.detach(), what=f"{op} forward under autograd")
    assert _rel(zz.grad, grads[0]) < 1e-2
    named = dict(mod.named_parameters())
    for k, g in zip(pp.keys(), grads[1:]):
        assert _rel(named[k].grad, g) < 1e-2, (k, _rel(named[k].grad, g))


@pytest.mark.parametrize("kind", ["trimul_out", "triatt_end"])
@pytest.mark.parametrize("c_z", [256, 200])
def test_dropout_wider_than_128_channels(kind, c_z):
    """Keep vectors of ceil(C / 128) 128-bit groups: C = 256 (two whole groups) and 200 (a
    partial second group), both dropout axes, the reference's own nn.Dropout draw packed
    (dropout_mask_from_multipliers) and the library's generator (dropout_mask_philox)."""
    dev = require_gpu()
    from genie_tk import ops
    B, N = 2, 37
    gen = torch.Generator().manual_seed(c_z + len(kind))
    z = torch.randn(B, N, N, c_z, generator=gen).to(dev)
    mask = torch.ones(B, N, N, device=dev)
    mask[-1, -3:, :] = 0
    params = to_dev(O.make_trimul_params(c_z, 32, gen, gate_bias=1.0) if kind.startswith("trimul")
                    else O.make_triatt_params(c_z, 32, 4, gen, gate_bias=1.0), dev)
    packed = ops.pack_trimul(params, dev) if kind.startswith("trimul") else ops.pack_triatt(params, dev, 4)
    upd = _oracle(kind, z, mask, params, 4)
    for rowwise in (True, False):
        shape = (B, 1, N, c_z) if rowwise else (B, N, 1, c_z)
        mult = (torch.rand(shape, generator=gen) > 0.3).float().to(dev) / 0.7
        drops = [(ops.dropout_mask_from_multipliers(mult, rowwise, 1 / 0.7), mult),
                 (ops.dropout_mask_philox(B, N, 0.3, seed=5, offset=int(rowwise), shared_across_rows=rowwise,
                                          device=dev, channels=c_z), None)]
        for drop, m in drops:
            assert tuple(drop.keep_bits.shape) == (B, N, 4 * ((c_z + 127) // 128))
            if m is None:
                bits = drop.keep_bits.cpu().numpy().view(np.uint32).reshape(-1, 4)
                m = D.multipliers_from_bits(bits, drop.scale, B, N, rowwise)[..., :c_z].to(dev)
            out = torch.empty_like(z)
            if kind.startswith("trimul"):
                ops.trimul_forward(z, mask, packed, True, out=out, add_residual=True, dropout=drop)
            else:
                ops.triatt_forward(z, mask, packed, False, out=out, add_residual=True, dropout=drop)
            torch.cuda.synchronize()
            assert_status_clean(dev)
            assert_parity(out, z + upd * m, what=f"{kind} c_z={c_z} dropout rowwise={rowwise}")
            dropped = (m == 0).expand_as(out)
            assert torch.equal(out[dropped], z[dropped])
