"""GPU parity of triangle attention (starting / ending node) through the C ABI."""

import math

import pytest
import torch

from golden_util import load_case
from gpu_util import assert_parity, assert_status_clean, require_gpu, to_dev
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu

LOG2E = 1.4426950408889634


def _oracle_intermediates(z, mask, p, starting, H=4):
    """q (scaled to log2 units), k, v, sigmoid gate, triangle bias (log2 units) and the gated
    attention output og, in the problem orientation (z^T for the ending node)."""
    x = z.float()
    m = mask.float()
    if not starting:
        x = x.transpose(1, 2)
        m = m.transpose(1, 2)
    x = O.layer_norm(x, p["layer_norm.weight"], p["layer_norm.bias"])
    B, N = x.shape[0], x.shape[1]
    d = 128 // H
    q = O.linear(x, p, "mha.linear_q").view(B, N, N, H, d).transpose(2, 3)
    k = O.linear(x, p, "mha.linear_k").view(B, N, N, H, d).transpose(2, 3)
    v = O.linear(x, p, "mha.linear_v").view(B, N, N, H, d).transpose(2, 3)
    g = torch.sigmoid(O.linear(x, p, "mha.linear_g"))
    tri = O.linear(x, p, "linear").permute(0, 3, 1, 2)
    s = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(d)
    s = s + (1e9 * (m - 1.0))[:, :, None, None, :] + tri[:, None]
    o = torch.matmul(torch.softmax(s, -1), v).transpose(2, 3).reshape(B, N, N, 128) * g
    return dict(q=q * LOG2E / math.sqrt(d), k=k, v=v, g=g, bias=tri * LOG2E, og=o)


@pytest.mark.parametrize("starting", [True, False])
def test_stages_match_oracle(starting):
    dev = require_gpu()
    from genie_tk import ops
    gen = torch.Generator().manual_seed(3)
    B, N = 1, 140
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = torch.ones(B, N, N, device=dev)
    mask[:, -9:, :] = 0
    mask[:, :, -7:] = 0
    mask[:, 5, :] = 0
    p = to_dev(O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0), dev)
    packed = ops.pack_triatt(p, dev, 4)
    ws, offs = ops.triatt_workspace(B, N, dev)
    ops.triatt_project(z, packed, starting, ws)
    ops.triatt_core(mask, starting, ws, B, N)
    torch.cuda.synchronize()
    got = ops.triatt_stage_views(ws, offs, B, N)
    ref = _oracle_intermediates(z, mask, p, starting)
    for name in ("q", "k", "v", "g"):
        assert_parity(got[name], ref[name], max_abs=1e-2, mean_abs=1e-3, what=name)
    # the bias is stored as bf16 (8-bit mantissa): bound it relative to its magnitude
    bias_err = (got["bias"][..., :N].float() - ref["bias"]).abs()
    assert (bias_err <= 2.0 ** -8 * ref["bias"].abs() + 1e-3).all(), float(bias_err.max())
    assert_parity(got["og"], ref["og"], max_abs=1e-2, mean_abs=1e-3, what="og")
    assert_status_clean(dev)


@pytest.mark.parametrize("name", ["triatt_start_c128", "triatt_end_c128"])
def test_module_matches_reference_golden(name):
    dev = require_gpu()
    import genie_tk
    op, dims, z, mask, params, out = load_case(name)
    cls = genie_tk.TriangleAttentionStartingNode if op == "triatt_start" else genie_tk.TriangleAttentionEndingNode
    mod = cls(dims["c_z"], dims["c_hidden"], dims["heads"]).to(dev)
    mod.load_state_dict(params)
    got = mod(z.to(dev), mask.to(dev))
    torch.cuda.synchronize()
    assert_parity(got, out, what=name)
    assert_status_clean(dev)


@pytest.mark.parametrize("cfg,N,starting", [(3, 96, True), (4, 96, False), (3, 200, False), (4, 257, True),
                                            (3, 512, True), (4, 384, False), (4, 768, False)])
def test_config_matches_oracle(cfg, N, starting):
    dev = require_gpu()
    import genie_tk
    z, mask, params = O.config_inputs(cfg, N=N)
    cls = genie_tk.TriangleAttentionStartingNode if starting else genie_tk.TriangleAttentionEndingNode
    mod = cls(128, 128, 4).to(dev)
    mod.load_state_dict(params)
    zd, md = z.to(dev), mask.to(dev)
    got = mod(zd, md)
    ref = O.triatt_forward(zd, md, to_dev(params, dev), starting=starting, no_heads=4, chunk_rows=64)
    assert_parity(got, ref, what=f"cfg{cfg} N={N}")
    z2 = zd.clone()
    with torch.no_grad():  # the in-place residual is a graph-less kernel call
        mod(z2, md, out=z2, add_residual=True)
    assert_parity(z2, zd + ref, what="residual in place")
    assert_status_clean(dev)


def test_no_mask_and_batch():
    dev = require_gpu()
    import genie_tk
    gen = torch.Generator().manual_seed(9)
    z = torch.randn(2, 64, 64, 128, generator=gen).to(dev)
    p = O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0, ln_random=True, bias_random=True)
    mod = genie_tk.TriangleAttentionEndingNode(128, 128, 4).to(dev)
    mod.load_state_dict(p)
    got = mod(z)
    ref = O.triatt_forward(z, None, to_dev(p, dev), starting=False, no_heads=4)
    assert_parity(got, ref, what="no mask, B=2")
    assert_status_clean(dev)
