"""Pin the fp32 oracle against golden vectors produced by the reference's own modules."""

import pytest
import torch

from golden_util import (GENERAL_CASES, LAYER_CASES, SINGLE_CASES, load_case, load_layer, load_stack,
                         load_transition, oracle_layer, oracle_run)
from oracle import triangle_oracle as O


@pytest.mark.parametrize("name", SINGLE_CASES + GENERAL_CASES)
def test_oracle_matches_reference_golden(name):
    op, dims, z, mask, params, out = load_case(name)
    got = oracle_run(op, dims, z, mask, params)
    torch.testing.assert_close(got, out, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("name", ["triatt_start_c128", "triatt_end_small"])
def test_oracle_row_chunking_is_exact(name):
    op, dims, z, mask, params, out = load_case(name)
    full = oracle_run(op, dims, z, mask, params)
    chunked = oracle_run(op, dims, z, mask, params, chunk_rows=3)
    torch.testing.assert_close(chunked, full, rtol=1e-5, atol=1e-6)


def test_oracle_stack_matches_reference_golden():
    z, mask, layers, out = load_stack()
    got = O.stack_forward(z, mask, layers, no_heads=4)
    torch.testing.assert_close(got, out, rtol=1e-4, atol=5e-5)


def test_oracle_transition_matches_reference_golden():
    z, mask, params, out = load_transition()
    torch.testing.assert_close(O.transition_forward(z, params), out, rtol=1e-4, atol=2e-5)
    tail = O.layer_tail(z, mask, params)
    torch.testing.assert_close(tail, (z + out) * mask.unsqueeze(-1), rtol=1e-5, atol=1e-6)
    assert float(tail[mask == 0].abs().max()) == 0.0


def test_oracle_transition_c64_matches_reference_golden():
    z, mask, params, out = load_transition("gen_transition_c64")
    torch.testing.assert_close(O.transition_forward(z, params), out, rtol=1e-4, atol=2e-5)


@pytest.mark.parametrize("name", LAYER_CASES)
def test_oracle_pair_transform_layer_matches_reference_golden(name):
    """A whole PairTransformLayer of the reference (eval mode) at its default shapes and at the
    shapes of its own layer test: the four triangle blocks, the transition and the mask."""
    dims, z, mask, blocks, out = load_layer(name)
    got = oracle_layer(z, mask, blocks, dims["heads"])
    torch.testing.assert_close(got, out, rtol=1e-4, atol=5e-5)


def test_known_answers():
    """Known answers derived from the reference math (not from its suite)."""
    gen = torch.Generator().manual_seed(5)
    z = torch.randn(1, 6, 6, 32, generator=gen)
    p = O.make_trimul_params(32, 16, gen, ln_random=True, bias_random=True)
    # mask = 0 everywhere -> a = b = 0 -> x = 0 -> LN_out(0) = beta.
    out = O.trimul_forward(z, torch.zeros(1, 6, 6), p, outgoing=True)
    zn = O.layer_norm(z, p["layer_norm_in.weight"], p["layer_norm_in.bias"])
    g = torch.sigmoid(O.linear(zn, p, "linear_g"))
    expect = (p["layer_norm_out.bias"] @ p["linear_z.weight"].t() + p["linear_z.bias"]) * g
    torch.testing.assert_close(out, expect, rtol=1e-5, atol=1e-6)
    # linear_o = 0 -> attention update is exactly b_o.
    pa = O.make_triatt_params(32, 16, 4, gen, bias_random=True)
    pa["mha.linear_o.weight"].zero_()
    out = O.triatt_forward(z, None, pa, starting=True, no_heads=4)
    torch.testing.assert_close(out, pa["mha.linear_o.bias"].expand_as(out))
    # ending node == starting node on the transposed pair tensor, transposed back.
    pa = O.make_triatt_params(32, 16, 4, gen, bias_random=True)
    m = (torch.rand(1, 6, 6, generator=gen) > 0.3).float()
    e = O.triatt_forward(z, m, pa, starting=False, no_heads=4)
    s = O.triatt_forward(z.transpose(1, 2), m.transpose(1, 2), pa, starting=True, no_heads=4).transpose(1, 2)
    torch.testing.assert_close(e, s)


def test_fully_masked_row_is_uniform_average():
    """All keys of row i masked: softmax over -1e9-shifted scores is uniform (fp32 absorbs the logits)."""
    gen = torch.Generator().manual_seed(6)
    z = torch.randn(1, 5, 5, 32, generator=gen)
    pa = O.make_triatt_params(32, 16, 4, gen)
    m = torch.ones(1, 5, 5)
    m[0, 1, :] = 0
    x = O.layer_norm(z, pa["layer_norm.weight"], pa["layer_norm.bias"])
    v = O.linear(x, pa, "mha.linear_v")[0, 1]              # [J, HD] values of row 1
    o = v.mean(dim=0, keepdim=True).expand(5, -1)
    o = o * torch.sigmoid(O.linear(x[0, 1], pa, "mha.linear_g"))
    expect = O.linear(o, pa, "mha.linear_o")
    got = O.triatt_forward(z, m, pa, starting=True, no_heads=4)[0, 1]
    torch.testing.assert_close(got, expect, rtol=1e-5, atol=1e-5)


def test_flop_model():
    assert O.flops_per_pair("layer", 1024) == 1536 * 1024 + 722944
