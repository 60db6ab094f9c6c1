"""Known answers and edge cases through the kernels, derived from the reference math
(src/genie_tk/triangle_mul.py:103-132, src/genie_tk/triangle_attention.py:100-143,
src/genie_tk/primitives.py:114-178). The same list is checked on the CPU oracle in
tests/test_oracle_golden.py, here on the B200:

* tiny pair grids, N = 1, 2, 3 and 8 (one partial tile everywhere), for all four blocks;
* an all-masked multiplicative update: a = b = 0, so x = 0 and LN_out(0) = beta_out, and the
  update is sigmoid(linear_g(LN_in(z))) * (beta_out W_z^T + b_z)
  (reference triangle_mul.py:114-132);
* linear_z = 0 gives sigmoid(...) * b_z; linear_o = 0 gives b_o (primitives.py:176);
* a fully masked attention row: every score is -1e9 plus terms that fp32 cannot resolve at
  that magnitude, so the softmax is uniform and the output is the plain average of v
  (triangle_attention.py:118, primitives.py:157-170);
* the ending node is the starting node of the transposed problem
  (triangle_attention.py:110-112, :140-141).
"""

import pytest
import torch

from gpu_util import assert_parity, assert_status_clean, require_gpu, to_dev
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


def _trimul(outgoing, params, dev):
    import genie_tk
    cls = genie_tk.TriangleMultiplicationOutgoing if outgoing else genie_tk.TriangleMultiplicationIncoming
    m = cls(128, 128).to(dev)
    m.load_state_dict(params)
    return m


def _triatt(starting, params, dev):
    import genie_tk
    cls = genie_tk.TriangleAttentionStartingNode if starting else genie_tk.TriangleAttentionEndingNode
    m = cls(128, 128, 4).to(dev)
    m.load_state_dict(params)
    return m


@pytest.mark.parametrize("N", [1, 2, 3, 8])
@pytest.mark.parametrize("B", [1, 2])
def test_tiny_grids_match_oracle(N, B):
    dev = require_gpu()
    gen = torch.Generator().manual_seed(10 * N + B)
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = (torch.rand(B, N, N, generator=gen) > 0.2).float().to(dev)
    with torch.no_grad():
        for outgoing in (True, False):
            p = to_dev(O.make_trimul_params(128, 128, gen, gate_bias=1.0), dev)
            got = _trimul(outgoing, p, dev)(z, mask)
            assert_parity(got, O.trimul_forward(z, mask, p, outgoing), what=f"trimul out={outgoing} N={N}")
        for starting in (True, False):
            p = to_dev(O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0), dev)
            got = _triatt(starting, p, dev)(z, mask)
            ref = O.triatt_forward(z, mask, p, starting, no_heads=4)
            assert_parity(got, ref, what=f"triatt start={starting} N={N}")
    assert_status_clean(dev)


@pytest.mark.parametrize("outgoing", [True, False])
def test_all_masked_trimul_is_the_gated_beta_projection(outgoing):
    dev = require_gpu()
    gen = torch.Generator().manual_seed(41)
    B, N = 1, 70
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = torch.zeros(B, N, N, device=dev)
    p = O.make_trimul_params(128, 128, gen, gate_bias=1.0)
    p["layer_norm_out.bias"] = 0.5 * torch.randn(128, generator=gen)
    p = to_dev(p, dev)
    with torch.no_grad():
        got = _trimul(outgoing, p, dev)(z, mask)
    zn = O.layer_norm(z, p["layer_norm_in.weight"], p["layer_norm_in.bias"])
    gate = torch.sigmoid(O.linear(zn, p, "linear_g"))
    y = p["layer_norm_out.bias"] @ p["linear_z.weight"].t() + p["linear_z.bias"]
    assert_parity(got, gate * y, what="all-masked trimul")
    assert_status_clean(dev)


def test_zero_output_weights_give_the_output_biases():
    dev = require_gpu()
    gen = torch.Generator().manual_seed(42)
    B, N = 1, 50
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = torch.ones(B, N, N, device=dev)
    pm = O.make_trimul_params(128, 128, gen, gate_bias=1.0)
    pm["linear_z.weight"].zero_()
    pm["linear_z.bias"] = torch.randn(128, generator=gen)
    pm = to_dev(pm, dev)
    pa = O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0)
    pa["mha.linear_o.weight"].zero_()
    pa["mha.linear_o.bias"] = torch.randn(128, generator=gen)
    pa = to_dev(pa, dev)
    with torch.no_grad():
        got_m = _trimul(True, pm, dev)(z, mask)
        got_a = _triatt(True, pa, dev)(z, mask)
    zn = O.layer_norm(z, pm["layer_norm_in.weight"], pm["layer_norm_in.bias"])
    assert_parity(got_m, torch.sigmoid(O.linear(zn, pm, "linear_g")) * pm["linear_z.bias"], what="W_z = 0")
    assert float((got_a - pa["mha.linear_o.bias"]).abs().max()) == 0.0
    assert_status_clean(dev)


@pytest.mark.parametrize("starting", [True, False])
def test_fully_masked_attention_is_the_average_of_v(starting):
    dev = require_gpu()
    gen = torch.Generator().manual_seed(43 + int(starting))
    B, N = 1, 90
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = torch.zeros(B, N, N, device=dev)
    p = to_dev(O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0), dev)
    with torch.no_grad():
        got = _triatt(starting, p, dev)(z, mask)
    x = z if starting else z.transpose(1, 2)
    xn = O.layer_norm(x, p["layer_norm.weight"], p["layer_norm.bias"])
    v = O.linear(xn, p, "mha.linear_v")                               # [B, i, k, H*d]
    vbar = v.mean(dim=2, keepdim=True).expand_as(v)                   # uniform over the keys of row i
    upd = O.linear(vbar * torch.sigmoid(O.linear(xn, p, "mha.linear_g")), p, "mha.linear_o")
    if not starting:
        upd = upd.transpose(1, 2)
    assert_parity(got, upd, what=f"fully masked start={starting}")
    assert_parity(got, O.triatt_forward(z, mask, p, starting, no_heads=4), what="vs oracle")
    assert_status_clean(dev)


def test_ending_node_is_the_starting_node_of_the_transpose():
    dev = require_gpu()
    gen = torch.Generator().manual_seed(44)
    B, N = 2, 131
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = (torch.rand(B, N, N, generator=gen) > 0.1).float().to(dev)
    p = to_dev(O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0), dev)
    with torch.no_grad():
        end = _triatt(False, p, dev)(z, mask)
        start_t = _triatt(True, p, dev)(z.transpose(1, 2).contiguous(), mask.transpose(1, 2).contiguous())
    assert torch.allclose(end, start_t.transpose(1, 2), rtol=0, atol=1e-5)
    assert_status_clean(dev)
