"""fp16 intermediates beyond +-65504 are reported, not silently clamped.

The tensor-core operands are fp16. For LayerNorm-normalised inputs and weights of the usual
1/fan_in scale every intermediate is far inside the fp16 range, and the parity tests run with
the status word clear. Weights scaled far beyond that push the a/b planes of the
multiplicative update, the q/k/v of attention or the transition's hidden rows past 65504;
the kernels then set GTK_STATUS_FP16_SATURATED in the caller's status word, so the caller
learns that the result is not the reference's.
"""

import pytest
import torch

from gpu_util import assert_status_clean, require_gpu, to_dev
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu

SATURATED = 0x40  # GTK_STATUS_FP16_SATURATED


def _status(dev):
    from genie_tk import ops
    return ops.check_status(dev)  # synchronises, returns and clears the word


@pytest.mark.parametrize("c_z,c", [(128, 128), (64, 32)])
@pytest.mark.parametrize("outgoing", [True, False])
def test_trimul_planes_beyond_fp16_range_are_reported(c_z, c, outgoing):
    dev = require_gpu()
    import genie_tk
    gen = torch.Generator().manual_seed(5)
    z = torch.randn(1, 40, 40, c_z, generator=gen).to(dev)
    p = O.make_trimul_params(c_z, c, gen, gate_bias=1.0)
    cls = genie_tk.TriangleMultiplicationOutgoing if outgoing else genie_tk.TriangleMultiplicationIncoming
    mod = cls(c_z, c).to(dev).eval()
    mod.load_state_dict(to_dev(p, dev))
    with torch.no_grad():
        mod(z)
    assert _status(dev) == 0, "normal weights must not saturate"
    big = dict(p)
    big["linear_a_p.weight"] = p["linear_a_p.weight"] * 3e4   # |a| ~ 3e4 * |xhat W| >> 65504
    mod.load_state_dict(to_dev(big, dev))
    with torch.no_grad():
        mod(z)
    assert _status(dev) & SATURATED


@pytest.mark.parametrize("c_in,c,H", [(128, 128, 4), (64, 32, 4)])
def test_attention_projections_beyond_fp16_range_are_reported(c_in, c, H):
    dev = require_gpu()
    import genie_tk
    gen = torch.Generator().manual_seed(6)
    z = torch.randn(1, 36, 36, c_in, generator=gen).to(dev)
    p = O.make_triatt_params(c_in, c, H, gen, gate_bias=1.0)
    p["mha.linear_v.weight"] = p["mha.linear_v.weight"] * 3e4
    mod = genie_tk.TriangleAttentionStartingNode(c_in, c, H).to(dev).eval()
    mod.load_state_dict(to_dev(p, dev))
    with torch.no_grad():
        mod(z)
    # both paths give the tensor cores v as fp16 (the tuned one from K3, the general one
    # through its fp16 operand planes): the clamp is reported
    assert _status(dev) & SATURATED


def test_transition_hidden_beyond_fp16_range_is_reported():
    dev = require_gpu()
    import genie_tk
    gen = torch.Generator().manual_seed(7)
    z = torch.randn(1, 30, 30, 128, generator=gen).to(dev)
    p = O.make_transition_params(128, 4, gen)
    p["linear_1.weight"] = p["linear_1.weight"] * 3e4
    mod = genie_tk.pair_transform.PairTransition(128, 4).to(dev).eval()
    mod.load_state_dict(to_dev(p, dev))
    with torch.no_grad():
        mod(z)
    assert _status(dev) & SATURATED
    assert_status_clean(dev)
