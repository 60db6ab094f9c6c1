"""GPU parity of the pair transition kernels (K5a + K5b through gtk_transition_forward) and of
PairTransformLayer, which now runs every one of its blocks on the library."""

import pytest
import torch

import genie_tk
from golden_util import load_transition
from gpu_util import assert_parity, assert_status_clean, require_gpu, to_dev
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


def test_transition_matches_reference_golden():
    dev = require_gpu()
    from genie_tk import ops
    z, mask, params, out = load_transition()
    packed = ops.pack_transition(to_dev(params, dev), dev)
    got = ops.transition_forward(z.to(dev), None, packed)
    torch.cuda.synchronize()
    assert_parity(got, out, what="transition golden")
    tail = ops.transition_forward(z.to(dev), mask.to(dev), packed, add_residual=True)
    assert_parity(tail, (z + out) * mask.unsqueeze(-1), what="transition golden, residual + mask")
    assert_status_clean(dev)


@pytest.mark.parametrize("B,N", [(1, 1), (1, 37), (2, 130), (1, 257)])
def test_transition_matches_oracle(B, N):
    dev = require_gpu()
    from genie_tk import ops
    gen = torch.Generator().manual_seed(1000 + N)
    z = 2.0 * torch.randn(B, N, N, 128, generator=gen) + 0.5
    mask = (torch.rand(B, N, N, generator=gen) > 0.25).float()
    params = O.make_transition_params(128, 4, gen)
    packed = ops.pack_transition(to_dev(params, dev), dev)
    zd = z.to(dev)
    got = ops.transition_forward(zd, None, packed)
    assert_status_clean(dev)  # a kernel that left early (timeout, bad launch) shows here first
    ref = O.transition_forward(z, params)
    d = (got.cpu() - ref).abs().amax(-1)
    bad = (d > 2e-2).nonzero()[:8].tolist()
    assert not bad, f"pairs (b, i, j) off by more than 2e-2: {bad} (of {int((d > 2e-2).sum())})"
    assert_parity(got, ref, what=f"transition N={N}")
    # in place: z = (z + transition(z)) * mask
    zz = zd.clone()
    ops.transition_forward(zz, mask.to(dev), packed, out=zz, add_residual=True)
    torch.cuda.synchronize()
    ref = O.layer_tail(z, mask, params)
    assert_parity(zz, ref, what=f"transition tail N={N}")
    assert float(zz.cpu()[mask == 0].abs().max()) == 0.0
    assert_status_clean(dev)


@pytest.mark.parametrize("n", [1, 2, 3])
def test_narrower_transition_runs_on_the_tuned_kernels(n):
    """c_p = 128 with an expansion n < 4: the hidden layer is zero-padded to 512 units in the
    packed weights (ReLU(0) = 0, zero W2 columns), so the result is the n-unit transition's."""
    dev = require_gpu()
    from genie_tk import ops
    gen = torch.Generator().manual_seed(70 + n)
    B, N = 1, 77
    z = torch.randn(B, N, N, 128, generator=gen)
    mask = (torch.rand(B, N, N, generator=gen) > 0.2).float()
    params = O.make_transition_params(128, n, gen)
    packed = ops.pack_transition(to_dev(params, dev), dev)
    zz = z.to(dev)
    ops.transition_forward(zz, mask.to(dev), packed, out=zz, add_residual=True)
    torch.cuda.synchronize()
    assert_parity(zz, O.layer_tail(z, mask, params), what=f"transition n={n}")
    assert_status_clean(dev)


def test_pair_transform_layer_matches_oracle():
    dev = require_gpu()
    B, N = 1, 64
    gen = torch.Generator().manual_seed(77)
    z = torch.randn(B, N, N, 128, generator=gen)
    mask = torch.ones(B, N, N)
    mask[:, -6:, :] = 0
    mask[:, :, -6:] = 0
    lp = {"tri_mul_out": O.make_trimul_params(128, 128, gen, gate_bias=1.0),
          "tri_mul_in": O.make_trimul_params(128, 128, gen, gate_bias=1.0),
          "tri_att_start": O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0),
          "tri_att_end": O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0)}
    tp = O.make_transition_params(128, 4, gen)
    layer = genie_tk.PairTransformLayer(c_p=128, c_hidden_mul=128, c_hidden_tri_att=128, n_head_tri=4).to(dev).eval()
    sd = {f"{blk}.{k}": v for blk, p in lp.items() for k, v in p.items()}
    sd.update({f"pair_transition.{k}": v for k, v in tp.items()})
    missing = set(layer.state_dict()) ^ set(sd)
    assert not missing, missing
    layer.load_state_dict(sd)
    with torch.no_grad():  # the fused in-place path
        got, _ = layer((z.to(dev), mask.to(dev)))
    tracked, _ = layer((z.to(dev), mask.to(dev)))  # parameters require grad: the autograd path
    torch.cuda.synchronize()
    ref = O.layer_tail(O.stack_forward(z, mask, [lp], no_heads=4), mask, tp)
    assert_parity(got, ref, what="PairTransformLayer")
    assert_parity(tracked, ref, what="PairTransformLayer under autograd")
    assert tracked.requires_grad
    assert_status_clean(dev)
