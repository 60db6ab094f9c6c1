"""GPU parity of the training-mode dropout folded into the residual epilogues.

The reference applies DropoutRowwise / DropoutColumnwise (src/genie_tk/pair_transform.py:26-61)
to each triangle update before its residual add (:182-189). The kernels take the mask as
keep bits; these tests check the bit generators bit-exactly against the oracle, each block's
``z + dropout(update)`` against the oracle for both mask axes and both block orientations,
and that a seeded training-mode PairTransformLayer draws exactly the masks the reference's
own nn.Dropout calls draw.
"""

import numpy as np
import pytest
import torch

from gpu_util import assert_parity, assert_status_clean, require_gpu, to_dev
from oracle import dropout_oracle as D
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


def _bits_np(mask) -> np.ndarray:
    return mask.keep_bits.cpu().numpy().view(np.uint32).reshape(-1, 4)


@pytest.mark.parametrize("seed,offset,p,n", [(0, 0, 0.25, 1), (1234, 7, 0.25, 3000),
                                             (2**40 + 17, 2**33 + 5, 0.1, 1025), (99, 0, 0.0, 64),
                                             (5, 3, 0.999, 200)])
def test_philox_keep_bits_match_oracle(seed, offset, p, n):
    dev = require_gpu()
    from genie_tk import ops
    m = ops.dropout_mask_philox(1, n, p, seed, offset, shared_across_rows=True, device=dev)
    torch.cuda.synchronize()
    got = _bits_np(m)
    ref = D.keep_bits_philox(seed, offset, p, n)
    assert np.array_equal(got, ref), "Philox keep bits differ from the oracle"
    assert m.scale == pytest.approx(1.0 / (1.0 - p))


def test_pack_keep_bits_match_oracle():
    dev = require_gpu()
    from genie_tk import ops
    gen = torch.Generator().manual_seed(3)
    B, N = 2, 37
    for rowwise in (True, False):
        keep = torch.rand(B, N, 128, generator=gen) > 0.3
        mult = keep.float() * (1 / 0.7)
        mult = mult.unsqueeze(1) if rowwise else mult.unsqueeze(2)
        m = ops.dropout_mask_from_multipliers(mult.to(dev), shared_across_rows=rowwise, scale=1 / 0.7)
        torch.cuda.synchronize()
        assert np.array_equal(_bits_np(m), D.pack_keep(keep.reshape(-1, 128).numpy()))


def _block_case(kind, N, B, seed):
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(B, N, N, 128, generator=gen)
    mask = torch.ones(B, N, N)
    mask[:, -3:, :] = 0
    mask[:, :, -5:] = 0
    if kind.startswith("trimul"):
        params = O.make_trimul_params(128, 128, gen, gate_bias=1.0)
    else:
        params = O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0)
    return z, mask, params


def _oracle_update(kind, z, mask, params):
    if kind == "trimul_out":
        return O.trimul_forward(z, mask, params, outgoing=True)
    if kind == "trimul_in":
        return O.trimul_forward(z, mask, params, outgoing=False)
    return O.triatt_forward(z, mask, params, starting=(kind == "triatt_start"), no_heads=4)


def _run(kind, zd, md, packed, out, add_residual, dropout):
    from genie_tk import ops
    if kind.startswith("trimul"):
        return ops.trimul_forward(zd, md, packed, kind == "trimul_out", out=out, add_residual=add_residual,
                                  dropout=dropout)
    return ops.triatt_forward(zd, md, packed, kind == "triatt_start", out=out, add_residual=add_residual,
                              dropout=dropout)


def _pack(kind, p, dev):
    from genie_tk import ops
    return ops.pack_trimul(p, dev) if kind.startswith("trimul") else ops.pack_triatt(p, dev, 4)


@pytest.mark.parametrize("kind", ["trimul_out", "trimul_in", "triatt_start", "triatt_end"])
@pytest.mark.parametrize("rowwise", [True, False])
@pytest.mark.parametrize("N,B,add_residual", [(96, 1, True), (200, 2, True), (130, 1, False)])
def test_block_dropout_matches_oracle(kind, rowwise, N, B, add_residual):
    dev = require_gpu()
    from genie_tk import ops
    z, mask, params = _block_case(kind, N, B, seed=N + 3 * B + (7 if rowwise else 0))
    p = to_dev(params, dev)
    packed = _pack(kind, p, dev)
    drop = ops.dropout_mask_philox(B, N, 0.25, seed=N * 31 + B, offset=int(rowwise), shared_across_rows=rowwise,
                                   device=dev)
    zd, md = z.to(dev), mask.to(dev)
    out = torch.empty_like(zd)
    _run(kind, zd, md, packed, out, add_residual, drop)
    torch.cuda.synchronize()
    assert_status_clean(dev)
    mult = D.multipliers_from_bits(_bits_np(drop), drop.scale, B, N, rowwise).to(dev)
    upd = _oracle_update(kind, zd, md, p) * mult
    ref = zd + upd if add_residual else upd
    assert_parity(out, ref, what=f"{kind} rowwise={rowwise} N={N}")
    # dropped channels contribute exactly nothing
    dropped = (mult == 0).expand_as(out)
    base = zd if add_residual else torch.zeros_like(zd)
    assert torch.equal(out[dropped], base[dropped])


@pytest.mark.parametrize("kind", ["trimul_out", "triatt_end"])
def test_keep_all_with_unit_scale_equals_plain_forward(kind):
    dev = require_gpu()
    from genie_tk import ops
    B, N = 1, 72
    z, mask, params = _block_case(kind, N, B, seed=11)
    p = to_dev(params, dev)
    packed = _pack(kind, p, dev)
    zd, md = z.to(dev), mask.to(dev)
    keep = ops.DropoutMask(torch.full((B, N, 4), -1, dtype=torch.int32, device=dev), 1.0, True)
    plain = torch.empty_like(zd)
    dropped = torch.empty_like(zd)
    _run(kind, zd, md, packed, plain, True, None)
    _run(kind, zd, md, packed, dropped, True, keep)
    torch.cuda.synchronize()
    assert_status_clean(dev)
    # one rounding of the update product apart at most
    assert torch.allclose(plain, dropped, rtol=1e-6, atol=1e-6)


def _layer_params(gen):
    lp = {"tri_mul_out": O.make_trimul_params(128, 128, gen, gate_bias=1.0),
          "tri_mul_in": O.make_trimul_params(128, 128, gen, gate_bias=1.0),
          "tri_att_start": O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0),
          "tri_att_end": O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0),
          "pair_transition": O.make_transition_params(128, 4, gen)}
    sd = {f"{blk}.{k}": v for blk, p in lp.items() for k, v in p.items()}
    return lp, sd


def test_training_layer_draws_the_reference_masks():
    """Seeded training-mode PairTransformLayer == the oracle layer fed with the masks that the
    reference's four nn.Dropout calls draw from the same CUDA generator state."""
    dev = require_gpu()
    import genie_tk
    B, N, p_drop = 1, 80, 0.25
    gen = torch.Generator().manual_seed(2024)
    z = torch.randn(B, N, N, 128, generator=gen)
    mask = torch.ones(B, N, N)
    mask[:, -4:, :] = 0
    mask[:, :, -4:] = 0
    lp, sd = _layer_params(gen)
    layer = genie_tk.PairTransformLayer(c_p=128, c_hidden_mul=128, c_hidden_tri_att=128, n_head_tri=4,
                                        tri_dropout=p_drop).to(dev)
    layer.load_state_dict(sd)
    layer.train()
    zd, md = z.to(dev), mask.to(dev)
    torch.cuda.manual_seed(1234)
    with torch.no_grad():  # the fused path: masks applied inside the residual epilogues
        got, _ = layer((zd, md))
    torch.cuda.synchronize()
    assert_status_clean(dev)
    # replay the reference's draws: DropoutRowwise x3 then DropoutColumnwise (pair_transform.py:182-189)
    torch.cuda.manual_seed(1234)
    drop = torch.nn.Dropout(p_drop).train()
    mults = [drop(torch.ones(B, 1, N, 128, device=dev)) for _ in range(3)]
    mults.append(drop(torch.ones(B, N, 1, 128, device=dev)))
    ref = D.pair_layer_forward(zd, md, {k: to_dev(v, dev) for k, v in lp.items()}, no_heads=4, drop_mults=mults)
    assert_parity(got, ref, what="training-mode PairTransformLayer")
    # and the masks really drop: eval mode gives a clearly different result
    layer.eval()
    with torch.no_grad():
        ev, _ = layer((zd, md))
    assert float((ev - got).abs().max()) > 0.1


def test_training_layer_with_zero_dropout_equals_eval():
    dev = require_gpu()
    import genie_tk
    B, N = 1, 48
    gen = torch.Generator().manual_seed(5)
    z = torch.randn(B, N, N, 128, generator=gen)
    mask = torch.ones(B, N, N)
    _, sd = _layer_params(gen)
    layer = genie_tk.PairTransformLayer(c_p=128, c_hidden_mul=128, c_hidden_tri_att=128, n_head_tri=4,
                                        tri_dropout=0.0).to(dev)
    layer.load_state_dict(sd)
    zd, md = z.to(dev), mask.to(dev)
    with torch.no_grad():
        tr, _ = layer.train()((zd, md))
        ev, _ = layer.eval()((zd, md))
    torch.cuda.synchronize()
    assert torch.equal(tr, ev)
    assert_status_clean(dev)


def test_dropout_custom_ops_match_ops():
    dev = require_gpu()
    import genie_tk  # noqa: F401  (registers torch.ops.genie_tk)
    from genie_tk import ops
    B, N = 1, 64
    z, mask, params = _block_case("trimul_out", N, B, seed=8)
    p = to_dev(params, dev)
    packed = ops.pack_trimul(p, dev)
    drop = ops.dropout_mask_philox(B, N, 0.25, seed=1, offset=0, shared_across_rows=True, device=dev)
    zd, md = z.to(dev), mask.to(dev)
    a = zd.clone()
    torch.ops.genie_tk.trimul_residual_dropout_(a, md, packed, True, drop.keep_bits, drop.scale, True)
    b = ops.trimul_forward(zd, md, packed, True, add_residual=True, dropout=drop)
    tz, tmask, tparams = _block_case("triatt_end", N, B, seed=9)
    tp = to_dev(tparams, dev)
    tpacked = ops.pack_triatt(tp, dev, 4)
    cdrop = ops.dropout_mask_philox(B, N, 0.25, seed=2, offset=0, shared_across_rows=False, device=dev)
    c = tz.to(dev).clone()
    torch.ops.genie_tk.triatt_residual_dropout_(c, tmask.to(dev), tpacked, False, 1e9, cdrop.keep_bits, cdrop.scale,
                                                False)
    d = ops.triatt_forward(tz.to(dev), tmask.to(dev), tpacked, False, add_residual=True, dropout=cdrop)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(c, d)
    assert_status_clean(dev)


@pytest.mark.parametrize("kind", ["trimul_out", "triatt_end"])
def test_dropout_epilogue_cost_is_small(kind):
    """The dropout instantiation of the residual epilogue reads 16 bytes of keep bits per pair
    (L2-resident) beside the 1 KB of residual traffic: the op may not slow down by more than
    10% at the benchmark size (the timings are printed, and appended as JSON lines to the
    file GTK_TIMING_JSON names)."""
    import json
    import os
    dev = require_gpu()
    from genie_tk import ops
    B, N = 1, 1024
    z, mask, params = _block_case(kind, N, B, seed=21)
    p = to_dev(params, dev)
    packed = _pack(kind, p, dev)
    zd, md = z.to(dev), mask.to(dev)
    drop = ops.dropout_mask_philox(B, N, 0.25, seed=3, offset=0, shared_across_rows=(kind != "triatt_end"),
                                   device=dev)
    out = torch.empty_like(zd)

    def timed(d):
        for _ in range(2):
            _run(kind, zd, md, packed, out, True, d)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(5):
            _run(kind, zd, md, packed, out, True, d)
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / 5

    t_plain = min(timed(None) for _ in range(2))
    t_drop = min(timed(drop) for _ in range(2))
    assert_status_clean(dev)
    row = {"case": f"{kind} N={N} residual", "plain_ms": round(t_plain, 4), "dropout_ms": round(t_drop, 4),
           "overhead": round(t_drop / t_plain - 1, 4)}
    print(json.dumps(row))
    if os.environ.get("GTK_TIMING_JSON"):
        with open(os.environ["GTK_TIMING_JSON"], "a") as f:
            f.write(json.dumps(row) + "\n")
    assert t_drop <= 1.10 * t_plain
