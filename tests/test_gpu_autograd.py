"""GPU checks of training support: gradients through the library's blocks against the
oracle's autograd (fp32, the reference math), the reference's own gradient-flow checks
(tests/test_triangle_mul.py:69-90, tests/test_triangle_attention.py:70-113: finite
gradients under masks), and a training step of PairTransformLayer with dropout.

The multiplicative update's backward contracts fp16 planes on the library's kernel and the
attention core runs forward and backward on fp16 tensor-core operands, so their gradients
are held to a relative L2 error of 1e-2; the transition and the embedding differentiate an
fp32 recomputation and are held to 1e-3 / 1e-4. A whole layer's gradients are evaluated at the
activations of the kernels' forward (bf16/fp16 operands, max-abs 2e-2 from fp32 per block)
rather than at the oracle's, and the five blocks compound that: 3e-2 there.
"""

import pytest
import torch

from gpu_util import assert_status_clean, require_gpu, to_dev
from oracle import dropout_oracle as D
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


def _rel(got, ref):
    got, ref = got.detach().float(), ref.detach().float()
    return float((got - ref).norm() / ref.norm().clamp_min(1e-30))


def _masked(B, N, gen):
    mask = torch.ones(B, N, N)
    mask[:, -3:, :] = 0
    mask[:, :, -2:] = 0
    return mask


@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("N", [24, 97])
def test_contraction_gradients_match_einsum(outgoing, N):
    dev = require_gpu()
    from genie_tk import autograd as AG
    gen = torch.Generator().manual_seed(N + int(outgoing))
    a = torch.randn(2, N, N, 128, generator=gen).to(dev).requires_grad_(True)
    b = torch.randn(2, N, N, 128, generator=gen).to(dev).requires_grad_(True)
    w = torch.randn(2, N, N, 128, generator=gen).to(dev) * 1e-6  # tiny gradients: scaling must keep them
    x = AG.contract(a, b, outgoing)
    ga, gb = torch.autograd.grad(x, [a, b], w)
    a2, b2 = a.detach().requires_grad_(True), b.detach().requires_grad_(True)
    eq = "bikc,bjkc->bijc" if outgoing else "bkic,bkjc->bijc"
    x2 = torch.einsum(eq, a2, b2)
    ga2, gb2 = torch.autograd.grad(x2, [a2, b2], w)
    assert _rel(x, x2) < 2e-3
    assert _rel(ga, ga2) < 2e-3 and _rel(gb, gb2) < 2e-3
    assert_status_clean(dev)


def _module_grads(mod, z, mask, w):
    zz = z.clone().requires_grad_(True)
    out = mod(zz, mask)
    grads = torch.autograd.grad((out * w).sum(), [zz] + list(mod.parameters()))
    return out, dict(zip(["z"] + [n for n, _ in mod.named_parameters()], grads))


def _oracle_grads(fn, params, z, w):
    zz = z.clone().requires_grad_(True)
    pp = {k: v.clone().requires_grad_(True) for k, v in params.items()}
    out = fn(zz, pp)
    grads = torch.autograd.grad((out * w).sum(), [zz] + list(pp.values()))
    return out, dict(zip(["z"] + list(pp.keys()), grads))


@pytest.mark.parametrize("outgoing", [True, False])
@pytest.mark.parametrize("N,B", [(48, 1), (77, 2)])
def test_trimul_gradients_match_oracle(outgoing, N, B):
    dev = require_gpu()
    import genie_tk
    gen = torch.Generator().manual_seed(3 * N + B)
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = _masked(B, N, gen).to(dev)
    w = torch.randn(B, N, N, 128, generator=gen).to(dev)
    params = to_dev(O.make_trimul_params(128, 128, gen, gate_bias=1.0), dev)
    cls = genie_tk.TriangleMultiplicationOutgoing if outgoing else genie_tk.TriangleMultiplicationIncoming
    mod = cls(128, 128).to(dev)
    mod.load_state_dict(params)
    out, g = _module_grads(mod, z, mask, w)
    ref, gr = _oracle_grads(lambda zz, pp: O.trimul_forward(zz, mask, pp, outgoing), params, z, w)
    torch.cuda.synchronize()
    assert_status_clean(dev)
    assert float((out - ref).detach().abs().max()) <= 2e-2
    for k, v in gr.items():
        assert _rel(g[k], v) < 1e-2, (k, _rel(g[k], v))


@pytest.mark.parametrize("starting", [True, False])
@pytest.mark.parametrize("N,B", [(40, 1), (67, 2)])
def test_triatt_gradients_match_oracle(starting, N, B):
    dev = require_gpu()
    import genie_tk
    gen = torch.Generator().manual_seed(5 * N + B + int(starting))
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = _masked(B, N, gen).to(dev)
    w = torch.randn(B, N, N, 128, generator=gen).to(dev)
    params = to_dev(O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0), dev)
    cls = genie_tk.TriangleAttentionStartingNode if starting else genie_tk.TriangleAttentionEndingNode
    mod = cls(128, 128, 4).to(dev)
    mod.load_state_dict(params)
    out, g = _module_grads(mod, z, mask, w)
    ref, gr = _oracle_grads(lambda zz, pp: O.triatt_forward(zz, mask, pp, starting, no_heads=4), params, z, w)
    torch.cuda.synchronize()
    assert_status_clean(dev)
    assert float((out - ref).detach().abs().max()) <= 2e-2
    for k, v in gr.items():
        assert _rel(g[k], v) < 1e-2, (k, _rel(g[k], v))


def _explicit_core(q, k, v, tri, mask, heads, inf=1e9):
    """o = softmax(q k^T / sqrt(d) + inf (mask - 1) + tri) v with explicit fp32 scores."""
    B, N, _, hd = q.shape
    d = hd // heads
    qh, kh, vh = (t.view(B, N, N, heads, d).transpose(-2, -3) for t in (q, k, v))
    s = torch.matmul(qh, kh.transpose(-1, -2)) * d ** -0.5 + tri[:, None]
    if mask is not None:
        s = s + (inf * (mask - 1.0))[:, :, None, None, :]
    return torch.matmul(torch.softmax(s, -1), vh).transpose(-2, -3).reshape(B, N, N, hd)


@pytest.mark.parametrize("B,N,H,d,with_mask,gscale", [(1, 70, 4, 32, True, 1.0), (2, 37, 4, 8, True, 1e-6),
                                                      (1, 130, 2, 64, False, 1.0), (1, 50, 3, 12, True, 3e4),
                                                      (1, 1, 1, 5, False, 1.0)])
def test_attention_core_kernels_match_explicit_scores(B, N, H, d, with_mask, gscale):
    """gtk_attn_core_forward / _backward against explicit fp32 scores and their autograd:
    ragged N (partial 64-row tiles, more than one tile, N = 1), head_dim 5 ... 64, fully
    masked rows, and output gradients scaled far from 1 (the kernels rescale them)."""
    dev = require_gpu()
    from genie_tk import ops
    gen = torch.Generator().manual_seed(N * 7 + d)
    q, k, v = (torch.randn(B, N, N, H * d, generator=gen).to(dev) for _ in range(3))
    tri = torch.randn(B, H, N, N, generator=gen).to(dev)
    mask = None
    if with_mask:
        mask = torch.ones(B, N, N)
        mask[:, -2:, :] = 0
        mask[:, :, -3:] = 0
        mask = mask.to(dev)
    do = (torch.randn(B, N, N, H * d, generator=gen) * gscale).to(dev)
    o, stats, pk = ops.attn_core_forward(q, k, v, tri, mask, H)
    dq, dk, dv, dtri = ops.attn_core_backward(pk, mask, stats, o, do)
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v, tri)]
    ref = _explicit_core(*leaves, mask, H)
    grads = torch.autograd.grad(ref, leaves, do)
    torch.cuda.synchronize()
    assert_status_clean(dev)
    assert _rel(o, ref) < 3e-3, _rel(o, ref)
    # with one key the softmax is constant and dq, dk, dtri are exactly zero: their error is
    # measured against a floor of 1e-2 of dv's norm (dv = do there) instead
    floor = 1e-2 * float(grads[2].norm())
    for name, a, b in zip(("dq", "dk", "dv", "dtri"), (dq, dk, dv, dtri), grads):
        assert torch.isfinite(a).all(), name
        err = float((a - b).norm())
        assert err < 1e-2 * max(float(b.norm()), floor), (name, _rel(a, b))


def test_transition_and_embedding_gradients_match_oracle():
    dev = require_gpu()
    import genie_tk
    gen = torch.Generator().manual_seed(31)
    B, N = 2, 33
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    w = torch.randn(B, N, N, 128, generator=gen).to(dev)
    tp = to_dev(O.make_transition_params(128, 4, gen), dev)
    tr = genie_tk.pair_transform.PairTransition(128, 4).to(dev)
    tr.load_state_dict(tp)
    _, g = _module_grads(tr, z, None, w)
    _, gr = _oracle_grads(lambda zz, pp: O.transition_forward(zz, pp), tp, z, w)
    for k, v in gr.items():
        assert _rel(g[k], v) < 1e-3, (k, _rel(g[k], v))
    c_s = 48
    s = torch.randn(B, N, c_s, generator=gen).to(dev).requires_grad_(True)
    m = (torch.rand(B, N, generator=gen) > 0.2).float().to(dev)
    emb = genie_tk.PairEmbedding(c_s, 128).to(dev)
    p, pm = emb(s, m)
    gs, gw, gb = torch.autograd.grad((p * w).sum(), [s, emb.weight, emb.bias])
    s2 = s.detach().clone().requires_grad_(True)
    ep = {"weight": emb.weight.detach().clone().requires_grad_(True),
          "bias": emb.bias.detach().clone().requires_grad_(True)}
    p2, pm2 = O.pair_embed(s2, m, ep)
    gs2, gw2, gb2 = torch.autograd.grad((p2 * w).sum(), [s2, ep["weight"], ep["bias"]])
    assert torch.equal(pm, pm2.to(pm.dtype))
    for a, b in ((gs, gs2), (gw, gw2), (gb, gb2)):
        assert _rel(a, b) < 1e-4
    assert_status_clean(dev)


def test_gradient_flow_under_masks_like_the_reference():
    """The reference's checks: gradients reach z, are finite, and a half-masked pair tensor
    gives finite outputs (test_triangle_mul.py:69-110, test_triangle_attention.py:70-113)."""
    dev = require_gpu()
    import genie_tk
    B, N = 1, 16
    z = torch.randn(B, N, N, 128, device=dev, requires_grad=True)
    mask = torch.ones(B, N, N, device=dev)
    mask[:, :, N // 2:] = 0
    for mod in (genie_tk.TriangleMultiplicationOutgoing(128, 128), genie_tk.TriangleMultiplicationIncoming(128, 128),
                genie_tk.TriangleAttentionStartingNode(128, 128, 4), genie_tk.TriangleAttentionEndingNode(128, 128, 4)):
        mod = mod.to(dev)
        z.grad = None
        out = mod(z, mask)
        out.sum().backward()
        assert z.grad is not None and torch.isfinite(z.grad).all() and torch.isfinite(out).all()
        assert all(p.grad is not None and torch.isfinite(p.grad).all() for p in mod.parameters())
    assert_status_clean(dev)


def test_pair_transform_layer_training_step_matches_oracle():
    """One training forward/backward of PairTransformLayer with dropout: the output and the
    gradients equal the oracle layer's, fed with the masks replayed from nn.Dropout."""
    dev = require_gpu()
    import genie_tk
    B, N, p_drop = 1, 40, 0.25
    gen = torch.Generator().manual_seed(77)
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = _masked(B, N, gen).to(dev)
    w = torch.randn(B, N, N, 128, generator=gen).to(dev)
    lp = {"tri_mul_out": O.make_trimul_params(128, 128, gen, gate_bias=1.0),
          "tri_mul_in": O.make_trimul_params(128, 128, gen, gate_bias=1.0),
          "tri_att_start": O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0),
          "tri_att_end": O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0),
          "pair_transition": O.make_transition_params(128, 4, gen)}
    layer = genie_tk.PairTransformLayer(c_p=128, c_hidden_mul=128, c_hidden_tri_att=128, n_head_tri=4,
                                        tri_dropout=p_drop).to(dev).train()
    layer.load_state_dict({f"{blk}.{k}": v for blk, p in lp.items() for k, v in p.items()})
    zz = z.clone().requires_grad_(True)
    torch.cuda.manual_seed(4321)
    out, _ = layer((zz, mask))
    (out * w).sum().backward()
    torch.cuda.synchronize()
    assert_status_clean(dev)
    torch.cuda.manual_seed(4321)
    drop = torch.nn.Dropout(p_drop).train()
    mults = [drop(torch.ones(B, 1, N, 128, device=dev)) for _ in range(3)]
    mults.append(drop(torch.ones(B, N, 1, 128, device=dev)))
    z2 = z.clone().requires_grad_(True)
    lp2 = {blk: {k: v.to(dev).requires_grad_(True) for k, v in p.items()} for blk, p in lp.items()}
    ref = D.pair_layer_forward(z2, mask, lp2, no_heads=4, drop_mults=mults)
    (ref * w).sum().backward()
    assert float((out - ref).detach().abs().max()) <= 2e-2
    assert _rel(zz.grad, z2.grad) < 3e-2
    named = dict(layer.named_parameters())
    for blk, p in lp2.items():
        for k, v in p.items():
            assert _rel(named[f"{blk}.{k}"].grad, v.grad) < 3e-2, (blk, k, _rel(named[f"{blk}.{k}"].grad, v.grad))


def test_bf16_model_trains_through_the_kernels():
    """A model converted with .to(torch.bfloat16) trains: the kernels take the fp32 copy of
    the pair tensor, the backward casts the bf16 parameters differentiably, and the
    gradients come back as bf16 close to the fp32 model's."""
    dev = require_gpu()
    import copy

    import genie_tk
    gen = torch.Generator().manual_seed(55)
    B, N = 1, 40
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = _masked(B, N, gen).to(dev)
    w = torch.randn(B, N, N, 128, generator=gen).to(dev)
    m1 = genie_tk.TriangleMultiplicationOutgoing(128, 128).to(dev)
    m1.load_state_dict(to_dev(O.make_trimul_params(128, 128, gen, gate_bias=1.0), dev))
    m2 = genie_tk.TriangleAttentionEndingNode(128, 128, 4).to(dev)
    m2.load_state_dict(to_dev(O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0), dev))
    for m32 in (m1, m2):
        m16 = copy.deepcopy(m32).to(torch.bfloat16)
        with torch.no_grad():  # compare at the same (bf16-rounded) weights
            for p16, p32 in zip(m16.parameters(), m32.parameters()):
                p32.copy_(p16.float())
        z32 = z.to(torch.bfloat16).float().requires_grad_(True)
        (m32(z32, mask) * w).sum().backward()
        z16 = z.to(torch.bfloat16).requires_grad_(True)
        out16 = m16(z16, mask)
        assert out16.dtype == torch.bfloat16
        (out16.float() * w).sum().backward()
        assert z16.grad.dtype == torch.bfloat16 and _rel(z16.grad, z32.grad) < 2e-2
        for p16, p32 in zip(m16.parameters(), m32.parameters()):
            assert p16.grad.dtype == torch.bfloat16
            assert _rel(p16.grad, p32.grad) < 2e-2
    assert_status_clean(dev)
