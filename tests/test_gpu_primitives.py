"""GPU checks of the reference's generic gated multi-head ``Attention`` module
(src/genie_tk/primitives.py:65-178) on the library's kernels: the projections on
``gtk_linear`` (the gate fused into the output projection's operand load) and the core on
``gtk_mha_forward`` (fp16 tensor-core operands, fp32 softmax), against the module's math
written out in fp32 PyTorch, with the biases the reference passes it -- a mask bias
[*, 1, 1, K] and a pair bias [*, H, Q, K] broadcast over batch axes -- and its gradients.
"""

import math

import pytest
import torch

from gpu_util import assert_status_clean, require_gpu

pytestmark = pytest.mark.gpu


def _rel(a, b):
    a, b = a.detach().float(), b.detach().float()
    return float((a - b).norm() / b.norm().clamp_min(1e-30))


def _definition(mod, q_x, k_x, v_x, biases):
    """primitives.py:124-178 in fp32."""
    H, d = mod.no_heads, mod.head_dim
    q = q_x @ mod.linear_q.weight.t()
    k = k_x @ mod.linear_k.weight.t()
    v = v_x @ mod.linear_v.weight.t()
    *batch, Q, _ = q.shape
    K = k.shape[-2]
    q = q.view(*batch, Q, H, d).transpose(-2, -3)
    k = k.view(*batch, K, H, d).transpose(-2, -3)
    v = v.view(*batch, K, H, d).transpose(-2, -3)
    a = torch.matmul(q, k.transpose(-1, -2)) / math.sqrt(d)
    for b in biases:
        a = a + b
    o = torch.matmul(torch.softmax(a, -1), v).transpose(-2, -3).reshape(*batch, Q, H * d)
    if mod.gating:
        o = o * torch.sigmoid(mod.linear_g(q_x))
    return mod.linear_o(o)


def _module(c_q, c_k, c_v, c_hidden, heads, gating, gen, dev):
    from genie_tk.primitives import Attention
    mod = Attention(c_q, c_k, c_v, c_hidden, heads, gating=gating)
    with torch.no_grad():
        for p in mod.parameters():  # the "final" / "gating" inits are zeros: use random weights
            p.copy_(torch.randn(p.shape, generator=gen) / math.sqrt(p.shape[-1]))
    return mod.to(dev)


@pytest.mark.parametrize("batch,Q,K,c_q,c_k,c_v,c_hidden,H,gating", [
    ((2, 3), 17, 29, 24, 20, 12, 32, 4, True),    # head_dim 8
    ((5,), 70, 70, 64, 64, 64, 64, 2, False),     # head_dim 32, two query tiles
    ((), 1, 130, 16, 8, 8, 48, 3, True),          # no batch axes, one query, head_dim 16
    ((1, 2, 2), 33, 65, 32, 32, 32, 128, 2, True),  # head_dim 64, three batch axes
])
def test_attention_matches_definition(batch, Q, K, c_q, c_k, c_v, c_hidden, H, gating):
    dev = require_gpu()
    gen = torch.Generator().manual_seed(Q * 31 + K)
    mod = _module(c_q, c_k, c_v, c_hidden, H, gating, gen, dev)
    q_x = torch.randn(*batch, Q, c_q, generator=gen).to(dev)
    k_x = torch.randn(*batch, K, c_k, generator=gen).to(dev)
    v_x = torch.randn(*batch, K, c_v, generator=gen).to(dev)
    keep = (torch.rand(*batch, 1, 1, K, generator=gen) > 0.2).float()
    keep[..., 0] = 1.0
    mask_bias = (1e9 * (keep - 1.0)).to(dev)
    pair_bias = torch.randn(*batch[:-1], 1, H, Q, K, generator=gen).to(dev) if batch else \
        torch.randn(H, Q, K, generator=gen).to(dev)
    biases = [mask_bias, pair_bias]
    with torch.no_grad():
        got = mod(q_x, k_x, v_x, biases=biases)
        ref = _definition(mod, q_x, k_x, v_x, biases)
    torch.cuda.synchronize()
    assert got.shape == ref.shape
    assert _rel(got, ref) < 3e-3, _rel(got, ref)
    assert float((got - ref).abs().max()) < 2e-2
    assert_status_clean(dev)


def test_attention_in_the_triangle_pattern():
    """The reference's starting-node call mha(x, x, x, biases=[mask_bias, triangle_bias])
    (triangle_attention.py:115-137): x [B, N, N, c], mask bias [B, N, 1, 1, N] and triangle
    bias [B, 1, H, N, N], both read in place through broadcast strides."""
    dev = require_gpu()
    gen = torch.Generator().manual_seed(11)
    B, N, c, H = 2, 45, 32, 4
    mod = _module(c, c, c, c, H, True, gen, dev)
    x = torch.randn(B, N, N, c, generator=gen).to(dev)
    mask = torch.ones(B, N, N)
    mask[1, :, -4:] = 0
    mask[0, -2:, :] = 0  # fully masked rows
    mask_bias = (1e9 * (mask - 1.0))[:, :, None, None, :].to(dev)
    tri = torch.randn(B, 1, H, N, N, generator=gen).to(dev)
    with torch.no_grad():
        got = mod(x, x, x, biases=[mask_bias, tri])
        ref = _definition(mod, x, x, x, [mask_bias, tri])
    torch.cuda.synchronize()
    assert _rel(got, ref) < 3e-3
    assert float((got - ref).abs().max()) < 2e-2
    assert_status_clean(dev)


def test_attention_gradients_match_definition():
    dev = require_gpu()
    gen = torch.Generator().manual_seed(5)
    mod = _module(24, 16, 16, 32, 4, True, gen, dev)
    q_x = torch.randn(3, 19, 24, generator=gen).to(dev).requires_grad_(True)
    kv = torch.randn(3, 23, 16, generator=gen).to(dev).requires_grad_(True)
    bias = torch.randn(3, 4, 19, 23, generator=gen).to(dev).requires_grad_(True)
    w = torch.randn(3, 19, 24, generator=gen).to(dev)
    out = mod(q_x, kv, kv, biases=[bias])
    grads = torch.autograd.grad((out * w).sum(), [q_x, kv, bias] + list(mod.parameters()))
    leaves = [t.detach().clone().requires_grad_(True) for t in (q_x, kv, bias)]
    ref = _definition(mod, leaves[0], leaves[1], leaves[1], [leaves[2]])
    rgrads = torch.autograd.grad((ref * w).sum(), leaves + list(mod.parameters()))
    torch.cuda.synchronize()
    assert _rel(out, ref) < 3e-3
    for a, b in zip(grads, rgrads):
        assert _rel(a, b) < 1e-4, _rel(a, b)  # the backward differentiates the fp32 math at the same inputs
    assert_status_clean(dev)


def test_linear_and_fused_layernorm_linear_match_torch():
    dev = require_gpu()
    from genie_tk import ops
    gen = torch.Generator().manual_seed(2)
    x = (2 * torch.randn(7, 9, 200, generator=gen) + 0.5).to(dev)
    gate = torch.randn(7, 9, 200, generator=gen).to(dev)
    w = (torch.randn(70, 200, generator=gen) / 200 ** 0.5).to(dev)
    b = torch.randn(70, generator=gen).to(dev)
    gamma = (1 + 0.1 * torch.randn(200, generator=gen)).to(dev)
    beta = (0.1 * torch.randn(200, generator=gen)).to(dev)
    ref_ln = torch.nn.functional.layer_norm(x, (200,), gamma, beta, 1e-5) @ w.t() + b
    assert float((ops.layernorm_linear(x, gamma, beta, w, b) - ref_ln).abs().max()) < 1e-4
    assert float((ops.linear(x, w, b) - (x @ w.t() + b)).abs().max()) < 1e-4
    assert float((ops.linear(x, w, None, gate=gate) - (x * torch.sigmoid(gate)) @ w.t()).abs().max()) < 1e-4
    assert_status_clean(dev)
