"""CPU checks of the training support's host logic (genie_tk.autograd): the differentiable
recomputations against the oracle and its autograd, and the contraction-gradient
identities of the multiplicative update. The library's contraction kernel and attention
core are replaced here by PyTorch functions with the same contracts; the kernels
themselves are covered by tests/test_gpu_autograd.py."""

import pytest
import torch

from oracle import triangle_oracle as O


def _rel(a, b):
    return float((a.detach() - b.detach()).norm() / b.detach().norm().clamp_min(1e-30))


def _einsum_contract(p, tp, q, tq, outgoing):
    """The contract of autograd._contract in fp32 einsums: out(P, Q) or inc(P, Q), with
    P / Q pair-transposed first when asked."""
    if tp:
        p = p.transpose(1, 2)
    if tq:
        q = q.transpose(1, 2)
    eq = "bikc,bjkc->bijc" if outgoing else "bkic,bkjc->bijc"
    return torch.einsum(eq, p, q)


def _torch_attn_core(q, k, v, tri, mask, heads, inf):
    """The contract of autograd._attn_core with explicit scores: q, k, v [B, N(i), N(j), H*d],
    tri [B, H, N(j), N(k)], mask [B, N(i), N(k)] or None."""
    B, N, _, hd = q.shape
    d = hd // heads
    qh, kh, vh = (t.view(B, N, N, heads, d).transpose(-2, -3) for t in (q, k, v))  # [B, i, H, j, d]
    s = torch.matmul(qh, kh.transpose(-1, -2)) * d ** -0.5 + tri[:, None]
    if mask is not None:
        s = s + (inf * (mask - 1.0))[:, :, None, None, :]
    return torch.matmul(torch.softmax(s, -1), vh).transpose(-2, -3).reshape(B, N, N, hd)


@pytest.fixture
def AG(monkeypatch):
    from genie_tk import autograd
    monkeypatch.setattr(autograd, "_contract", _einsum_contract)
    monkeypatch.setattr(autograd, "_attn_core", _torch_attn_core)
    return autograd


def _case(seed, B=1, N=11):
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(B, N, N, 128, generator=gen, dtype=torch.float64).float()
    mask = torch.ones(B, N, N)
    mask[:, -2:, :] = 0
    mask[:, :, -3:] = 0
    w = torch.randn(B, N, N, 128, generator=gen)
    return gen, z, mask, w


@pytest.mark.parametrize("outgoing", [True, False])
def test_contraction_gradient_identities(AG, outgoing):
    gen, _, _, _ = _case(1)
    a = torch.randn(2, 9, 9, 16, generator=gen, requires_grad=True)
    b = torch.randn(2, 9, 9, 16, generator=gen, requires_grad=True)
    w = torch.randn(2, 9, 9, 16, generator=gen)
    ga, gb = torch.autograd.grad(AG.contract(a, b, outgoing), [a, b], w)
    eq = "bikc,bjkc->bijc" if outgoing else "bkic,bkjc->bijc"
    ga2, gb2 = torch.autograd.grad(torch.einsum(eq, a, b), [a, b], w)
    assert _rel(ga, ga2) < 1e-6 and _rel(gb, gb2) < 1e-6


@pytest.mark.parametrize("outgoing", [True, False])
def test_trimul_recompute_and_gradients_match_oracle(AG, outgoing):
    gen, z, mask, w = _case(2)
    p = O.make_trimul_params(128, 128, gen, gate_bias=1.0)
    z1 = z.clone().requires_grad_(True)
    p1 = {k: v.clone().requires_grad_(True) for k, v in p.items()}
    out = AG.trimul_recompute(z1, mask, p1, outgoing)
    g1 = torch.autograd.grad((out * w).sum(), [z1] + list(p1.values()))
    z2 = z.clone().requires_grad_(True)
    p2 = {k: v.clone().requires_grad_(True) for k, v in p.items()}
    ref = O.trimul_forward(z2, mask, p2, outgoing)
    g2 = torch.autograd.grad((ref * w).sum(), [z2] + list(p2.values()))
    assert float((out - ref).detach().abs().max()) < 1e-4
    for a, b in zip(g1, g2):
        assert _rel(a, b) < 1e-4


@pytest.mark.parametrize("starting", [True, False])
@pytest.mark.parametrize("c_in,c,H", [(128, 128, 4), (64, 32, 4)])
def test_attention_recompute_and_gradients_match_oracle(AG, starting, c_in, c, H):
    """The recomputation around the attention core (orientation, LayerNorm, projections,
    triangle bias, gate, output projection) and its gradients, against the oracle."""
    gen, z, mask, w = _case(3 + int(starting))
    z, w = z[..., :c_in].contiguous(), w[..., :c_in].contiguous()
    p = O.make_triatt_params(c_in, c, H, gen, gate_bias=1.0)
    zl = z.clone().requires_grad_(True)
    pl = {k: v.clone().requires_grad_(True) for k, v in p.items()}
    out = AG.triatt_recompute(zl, mask, pl, starting, H, 1e9)
    got = torch.autograd.grad((out * w).sum(), [zl] + list(pl.values()))
    z2 = z.clone().requires_grad_(True)
    p2 = {k: v.clone().requires_grad_(True) for k, v in p.items()}
    ref = O.triatt_forward(z2, mask, p2, starting, no_heads=H)
    g2 = torch.autograd.grad((ref * w).sum(), [z2] + list(p2.values()))
    assert float((out - ref).detach().abs().max()) < 1e-4
    for name, a, b in zip(["z"] + list(p), got, g2):
        assert a is not None, name
        assert _rel(a, b) < 1e-4, (name, _rel(a, b))


def test_transition_recompute_matches_oracle(AG):
    gen, z, _, w = _case(5)
    p = O.make_transition_params(128, 4, gen)
    out = AG.transition_recompute(z, p)
    assert float((out - O.transition_forward(z, p)).abs().max()) < 1e-4


def test_needs_grad_follows_autograd_state(AG):
    lin = torch.nn.Linear(2, 2)
    x = torch.zeros(2)
    assert AG.needs_grad(x, lin)
    with torch.no_grad():
        assert not AG.needs_grad(x, lin)
    for q in lin.parameters():
        q.requires_grad_(False)
    assert not AG.needs_grad(x, lin)
    assert AG.needs_grad(x.requires_grad_(True), lin)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_half_precision_parameters_get_gradients_in_their_dtype(AG, dtype):
    """A model converted to bf16 / fp16: the fp32 recomputations cast its parameters
    differentiably, so the gradients come back in the parameters' dtype and equal the fp32
    model's gradients evaluated at the rounded parameters."""
    gen, z, mask, w = _case(7, N=9)
    for kind in ("trimul", "triatt", "transition"):
        if kind == "trimul":
            p = O.make_trimul_params(128, 128, gen, gate_bias=1.0)
        elif kind == "triatt":
            p = O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0)
        else:
            p = O.make_transition_params(128, 4, gen)
        half = {k: v.to(dtype).requires_grad_(True) for k, v in p.items()}
        full = {k: v.detach().float().requires_grad_(True) for k, v in half.items()}
        grads = []
        for params in (half, full):
            leaves = list(params.values())
            if kind == "trimul":
                out = AG.trimul_recompute(z, mask, params, True)
            elif kind == "transition":
                out = AG.transition_recompute(z, params)
            else:
                out = AG.triatt_recompute(z, mask, params, True, 4, 1e9)
            grads.append(torch.autograd.grad((out * w).sum(), leaves))
        for gh, gf, t in zip(grads[0], grads[1], half.values()):
            assert gh.dtype == t.dtype, (kind, gh.dtype)
            assert _rel(gh.float(), gf) < 1e-2, (kind, _rel(gh.float(), gf))


def test_tf32_switch_restores_the_global_flag(AG, monkeypatch):
    """The recompute enables TF32 matmuls only inside its own scope, and not at all when
    RECOMPUTE_TF32 is off."""
    torch.backends.cuda.matmul.allow_tf32 = False
    with AG._Tf32():
        assert torch.backends.cuda.matmul.allow_tf32
    assert not torch.backends.cuda.matmul.allow_tf32
    monkeypatch.setattr(AG, "RECOMPUTE_TF32", False)
    with AG._Tf32():
        assert not torch.backends.cuda.matmul.allow_tf32
    assert not torch.backends.cuda.matmul.allow_tf32
