"""Training support: autograd for the blocks whose forward runs on the library's kernels.

The reference trains through PyTorch autograd over its PyTorch path (its only working
path; the gradient tests are tests/test_triangle_mul.py:69-90 and
tests/test_triangle_attention.py:70-113). Here every forward still runs on the library's
kernels. Each block is a ``torch.autograd.Function`` whose backward differentiates a
recomputation of the block's math on the GPU:

* Triangle multiplicative update (triangle_mul.py:103-132): the per-pair parts
  (LayerNorms, gated projections, output gate, all O(N^2)) are recomputed with PyTorch
  ops, and the two O(N^3) contractions of the backward, plus the one of the recompute,
  run on the library's tcgen05 contraction kernel (``gtk_trimul_contract``). The
  contraction's gradients are again contractions of the same two kinds:
    outgoing  X = out(A, B):  dA = inc(dX^T, B),  dB = inc(dX, A)
    incoming  X = inc(A, B):  dA = out(B, dX),    dB = out(A, dX^T)
  where out(P, Q)[i,j] = sum_k P[i,k] Q[j,k], inc(P, Q)[i,j] = sum_k P[k,i] Q[k,j] and
  ^T swaps the two pair axes. Operands go to the kernel as fp16 planes scaled by their
  own max-abs, so gradients of any magnitude keep 11 significant bits.
* Triangle attention (triangle_attention.py:100-143, primitives.py:114-178): the
  LayerNorm, the projections, the gate and the triangle bias are recomputed with PyTorch
  ops; the attention core between them runs forward and backward on the library's
  tensor-core kernels (``gtk_attn_core_forward`` / ``gtk_attn_core_backward``), which never
  form the [B, N, H, N, N] scores: dq, dk, dv and the triangle bias's gradient come
  straight from the kernels.
* Pair transition (pair_transform.py:78-84): recomputed and differentiated with
  PyTorch ops.

The recomputations are fp32. Their GEMMs in the multiplicative update and the attention
run on TF32 tensor cores while ``RECOMPUTE_TF32`` is true (the default): products with a
10-bit mantissa and fp32 accumulation, relative error ~1e-3 against fp32, where the
reference's bf16 autograd has ~1e-2. Set it to False for fp32 CUDA-core GEMMs. The
transition's recompute is always fp32. A block with no input or parameter that requires a
gradient never builds any of this: its forward is the plain kernel call.
"""

from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch
import torch.nn.functional as F
from torch import Tensor

from . import ops

LN_EPS = 1e-5

# TF32 tensor cores for the GEMMs of the multiplicative-update and attention recomputes
RECOMPUTE_TF32 = True


class _Tf32:
    """Enables TF32 matmuls for the enclosed recompute (when RECOMPUTE_TF32), then restores."""

    def __enter__(self):
        self._old = torch.backends.cuda.matmul.allow_tf32
        if RECOMPUTE_TF32:
            torch.backends.cuda.matmul.allow_tf32 = True
        return self

    def __exit__(self, *exc):
        torch.backends.cuda.matmul.allow_tf32 = self._old
        return False


def needs_grad(x: Tensor, module: torch.nn.Module) -> bool:
    """True when autograd must track a forward on ``x`` through ``module``."""
    return torch.is_grad_enabled() and (x.requires_grad or any(p.requires_grad for p in module.parameters()))


# --------------------------------------------------------------------------------------
# The N^3 contraction on the library's kernel
# --------------------------------------------------------------------------------------

# out(P, Q) / inc(P, Q) of fp32 pair tensors on the contraction kernel (module-level name,
# so that tests on the CPU can put an einsum with the same contract in its place)
_contract = ops.pair_contract


class _Contract(torch.autograd.Function):
    """x = out(a, b) (outgoing) or inc(a, b) (incoming), both operands fp32 [B, N, N, C]."""

    @staticmethod
    def forward(ctx, a: Tensor, b: Tensor, outgoing: bool) -> Tensor:
        ctx.save_for_backward(a, b)
        ctx.outgoing = outgoing
        return _contract(a, False, b, False, outgoing)

    @staticmethod
    def backward(ctx, dx: Tensor):
        a, b = ctx.saved_tensors
        dx = dx.contiguous()
        if ctx.outgoing:
            da = _contract(dx, True, b, False, outgoing=False) if ctx.needs_input_grad[0] else None
            db = _contract(dx, False, a, False, outgoing=False) if ctx.needs_input_grad[1] else None
        else:
            da = _contract(b, False, dx, False, outgoing=True) if ctx.needs_input_grad[0] else None
            db = _contract(a, False, dx, True, outgoing=True) if ctx.needs_input_grad[1] else None
        return da, db, None


def contract(a: Tensor, b: Tensor, outgoing: bool) -> Tensor:
    """Differentiable triangle contraction on the library's kernel (fp32 pair tensors)."""
    return _Contract.apply(a, b, outgoing)


# --------------------------------------------------------------------------------------
# Recomputations (the reference math, differentiable)
# --------------------------------------------------------------------------------------

def _linear(x: Tensor, p: Dict[str, Tensor], name: str) -> Tensor:
    return F.linear(x, p[name + ".weight"], p.get(name + ".bias"))


def _fp32(p: Dict[str, Tensor]) -> Dict[str, Tensor]:
    """The parameters as fp32 (a differentiable cast: a bf16 / fp16 model gets its gradients
    back in its own dtype)."""
    return {k: v.float() for k, v in p.items()}


def _mask_or_ones(z: Tensor, mask: Optional[Tensor]) -> Tensor:
    return torch.ones(z.shape[:-1], dtype=z.dtype, device=z.device) if mask is None else mask.to(z.dtype)


def _linear_cat(x: Tensor, p: Dict[str, Tensor], names: Sequence[str]) -> List[Tensor]:
    """The projections `names` of one input as one GEMM over their concatenated weights (the
    input is read once, and its gradient comes out of one GEMM instead of a sum of several);
    the results are views of the one output, in order."""
    ws = [p[n + ".weight"] for n in names]
    bs = [p.get(n + ".bias") for n in names]
    if all(b is None for b in bs):
        bias = None
    else:
        bias = torch.cat([b if b is not None else w.new_zeros(w.shape[0]) for w, b in zip(ws, bs)])
    y = F.linear(x, torch.cat(ws), bias)
    return list(torch.split(y, [w.shape[0] for w in ws], dim=-1))


def trimul_recompute(z: Tensor, mask: Optional[Tensor], p: Dict[str, Tensor], outgoing: bool) -> Tensor:
    """The update of the triangle multiplicative block (triangle_mul.py:103-132), fp32,
    with the contraction on the library's kernel."""
    p = _fp32(p)
    m = _mask_or_ones(z, mask).unsqueeze(-1)
    zn = F.layer_norm(z, (z.shape[-1],), p["layer_norm_in.weight"], p["layer_norm_in.bias"], LN_EPS)
    ap, ag, bp, bg, g = _linear_cat(zn, p, ["linear_a_p", "linear_a_g", "linear_b_p", "linear_b_g", "linear_g"])
    a = ap * torch.sigmoid(ag) * m
    b = bp * torch.sigmoid(bg) * m
    x = contract(a, b, outgoing)
    x = F.layer_norm(x, (x.shape[-1],), p["layer_norm_out.weight"], p["layer_norm_out.bias"], LN_EPS)
    return _linear(x, p, "linear_z") * torch.sigmoid(g)


class _AttnCore(torch.autograd.Function):
    """The attention core o = softmax(q k^T / sqrt(d) + inf (mask - 1) + tri) v on the
    library's kernels, with their backward. Keeps the fp16 operand planes of the forward
    (half the bytes of q, k, v) for the backward."""

    @staticmethod
    def forward(ctx, q, k, v, tri, mask, heads, inf):
        o, stats, pk = ops.attn_core_forward(q, k, v, tri, mask, heads, inf)
        ctx.save_for_backward(pk.q, pk.k, pk.v, pk.tri, mask, stats, o)
        ctx.dims, ctx.inf = (pk.B, pk.N, pk.heads, pk.head_dim), inf
        return o

    @staticmethod
    def backward(ctx, do):
        qh, kh, vh, th, mask, stats, o = ctx.saved_tensors
        pk = ops.AttnCorePacked(qh, kh, vh, th, *ctx.dims)
        dq, dk, dv, dtri = ops.attn_core_backward(pk, mask, stats, o, do, ctx.inf)
        return dq, dk, dv, dtri, None, None, None


def _native_attn_core(q: Tensor, k: Tensor, v: Tensor, tri: Tensor, mask: Optional[Tensor], heads: int,
                      inf: float) -> Tensor:
    return _AttnCore.apply(q, k, v, tri, mask, heads, inf)


# q, k, v [B, N(i), N(j), H*d], tri [B, H, N(j), N(k)], mask [B, N(i), N(k)] or None -> o like q
# (module-level name, so that tests on the CPU can put a PyTorch version in its place)
_attn_core = _native_attn_core


def triatt_recompute(z: Tensor, mask: Optional[Tensor], p: Dict[str, Tensor], starting: bool, heads: int,
                     inf: float) -> Tensor:
    """The update of the triangle attention block (triangle_attention.py:100-143), fp32, with
    the attention core on the library's kernels: orientation, LayerNorm, the projections
    q, k, v, g and the triangle bias [B, H, N, N] (one GEMM), the core, the gate and W_o."""
    p = _fp32(p)
    x, m = z, mask
    if not starting:
        x = x.transpose(-2, -3)
        m = None if m is None else m.transpose(-1, -2)
    xn = F.layer_norm(x, (x.shape[-1],), p["layer_norm.weight"], p["layer_norm.bias"], LN_EPS)
    q, k, v, g, tri = _linear_cat(xn, p, ["mha.linear_q", "mha.linear_k", "mha.linear_v", "mha.linear_g", "linear"])
    m = None if m is None else m.float().contiguous()
    o = _attn_core(q.contiguous(), k.contiguous(), v.contiguous(), tri.permute(0, 3, 1, 2).contiguous(), m, heads,
                   inf)
    o = o * torch.sigmoid(g)
    out = _linear(o, p, "mha.linear_o")
    return out if starting else out.transpose(-2, -3)


def transition_recompute(z: Tensor, p: Dict[str, Tensor]) -> Tensor:
    """PairTransition.forward (pair_transform.py:78-84) in fp32."""
    p = _fp32(p)
    x = F.layer_norm(z, (z.shape[-1],), p["layer_norm.weight"], p["layer_norm.bias"], LN_EPS)
    return _linear(torch.relu(_linear(x, p, "linear_1")), p, "linear_2")


# --------------------------------------------------------------------------------------
# Block functions: forward on the kernels, backward through the recomputation
# --------------------------------------------------------------------------------------

def _leaves(z: Tensor, params: Sequence[Tensor]):
    zl = z.detach().requires_grad_(z.requires_grad)
    pl = [t.detach().requires_grad_(t.requires_grad) for t in params]
    return zl, pl


def _grads(out: Tensor, zl: Tensor, pl: List[Tensor], dU: Tensor):
    wanted = [t for t in [zl] + pl if t.requires_grad]
    got = torch.autograd.grad(out, wanted, dU, allow_unused=True) if wanted else []
    it = iter(got)
    return [next(it) if t.requires_grad else None for t in [zl] + pl]


class TriMulFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z, mask, packed, outgoing, *params):
        ctx.save_for_backward(z, mask, *params)
        ctx.outgoing = outgoing
        return ops.trimul_forward(z, mask, packed, outgoing)

    @staticmethod
    def backward(ctx, dU):
        z, mask, *params = ctx.saved_tensors
        with torch.enable_grad(), _Tf32():
            zl, pl = _leaves(z.float(), params)
            out = trimul_recompute(zl, mask, dict(zip(ops.TRIMUL_KEYS, pl)), ctx.outgoing)
            g = _grads(out, zl, pl, dU.float())
        return (g[0], None, None, None, *g[1:])


class TriAttFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z, mask, packed, starting, inf, heads, *params):
        ctx.save_for_backward(z, mask, *params)
        ctx.starting, ctx.inf, ctx.heads = starting, inf, heads
        return ops.triatt_forward(z, mask, packed, starting, inf=inf)

    @staticmethod
    def backward(ctx, dU):
        z, mask, *params = ctx.saved_tensors
        with torch.enable_grad(), _Tf32():
            zl, pl = _leaves(z.float(), params)
            out = triatt_recompute(zl, mask, dict(zip(ops.TRIATT_KEYS, pl)), ctx.starting, ctx.heads, ctx.inf)
            g = _grads(out, zl, pl, dU.float())
        return (g[0], None, None, None, None, None, *g[1:])


class TransitionFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z, packed, *params):
        ctx.save_for_backward(z, *params)
        return ops.transition_forward(z, None, packed)

    @staticmethod
    def backward(ctx, dU):
        z, *params = ctx.saved_tensors
        with torch.enable_grad():
            zl, pl = _leaves(z.float(), params)
            out = transition_recompute(zl, dict(zip(ops.TRANSITION_KEYS, pl)))
            g = _grads(out, zl, pl, dU.float())
        return (g[0], None, *g[1:])


class PairEmbedFn(torch.autograd.Function):
    """p[b,i,j] = s_i W_a^T + s_j W_b^T + bias (examples/basic_usage.py:181-199) on the pair
    embedding kernels. With p = U_i + V_j the backward is closed-form and O(N^2 c):
    dU_i = sum_j dp_ij, dV_j = sum_i dp_ij, ds = dU W_a + dV W_b, dW = [dU^T s | dV^T s],
    dbias = sum dV. The pair mask carries no gradient."""

    @staticmethod
    def forward(ctx, s, mask, weight, bias):
        ctx.save_for_backward(s, weight)
        ctx.has_bias = bias is not None
        ctx.bias_dtype = None if bias is None else bias.dtype
        p, pm = ops.pair_embed(s, mask, weight, bias, with_mask=mask is not None)
        if pm is not None:
            ctx.mark_non_differentiable(pm)
        return p, pm

    @staticmethod
    def backward(ctx, dp, dpm):
        s, weight = ctx.saved_tensors
        c_s, c_p = s.shape[-1], weight.shape[0]
        dp = dp.float()
        du = dp.sum(2)  # [B, N(i), c_p]
        dv = dp.sum(1)  # [B, N(j), c_p]
        sf = s.float().reshape(-1, c_s)
        w = weight.float()
        ds = dw = db = None
        if ctx.needs_input_grad[0]:
            ds = (du @ w[:, :c_s] + dv @ w[:, c_s:]).to(s.dtype)
        if ctx.needs_input_grad[2]:
            dw = torch.cat([du.reshape(-1, c_p).t() @ sf, dv.reshape(-1, c_p).t() @ sf], dim=1).to(weight.dtype)
        if ctx.has_bias and ctx.needs_input_grad[3]:
            db = dv.sum((0, 1)).to(ctx.bias_dtype)
        return ds, None, dw, db
