"""``genie_tk._C``: the reference's native module, same names, arguments and meaning, on the
B200 library.

The reference declares six functions in kernels/bindings.cpp:69-101 (module ``_C``). In the
reference the module never links: ``triangle_mul.py:134-169`` would call the two contraction
functions, ``triangle_attention.py:145-179`` falls back to PyTorch before calling the
attention ones, and the LayerNorm ones are not called at all. Code that imports
``genie_tk._C`` and calls these functions gets them here:

  triangle_mul_outgoing(a, b, mask)   x[b,i,j,c] = sum_k a[b,i,k,c] b[b,j,k,c]
  triangle_mul_incoming(a, b, mask)   x[b,i,j,c] = sum_k a[b,k,i,c] b[b,k,j,c]
      a, b [B, N, N, C] (bf16 in the reference's caller, already multiplied by the mask,
      triangle_mul.py:146-152); mask [B, N, N] (validated; like the reference kernel's, it
      does not enter x). Runs on the contraction kernel (fp16 operand planes scaled by
      their max-abs, fp32 accumulation). Returns a's dtype.
  triangle_attention_starting(q, k, v, bias, mask, scale)
      o[b,h,i,j,:] = sum_k softmax_k(scale q[b,h,i,j].k[b,h,i,k] + bias[b,h,j,k]
                                     + 1e9 (mask[b,i,k] - 1)) v[b,h,i,k,:]
      q, k, v [B, H, N, N, D] (triangle_attention.cuh:110-112), bias [B, H, N, N], mask
      [B, N, N]. The reference kernel's H = 4, D = 32 runs on the tuned tcgen05 attention
      core; any other H and D <= 64 on the tensor-core attention core of the training path
      (gtk_attn_core_forward). Returns q's dtype.
  triangle_attention_ending(q, k, v, bias, mask, scale)
      the same around the ending node: the starting form on q, k, v and mask with their two
      pair axes swapped, the result swapped back; bias is in the problem frame, as the
      reference computes it from the transposed pair tensor (triangle_attention.py:110-129).
  layernorm(x, gamma, beta, eps=1e-5)
      LayerNorm over the last axis (kernels/fused_layernorm/layernorm.cu:17-44), fp32.
  fused_layernorm_linear(x, gamma, beta, weight, bias=None, eps=1e-5)
      LayerNorm(x) @ weight (+ bias) with weight [D_in, D_out], the reference's layout
      (layernorm.cu:46-76), in one kernel (gtk_layernorm_linear): the rows are normalised
      as the GEMM loads them and never reach memory. fp32.

Errors are ``RuntimeError``, as the reference's TORCH_CHECKs raise. CUDA tensors only.
"""

from __future__ import annotations

import math
from typing import Optional

import torch
from torch import Tensor

from . import ops

_INF = 1e9  # the reference's mask constant (triangle_attention.py:118)
_LOG2E = 1.0 / math.log(2.0)


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise RuntimeError(f"genie_tk (B200) _C: {msg}")


def _cuda(t: Tensor, name: str) -> None:
    _check(isinstance(t, Tensor) and t.is_cuda, f"{name} must be a CUDA tensor")


def _contract(a: Tensor, b: Tensor, mask: Optional[Tensor], outgoing: bool) -> Tensor:
    _cuda(a, "a")
    _cuda(b, "b")
    _check(a.dim() == 4 and a.shape == b.shape and a.shape[1] == a.shape[2], "a and b must both be [B, N, N, C]")
    if mask is not None:
        _cuda(mask, "mask")
        _check(tuple(mask.shape) == tuple(a.shape[:3]), "mask must be [B, N, N]")
    with torch.no_grad():
        x = ops.pair_contract(a, False, b, False, outgoing)
    return x.to(a.dtype)


def triangle_mul_outgoing(a: Tensor, b: Tensor, mask: Optional[Tensor]) -> Tensor:
    """x[b,i,j,c] = sum_k a[b,i,k,c] b[b,j,k,c] (Algorithm 11's contraction)."""
    return _contract(a, b, mask, True)


def triangle_mul_incoming(a: Tensor, b: Tensor, mask: Optional[Tensor]) -> Tensor:
    """x[b,i,j,c] = sum_k a[b,k,i,c] b[b,k,j,c] (Algorithm 12's contraction)."""
    return _contract(a, b, mask, False)


def _attention(q: Tensor, k: Tensor, v: Tensor, bias: Tensor, mask: Optional[Tensor], scale: float,
               starting: bool) -> Tensor:
    for t, n in ((q, "q"), (k, "k"), (v, "v"), (bias, "bias")):
        _cuda(t, n)
    _check(q.dim() == 5 and q.shape == k.shape == v.shape, "q, k, v must be [B, H, N, N, D] of one shape")
    B, H, N, N2, D = q.shape
    _check(N == N2, "q, k, v must be [B, H, N, N, D]")
    _check(1 <= D <= 64, "the attention kernels support head dims up to 64")
    _check(tuple(bias.shape) == (B, H, N, N), "bias must be [B, H, N, N]")
    if mask is not None:
        _cuda(mask, "mask")
        _check(tuple(mask.shape) == (B, N, N), "mask must be [B, N, N]")
    if not starting:  # End(q, k, v, mask) = Start(q^T, k^T, v^T, mask^T)^T in the pair axes
        q, k, v = (t.transpose(2, 3) for t in (q, k, v))
        mask = None if mask is None else mask.transpose(1, 2)
    with torch.no_grad():
        if H == ops.SUPPORTED_HEADS and H * D == ops.SUPPORTED_C:
            o = _tuned_core(q, k, v, bias, mask, scale)
        else:
            # the training core's layout: [B, i, j, H*D] fp32; it divides q.k by sqrt(D)
            qf, kf, vf = (t.float().permute(0, 2, 3, 1, 4).reshape(B, N, N, H * D) for t in (q, k, v))
            qf = (qf * (float(scale) * math.sqrt(D))).contiguous()
            m = None if mask is None else mask.float().contiguous()
            of, _, _ = ops.attn_core_forward(qf, kf.contiguous(), vf.contiguous(), bias.float().contiguous(), m, H,
                                             _INF)
            o = of.view(B, N, N, H, D).permute(0, 3, 1, 2, 4)  # [B, H, i, j, D]
        if not starting:
            o = o.transpose(2, 3)
        return o.to(q.dtype).contiguous()


def _tuned_core(q: Tensor, k: Tensor, v: Tensor, bias: Tensor, mask: Optional[Tensor], scale: float) -> Tensor:
    """The starting-node core at H = 4, D = 32 on the tuned kernel; o [B, H, i, j, D] fp32."""
    B, H, N, _, D = q.shape
    ws, offs = ops.triatt_workspace(B, N, q.device)
    st = ops.triatt_stage_views(ws, offs, B, N)
    # the core's operand layout: q, k, v [B, i, H, j, D] fp16, q times scale * log2(e)
    # (the core's softmax is base 2); bias [B, H, j, k] bf16 in log2 units; gate = 1
    st["q"].copy_((q.float() * (float(scale) * _LOG2E)).permute(0, 2, 1, 3, 4))
    st["k"].copy_(k.permute(0, 2, 1, 3, 4))
    st["v"].copy_(v.permute(0, 2, 1, 3, 4))
    st["bias"][..., :N].copy_(bias.float() * _LOG2E)
    st["g"].fill_(1.0)
    m = None if mask is None else mask.float().contiguous()
    ops.triatt_core(m, True, ws, B, N, inf=_INF)
    return st["og"].view(B, N, N, H, D).permute(0, 3, 1, 2, 4).float()


def triangle_attention_starting(q: Tensor, k: Tensor, v: Tensor, bias: Tensor, mask: Optional[Tensor],
                                scale: float) -> Tensor:
    """Triangle attention around the starting node (Algorithm 13's attention core)."""
    return _attention(q, k, v, bias, mask, scale, True)


def triangle_attention_ending(q: Tensor, k: Tensor, v: Tensor, bias: Tensor, mask: Optional[Tensor],
                              scale: float) -> Tensor:
    """Triangle attention around the ending node (Algorithm 14's attention core)."""
    return _attention(q, k, v, bias, mask, scale, False)


def _layernorm_fp32(x: Tensor, gamma: Tensor, beta: Tensor, eps: float) -> Tensor:
    for t, n in ((x, "x"), (gamma, "gamma"), (beta, "beta")):
        _cuda(t, n)
    _check(x.dim() >= 1 and x.shape[-1] >= 1, "x must have a last axis")
    _check(gamma.numel() == x.shape[-1] and beta.numel() == x.shape[-1], "gamma and beta must match x's last axis")
    with torch.no_grad():
        return ops.layernorm(x, gamma, beta, eps)


def layernorm(x: Tensor, gamma: Tensor, beta: Tensor, eps: float = 1e-5) -> Tensor:
    """LayerNorm over the last axis, fp32 (the result has x's dtype)."""
    return _layernorm_fp32(x, gamma, beta, eps).to(x.dtype)


def fused_layernorm_linear(x: Tensor, gamma: Tensor, beta: Tensor, weight: Tensor, bias: Optional[Tensor] = None,
                           eps: float = 1e-5) -> Tensor:
    """LayerNorm(x) @ weight (+ bias), weight [D_in, D_out] as in the reference; one kernel."""
    for t, n in ((x, "x"), (gamma, "gamma"), (beta, "beta"), (weight, "weight")):
        _cuda(t, n)
    _check(x.dim() >= 1 and x.shape[-1] >= 1, "x must have a last axis")
    _check(gamma.numel() == x.shape[-1] and beta.numel() == x.shape[-1], "gamma and beta must match x's last axis")
    _check(weight.dim() == 2 and weight.shape[0] == x.shape[-1], "weight must be [D_in, D_out]")
    if bias is not None:
        _cuda(bias, "bias")
        _check(bias.numel() == weight.shape[1], "bias must have D_out elements")
    with torch.no_grad():
        out = ops.layernorm_linear(x.float(), gamma.float(), beta.float(), weight.float().t().contiguous(),
                                   None if bias is None else bias.float(), eps)
        return out.to(x.dtype)
