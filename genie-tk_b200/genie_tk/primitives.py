"""Parameter-holding building blocks with the reference's names and initialisers.

Mirrors src/genie_tk/primitives.py of northws/Genie-TK: ``Linear`` with the AF2
initialisers (default / final / gating / normal, primitives.py:17-40) and the gated
multi-head ``Attention`` (primitives.py:65-178). The parameter names are identical so
reference ``state_dict``s load unchanged. Inside the triangle blocks the attention runs
fused in their own kernels; called on its own, ``Attention.forward`` runs its projections
on the library's linear kernel (``gtk_linear``, the gate fused into the output
projection's operand load) and the attention core on the tensor-core kernel
(``gtk_mha_forward``), which reads the biases in place through broadcast strides.
"""

from __future__ import annotations

import math
from typing import List, Optional

import torch
import torch.nn as nn
from torch import Tensor

from . import ops


def _init_weights(linear: nn.Linear, init: str = "default", std: float = 0.02) -> None:
    """AF2 initialisers, same semantics as primitives.py:17-40 of the reference."""
    if init == "default":
        nn.init.kaiming_uniform_(linear.weight, a=math.sqrt(5))
        if linear.bias is not None:
            fan_in = linear.weight.shape[1]
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(linear.bias, -bound, bound)
    elif init == "final":
        nn.init.zeros_(linear.weight)
        if linear.bias is not None:
            nn.init.zeros_(linear.bias)
    elif init == "gating":
        nn.init.zeros_(linear.weight)
        if linear.bias is not None:
            nn.init.ones_(linear.bias)
    elif init == "normal":
        nn.init.normal_(linear.weight, std=std)
        if linear.bias is not None:
            nn.init.zeros_(linear.bias)
    else:
        raise ValueError(f"unknown init {init!r}")


class Linear(nn.Linear):
    """nn.Linear with an AF2 initialiser (reference primitives.py:43-62)."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, init: str = "default"):
        super().__init__(in_features, out_features, bias=bias)
        _init_weights(self, init)


def _attention_math(mod: "Attention", q_x: Tensor, k_x: Tensor, v_x: Tensor, biases: List[Tensor],
                    params: List[Tensor]) -> Tensor:
    """The reference's Attention.forward (primitives.py:114-178) in fp32 PyTorch ops; the
    differentiable recomputation behind the kernels' forward."""
    wq, wk, wv, wo, bo = params[:5]
    H, d = mod.no_heads, mod.head_dim
    q = q_x.float() @ wq.float().t()
    k = k_x.float() @ wk.float().t()
    v = v_x.float() @ wv.float().t()
    *batch, Q, _ = q.shape
    K = k.shape[-2]
    q = q.view(*batch, Q, H, d).transpose(-2, -3)
    k = k.view(*batch, K, H, d).transpose(-2, -3)
    v = v.view(*batch, K, H, d).transpose(-2, -3)
    a = torch.matmul(q, k.transpose(-1, -2)) * (1.0 / math.sqrt(d))
    for b in biases:
        a = a + b.float()
    o = torch.matmul(torch.softmax(a, dim=-1), v).transpose(-2, -3).reshape(*batch, Q, H * d)
    if mod.gating:
        wg, bg = params[5:7]
        o = o * torch.sigmoid(q_x.float() @ wg.float().t() + bg.float())
    return o @ wo.float().t() + bo.float()


def _attention_kernels(mod: "Attention", q_x: Tensor, k_x: Tensor, v_x: Tensor, biases: List[Tensor],
                       params: List[Tensor]) -> Tensor:
    """Attention.forward on the library's kernels (fp32 results)."""
    wq, wk, wv, wo, bo = (t.detach().float() for t in params[:5])
    qf, kf, vf = q_x.detach().float(), k_x.detach().float(), v_x.detach().float()
    q = ops.linear(qf, wq)
    k = ops.linear(kf, wk)
    v = ops.linear(vf, wv)
    o = ops.mha_forward(q, k, v, mod.no_heads, 1.0 / math.sqrt(mod.head_dim), [b.detach() for b in biases])
    gate = None
    if mod.gating:
        wg, bg = (t.detach().float() for t in params[5:7])
        gate = ops.linear(qf, wg, bg)
    return ops.linear(o, wo, bo, gate=gate)


class _AttentionFn(torch.autograd.Function):
    """Forward on the kernels; backward through the fp32 recomputation."""

    @staticmethod
    def forward(ctx, mod, n_bias, q_x, k_x, v_x, *rest):
        biases, params = list(rest[:n_bias]), list(rest[n_bias:])
        ctx.mod, ctx.n_bias = mod, n_bias
        ctx.save_for_backward(q_x, k_x, v_x, *rest)
        return _attention_kernels(mod, q_x, k_x, v_x, biases, params).to(q_x.dtype)

    @staticmethod
    def backward(ctx, dout):
        q_x, k_x, v_x, *rest = ctx.saved_tensors
        inputs = [q_x, k_x, v_x] + rest
        with torch.enable_grad():
            leaves = [t.detach().requires_grad_(t.requires_grad) for t in inputs]
            biases, params = leaves[3:3 + ctx.n_bias], leaves[3 + ctx.n_bias:]
            out = _attention_math(ctx.mod, leaves[0], leaves[1], leaves[2], biases, params)
            wanted = [t for t in leaves if t.requires_grad]
            got = iter(torch.autograd.grad(out, wanted, dout.float(), allow_unused=True) if wanted else [])
            grads = [next(got) if t.requires_grad else None for t in leaves]
        grads = [None if g is None else g.to(t.dtype) for g, t in zip(grads, inputs)]
        return (None, None, *grads)


class Attention(nn.Module):
    """Gated multi-head attention with additive biases (reference primitives.py:65-178).

    ``linear_q/k/v`` without bias, ``linear_o`` (init "final"), ``linear_g`` (init
    "gating"). ``forward(q_x [*, Q, c_q], k_x [*, K, c_k], v_x [*, K, c_v], biases)`` with
    each bias broadcastable to [*, H, Q, K] returns [*, Q, c_q] in q_x's dtype, computed on
    the library's kernels (CUDA tensors only; head_dim <= 64). Under autograd the backward
    differentiates an fp32 recomputation of the same math.
    """

    def __init__(self, c_q: int, c_k: int, c_v: int, c_hidden: int, no_heads: int, gating: bool = True):
        super().__init__()
        self.c_q = c_q
        self.c_k = c_k
        self.c_v = c_v
        self.c_hidden = c_hidden
        self.no_heads = no_heads
        self.gating = gating
        assert c_hidden % no_heads == 0
        self.head_dim = c_hidden // no_heads
        self.linear_q = Linear(c_q, c_hidden, bias=False)
        self.linear_k = Linear(c_k, c_hidden, bias=False)
        self.linear_v = Linear(c_v, c_hidden, bias=False)
        self.linear_o = Linear(c_hidden, c_q, init="final")
        if gating:
            self.linear_g = Linear(c_q, c_hidden, init="gating")
        self.sigmoid = nn.Sigmoid()
        self.softmax = nn.Softmax(dim=-1)

    def _params(self) -> List[Tensor]:
        ps = [self.linear_q.weight, self.linear_k.weight, self.linear_v.weight, self.linear_o.weight,
              self.linear_o.bias]
        if self.gating:
            ps += [self.linear_g.weight, self.linear_g.bias]
        return ps

    def forward(self, q_x: Tensor, k_x: Tensor, v_x: Tensor, biases: Optional[List[Tensor]] = None) -> Tensor:
        biases = [b for b in (biases or []) if b is not None]
        params = self._params()
        tracked = torch.is_grad_enabled() and any(t.requires_grad for t in [q_x, k_x, v_x] + biases + params)
        if tracked:
            return _AttentionFn.apply(self, len(biases), q_x, k_x, v_x, *biases, *params)
        return _attention_kernels(self, q_x, k_x, v_x, biases, params).to(q_x.dtype)
