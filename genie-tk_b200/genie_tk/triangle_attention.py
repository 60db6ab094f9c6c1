"""Triangle attention (AlphaFold2 Algorithms 13 & 14) on the B200 kernels.

Drop-in for src/genie_tk/triangle_attention.py of northws/Genie-TK: same class names,
constructor arguments (``c_hidden`` is the total hidden size, ``head_dim = c_hidden //
no_heads``), parameter names and ``forward(x, mask=None) -> update``. The forward
(reference ``_forward_pytorch``, triangle_attention.py:100-143 with primitives.py:114-178)
runs as three sm_100a kernels behind ``gtk_triatt_forward``: LN + projections, a
flash-style attention that never materialises the N^3 scores, and the gated output
projection. The ending node reads and writes the pair tensor transposed through its
TMA descriptors instead of copying it.
"""

from __future__ import annotations

from functools import partialmethod
from typing import Optional

import torch
import torch.nn as nn
from torch import Tensor

from . import autograd, ops
from .primitives import Attention, Linear
from .triangle_mul import _PackCache


class TriangleAttention(nn.Module):
    """Triangle attention (reference triangle_attention.py:34-199). c_in = c_hidden = 128 with
    4 heads runs on the tuned kernels; every other shape (c_hidden a multiple of the heads,
    head_dim <= 64, up to 32 heads and 512 channels) on the general-shape path."""

    def __init__(self, c_in: int, c_hidden: int, no_heads: int, starting: bool = True, inf: float = 1e9,
                 use_fused_kernel: bool = True):
        super().__init__()
        self.c_in = c_in
        self.c_hidden = c_hidden
        self.no_heads = no_heads
        self.starting = starting
        self.inf = inf
        self.use_fused_kernel = use_fused_kernel
        self.layer_norm = nn.LayerNorm(c_in)
        self.linear = Linear(c_in, no_heads, bias=False, init="normal")
        self.mha = Attention(c_q=c_in, c_k=c_in, c_v=c_in, c_hidden=c_hidden, no_heads=no_heads)
        self._pack = _PackCache()

    def packed_weights(self, device: torch.device) -> Tensor:
        sd = {k: v for k, v in self.state_dict(keep_vars=True).items()}
        return self._pack.get(self, lambda: ops.pack_triatt(sd, device, self.no_heads))

    def forward(self, x: Tensor, mask: Optional[Tensor] = None, *, out: Optional[Tensor] = None,
                add_residual: bool = False, dropout: Optional[ops.DropoutMask] = None) -> Tensor:
        """Return the update for ``x`` ``[B, N, N, c_in]`` (``mask`` ``[B, N, N]``).

        ``add_residual=True`` returns ``x + update`` (``out=x`` updates in place, fp32).
        ``dropout`` (an ``ops.DropoutMask``) multiplies the update by a training-mode channel
        dropout mask before the residual add, inside the kernel's epilogue.
        """
        if not x.is_cuda:
            raise RuntimeError("genie_tk (B200): TriangleAttention runs on CUDA tensors only")
        packed = self.packed_weights(x.device)
        if autograd.needs_grad(x, self):
            # training: forward on the kernels, backward through a recomputation whose
            # attention core runs forward and backward on the tensor-core kernels
            if out is not None or dropout is not None:
                raise RuntimeError("genie_tk (B200): out= and dropout= are inference-only; under autograd "
                                   "use the returned update (and nn.Dropout) instead")
            sd = dict(self.named_parameters())
            upd = autograd.TriAttFn.apply(x.float().contiguous(), mask, packed, self.starting, float(self.inf),
                                          self.no_heads, *[sd[k] for k in ops.TRIATT_KEYS])
            res = x.float() + upd if add_residual else upd
            return res if res.dtype == x.dtype else res.to(x.dtype)
        if out is None and not add_residual and dropout is None:
            res = torch.ops.genie_tk.triatt_forward(x, mask, packed, self.starting, float(self.inf))
        else:
            res = ops.triatt_forward(x, mask, packed, self.starting, inf=self.inf, out=out, add_residual=add_residual,
                                     dropout=dropout)
        return res if res.dtype == x.dtype or out is not None else res.to(x.dtype)


class TriangleAttentionStartingNode(TriangleAttention):
    """Algorithm 13 (reference triangle_attention.py:202-209)."""

    __init__ = partialmethod(TriangleAttention.__init__, starting=True)


class TriangleAttentionEndingNode(TriangleAttention):
    """Algorithm 14 (reference triangle_attention.py:212-219)."""

    __init__ = partialmethod(TriangleAttention.__init__, starting=False)
