"""Triangle multiplicative update (AlphaFold2 Algorithms 11 & 12) on the B200 kernels.

Drop-in for src/genie_tk/triangle_mul.py of northws/Genie-TK: same class names,
constructor arguments, parameter names (``state_dict`` compatible) and
``forward(z, mask=None) -> update`` on pair tensors ``[B, N, N, c_z]``. The whole
forward (reference ``_forward_pytorch``, triangle_mul.py:103-132) runs as three sm_100a
kernels behind ``gtk_trimul_forward``; there is no PyTorch compute path here.
"""

from __future__ import annotations

from functools import partialmethod
from typing import Optional

import torch
import torch.nn as nn
from torch import Tensor

from . import autograd, ops
from .primitives import Linear


class _PackCache:
    """Packed fp16 weights, rebuilt when a parameter tensor or its version changes."""

    def __init__(self):
        self.key = None
        self.packed = None

    def get(self, module: nn.Module, build):
        params = list(module.parameters())
        key = tuple((p.data_ptr(), p._version, p.device) for p in params)
        if key != self.key:
            self.packed = build()
            self.key = key
        return self.packed


class TriangleMultiplicativeUpdate(nn.Module):
    """Triangle multiplicative update (reference triangle_mul.py:33-185).

    Args:
        c_z: pair channels
        c_hidden: hidden channels of the projections. c_z = c_hidden = 128 runs on the tuned
            kernels; every other shape up to 512 channels on the general-shape path
        _outgoing: Algorithm 11 (True) or 12 (False)
        use_fused_kernel: kept for signature compatibility; the fused kernels are the
            only implementation in this package
    """

    def __init__(self, c_z: int, c_hidden: int, _outgoing: bool = True, use_fused_kernel: bool = True):
        super().__init__()
        self.c_z = c_z
        self.c_hidden = c_hidden
        self._outgoing = _outgoing
        self.use_fused_kernel = use_fused_kernel
        self.linear_a_p = Linear(c_z, c_hidden)
        self.linear_a_g = Linear(c_z, c_hidden, init="gating")
        self.linear_b_p = Linear(c_z, c_hidden)
        self.linear_b_g = Linear(c_z, c_hidden, init="gating")
        self.linear_g = Linear(c_z, c_z, init="gating")
        self.linear_z = Linear(c_hidden, c_z, init="final")
        self.layer_norm_in = nn.LayerNorm(c_z)
        self.layer_norm_out = nn.LayerNorm(c_hidden)
        self.sigmoid = nn.Sigmoid()
        self._pack = _PackCache()

    def packed_weights(self, device: torch.device) -> Tensor:
        sd = {k: v for k, v in self.state_dict(keep_vars=True).items()}
        return self._pack.get(self, lambda: ops.pack_trimul(sd, device))

    def forward(self, z: Tensor, mask: Optional[Tensor] = None, *, out: Optional[Tensor] = None,
                add_residual: bool = False, dropout: Optional[ops.DropoutMask] = None) -> Tensor:
        """Return the update for ``z`` ``[B, N, N, c_z]`` (``mask`` ``[B, N, N]``).

        ``add_residual=True`` returns ``z + update`` (``out=z`` updates in place, fp32).
        ``dropout`` (an ``ops.DropoutMask``) multiplies the update by a training-mode channel
        dropout mask before the residual add, inside the kernel's epilogue.
        """
        if not z.is_cuda:
            raise RuntimeError("genie_tk (B200): TriangleMultiplicativeUpdate runs on CUDA tensors only")
        packed = self.packed_weights(z.device)
        if autograd.needs_grad(z, self):
            # training: the forward still runs on the kernels; the backward differentiates a
            # recomputation whose contractions run on the library's contraction kernel
            if out is not None or dropout is not None:
                raise RuntimeError("genie_tk (B200): out= and dropout= are inference-only; under autograd "
                                   "use the returned update (and nn.Dropout) instead")
            sd = dict(self.named_parameters())
            upd = autograd.TriMulFn.apply(z.float().contiguous(), mask, packed, self._outgoing,
                                          *[sd[k] for k in ops.TRIMUL_KEYS])
            res = z.float() + upd if add_residual else upd
            return res if res.dtype == z.dtype else res.to(z.dtype)
        if out is None and not add_residual and dropout is None:
            res = torch.ops.genie_tk.trimul_forward(z, mask, packed, self._outgoing)
        else:
            res = ops.trimul_forward(z, mask, packed, self._outgoing, out=out, add_residual=add_residual,
                                     dropout=dropout)
        return res if res.dtype == z.dtype or out is not None else res.to(z.dtype)


class TriangleMultiplicationOutgoing(TriangleMultiplicativeUpdate):
    """Algorithm 11: z_ij += sum_k a_ik * b_jk (reference triangle_mul.py:188-195)."""

    __init__ = partialmethod(TriangleMultiplicativeUpdate.__init__, _outgoing=True)


class TriangleMultiplicationIncoming(TriangleMultiplicativeUpdate):
    """Algorithm 12: z_ij += sum_k a_ki * b_kj (reference triangle_mul.py:198-205)."""

    __init__ = partialmethod(TriangleMultiplicativeUpdate.__init__, _outgoing=False)
