"""Pair transform layer / network (reference src/genie_tk/pair_transform.py).

The four triangle blocks run on the B200 kernels with the residual add fused into
their epilogues (``add_residual=True``) whenever the residual can be taken in place.
``PairTransition`` (LN -> 4x expand -> ReLU -> project) runs on the two transition
kernels (``gtk_transition_forward``); inside ``PairTransformLayer`` its residual add and
the layer's final mask multiply are folded into the second one. In training mode the
row/column dropout of the four triangle updates is applied inside the same residual
epilogues: each mask is drawn with the reference's own ``nn.Dropout`` call (same shape,
dtype and generator, so a seeded run draws the reference's masks) and handed to the
kernels as keep bits.
"""

from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn
from torch import Tensor

from . import autograd, ops
from .primitives import Linear
from .triangle_attention import TriangleAttentionEndingNode, TriangleAttentionStartingNode
from .triangle_mul import TriangleMultiplicationIncoming, TriangleMultiplicationOutgoing, _PackCache


class _SharedDropout(nn.Module):
    """Dropout whose mask is shared along one pair axis (``_shared_dim``: -3 rows, -2 columns)."""

    _shared_dim = -3

    def __init__(self, p: float):
        super().__init__()
        self.p = p
        self.dropout = nn.Dropout(p)

    def _multipliers(self, shape, dtype: torch.dtype, device: torch.device) -> Tensor:
        shape = list(shape)
        shape[self._shared_dim] = 1
        return self.dropout(torch.ones(shape, dtype=dtype, device=device))

    def forward(self, x: Tensor) -> Tensor:
        if not self.training or self.p == 0:
            return x
        return x * self._multipliers(x.shape, x.dtype, x.device)

    def keep_mask(self, shape, dtype: torch.dtype, device: torch.device) -> Optional[ops.DropoutMask]:
        """The mask ``forward`` would draw for an update of ``shape`` / ``dtype`` (the same
        ``nn.Dropout`` call, so the same random numbers), as keep bits for the residual
        epilogues; None in eval mode or for p = 0."""
        if not self.training or self.p == 0:
            return None
        mult = self._multipliers(shape, dtype, device)
        scale = 0.0 if self.p >= 1 else float(torch.tensor(1.0 / (1.0 - self.p), dtype=torch.float64).to(dtype))
        return ops.dropout_mask_from_multipliers(mult, shared_across_rows=self._shared_dim == -3, scale=scale)


class DropoutRowwise(_SharedDropout):
    """Dropout with one mask shared across rows (reference pair_transform.py:26-42)."""

    _shared_dim = -3


class DropoutColumnwise(_SharedDropout):
    """Dropout with one mask shared across columns (reference pair_transform.py:45-61)."""

    _shared_dim = -2


class PairTransition(nn.Module):
    """Pair feed-forward (reference pair_transform.py:64-84): LN -> Linear(c_p, n c_p) ->
    ReLU -> Linear(n c_p, c_p). c_p = 128 with n = 4 runs on the tuned transition kernels,
    other shapes on the general-shape path."""

    def __init__(self, c_p: int, n: int = 4):
        super().__init__()
        self.c_p = c_p
        self.n = n
        self.layer_norm = nn.LayerNorm(c_p)
        self.linear_1 = Linear(c_p, c_p * n)
        self.relu = nn.ReLU()
        self.linear_2 = Linear(c_p * n, c_p, init="final")
        self._pack = _PackCache()

    def packed_weights(self, device: torch.device) -> Tensor:
        sd = {k: v for k, v in self.state_dict(keep_vars=True).items()}
        return self._pack.get(self, lambda: ops.pack_transition(sd, device))

    def _check(self, p: Tensor) -> None:
        if not p.is_cuda:
            raise RuntimeError("genie_tk (B200): PairTransition runs on CUDA tensors only")

    def forward(self, p: Tensor, mask: Optional[Tensor] = None) -> Tensor:
        """The update (the reference ignores ``mask`` here, and so does this)."""
        self._check(p)
        if autograd.needs_grad(p, self):
            sd = dict(self.named_parameters())
            res = autograd.TransitionFn.apply(p.float().contiguous(), self.packed_weights(p.device),
                                              *[sd[k] for k in ops.TRANSITION_KEYS])
        else:
            res = torch.ops.genie_tk.transition_forward(p, self.packed_weights(p.device))
        return res if res.dtype == p.dtype else res.to(p.dtype)

    def residual_masked_(self, p: Tensor, p_mask: Optional[Tensor]) -> Tensor:
        """p = (p + transition(p)) * p_mask, in place on a contiguous fp32 ``p`` (the tail of
        PairTransformLayer.forward, pair_transform.py:190-193, in one kernel pass)."""
        self._check(p)
        return ops.transition_forward(p, p_mask, self.packed_weights(p.device), out=p, add_residual=True)


class PairEmbedding(nn.Module):
    """Initial pair representation from the single representation (reference
    examples/basic_usage.py:170-199): ``p[b,i,j] = Linear(2 c_s, c_p)([s_i ; s_j])`` and the
    pair mask ``p_mask[b,i,j] = mask[b,i] * mask[b,j]``. Holds the ``weight`` / ``bias`` of
    that ``nn.Linear(c_s * 2, c_p)`` (state-dict compatible with it) and runs on the pair
    embedding kernels, which never form the concatenated [B, N, N, 2 c_s] tensor. Any c_p
    in 1..4096.
    """

    def __init__(self, c_s: int, c_p: int):
        super().__init__()
        self.c_s = c_s
        self.c_p = c_p
        lin = nn.Linear(c_s * 2, c_p)
        self.weight = lin.weight
        self.bias = lin.bias

    def forward(self, s: Tensor, mask: Optional[Tensor] = None) -> Tuple[Tensor, Optional[Tensor]]:
        """(p [B, N, N, c_p] fp32, p_mask [B, N, N] or None when ``mask`` is None)."""
        if not s.is_cuda:
            raise RuntimeError("genie_tk (B200): PairEmbedding runs on CUDA tensors only")
        if autograd.needs_grad(s, self):
            p, pm = autograd.PairEmbedFn.apply(s, mask, self.weight, self.bias)
            return p, pm
        p, pm = ops.pair_embed(s, mask, self.weight, self.bias, with_mask=mask is not None)
        return p, pm


class PairTransformLayer(nn.Module):
    """One pair transform layer (reference pair_transform.py:87-195)."""

    def __init__(self, c_p: int, include_mul_update: bool = True, include_tri_att: bool = True,
                 c_hidden_mul: int = 128, c_hidden_tri_att: int = 32, n_head_tri: int = 4,
                 tri_dropout: float = 0.25, pair_transition_n: int = 4, use_fused_kernel: bool = True):
        super().__init__()
        self.include_mul_update = include_mul_update
        self.include_tri_att = include_tri_att
        if include_mul_update:
            self.tri_mul_out = TriangleMultiplicationOutgoing(c_z=c_p, c_hidden=c_hidden_mul,
                                                              use_fused_kernel=use_fused_kernel)
            self.tri_mul_in = TriangleMultiplicationIncoming(c_z=c_p, c_hidden=c_hidden_mul,
                                                             use_fused_kernel=use_fused_kernel)
        if include_tri_att:
            self.tri_att_start = TriangleAttentionStartingNode(c_in=c_p, c_hidden=c_hidden_tri_att,
                                                               no_heads=n_head_tri, use_fused_kernel=use_fused_kernel)
            self.tri_att_end = TriangleAttentionEndingNode(c_in=c_p, c_hidden=c_hidden_tri_att, no_heads=n_head_tri,
                                                           use_fused_kernel=use_fused_kernel)
        self.pair_transition = PairTransition(c_p, pair_transition_n)
        self.dropout_row = DropoutRowwise(tri_dropout)
        self.dropout_col = DropoutColumnwise(tri_dropout)

    def forward(self, inputs: Tuple[Tensor, Tensor]) -> Tuple[Tensor, Tensor]:
        p, p_mask = inputs
        if not p.is_cuda:
            raise RuntimeError("genie_tk (B200): PairTransformLayer runs on CUDA tensors only")
        dtype = p.dtype
        if autograd.needs_grad(p, self):
            return self._forward_autograd(p, p_mask)
        p = p.float().clone()
        blocks = []
        if self.include_mul_update:
            blocks += [(self.tri_mul_out, self.dropout_row), (self.tri_mul_in, self.dropout_row)]
        if self.include_tri_att:
            blocks += [(self.tri_att_start, self.dropout_row), (self.tri_att_end, self.dropout_col)]
        for block, drop in blocks:
            # p += dropout(update), the dropout (training mode only) applied in the epilogue
            block(p, p_mask, out=p, add_residual=True, dropout=drop.keep_mask(p.shape, dtype, p.device))
        # p = (p + transition(p)) * mask in one pass (p is a private contiguous fp32 copy)
        self.pair_transition.residual_masked_(p, p_mask)
        return (p.to(dtype), p_mask)

    def _forward_autograd(self, p: Tensor, p_mask: Tensor) -> Tuple[Tensor, Tensor]:
        """The reference's out-of-place chain (pair_transform.py:177-195), every block's forward
        on the kernels and differentiable; the dropout draws exactly as the reference does."""
        dtype = p.dtype
        p = p.float()
        if self.include_mul_update:
            p = p + self.dropout_row(self.tri_mul_out(p, p_mask))
            p = p + self.dropout_row(self.tri_mul_in(p, p_mask))
        if self.include_tri_att:
            p = p + self.dropout_row(self.tri_att_start(p, p_mask))
            p = p + self.dropout_col(self.tri_att_end(p, p_mask))
        p = p + self.pair_transition(p, p_mask)
        p = p * p_mask.unsqueeze(-1).to(p.dtype)
        return (p.to(dtype), p_mask)


class PairTransformNet(nn.Module):
    """Stack of PairTransformLayers (reference pair_transform.py:198-258)."""

    def __init__(self, c_p: int, n_layers: int, include_mul_update: bool = True, include_tri_att: bool = True,
                 c_hidden_mul: int = 128, c_hidden_tri_att: int = 32, n_head_tri: int = 4,
                 tri_dropout: float = 0.25, pair_transition_n: int = 4, use_fused_kernel: bool = True):
        super().__init__()
        self.layers = nn.ModuleList([
            PairTransformLayer(c_p=c_p, include_mul_update=include_mul_update, include_tri_att=include_tri_att,
                               c_hidden_mul=c_hidden_mul, c_hidden_tri_att=c_hidden_tri_att, n_head_tri=n_head_tri,
                               tri_dropout=tri_dropout, pair_transition_n=pair_transition_n,
                               use_fused_kernel=use_fused_kernel)
            for _ in range(n_layers)])

    def forward(self, p: Tensor, p_mask: Tensor) -> Tensor:
        for layer in self.layers:
            p, p_mask = layer((p, p_mask))
        return p
