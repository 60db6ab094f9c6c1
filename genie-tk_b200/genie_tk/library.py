"""The C-ABI entry points as PyTorch operators (``torch.ops.genie_tk.*``).

Each operator is a ``torch.library.custom_op`` whose implementation enqueues the library's
kernels on the current CUDA stream (``ops.trimul_forward`` / ``ops.triatt_forward``), with
outputs from the caching allocator, so it can be captured in a CUDA graph and is opaque to
``torch.compile`` (the fake implementations give it shapes without running anything). They
replace the pybind functions the reference declares in ``kernels/bindings.cpp:13-65``
(``triangle_mul_outgoing`` / ``_incoming``, ``triangle_attention_starting`` / ``_ending``),
taking the module's packed weights instead of pre-projected operands because the B200
kernels fuse the projections.

  genie_tk::trimul_forward(z, mask, packed, outgoing) -> update
  genie_tk::triatt_forward(z, mask, packed, starting, inf) -> update
  genie_tk::trimul_residual_(z, mask, packed, outgoing)        z += update, in place
  genie_tk::triatt_residual_(z, mask, packed, starting, inf)   z += update, in place
  genie_tk::transition_forward(z, packed) -> update            the pair transition
  genie_tk::transition_residual_(z, mask, packed)              z = (z + update) * mask, in place
  genie_tk::trimul_residual_dropout_(z, mask, packed, outgoing, keep_bits, scale, shared_across_rows)
  genie_tk::triatt_residual_dropout_(z, mask, packed, starting, inf, keep_bits, scale, shared_across_rows)
                                                               z += dropout(update), in place

``z`` is ``[B, N, N, C]`` (any float dtype; fp32 in place), ``mask`` ``[B, N, N]`` or
None, ``packed`` the uint8 buffer of ``ops.pack_trimul`` / ``ops.pack_triatt`` /
``ops.pack_transition``; ``keep_bits`` the int32 [B, N, 4 ceil(C / 128)] keep bits of an
``ops.DropoutMask``. No operator has an autograd formula: the kernels are forward-only.
"""

from __future__ import annotations

from typing import Optional

import torch
from torch import Tensor

from . import ops


@torch.library.custom_op("genie_tk::trimul_forward", mutates_args=())
def trimul_forward(z: Tensor, mask: Optional[Tensor], packed: Tensor, outgoing: bool) -> Tensor:
    """Update of the triangle multiplicative block (fp32)."""
    return ops.trimul_forward(z, mask, packed, outgoing)


@trimul_forward.register_fake
def _trimul_forward_fake(z, mask, packed, outgoing):
    return torch.empty(z.shape, dtype=torch.float32, device=z.device)


@torch.library.custom_op("genie_tk::triatt_forward", mutates_args=())
def triatt_forward(z: Tensor, mask: Optional[Tensor], packed: Tensor, starting: bool, inf: float) -> Tensor:
    """Update of triangle attention around the starting / ending node (fp32)."""
    return ops.triatt_forward(z, mask, packed, starting, inf=inf)


@triatt_forward.register_fake
def _triatt_forward_fake(z, mask, packed, starting, inf):
    return torch.empty(z.shape, dtype=torch.float32, device=z.device)


@torch.library.custom_op("genie_tk::trimul_residual_", mutates_args=("z",))
def trimul_residual_(z: Tensor, mask: Optional[Tensor], packed: Tensor, outgoing: bool) -> None:
    """z += update of the triangle multiplicative block, in place (z fp32 contiguous)."""
    ops.trimul_forward(z, mask, packed, outgoing, out=z, add_residual=True)


@trimul_residual_.register_fake
def _trimul_residual_fake(z, mask, packed, outgoing):
    return None


@torch.library.custom_op("genie_tk::triatt_residual_", mutates_args=("z",))
def triatt_residual_(z: Tensor, mask: Optional[Tensor], packed: Tensor, starting: bool, inf: float) -> None:
    """z += update of triangle attention, in place (z fp32 contiguous)."""
    ops.triatt_forward(z, mask, packed, starting, inf=inf, out=z, add_residual=True)


@triatt_residual_.register_fake
def _triatt_residual_fake(z, mask, packed, starting, inf):
    return None


@torch.library.custom_op("genie_tk::transition_forward", mutates_args=())
def transition_forward(z: Tensor, packed: Tensor) -> Tensor:
    """Update of the pair transition (LN -> 4x expand -> ReLU -> project), fp32."""
    return ops.transition_forward(z, None, packed)


@transition_forward.register_fake
def _transition_forward_fake(z, packed):
    return torch.empty(z.shape, dtype=torch.float32, device=z.device)


@torch.library.custom_op("genie_tk::transition_residual_", mutates_args=("z",))
def transition_residual_(z: Tensor, mask: Optional[Tensor], packed: Tensor) -> None:
    """z = (z + transition(z)) * mask, in place (z fp32 contiguous; no mask: just the residual)."""
    ops.transition_forward(z, mask, packed, out=z, add_residual=True)


@transition_residual_.register_fake
def _transition_residual_fake(z, mask, packed):
    return None


@torch.library.custom_op("genie_tk::trimul_residual_dropout_", mutates_args=("z",))
def trimul_residual_dropout_(z: Tensor, mask: Optional[Tensor], packed: Tensor, outgoing: bool, keep_bits: Tensor,
                             scale: float, shared_across_rows: bool) -> None:
    """z += dropout(update of the triangle multiplicative block), in place (z fp32 contiguous)."""
    ops.trimul_forward(z, mask, packed, outgoing, out=z, add_residual=True,
                       dropout=ops.DropoutMask(keep_bits, scale, shared_across_rows))


@trimul_residual_dropout_.register_fake
def _trimul_residual_dropout_fake(z, mask, packed, outgoing, keep_bits, scale, shared_across_rows):
    return None


@torch.library.custom_op("genie_tk::triatt_residual_dropout_", mutates_args=("z",))
def triatt_residual_dropout_(z: Tensor, mask: Optional[Tensor], packed: Tensor, starting: bool, inf: float,
                             keep_bits: Tensor, scale: float, shared_across_rows: bool) -> None:
    """z += dropout(update of triangle attention), in place (z fp32 contiguous)."""
    ops.triatt_forward(z, mask, packed, starting, inf=inf, out=z, add_residual=True,
                       dropout=ops.DropoutMask(keep_bits, scale, shared_across_rows))


@triatt_residual_dropout_.register_fake
def _triatt_residual_dropout_fake(z, mask, packed, starting, inf, keep_bits, scale, shared_across_rows):
    return None
