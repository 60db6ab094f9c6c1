"""Parameter-holding building blocks with the reference's names and initialisers.

Mirrors src/genie_tk/primitives.py of northws/Genie-TK: ``Linear`` with the AF2
initialisers (default / final / gating / normal, primitives.py:17-40) and the gated
multi-head ``Attention`` parameter set (primitives.py:78-112). The parameter names are
identical so reference ``state_dict``s load unchanged. The attention arithmetic itself
runs fused inside ``TriangleAttention`` on the B200 kernels.
"""

from __future__ import annotations

import math
from typing import List, Optional

import torch.nn as nn
from torch import Tensor


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


class Attention(nn.Module):
    """Parameters of the gated multi-head attention (reference primitives.py:65-112).

    ``linear_q/k/v`` without bias, ``linear_o`` (init "final"), ``linear_g`` (init
    "gating"). Used by ``TriangleAttention``, whose fused kernel consumes these
    parameters; calling this module on its own is not part of the B200 path.
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

    def forward(self, q_x: Tensor, k_x: Tensor, v_x: Tensor, biases: Optional[List[Tensor]] = None) -> Tensor:
        raise NotImplementedError(
            "genie_tk (B200): generic Attention is evaluated only inside the fused TriangleAttention kernels")
