"""The triangle pair stack: ``z += TriMulOut(z); z += TriMulIn(z); z += TriAttStart(z);
z += TriAttEnd(z)`` per layer, on an fp32 residual stream updated in place.

This is the explicit residual chain of the reference's examples/basic_usage.py:44-78
(equal to PairTransformLayer.forward, pair_transform.py:162-195, without the
PairTransition block and the final mask multiply). Each block is one
``gtk_*_forward`` call with the residual add fused into its last kernel, so a layer is
twelve kernel launches; ``capture_graph`` records a whole stack into one CUDA graph.
"""

from __future__ import annotations

from typing import Dict, List, Optional

import torch
import torch.nn as nn
from torch import Tensor

from . import ops
from .triangle_attention import TriangleAttentionEndingNode, TriangleAttentionStartingNode
from .triangle_mul import TriangleMultiplicationIncoming, TriangleMultiplicationOutgoing

OP_NAMES = ("tri_mul_out", "tri_mul_in", "tri_att_start", "tri_att_end")


class TriangleStackLayer(nn.Module):
    def __init__(self, c_z: int = 128, c_hidden_mul: int = 128, c_hidden_att: int = 128, no_heads: int = 4):
        super().__init__()
        self.tri_mul_out = TriangleMultiplicationOutgoing(c_z, c_hidden_mul)
        self.tri_mul_in = TriangleMultiplicationIncoming(c_z, c_hidden_mul)
        self.tri_att_start = TriangleAttentionStartingNode(c_z, c_hidden_att, no_heads)
        self.tri_att_end = TriangleAttentionEndingNode(c_z, c_hidden_att, no_heads)

    def forward_(self, z: Tensor, mask: Optional[Tensor]) -> Tensor:
        """In-place layer on an fp32 contiguous CUDA pair tensor."""
        for name in OP_NAMES:
            getattr(self, name)(z, mask, out=z, add_residual=True)
        return z


class TrianglePairStack(nn.Module):
    """``n_layers`` x [TriMulOut, TriMulIn, TriAttStart, TriAttEnd] with residual adds."""

    def __init__(self, n_layers: int, c_z: int = 128, c_hidden_mul: int = 128, c_hidden_att: int = 128,
                 no_heads: int = 4):
        super().__init__()
        self.layers = nn.ModuleList(
            [TriangleStackLayer(c_z, c_hidden_mul, c_hidden_att, no_heads) for _ in range(n_layers)])

    def load_layer_params(self, layers: List[Dict[str, Dict[str, Tensor]]]) -> None:
        """Load per-layer reference state dicts ``[{op_name: state_dict}, ...]``."""
        for layer, lp in zip(self.layers, layers):
            for name in OP_NAMES:
                getattr(layer, name).load_state_dict(lp[name])

    @torch.no_grad()
    def forward_(self, z: Tensor, mask: Optional[Tensor] = None) -> Tensor:
        """Run the stack in place on ``z`` (fp32, contiguous, CUDA); returns ``z``."""
        if not (z.is_cuda and z.dtype == torch.float32 and z.is_contiguous()):
            raise RuntimeError("TrianglePairStack.forward_ needs a contiguous fp32 CUDA tensor")
        for layer in self.layers:
            layer.forward_(z, mask)
        return z

    @torch.no_grad()
    def forward(self, z: Tensor, mask: Optional[Tensor] = None) -> Tensor:
        if not z.is_cuda:
            raise RuntimeError("genie_tk (B200): TrianglePairStack runs on CUDA tensors only")
        zf = z.float().contiguous().clone()
        mf = None if mask is None else mask.float().contiguous()
        self.forward_(zf, mf)
        return zf if z.dtype == torch.float32 else zf.to(z.dtype)

    @torch.no_grad()
    def prepare(self, z: Tensor) -> None:
        """Pack all weights and size the workspaces for ``z``'s shape (call before graph capture)."""
        for layer in self.layers:
            for name in OP_NAMES:
                getattr(layer, name).packed_weights(z.device)
        B, N = z.shape[0], z.shape[1]
        lib = ops._lib.load()
        need = max(lib.gtk_trimul_workspace_bytes(B, N, 128, 128),
                   lib.gtk_triatt_workspace_bytes(B, N, 128, 128, 4))
        ops.workspace(z.device, need)
        ops.status_buffer(z.device)

    def capture_graph(self, z: Tensor, mask: Optional[Tensor] = None) -> "torch.cuda.CUDAGraph":
        """Capture ``forward_(z, mask)`` into a CUDA graph (replay updates ``z`` in place)."""
        self.prepare(z)
        s = torch.cuda.Stream(device=z.device)
        s.wait_stream(torch.cuda.current_stream(z.device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self.forward_(z, mask)
        torch.cuda.current_stream(z.device).wait_stream(s)
        return g
