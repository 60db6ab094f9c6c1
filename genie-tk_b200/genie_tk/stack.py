"""The triangle pair stack: ``z += TriMulOut(z); z += TriMulIn(z); z += TriAttStart(z);
z += TriAttEnd(z)`` per layer, on an fp32 residual stream updated in place.

This is the explicit residual chain of the reference's examples/basic_usage.py:44-78
(equal to PairTransformLayer.forward, pair_transform.py:162-195, without the
PairTransition block and the final mask multiply). Each block is three kernels (its
stage entry points, with the residual add fused into the last one), so a layer is twelve
kernel launches on one stream sharing one workspace; ``capture_graph`` records a whole
stack into one CUDA graph.
"""

from __future__ import annotations

from typing import Callable, Dict, List, Optional

import torch
import torch.nn as nn
from torch import Tensor

from . import ops
from .triangle_attention import TriangleAttentionEndingNode, TriangleAttentionStartingNode
from .triangle_mul import TriangleMultiplicationIncoming, TriangleMultiplicationOutgoing

OP_NAMES = ("tri_mul_out", "tri_mul_in", "tri_att_start", "tri_att_end")
KERNELS_PER_LAYER = 12

# hook(label) is called before and after every kernel launch when given (bench timing)
Hook = Optional[Callable[[str], None]]


class TriangleStackLayer(nn.Module):
    def __init__(self, c_z: int = 128, c_hidden_mul: int = 128, c_hidden_att: int = 128, no_heads: int = 4):
        super().__init__()
        self.tri_mul_out = TriangleMultiplicationOutgoing(c_z, c_hidden_mul)
        self.tri_mul_in = TriangleMultiplicationIncoming(c_z, c_hidden_mul)
        self.tri_att_start = TriangleAttentionStartingNode(c_z, c_hidden_att, no_heads)
        self.tri_att_end = TriangleAttentionEndingNode(c_z, c_hidden_att, no_heads)


class TrianglePairStack(nn.Module):
    """``n_layers`` x [TriMulOut, TriMulIn, TriAttStart, TriAttEnd] with residual adds."""

    def __init__(self, n_layers: int, c_z: int = 128, c_hidden_mul: int = 128, c_hidden_att: int = 128,
                 no_heads: int = 4):
        super().__init__()
        self.layers = nn.ModuleList(
            [TriangleStackLayer(c_z, c_hidden_mul, c_hidden_att, no_heads) for _ in range(n_layers)])
        self._ws = None

    def load_layer_params(self, layers: List[Dict[str, Dict[str, Tensor]]]) -> None:
        """Load per-layer reference state dicts ``[{op_name: state_dict}, ...]``."""
        for layer, lp in zip(self.layers, layers):
            for name in OP_NAMES:
                getattr(layer, name).load_state_dict(lp[name])

    @torch.no_grad()
    def prepare(self, B: int, N: int, device: torch.device) -> None:
        """Pack all weights and allocate the shared workspace (call before graph capture)."""
        for layer in self.layers:
            for name in OP_NAMES:
                getattr(layer, name).packed_weights(device)
        lib = ops._lib.load()
        ld = ops.plane_pitch(N)
        plane_bytes = (B * N * 128 * ld * 2 + 255) // 256 * 256
        tri_bytes = lib.gtk_triatt_workspace_bytes(B, N, 128, 128, 4)
        need = max(3 * plane_bytes, tri_bytes)
        if self._ws is None or self._ws[0].numel() < need or self._ws[1] != (B, N):
            ws = torch.empty(need, dtype=torch.uint8, device=device)
            self._ws = (ws, (B, N), plane_bytes)
        ops.status_buffer(device)

    def _run(self, z_in: Tensor, z: Tensor, mask: Optional[Tensor], hook: Hook) -> None:
        B, N = z.shape[0], z.shape[1]
        self.prepare(B, N, z.device)
        ws, _, plane_bytes = self._ws
        lib = ops._lib.load()
        st = ops.status_buffer(z.device)
        stream = ops._stream(z.device)
        P = ops._ptr
        ld = ops.plane_pitch(N)
        ap, bp, xp = (ops.ctypes.c_void_p(ws.data_ptr() + k * plane_bytes) for k in range(3))
        xs = 1.0 / N
        src = z_in
        h = hook or (lambda label: None)
        for layer in self.layers:
            for name in OP_NAMES:
                mod = getattr(layer, name)
                packed = mod.packed_weights(z.device)
                if name.startswith("tri_mul"):
                    outgoing = name == "tri_mul_out"
                    h("trimul_project")
                    ops._lib.check(lib.gtk_trimul_project(P(src), P(mask), P(packed), ap, bp, ld, B, N, N, P(st),
                                                          stream), "gtk_trimul_project")
                    h("trimul_contract")
                    ops._lib.check(lib.gtk_trimul_contract(int(outgoing), ap, bp, xp, B, 128, N, N, N, ld, ld, ld, xs,
                                                           P(st), stream), "gtk_trimul_contract")
                    h("trimul_finish")
                    ops._lib.check(lib.gtk_trimul_finish(P(src), xp, ld, xs, P(packed), P(z), 1, B, N, N, P(st),
                                                         stream), "gtk_trimul_finish")
                    h("end")
                else:
                    starting = name == "tri_att_start"
                    h("triatt_project")
                    ops._lib.check(lib.gtk_triatt_project(int(starting), P(src), P(packed), P(ws), B, N, N, 0,
                                                          P(st), stream), "gtk_triatt_project")
                    h("triatt_core")
                    ops._lib.check(lib.gtk_triatt_core(int(starting), P(mask), P(ws), B, N, N, 0, float(mod.inf),
                                                       P(st), stream), "gtk_triatt_core")
                    h("triatt_finish")
                    ops._lib.check(lib.gtk_triatt_finish(int(starting), P(src), P(packed), P(ws), P(z), 1, B, N,
                                                         N, P(st), stream), "gtk_triatt_finish")
                    h("end")
                src = z

    @torch.no_grad()
    def forward_into(self, z_in: Tensor, z_out: Tensor, mask: Optional[Tensor] = None, hook: Hook = None) -> Tensor:
        """``z_out = stack(z_in)``; z_in is read by the first block only and left unchanged."""
        for t, n in ((z_in, "z_in"), (z_out, "z_out")):
            if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous() and t.shape[-1] == 128):
                raise RuntimeError(f"TrianglePairStack: {n} must be a contiguous fp32 CUDA [B, N, N, 128] tensor")
        if mask is not None:
            mask = mask.float().contiguous()
        self._run(z_in, z_out, mask, hook)
        return z_out

    @torch.no_grad()
    def forward_(self, z: Tensor, mask: Optional[Tensor] = None, hook: Hook = None) -> Tensor:
        """Run the stack in place on ``z`` (fp32, contiguous, CUDA); returns ``z``."""
        return self.forward_into(z, z, mask, hook)

    @torch.no_grad()
    def forward(self, z: Tensor, mask: Optional[Tensor] = None) -> Tensor:
        if not z.is_cuda:
            raise RuntimeError("genie_tk (B200): TrianglePairStack runs on CUDA tensors only")
        zin = z.float().contiguous()
        out = torch.empty_like(zin)
        self.forward_into(zin, out, mask)
        return out if z.dtype == torch.float32 else out.to(z.dtype)

    def capture_graph(self, z_in: Tensor, z_out: Tensor, mask: Optional[Tensor] = None) -> "torch.cuda.CUDAGraph":
        """Capture ``forward_into(z_in, z_out, mask)`` into a CUDA graph."""
        B, N = z_in.shape[0], z_in.shape[1]
        self.prepare(B, N, z_in.device)
        if mask is not None:
            mask = mask.float().contiguous()
        self.forward_into(z_in, z_out, mask)  # warm the tensor-map / attribute caches outside capture
        torch.cuda.synchronize(z_in.device)
        s = torch.cuda.Stream(device=z_in.device)
        s.wait_stream(torch.cuda.current_stream(z_in.device))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            with torch.cuda.graph(g, stream=s):
                self._run(z_in, z_out, mask, None)
        torch.cuda.current_stream(z_in.device).wait_stream(s)
        return g
