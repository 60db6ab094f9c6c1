"""CPU stand-ins for the stage kernels, for testing the row-sharded driver without a GPU.

Test infrastructure only. ``genie_tk.sharded`` runs its per-rank program over a
``stage_ops`` object; on a GPU that is ``CudaStageOps`` (the library's kernels). This
class implements the same calls on CPU tensors with the oracle's fp32 math
(``oracle.triangle_oracle.layer_norm`` / ``linear``), writing every intermediate in the
exact byte layout the kernels use (fp16 planes with the 1/N contraction scale, q scaled
by log2(e)/sqrt(d), the bf16 triangle bias in log2 units in its [N][B][H][ldn] region),
so the driver's offsets, packing, collectives and row bookkeeping are exercised as they
are on the GPU. Workspace offsets come from the library's own host function.
"""

from __future__ import annotations

import math

import torch

from genie_tk import _lib
from oracle import triangle_oracle as O

C, H, D = 128, 4, 32
LOG2E = 1.0 / math.log(2.0)


def _typed(buf: torch.Tensor, dtype, shape):
    n = 1
    for s in shape:
        n *= s
    nbytes = n * torch.empty((), dtype=dtype).element_size()
    assert buf.numel() >= nbytes, (buf.numel(), nbytes)
    return buf[:nbytes].view(dtype).view(*shape)


class CpuStageOps:
    def __init__(self):
        self.lib = _lib.load()

    def alloc(self, nbytes: int) -> torch.Tensor:
        return torch.zeros(max(int(nbytes), 256), dtype=torch.uint8)

    @staticmethod
    def _p(mod):
        return {k: v.detach().float() for k, v in mod.state_dict().items()}

    def triatt_layout(self, B, rows, N):
        import ctypes
        offs = (ctypes.c_int64 * 7)()
        assert self.lib.gtk_triatt_workspace_offsets(B, rows, N, offs) == 0
        return {k: int(offs[n]) for n, k in enumerate(("q", "k", "v", "g", "og", "bias", "total"))}

    # ------------------------------------------------------------------ TriMul
    def trimul_project(self, mod, z, mask, a, b, B, rows, N):
        _, av, bv = O.trimul_prepare(z, mask, self._p(mod))
        _typed(a, torch.float16, (B, rows, C, N)).copy_(av.permute(0, 1, 3, 2))
        _typed(b, torch.float16, (B, rows, C, N)).copy_(bv.permute(0, 1, 3, 2))

    def trimul_project_to(self, mod, z, mask, a_dst, b_dst, B, rows, N, row0):
        _, av, bv = O.trimul_prepare(z, mask, self._p(mod))
        P = len(a_dst.tensors)
        CP = C // P
        for dst, val in ((a_dst, av), (b_dst, bv)):
            planes = val.permute(0, 1, 3, 2)                       # [B][rows][C][N]
            for q, t in enumerate(dst.tensors):
                _typed(t, torch.float16, (B, N, CP, N))[:, row0:row0 + rows].copy_(planes[:, :, q * CP:(q + 1) * CP])

    def trimul_contract(self, outgoing, a, b, x, B, M, Nj, K, lda, ldb, ldx, xs, channels=C):
        Cc = channels
        if outgoing:
            A = _typed(a, torch.float16, (B, M, Cc, lda))[..., :K].float()
            Bm = _typed(b, torch.float16, (B, Nj, Cc, ldb))[..., :K].float()
            X = torch.einsum("bmck,bnck->bmcn", A, Bm)
        else:
            A = _typed(a, torch.float16, (B, K, Cc, lda))[..., :M].float()
            Bm = _typed(b, torch.float16, (B, K, Cc, ldb))[..., :Nj].float()
            X = torch.einsum("bkcm,bkcn->bmcn", A, Bm)
        _typed(x, torch.float16, (B, M, Cc, ldx))[..., :Nj].copy_(X * xs)

    def trimul_finish(self, mod, z, x, ldx, xs, B, rows, N, out):
        p = self._p(mod)
        X = _typed(x, torch.float16, (B, rows, C, ldx))[..., :N].float().permute(0, 1, 3, 2) / xs
        zn = O.layer_norm(z, p["layer_norm_in.weight"], p["layer_norm_in.bias"])
        g = torch.sigmoid(O.linear(zn, p, "linear_g"))
        u = O.linear(O.layer_norm(X, p["layer_norm_out.weight"], p["layer_norm_out.bias"]), p, "linear_z")
        out.copy_(z + u * g)

    # ------------------------------------------------------------------ TriAtt (starting orientation)
    def _views(self, ws, B, rows, N):
        lay = self.triatt_layout(B, rows, N)
        ldn = (N + 7) // 8 * 8

        def at(name, dtype, shape):
            return _typed(ws[lay[name]:], dtype, shape)
        return dict(q=at("q", torch.float16, (B, rows, H, N, D)), k=at("k", torch.float16, (B, rows, H, N, D)),
                    v=at("v", torch.float16, (B, rows, H, N, D)), g=at("g", torch.float16, (B, rows, N, C)),
                    og=at("og", torch.float16, (B, rows, N, C)),
                    bias=at("bias", torch.bfloat16, (N, B, H, ldn)))

    def triatt_project(self, mod, z, ws, B, rows, N, row0):
        p = self._p(mod)
        v = self._views(ws, B, rows, N)
        x = O.layer_norm(z, p["layer_norm.weight"], p["layer_norm.bias"])
        for name, scale in (("q", LOG2E / math.sqrt(D)), ("k", 1.0), ("v", 1.0)):
            t = O.linear(x, p, f"mha.linear_{name}") * scale
            v[name].copy_(t.view(B, rows, N, H, D).permute(0, 1, 3, 2, 4))
        v["g"].copy_(torch.sigmoid(O.linear(x, p, "mha.linear_g")))
        tri = O.linear(x, p, "linear") * LOG2E                        # [B, rows, N(k), H]
        v["bias"][row0:row0 + rows, :, :, :N].copy_(tri.permute(1, 0, 3, 2))

    def triatt_core(self, mod, mask, ws, B, rows, N, row0):
        v = self._views(ws, B, rows, N)
        q, k, vv = v["q"].float(), v["k"].float(), v["v"].float()
        s = torch.matmul(q, k.transpose(-1, -2))                        # [B, rows, H, J, K]
        if mask is not None:
            mb = (mask[:, row0:row0 + rows].float() - 1.0) * (float(mod.inf) * LOG2E)
            s = s + mb[:, :, None, None, :]
        bias = v["bias"][:, :, :, :N].float().permute(1, 2, 0, 3)       # [B, H, J, K]
        s = s + bias[:, None]
        s = s - s.amax(-1, keepdim=True)
        e = torch.exp2(s)
        o = torch.matmul(e / e.sum(-1, keepdim=True), vv)              # [B, rows, H, J, D]
        o = o.permute(0, 1, 3, 2, 4).reshape(B, rows, N, C) * v["g"].float()
        v["og"].copy_(o)

    def triatt_finish(self, mod, z, ws, B, rows, N):
        v = self._views(ws, B, rows, N)
        z.add_(O.linear(v["og"].float(), self._p(mod), "mha.linear_o"))

    def trimul_contract_to(self, outgoing, a, b, B, M, Nj, K, lda, ldb, xs, channels, dst, c_off, ld_dst):
        # gtk_trimul_contract_to_peers: the contraction, then rows of rank p -> p's x planes
        P = len(dst.tensors)
        R = M // P
        x = torch.empty(B * M * channels * ld_dst * 2, dtype=torch.uint8)
        self.trimul_contract(outgoing, a, b, x, B, M, Nj, K, lda, ldb, ld_dst, xs, channels)
        X = _typed(x, torch.float16, (B, M, channels, ld_dst))
        for p, t in enumerate(dst.tensors):
            _typed(t, torch.float16, (B, R, C, ld_dst))[:, :, c_off:c_off + channels].copy_(X[:, p * R:(p + 1) * R])

    def triatt_finish_to(self, mod, z, ws, B, rows, N, row0, dst):
        # gtk_triatt_finish_to_peers: z + update, pair-transposed into every rank's shard
        v = self._views(ws, B, rows, N)
        out = z + O.linear(v["og"].float(), self._p(mod), "mha.linear_o")
        self.push_pair_transpose(out.contiguous(), dst, B, rows, N, len(dst.tensors), N, row0)

    # ------------------------------------------------------------------ data movement
    def copy_2d(self, dst, dpitch, src, spitch, width, height):
        assert dst.dtype == torch.uint8 and src.dtype == torch.uint8
        assert (height - 1) * dpitch + width <= dst.numel() and (height - 1) * spitch + width <= src.numel()
        d = dst.as_strided((height, width), (dpitch, 1))
        d.copy_(src.as_strided((height, width), (spitch, 1)))

    def copy_3d(self, dst, dpitch, dslab, src, spitch, sslab, width, height, depth):
        for k in range(depth):
            self.copy_2d(dst[k * dslab:], dpitch, src[k * sslab:], spitch, width, height)

    def push_3d(self, dst, doff, dpitch, src, spitch, sslab, width, height):
        # slab k -> rank k's buffer (ranks emulated in one process: dst.tensors)
        for k, t in enumerate(dst.tensors):
            self.copy_2d(t[doff:], dpitch, src[k * sslab:], spitch, width, height)

    def push_pair_transpose(self, src, dst, B, R, Cn, P, ndst, row0):
        CP = Cn // P
        s = src.reshape(B, R, P, CP, C)
        for q, t in enumerate(dst.tensors):
            _typed(t, torch.float32, (B, CP, ndst, C))[:, :, row0:row0 + R].copy_(s[:, :, q].permute(0, 2, 1, 3))

    def pair_transpose_pack(self, src, dst, B, R, Cn, P):
        s = src.reshape(B, R, P, Cn // P, C).permute(2, 0, 3, 1, 4)     # [P][B][Cn/P][R][C]
        _typed(dst, torch.float32, (P, B, Cn // P, R, C)).copy_(s)
