"""Thin PyTorch-facing wrappers over the C ABI (``include/genie_tk_b200.h``).

PyTorch is used here only for device memory and streams: every tensor handed to the
library is a CUDA tensor of the right dtype and layout, outputs and workspaces are
allocated with ``torch.empty`` on the current stream, and the kernels are enqueued on
``torch.cuda.current_stream()``. Nothing here computes on the CPU; a CPU tensor, an
unsupported shape or a missing library raises.
"""

from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Dict, Optional

import torch

from . import _lib

SUPPORTED_C = 128
SUPPORTED_HEADS = 4

_status_bufs: Dict[int, torch.Tensor] = {}
_workspaces: Dict[tuple, torch.Tensor] = {}


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def status_buffer(device: torch.device) -> torch.Tensor:
    """Per-device uint32 status word the kernels OR their timeout bits into."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _status_bufs.get(idx)
    if buf is None:
        buf = torch.zeros(1, dtype=torch.int32, device=torch.device("cuda", idx))
        _status_bufs[idx] = buf
    return buf


def check_status(device: torch.device, reset: bool = True) -> int:
    """Synchronise and return the device status word (0 = no kernel timed out)."""
    buf = status_buffer(device)
    val = int(buf.item())
    if reset and val:
        buf.zero_()
    return val


def workspace(device: torch.device, nbytes: int, tag: str = "ws") -> torch.Tensor:
    """A cached uint8 scratch buffer of at least ``nbytes`` on ``device`` (grown, never shrunk)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, tag)
    buf = _workspaces.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(nbytes, 256), dtype=torch.uint8, device=torch.device("cuda", idx))
        _workspaces[key] = buf
    return buf


def release_workspaces() -> None:
    _workspaces.clear()


def _require_cuda(t: torch.Tensor, name: str, dtype=None) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise RuntimeError(f"genie_tk (B200): {name} must be a CUDA tensor; this package has no CPU path")
    if dtype is not None and t.dtype != dtype:
        raise TypeError(f"genie_tk (B200): {name} must be {dtype}, got {t.dtype}")


def packed_dims(packed: torch.Tensor, default: tuple) -> tuple:
    """The shape a packed weight buffer was built for (recorded by the ``pack_*`` functions);
    ``default`` for a buffer packed elsewhere."""
    return tuple(getattr(packed, "_gtk_dims", default))


def prepare_pair(z: torch.Tensor, mask: Optional[torch.Tensor], c_expected: int):
    """Validate a pair tensor [B, N, N, C] and its mask; return contiguous fp32 views."""
    _require_cuda(z, "z")
    if z.dim() != 4 or z.shape[1] != z.shape[2]:
        raise ValueError(f"pair tensor must be [B, N, N, C], got {tuple(z.shape)}")
    if z.shape[-1] != c_expected:
        raise NotImplementedError(f"genie_tk (B200): channel count {z.shape[-1]} not supported (need {c_expected})")
    zf = z.contiguous() if z.dtype == torch.float32 else z.float().contiguous()
    mf = None
    if mask is not None:
        _require_cuda(mask, "mask")
        if tuple(mask.shape) != tuple(z.shape[:3]):
            raise ValueError(f"mask must be [B, N, N], got {tuple(mask.shape)}")
        mf = mask.float().contiguous() if mask.dtype != torch.float32 else mask.contiguous()
    return zf, mf


# --------------------------------------------------------------------------------------
# Training-mode channel dropout of the residual updates (reference pair_transform.py:26-61)
# --------------------------------------------------------------------------------------

@dataclass
class DropoutMask:
    """A DropoutRowwise / DropoutColumnwise mask as the residual epilogues consume it.

    ``keep_bits`` is int32 [B, N, 4 G] on the GPU, G = ceil(C / 128): 128 G bits per
    (b, residue), bit c % 32 of word c // 32 set when channel c is kept. ``shared_across_rows``: DropoutRowwise (the mask [B, 1, N, C] varies
    with the column j), else DropoutColumnwise ([B, N, 1, C], varies with the row i). Kept
    channels of the update are multiplied by ``scale``."""

    keep_bits: torch.Tensor
    scale: float
    shared_across_rows: bool

    def _struct(self, B: int, N: int, C: int = SUPPORTED_C):
        kb = self.keep_bits
        _require_cuda(kb, "keep_bits", torch.int32)
        W = 4 * ((C + 127) // 128)
        if tuple(kb.shape) != (B, N, W) or not kb.is_contiguous():
            raise ValueError(f"keep_bits must be a contiguous int32 [B, N, {W}] for {C} channels, "
                             f"got {tuple(kb.shape)}")
        return _lib.Dropout(ctypes.c_void_p(kb.data_ptr()), float(self.scale), int(bool(self.shared_across_rows)))


def dropout_mask_from_multipliers(mult: torch.Tensor, shared_across_rows: bool, scale: float) -> DropoutMask:
    """Pack a multiplier tensor drawn the reference's way (``nn.Dropout`` applied to ones of
    shape [B, 1, N, C] for rows, [B, N, 1, C] for columns; 0 = dropped) into keep bits."""
    lib = _lib.load()
    _require_cuda(mult, "multipliers")
    if mult.dim() != 4 or mult.shape[1 if shared_across_rows else 2] != 1:
        want = "[B, 1, N, C]" if shared_across_rows else "[B, N, 1, C]"
        raise ValueError(f"dropout multipliers must be {want}, got {tuple(mult.shape)}")
    C = mult.shape[-1]
    G = (C + 127) // 128  # 128-channel groups per keep vector
    B = mult.shape[0]
    N = mult.shape[2] if shared_across_rows else mult.shape[1]
    m = mult.reshape(B * N, C).float()
    if C < 128 * G:  # channels past C do not exist; their bits are never read
        m = torch.nn.functional.pad(m, (0, 128 * G - C), value=1.0)
    m = m.contiguous()
    bits = torch.empty(B, N, 4 * G, dtype=torch.int32, device=mult.device)
    _lib.check(lib.gtk_dropout_pack_keep_bits(_ptr(m), B * N * G, _ptr(bits), _stream(mult.device)),
               "gtk_dropout_pack_keep_bits")
    bits._gtk_keepalive = m
    return DropoutMask(bits, float(scale), bool(shared_across_rows))


def dropout_mask_philox(B: int, N: int, p: float, seed: int, offset: int, shared_across_rows: bool,
                        device: torch.device, channels: int = SUPPORTED_C) -> DropoutMask:
    """A dropout mask for ``channels`` channels from the library's Philox4x32-10 generator
    (gtk_dropout_keep_bits_philox): reproducible from (seed, offset) alone, independent of
    torch's generator state."""
    lib = _lib.load()
    if not 0.0 <= p < 1.0:
        raise ValueError("dropout probability must be in [0, 1)")
    G = (int(channels) + 127) // 128
    bits = torch.empty(B, N, 4 * G, dtype=torch.int32, device=device)
    _lib.check(lib.gtk_dropout_keep_bits_philox(int(seed) & (2**64 - 1), int(offset) & (2**64 - 1), float(p), B * N * G,
                                                _ptr(bits), _stream(bits.device)), "gtk_dropout_keep_bits_philox")
    return DropoutMask(bits, 1.0 / (1.0 - p), bool(shared_across_rows))


# --------------------------------------------------------------------------------------
# Triangle multiplicative update
# --------------------------------------------------------------------------------------

TRIMUL_KEYS = ("layer_norm_in.weight", "layer_norm_in.bias", "linear_a_p.weight", "linear_a_p.bias",
               "linear_a_g.weight", "linear_a_g.bias", "linear_b_p.weight", "linear_b_p.bias",
               "linear_b_g.weight", "linear_b_g.bias", "linear_g.weight", "linear_g.bias",
               "linear_z.weight", "linear_z.bias", "layer_norm_out.weight", "layer_norm_out.bias")


def pack_trimul(params: Dict[str, torch.Tensor], device: torch.device) -> torch.Tensor:
    """Pack fp32 module parameters (reference state_dict keys) into the kernels' buffer."""
    lib = _lib.load()
    c_hidden, c_z = (int(x) for x in params["linear_a_p.weight"].shape)
    nbytes = lib.gtk_trimul_packed_bytes(c_z, c_hidden)
    if nbytes == 0:
        raise NotImplementedError(f"genie_tk (B200): triangle multiplication with c_z = {c_z}, c_hidden = {c_hidden} "
                                  "is beyond the library's limits (1..512 channels)")
    tensors = []
    for k in TRIMUL_KEYS:
        t = params[k].detach()
        _require_cuda(t, k)
        tensors.append(t.float().contiguous())
    packed = torch.empty(nbytes, dtype=torch.uint8, device=device)
    st = _lib.TrimulParams(*[ctypes.c_void_p(t.data_ptr()) for t in tensors])
    _lib.check(lib.gtk_trimul_pack(ctypes.byref(st), c_z, c_hidden, _ptr(packed), nbytes, _stream(device)),
               "gtk_trimul_pack")
    packed._gtk_keepalive = tensors  # fp32 copies must live until the pack kernel ran
    packed._gtk_dims = (c_z, c_hidden)
    return packed


def trimul_forward(z: torch.Tensor, mask: Optional[torch.Tensor], packed: torch.Tensor, outgoing: bool,
                   out: Optional[torch.Tensor] = None, add_residual: bool = False,
                   dropout: Optional[DropoutMask] = None) -> torch.Tensor:
    """update (or z + update) of the triangle multiplicative block; fp32 [B, N, N, c_z].
    ``dropout`` multiplies the update by a channel dropout mask inside the epilogue. The
    channel counts are those ``packed`` was built for (``pack_trimul``)."""
    lib = _lib.load()
    c_z, c_hidden = packed_dims(packed, (SUPPORTED_C, SUPPORTED_C))
    zf, mf = prepare_pair(z, mask, c_z)
    B, N = zf.shape[0], zf.shape[1]
    if out is None:
        out = torch.empty_like(zf)
    _require_cuda(out, "out", torch.float32)
    nbytes = lib.gtk_trimul_workspace_bytes(B, N, c_z, c_hidden)
    ws = workspace(zf.device, nbytes)
    if dropout is None:
        rc = lib.gtk_trimul_forward(int(outgoing), _ptr(zf), _ptr(mf), _ptr(packed), _ptr(out), int(add_residual),
                                    _ptr(ws), ws.numel(), B, N, c_z, c_hidden,
                                    _ptr(status_buffer(zf.device)), _stream(zf.device))
        _lib.check(rc, "gtk_trimul_forward")
        return out
    d = dropout._struct(B, N, c_z)
    rc = lib.gtk_trimul_forward_dropout(int(outgoing), _ptr(zf), _ptr(mf), _ptr(packed), _ptr(out), int(add_residual),
                                        ctypes.byref(d), _ptr(ws), ws.numel(), B, N, c_z, c_hidden,
                                        _ptr(status_buffer(zf.device)), _stream(zf.device))
    _lib.check(rc, "gtk_trimul_forward_dropout")
    return out


def plane_pitch(N: int) -> int:
    return int(_lib.load().gtk_plane_pitch(N))


def trimul_project(z: torch.Tensor, mask: Optional[torch.Tensor], packed: torch.Tensor):
    """Stage K1: a, b planes [B, R, 128, ld] (fp16) for the pair rows of z [B, R, N, 128]."""
    lib = _lib.load()
    _require_cuda(z, "z", torch.float32)
    B, R, N = z.shape[0], z.shape[1], z.shape[2]
    ld = plane_pitch(N)
    a = torch.empty(B, R, SUPPORTED_C, ld, dtype=torch.float16, device=z.device)
    b = torch.empty_like(a)
    _lib.check(lib.gtk_trimul_project(_ptr(z.contiguous()), _ptr(mask), _ptr(packed), _ptr(a), _ptr(b), ld, B, R, N,
                                      _ptr(status_buffer(z.device)), _stream(z.device)), "gtk_trimul_project")
    return a, b


def trimul_contract(a: torch.Tensor, b: torch.Tensor, outgoing: bool, M: int, Nj: int, K: int,
                    out: Optional[torch.Tensor] = None, out_scale: float = 1.0) -> torch.Tensor:
    """Stage K2 on fp16 plane buffers a [B, *, C, lda], b [B, *, C, ldb]; returns x * out_scale
    as fp16 planes [B, M, C, ldx]."""
    lib = _lib.load()
    _require_cuda(a, "a", torch.float16)
    _require_cuda(b, "b", torch.float16)
    B, C = a.shape[0], a.shape[2]
    if out is None:
        out = torch.empty(B, M, C, plane_pitch(Nj), dtype=torch.float16, device=a.device)
    _lib.check(lib.gtk_trimul_contract(int(outgoing), _ptr(a), _ptr(b), _ptr(out), B, C, M, Nj, K, a.shape[3],
                                       b.shape[3], out.shape[3], float(out_scale), _ptr(status_buffer(a.device)),
                                       _stream(a.device)), "gtk_trimul_contract")
    return out


def _pair_planes(t: torch.Tensor, transpose: bool):
    """fp32 pair tensor [B, N, N, C] -> (fp16 planes [B, N, C, ld] of t / amax, amax).
    Plane row r, column col hold t[b, r, col, c] (``transpose``: t[b, col, r, c])."""
    B, N, _, C = t.shape
    amax = t.detach().abs().amax().clamp_min(1e-30)
    view = t.permute(0, 2, 3, 1) if transpose else t.permute(0, 1, 3, 2)
    planes = torch.zeros(B, N, C, plane_pitch(N), dtype=torch.float16, device=t.device)
    planes[..., :N] = (view / amax).to(torch.float16)
    return planes, amax


def pair_contract(p: torch.Tensor, transpose_p: bool, q: torch.Tensor, transpose_q: bool,
                  outgoing: bool) -> torch.Tensor:
    """The triangle contraction of two pair tensors [B, N, N, C] on the contraction kernel:
    out(P, Q)[b,i,j,c] = sum_k P[b,i,k,c] Q[b,j,k,c] (``outgoing``) or
    inc(P, Q)[b,i,j,c] = sum_k P[b,k,i,c] Q[b,k,j,c], with P / Q pair-transposed first when
    asked. Each operand goes to the kernel as fp16 planes scaled by its own max-abs (11
    significant bits at any magnitude); the result is fp32."""
    _require_cuda(p, "p")
    _require_cuda(q, "q")
    if p.dim() != 4 or p.shape != q.shape or p.shape[1] != p.shape[2]:
        raise ValueError(f"pair tensors must both be [B, N, N, C], got {tuple(p.shape)} and {tuple(q.shape)}")
    N = p.shape[1]
    pp, sp = _pair_planes(p.float(), transpose_p)
    qp, sq = _pair_planes(q.float(), transpose_q)
    x = trimul_contract(pp, qp, outgoing, N, N, N, out_scale=1.0 / N)
    return x[..., :N].permute(0, 1, 3, 2).float() * (sp * sq * N)


def trimul_finish(z: torch.Tensor, x: torch.Tensor, packed: torch.Tensor, x_scale: float,
                  out: Optional[torch.Tensor] = None, add_residual: bool = False) -> torch.Tensor:
    """Stage K2e: LN_out + linear_z + gate (+ residual) for z [B, R, N, 128] and x planes
    written with ``out_scale = x_scale``."""
    lib = _lib.load()
    _require_cuda(z, "z", torch.float32)
    B, R, N = z.shape[0], z.shape[1], z.shape[2]
    if out is None:
        out = torch.empty_like(z)
    _lib.check(lib.gtk_trimul_finish(_ptr(z), _ptr(x), x.shape[3], float(x_scale), _ptr(packed), _ptr(out),
                                     int(add_residual), B, R, N, _ptr(status_buffer(z.device)), _stream(z.device)),
               "gtk_trimul_finish")
    return out


# --------------------------------------------------------------------------------------
# Triangle attention
# --------------------------------------------------------------------------------------

TRIATT_KEYS = ("layer_norm.weight", "layer_norm.bias", "linear.weight", "mha.linear_q.weight",
               "mha.linear_k.weight", "mha.linear_v.weight", "mha.linear_g.weight", "mha.linear_g.bias",
               "mha.linear_o.weight", "mha.linear_o.bias")


def pack_triatt(params: Dict[str, torch.Tensor], device: torch.device, heads: int) -> torch.Tensor:
    lib = _lib.load()
    c_in = int(params["layer_norm.weight"].shape[0])
    c_hidden = int(params["mha.linear_q.weight"].shape[0])
    nbytes = lib.gtk_triatt_packed_bytes(c_in, c_hidden, heads)
    if nbytes == 0:
        raise NotImplementedError(f"genie_tk (B200): triangle attention with c_in = {c_in}, c_hidden = {c_hidden}, "
                                  f"{heads} heads is beyond the library's limits (c_hidden a multiple of the heads, "
                                  "head_dim <= 64, <= 32 heads, <= 512 channels)")
    tensors = []
    for k in TRIATT_KEYS:
        t = params[k].detach()
        _require_cuda(t, k)
        tensors.append(t.float().contiguous())
    packed = torch.empty(nbytes, dtype=torch.uint8, device=device)
    st = _lib.TriattParams(*[ctypes.c_void_p(t.data_ptr()) for t in tensors])
    _lib.check(lib.gtk_triatt_pack(ctypes.byref(st), c_in, c_hidden, heads, _ptr(packed), nbytes, _stream(device)),
               "gtk_triatt_pack")
    packed._gtk_keepalive = tensors
    packed._gtk_dims = (c_in, c_hidden, heads)
    return packed


def triatt_forward(z: torch.Tensor, mask: Optional[torch.Tensor], packed: torch.Tensor, starting: bool,
                   inf: float = 1e9, out: Optional[torch.Tensor] = None, add_residual: bool = False,
                   dropout: Optional[DropoutMask] = None) -> torch.Tensor:
    """update (or z + update) of triangle attention around the starting / ending node.
    ``dropout`` multiplies the update by a channel dropout mask inside the epilogue. The
    shape (c_in, c_hidden, heads) is the one ``packed`` was built for (``pack_triatt``)."""
    lib = _lib.load()
    c_in, c_hidden, heads = packed_dims(packed, (SUPPORTED_C, SUPPORTED_C, SUPPORTED_HEADS))
    zf, mf = prepare_pair(z, mask, c_in)
    B, N = zf.shape[0], zf.shape[1]
    if out is None:
        out = torch.empty_like(zf)
    _require_cuda(out, "out", torch.float32)
    nbytes = lib.gtk_triatt_workspace_bytes(B, N, c_in, c_hidden, heads)
    ws = workspace(zf.device, nbytes)
    if dropout is None:
        rc = lib.gtk_triatt_forward(int(starting), _ptr(zf), _ptr(mf), _ptr(packed), _ptr(out), int(add_residual),
                                    _ptr(ws), ws.numel(), B, N, c_in, c_hidden, heads, float(inf),
                                    _ptr(status_buffer(zf.device)), _stream(zf.device))
        _lib.check(rc, "gtk_triatt_forward")
        return out
    d = dropout._struct(B, N, c_in)
    rc = lib.gtk_triatt_forward_dropout(int(starting), _ptr(zf), _ptr(mf), _ptr(packed), _ptr(out), int(add_residual),
                                        ctypes.byref(d), _ptr(ws), ws.numel(), B, N, c_in, c_hidden,
                                        heads, float(inf), _ptr(status_buffer(zf.device)),
                                        _stream(zf.device))
    _lib.check(rc, "gtk_triatt_forward_dropout")
    return out


def triatt_workspace(B: int, N: int, device: torch.device, rows: Optional[int] = None):
    """A stage workspace for ``rows`` problem rows (default all N) and the byte offsets of
    q, k, v, g, og, bias inside it."""
    lib = _lib.load()
    rows = N if rows is None else rows
    offs = (ctypes.c_int64 * 7)()
    _lib.check(lib.gtk_triatt_workspace_offsets(B, rows, N, offs), "gtk_triatt_workspace_offsets")
    ws = torch.empty(int(offs[6]), dtype=torch.uint8, device=device)
    return ws, {k: int(offs[n]) for n, k in enumerate(("q", "k", "v", "g", "og", "bias"))}


def triatt_stage_views(ws: torch.Tensor, offs, B: int, N: int, rows: Optional[int] = None):
    """Views of the attention intermediates inside a workspace (problem orientation): q, k, v,
    g, og fp16 over the ``rows`` local rows; the triangle bias bf16 over all N rows, viewed
    as [B, H, N, ldn] (it is stored [N][B][H][ldn])."""
    rows = N if rows is None else rows

    def view(name, nelem, shape, dtype=torch.float16):
        o = offs[name]
        return ws[o:o + 2 * nelem].view(dtype).view(*shape)
    H, d = SUPPORTED_HEADS, SUPPORTED_C // SUPPORTED_HEADS
    ldn = plane_pitch(N)
    return {
        "q": view("q", B * rows * H * N * d, (B, rows, H, N, d)),
        "k": view("k", B * rows * H * N * d, (B, rows, H, N, d)),
        "v": view("v", B * rows * H * N * d, (B, rows, H, N, d)),
        "g": view("g", B * rows * N * SUPPORTED_C, (B, rows, N, SUPPORTED_C)),
        "og": view("og", B * rows * N * SUPPORTED_C, (B, rows, N, SUPPORTED_C)),
        "bias": view("bias", N * B * H * ldn, (N, B, H, ldn), torch.bfloat16).permute(1, 2, 0, 3),
    }


def triatt_project(z: torch.Tensor, packed: torch.Tensor, starting: bool, ws: torch.Tensor, N: Optional[int] = None,
                   row0: int = 0) -> None:
    """q, k, v, g and the triangle-bias rows of the pair rows in ``z`` ([B, rows, N, 128];
    rows = N unless ``z`` is one shard of a row-sharded pair tensor starting at ``row0``)."""
    lib = _lib.load()
    _require_cuda(z, "z", torch.float32)
    B, R = z.shape[0], z.shape[1]
    N = z.shape[2] if N is None else N
    _lib.check(lib.gtk_triatt_project(int(starting), _ptr(z), _ptr(packed), _ptr(ws), B, R, N, row0,
                                      _ptr(status_buffer(z.device)), _stream(z.device)), "gtk_triatt_project")


def triatt_core(mask: Optional[torch.Tensor], starting: bool, ws: torch.Tensor, B: int, N: int,
                inf: float = 1e9, rows: Optional[int] = None, row0: int = 0) -> None:
    lib = _lib.load()
    rows = N if rows is None else rows
    _lib.check(lib.gtk_triatt_core(int(starting), _ptr(mask), _ptr(ws), B, rows, N, row0, float(inf),
                                   _ptr(status_buffer(ws.device)), _stream(ws.device)), "gtk_triatt_core")


def triatt_finish(z: Optional[torch.Tensor], packed: torch.Tensor, starting: bool, ws: torch.Tensor,
                  out: torch.Tensor, add_residual: bool = False) -> torch.Tensor:
    lib = _lib.load()
    B, R, N = out.shape[0], out.shape[1], out.shape[2]
    _lib.check(lib.gtk_triatt_finish(int(starting), _ptr(z), _ptr(packed), _ptr(ws), _ptr(out), int(add_residual), B,
                                     R, N, _ptr(status_buffer(out.device)), _stream(out.device)),
               "gtk_triatt_finish")
    return out


# --------------------------------------------------------------------------------------
# Pair transition (LayerNorm -> 4x expand -> ReLU -> project), residual and mask folded in
# --------------------------------------------------------------------------------------

TRANSITION_KEYS = ("layer_norm.weight", "layer_norm.bias", "linear_1.weight", "linear_1.bias", "linear_2.weight",
                   "linear_2.bias")


def pack_transition(params: Dict[str, torch.Tensor], device: torch.device) -> torch.Tensor:
    """Pack a PairTransition's fp32 parameters (reference state_dict keys)."""
    lib = _lib.load()
    c_p = int(params["layer_norm.weight"].shape[0])
    hid = int(params["linear_1.weight"].shape[0])
    nbytes = lib.gtk_transition_packed_bytes(c_p, hid // c_p) if hid % c_p == 0 else 0
    if nbytes == 0:
        raise NotImplementedError(f"genie_tk (B200): pair transition with c_p = {c_p}, hidden {hid} is beyond the "
                                  "library's limits (hidden a multiple of c_p, c_p <= 512, hidden <= 2048)")
    tensors = []
    for k in TRANSITION_KEYS:
        t = params[k].detach()
        _require_cuda(t, k)
        tensors.append(t.float().contiguous())
    packed = torch.empty(nbytes, dtype=torch.uint8, device=device)
    st = _lib.TransitionParams(*[ctypes.c_void_p(t.data_ptr()) for t in tensors])
    _lib.check(lib.gtk_transition_pack(ctypes.byref(st), c_p, hid // c_p, _ptr(packed), nbytes, _stream(device)),
               "gtk_transition_pack")
    packed._gtk_keepalive = tensors
    packed._gtk_dims = (c_p, hid // c_p)
    return packed


def transition_forward(z: torch.Tensor, mask: Optional[torch.Tensor], packed: torch.Tensor,
                       out: Optional[torch.Tensor] = None, add_residual: bool = False) -> torch.Tensor:
    """transition(z), or z + transition(z) (add_residual), times mask[b, i, j] when a mask
    is given; fp32 [B, N, N, c_p]. ``out=z`` updates in place. (c_p, n) are the ones
    ``packed`` was built for (``pack_transition``)."""
    lib = _lib.load()
    c_p, n = packed_dims(packed, (SUPPORTED_C, 4))
    zf, mf = prepare_pair(z, mask, c_p)
    B, N = zf.shape[0], zf.shape[1]
    if out is None:
        out = torch.empty_like(zf)
    _require_cuda(out, "out", torch.float32)
    nbytes = lib.gtk_transition_workspace_bytes(B, N, c_p, n)
    ws = workspace(zf.device, nbytes, tag="transition")
    rc = lib.gtk_transition_forward(_ptr(zf), _ptr(mf), _ptr(packed), _ptr(out), int(add_residual), _ptr(ws),
                                    ws.numel(), B, N, c_p, n, _ptr(status_buffer(zf.device)),
                                    _stream(zf.device))
    _lib.check(rc, "gtk_transition_forward")
    return out


# --------------------------------------------------------------------------------------
# The attention core for training (gtk_attn_core_forward / gtk_attn_core_backward)
# --------------------------------------------------------------------------------------

def _core_args(q, k, v, tri, mask, heads):
    for name, t in (("q", q), ("k", k), ("v", v), ("tri", tri)):
        _require_cuda(t, name, torch.float32)
        if not t.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    B, N, N2, hd = q.shape
    if N2 != N or k.shape != q.shape or v.shape != q.shape or hd % heads:
        raise ValueError("q, k, v must be [B, N, N, heads * head_dim]")
    if tuple(tri.shape) != (B, heads, N, N):
        raise ValueError(f"tri must be [B, heads, N, N] = {(B, heads, N, N)}, got {tuple(tri.shape)}")
    if mask is not None:
        _require_cuda(mask, "mask", torch.float32)
        if tuple(mask.shape) != (B, N, N) or not mask.is_contiguous():
            raise ValueError("mask must be a contiguous fp32 [B, N, N] tensor")
    return B, N, hd // heads


@dataclass
class AttnCorePacked:
    """The attention core's fp16 operand planes (gtk_attn_core_pack / _pack_bias)."""
    q: torch.Tensor
    k: torch.Tensor
    v: torch.Tensor
    tri: torch.Tensor
    B: int
    N: int
    heads: int
    head_dim: int


def attn_core_pack(x: torch.Tensor, heads: int, scale: float = 1.0) -> torch.Tensor:
    """fp32 [B, N, N, heads * d] -> the fp16 plane [B, N, heads, N, Dp] (times ``scale``)."""
    lib = _lib.load()
    B, N, _, hd = x.shape
    d = hd // heads
    nbytes = lib.gtk_attn_core_packed_bytes(B, N, heads, d)
    if nbytes == 0:
        raise ValueError("attention core: head_dim must be 1 .. 64")
    out = torch.empty(nbytes // 2, dtype=torch.float16, device=x.device)
    _lib.check(lib.gtk_attn_core_pack(_ptr(x), B, N, heads, d, float(scale), _ptr(out), _stream(x.device)),
               "gtk_attn_core_pack")
    return out


def attn_core_pack_bias(tri: torch.Tensor) -> torch.Tensor:
    """fp32 tri [B, H, N, N] -> the fp16 plane [B, H, N, Np]."""
    lib = _lib.load()
    B, H, N, _ = tri.shape
    out = torch.empty(lib.gtk_attn_core_bias_bytes(B, N, H) // 2, dtype=torch.float16, device=tri.device)
    _lib.check(lib.gtk_attn_core_pack_bias(_ptr(tri), B, N, H, _ptr(out), _stream(tri.device)),
               "gtk_attn_core_pack_bias")
    return out


def attn_core_forward(q, k, v, tri, mask, heads: int, inf: float = 1e9):
    """o = softmax(q k^T / sqrt(d) + inf (mask - 1) + tri) v per (b, i, h), the softmax
    statistics [B, N, heads, N, 2] and the packed operands (for the backward), without
    forming the scores. q, k, v fp32 [B, N, N, heads * d], tri fp32 [B, heads, N, N]."""
    lib = _lib.load()
    B, N, d = _core_args(q, k, v, tri, mask, heads)
    pk = AttnCorePacked(attn_core_pack(q, heads), attn_core_pack(k, heads), attn_core_pack(v, heads),
                        attn_core_pack_bias(tri), B, N, heads, d)
    o = torch.empty_like(q)
    stats = torch.empty(B, N, heads, N, 2, dtype=torch.float32, device=q.device)
    _lib.check(lib.gtk_attn_core_forward(_ptr(pk.q), _ptr(pk.k), _ptr(pk.v), _ptr(pk.tri), _ptr(mask), B, N, heads,
                                         d, float(inf), _ptr(o), _ptr(stats), _stream(q.device)),
               "gtk_attn_core_forward")
    return o, stats, pk


def attn_core_backward(pk: AttnCorePacked, mask, stats, o, do, inf: float = 1e9):
    """(dq, dk, dv, dtri) of the attention core for the output gradient ``do``.

    ``do`` enters its fp16 plane times a power of two that brings its largest element into
    [0.5, 1), so gradients of any magnitude keep 11 bits."""
    lib = _lib.load()
    B, N, H, d = pk.B, pk.N, pk.heads, pk.head_dim
    do = do.float().contiguous()
    dq, dk, dv = (torch.empty(B, N, N, H * d, dtype=torch.float32, device=do.device) for _ in range(3))
    dtri = torch.empty(B, H, N, N, dtype=torch.float32, device=do.device)
    amax = float(do.abs().max())
    if amax == 0.0:
        return dq.zero_(), dk.zero_(), dv.zero_(), dtri.zero_()
    if not math.isfinite(amax):
        raise ValueError("attention core backward: the output gradient is not finite")
    scale = math.ldexp(1.0, -math.frexp(amax)[1])  # amax * scale in [0.5, 1)
    dsum = (do * o).view(B, N, N, H, d).sum(-1).permute(0, 1, 3, 2).contiguous()  # [B, N(i), H, N(j)]
    doh = attn_core_pack(do, H, scale)
    _lib.check(lib.gtk_attn_core_backward(_ptr(pk.q), _ptr(pk.k), _ptr(pk.v), _ptr(pk.tri), _ptr(mask), _ptr(stats),
                                          _ptr(doh), _ptr(dsum), scale, B, N, H, d, float(inf), _ptr(dq), _ptr(dk),
                                          _ptr(dv), _ptr(dtri), _stream(do.device)), "gtk_attn_core_backward")
    return dq, dk, dv, dtri


# --------------------------------------------------------------------------------------
# LayerNorm over the last axis (the reference's _C.layernorm)
# --------------------------------------------------------------------------------------

def layernorm(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, eps: float = 1e-5,
              out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """LayerNorm over the last axis in fp32 (gtk_layernorm); returns fp32 of x's shape."""
    lib = _lib.load()
    _require_cuda(x, "x")
    D = x.shape[-1]
    xf = x.float().contiguous()
    g = gamma.detach().float().contiguous()
    b = beta.detach().float().contiguous()
    _require_cuda(g, "gamma")
    _require_cuda(b, "beta")
    if g.numel() != D or b.numel() != D:
        raise ValueError(f"gamma and beta must have {D} elements")
    if out is None:
        out = torch.empty_like(xf)
    _require_cuda(out, "out", torch.float32)
    rows = xf.numel() // D
    _lib.check(lib.gtk_layernorm(_ptr(xf), _ptr(g), _ptr(b), _ptr(out), rows, D, float(eps), _stream(x.device)),
               "gtk_layernorm")
    return out


# --------------------------------------------------------------------------------------
# Pair embedding producer: p[b,i,j] = Linear(2 c_s, c_p)([s_i ; s_j]), p_mask = m_i m_j
# --------------------------------------------------------------------------------------

def pair_embed(s: torch.Tensor, mask: Optional[torch.Tensor], weight: torch.Tensor, bias: Optional[torch.Tensor],
               rows: Optional[int] = None, row0: int = 0, with_mask: bool = True):
    """Pair representation [B, rows, N, c_p] fp32 (rows row0 .. row0+rows-1 of the N x N
    grid; all by default) and, with ``with_mask``, the pair mask [B, rows, N]."""
    lib = _lib.load()
    _require_cuda(s, "s")
    if s.dim() != 3:
        raise ValueError(f"s must be [B, N, c_s], got {tuple(s.shape)}")
    B, N, c_s = s.shape
    c_p = weight.shape[0]
    if not 1 <= c_p <= 4096:
        raise NotImplementedError(f"genie_tk (B200): pair embedding takes c_p in 1..4096, got {c_p}")
    if tuple(weight.shape) != (c_p, 2 * c_s):
        raise ValueError(f"weight must be [c_p, 2 c_s] = [{c_p}, {2 * c_s}], got {tuple(weight.shape)}")
    rows = N if rows is None else int(rows)
    sf = s.float().contiguous()
    wf = weight.detach().float().contiguous()
    _require_cuda(wf, "weight")
    bf = None if bias is None else bias.detach().float().contiguous()
    mf = None
    if mask is not None:
        _require_cuda(mask, "mask")
        if tuple(mask.shape) != (B, N):
            raise ValueError(f"mask must be [B, N], got {tuple(mask.shape)}")
        mf = mask.float().contiguous()
    out = torch.empty(B, rows, N, c_p, dtype=torch.float32, device=s.device)
    pm = torch.empty(B, rows, N, dtype=torch.float32, device=s.device) if with_mask else None
    nbytes = lib.gtk_pair_embed_workspace_bytes(B, N, c_p)
    ws = workspace(s.device, nbytes, tag="embed")
    _lib.check(lib.gtk_pair_embed(_ptr(sf), _ptr(mf), _ptr(wf), _ptr(bf), _ptr(out), _ptr(pm), _ptr(ws), ws.numel(),
                                  B, N, rows, int(row0), c_s, c_p, _stream(s.device)), "gtk_pair_embed")
    return out, pm


# --------------------------------------------------------------------------------------
# Linear layers and the generic attention core of the reference's Attention module
# --------------------------------------------------------------------------------------

def _rows_2d(x: torch.Tensor, name: str) -> torch.Tensor:
    _require_cuda(x, name, torch.float32)
    return x.reshape(-1, x.shape[-1]).contiguous()


def _weight(weight: torch.Tensor, d_in: int) -> torch.Tensor:
    _require_cuda(weight, "weight", torch.float32)
    if weight.dim() != 2 or weight.shape[1] != d_in:
        raise ValueError(f"weight must be [D_out, {d_in}], got {tuple(weight.shape)}")
    return weight.contiguous()


def _bias(bias: Optional[torch.Tensor], d_out: int) -> Optional[torch.Tensor]:
    if bias is None:
        return None
    _require_cuda(bias, "bias", torch.float32)
    if bias.numel() != d_out:
        raise ValueError(f"bias must have {d_out} elements")
    return bias.contiguous()


def layernorm_linear(x: torch.Tensor, gamma: torch.Tensor, beta: torch.Tensor, weight: torch.Tensor,
                     bias: Optional[torch.Tensor] = None, eps: float = 1e-5) -> torch.Tensor:
    """LayerNorm(x) weight^T + bias in one kernel (gtk_layernorm_linear); weight [D_out, D_in]."""
    lib = _lib.load()
    x2 = _rows_2d(x, "x")
    D_in = x2.shape[1]
    w = _weight(weight, D_in)
    b = _bias(bias, w.shape[0])
    for t, n in ((gamma, "gamma"), (beta, "beta")):
        _require_cuda(t, n, torch.float32)
        if t.numel() != D_in:
            raise ValueError(f"{n} must have {D_in} elements")
    out = torch.empty(x2.shape[0], w.shape[0], dtype=torch.float32, device=x.device)
    _lib.check(lib.gtk_layernorm_linear(_ptr(x2), _ptr(gamma.contiguous()), _ptr(beta.contiguous()), _ptr(w), _ptr(b),
                                        _ptr(out), x2.shape[0], D_in, w.shape[0], float(eps), _stream(x.device)),
               "gtk_layernorm_linear")
    return out.view(*x.shape[:-1], w.shape[0])


def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor] = None,
           gate: Optional[torch.Tensor] = None) -> torch.Tensor:
    """(x * sigmoid(gate)) weight^T + bias (gtk_linear); weight [D_out, D_in], gate like x."""
    lib = _lib.load()
    x2 = _rows_2d(x, "x")
    D_in = x2.shape[1]
    w = _weight(weight, D_in)
    b = _bias(bias, w.shape[0])
    g = None
    if gate is not None:
        if gate.shape != x.shape:
            raise ValueError("gate must have x's shape")
        g = _rows_2d(gate, "gate")
    out = torch.empty(x2.shape[0], w.shape[0], dtype=torch.float32, device=x.device)
    _lib.check(lib.gtk_linear(_ptr(x2), _ptr(g), _ptr(w), _ptr(b), _ptr(out), x2.shape[0], D_in, w.shape[0],
                              _stream(x.device)), "gtk_linear")
    return out.view(*x.shape[:-1], w.shape[0])


def _merged_stride(shape, strides):
    """The one stride of axes that index memory as a single merged axis, or None."""
    dims = [(n, st) for n, st in zip(shape, strides) if n != 1]
    for (_, s_outer), (n_inner, s_inner) in zip(dims, dims[1:]):
        if s_outer != s_inner * n_inner:
            return None
    return dims[-1][1] if dims else 0


def _bias_layout(biases, batch: tuple, heads: int, Q: int, K: int):
    """Biases broadcastable to [*batch, heads, Q, K] as tensors with five element strides
    over (l0, l1, h, q, k), for one split of the batch axes into two levels L0 x L1:
    broadcast axes read with stride 0, in place. A bias whose batch axes fit no common split
    is made contiguous first."""
    full = tuple(batch) + (heads, Q, K)
    exp = []
    for b in biases:
        if b.dim() > len(full):
            raise ValueError(f"bias of shape {tuple(b.shape)} does not broadcast to {full}")
        exp.append(b.float().expand(*full))
    nb = len(batch)

    def split_ok(p, tensors):
        return all(_merged_stride(batch[:p], t.stride()[:p]) is not None and
                   _merged_stride(batch[p:], t.stride()[p:nb]) is not None for t in tensors)

    split = next((p for p in range(nb + 1) if split_ok(p, exp)), None)
    if split is None:
        exp = [t if split_ok(0, [t]) else t.contiguous() for t in exp]
        split = 0
    L0 = math.prod(batch[:split])
    L1 = math.prod(batch[split:])
    out = []
    for t in exp:
        st = t.stride()
        strides = torch.tensor([_merged_stride(batch[:split], st[:split]),
                                _merged_stride(batch[split:], st[split:nb]), st[nb], st[nb + 1], st[nb + 2]],
                               dtype=torch.int64)
        out.append((t, strides))
    return out, L0, L1


def mha_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, heads: int, scale: float,
                biases: Optional[list] = None) -> torch.Tensor:
    """o[*, Q, H*d] = softmax(scale q k^T + sum(biases)) v per head (gtk_mha_forward).

    q [*, Q, H*d], k, v [*, K, H*d] fp32; each bias broadcastable to [*, H, Q, K] (at most
    two; more are summed first)."""
    lib = _lib.load()
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _require_cuda(t, n, torch.float32)
    batch = tuple(q.shape[:-2])
    Q, hd = q.shape[-2], q.shape[-1]
    K = k.shape[-2]
    if tuple(k.shape[:-2]) != batch or k.shape != v.shape or k.shape[-1] != hd or hd % heads:
        raise ValueError("q [*, Q, H*d], k and v [*, K, H*d] with one batch shape")
    d = hd // heads
    biases = [b.to(q.device) for b in (biases or []) if b is not None]
    if len(biases) > 2:
        biases = [sum(biases[1:], biases[0])]
    L = math.prod(batch)
    q3, k3, v3 = (t.reshape(L, -1, hd).contiguous() for t in (q, k, v))
    o = torch.empty(L, Q, hd, dtype=torch.float32, device=q.device)
    layout, L0, L1 = _bias_layout(biases, batch, heads, Q, K)
    layout += [(None, None)] * (2 - len(layout))
    (b0, s0), (b1, s1) = layout
    sp = [None if st is None else ctypes.c_void_p(st.data_ptr()) for st in (s0, s1)]
    _lib.check(lib.gtk_mha_forward(_ptr(q3), _ptr(k3), _ptr(v3), _ptr(b0), sp[0], _ptr(b1), sp[1], L0, L1, Q, K,
                                   heads, d, float(scale), _ptr(o), _stream(q.device)), "gtk_mha_forward")
    return o.view(*batch, Q, hd)
