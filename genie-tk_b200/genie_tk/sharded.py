"""Row-sharded triangle pair stack: the pair tensor [B, N, N, 128] split over its first
pair index i across P ranks (one process per GPU), R = N / P rows per rank.

Each op needs one exchange between the ranks; the kernels run on local data only and
every exchange goes through the collective into local memory first:

  TriMulOut / TriMulIn   x[i,j,c] = sum_k a[i,k,c] b[j,k,c] (outgoing) or a[k,i,c] b[k,j,c]
              (incoming), two exchanges to choose from (``trimul_exchange``):
              "channels": the per-channel contractions are independent, so after projecting
              its rows each rank trades planes with an all-to-all from row shards to channel
              shards (all N rows, its C/P channels), runs full N x N contractions for its
              channels (outgoing and incoming alike), and an all-to-all of x brings the rows
              back for the LN_out / gate epilogue: 3 (P-1)/P planes per rank and op (84 MB at
              N = 1024, P = 8);
              "gather": the b planes are all-gathered (every rank needs all rows j) and, for
              the incoming update, an all-to-all gives each rank its columns i of every row
              k of a; local rows i are contracted against all j: (P-1) planes (+ (P-1)/P).
              "auto": channels whenever the x exchange is fused into the contraction's stores
              (peer exchange, rows per rank a multiple of 128), else the one that moves
              fewer bytes (gather for P <= 3).
  TriAttStart local rows i; the triangle bias bias[h, j, k] is needed for all rows j, so
              each rank computes its rows and the bias region is all-gathered.
  TriAttEnd   End(z) = Start(z^T)^T with the mask transposed: an all-to-all transpose
              (gtk_pair_transpose_pack + gtk_copy_2d) turns the row shard into the shard of
              z^T, the starting-node stages run on it with the residual added in place,
              and the same transpose brings the updated shard back.

The per-rank program is a generator that yields its collectives (``("all_gather", out,
inp)`` / ``("all_to_all", out, inp)`` on uint8 views), so the same code runs on real
ranks (``forward_`` with ``torch.distributed``: NCCL on GPUs) and on P ranks emulated in
one process (``run_emulated``, used to check the sharding on a single device). The stage
computations go through a ``stage_ops`` object; the default, ``CudaStageOps``, calls the
library's kernels, and there is no CPU implementation in this package.

The reference has no multi-GPU path (its modules run on one device); this follows the
row sharding of the pair stack over i with all-gather / all-to-all exchanges.
"""

from __future__ import annotations

import ctypes
from typing import Dict, Generator, List, Optional, Tuple

import torch
from torch import Tensor

from . import ops
from .stack import OP_NAMES, TrianglePairStack

C = 128
H = 4
PAIR_BYTES = C * 4

Request = Tuple[str, Tensor, Tensor]


class ShardSpec:
    """Rows owned by ``rank`` out of ``world`` for a [B, N, N, 128] pair tensor."""

    def __init__(self, B: int, N: int, world: int, rank: int):
        if world < 1 or not 0 <= rank < world:
            raise ValueError(f"bad world/rank {world}/{rank}")
        if N % world:
            raise ValueError(f"N = {N} is not divisible by the {world} ranks")
        R = N // world
        if R % 8:
            raise ValueError(f"rows per rank N / P = {R} must be a multiple of 8 (16-byte plane slices)")
        self.B, self.N, self.P, self.rank = B, N, world, rank
        self.R = R
        self.row0 = rank * R

    def rows(self) -> slice:
        return slice(self.row0, self.row0 + self.R)


class CudaStageOps:
    """The stage computations on this rank's GPU, through the C ABI.

    ``push``: "kernel" moves the peer pushes of strided slabs (``push_3d``) with the push
    kernel; "dma" issues one ``cudaMemcpy2DAsync`` per destination rank on the same stream
    (the copy engines, no SM time). The pair-grid transposes always use their kernel."""

    def __init__(self, device: torch.device, push: str = "kernel"):
        if push not in ("kernel", "dma"):
            raise ValueError(f"push must be 'kernel' or 'dma', got {push!r}")
        self.device = device
        self.push = push
        self.lib = ops._lib.load()
        self.status = ops.status_buffer(device)

    def alloc(self, nbytes: int) -> Tensor:
        return torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=self.device)

    def _s(self):
        return ops._stream(self.device)

    def _chk(self, rc, what):
        ops._lib.check(rc, what)

    def trimul_project(self, mod, z, mask, a, b, B, rows, N):
        P = ops._ptr
        self._chk(self.lib.gtk_trimul_project(P(z), P(mask), P(mod.packed_weights(self.device)), P(a), P(b), N, B,
                                              rows, N, P(self.status), self._s()), "gtk_trimul_project")

    def trimul_contract(self, outgoing, a, b, x, B, M, Nj, K, lda, ldb, ldx, xs, channels=C):
        P = ops._ptr
        self._chk(self.lib.gtk_trimul_contract(int(outgoing), P(a), P(b), P(x), B, channels, M, Nj, K, lda, ldb, ldx,
                                               xs, P(self.status), self._s()), "gtk_trimul_contract")

    def trimul_finish(self, mod, z, x, ldx, xs, B, rows, N, out):
        P = ops._ptr
        self._chk(self.lib.gtk_trimul_finish(P(z), P(x), ldx, xs, P(mod.packed_weights(self.device)), P(out), 1, B,
                                             rows, N, P(self.status), self._s()), "gtk_trimul_finish")

    def triatt_project(self, mod, z, ws, B, rows, N, row0):
        P = ops._ptr
        self._chk(self.lib.gtk_triatt_project(1, P(z), P(mod.packed_weights(self.device)), P(ws), B, rows, N, row0,
                                              P(self.status), self._s()), "gtk_triatt_project")

    def triatt_core(self, mod, mask, ws, B, rows, N, row0):
        P = ops._ptr
        self._chk(self.lib.gtk_triatt_core(1, P(mask), P(ws), B, rows, N, row0, float(mod.inf), P(self.status),
                                           self._s()), "gtk_triatt_core")

    def triatt_finish(self, mod, z, ws, B, rows, N):
        P = ops._ptr
        self._chk(self.lib.gtk_triatt_finish(1, P(z), P(mod.packed_weights(self.device)), P(ws), P(z), 1, B, rows,
                                             N, P(self.status), self._s()), "gtk_triatt_finish")

    def trimul_contract_to(self, outgoing, a, b, B, M, Nj, K, lda, ldb, xs, channels, dst: "PeerBuffer", c_off,
                           ld_dst):
        """K2 of the channel-sharded exchange with the x scatter fused into its stores: the x
        tiles of rows owned by rank p go straight into p's x planes at channels c_off.."""
        P = ops._ptr
        bases = (ctypes.c_uint64 * len(dst.addrs))(*dst.addrs)
        self._chk(self.lib.gtk_trimul_contract_to_peers(int(outgoing), P(a), P(b), bases, len(dst.addrs), B, channels,
                                                        M, Nj, K, lda, ldb, C, c_off, ld_dst, xs, P(self.status),
                                                        self._s()), "gtk_trimul_contract_to_peers")

    def triatt_finish_to(self, mod, z, ws, B, rows, N, row0, dst: "PeerBuffer"):
        """K4e with the pair-grid transpose fused into its stores: z + update, transposed,
        straight into every rank's shard of ``dst``."""
        P = ops._ptr
        bases = (ctypes.c_uint64 * len(dst.addrs))(*dst.addrs)
        self._chk(self.lib.gtk_triatt_finish_to_peers(P(z), P(mod.packed_weights(self.device)), P(ws), bases,
                                                      len(dst.addrs), B, rows, N, row0, 1, P(self.status),
                                                      self._s()), "gtk_triatt_finish_to_peers")

    def copy_2d(self, dst, dpitch, src, spitch, width, height):
        self._chk(self.lib.gtk_copy_2d(ops._ptr(dst), dpitch, ops._ptr(src), spitch, width, height, self._s()),
                  "gtk_copy_2d")

    def copy_3d(self, dst, dpitch, dslab, src, spitch, sslab, width, height, depth):
        self._chk(self.lib.gtk_copy_3d(ops._ptr(dst), dpitch, dslab, ops._ptr(src), spitch, sslab, width, height,
                                       depth, self._s()), "gtk_copy_3d")

    def pair_transpose_pack(self, src, dst, B, R, Cn, P):
        self._chk(self.lib.gtk_pair_transpose_pack(ops._ptr(src), ops._ptr(dst), B, R, Cn, P, self._s()),
                  "gtk_pair_transpose_pack")

    def trimul_project_to(self, mod, z, mask, a_dst: "PeerBuffer", b_dst: "PeerBuffer", B, rows, N, row0):
        """K1 for a shard, writing channel group q of the planes straight into a_dst / b_dst
        of rank q (rows row0.. of its [B][N][128/P][N] channel shard)."""
        P = len(a_dst.addrs)
        At = ctypes.c_void_p * P
        a_tab = At(*[ctypes.c_void_p(a) for a in a_dst.addrs])
        b_tab = At(*[ctypes.c_void_p(a) for a in b_dst.addrs])
        self._chk(self.lib.gtk_trimul_project_sharded(ops._ptr(z), ops._ptr(mask), ops._ptr(mod.packed_weights(self.device)),
                                                      a_tab, b_tab, P, N, row0, N, B, rows, N, ops._ptr(self.status),
                                                      self._s()), "gtk_trimul_project_sharded")

    def push_3d(self, dst: "PeerBuffer", doff, dpitch, src, spitch, sslab, width, height):
        if self.push == "dma":
            base = src.data_ptr()
            for k, addr in enumerate(dst.addrs):
                self._chk(self.lib.gtk_copy_2d_dma(ctypes.c_void_p(addr + doff), dpitch,
                                                   ctypes.c_void_p(base + k * sslab), spitch, width, height,
                                                   self._s()), "gtk_copy_2d_dma")
            return
        self._chk(self.lib.gtk_push_3d(ops._ptr(dst.ptrs), dst.ptrs.numel(), doff, dpitch, ops._ptr(src), spitch, sslab,
                                       width, height, self._s()), "gtk_push_3d")

    def push_pair_transpose(self, src, dst: "PeerBuffer", B, R, Cn, P, ndst, row0):
        self._chk(self.lib.gtk_push_pair_transpose(ops._ptr(src), ops._ptr(dst.ptrs), B, R, Cn, P, ndst, row0,
                                                   self._s()), "gtk_push_pair_transpose")

    def triatt_layout(self, B, rows, N) -> Dict[str, int]:
        offs = (ctypes.c_int64 * 7)()
        self._chk(self.lib.gtk_triatt_workspace_offsets(B, rows, N, offs), "gtk_triatt_workspace_offsets")
        return {k: int(offs[n]) for n, k in enumerate(("q", "k", "v", "g", "og", "bias", "total"))}


def _round256(n: int) -> int:
    return (int(n) + 255) // 256 * 256


class PeerBuffer:
    """A receive buffer that every rank may write into: this rank's ``local`` uint8 tensor
    and ``ptrs``, a device int64 tensor with the base address of the same buffer on every
    rank (peer buffers mapped into this process, or, for ranks emulated in one process,
    their local tensors, which are also listed in ``tensors``)."""

    def __init__(self, local: Tensor, addrs: List[int], device, tensors: Optional[List[Tensor]] = None):
        self.local, self.addrs, self.tensors = local, list(addrs), tensors
        self.ptrs = torch.tensor(self.addrs, dtype=torch.int64, device=device)


class _CudaArray:
    """Exposes a device allocation to ``torch.as_tensor`` (``__cuda_array_interface__``)."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 3, "strides": None}


class ShardedTrianglePairStack:
    """One rank's share of a :class:`TrianglePairStack` whose pair tensor is row-sharded.

    ``forward_(z_local, mask)`` updates this rank's rows ``z_local`` [B, N/P, N, 128] (fp32)
    in place; ``mask`` is the whole [B, N, N] mask (or None), identical on every rank.

    ``exchange``: "nccl" runs the exchanges as NCCL collectives on packed chunks; "peer"
    pushes every rank's share straight into the peers' buffers with the exchange kernels
    (CUDA IPC mappings over NVLink) and orders them with a device-side barrier. Peer mode
    needs ``connect(group, B, N)`` once (a collective) before ``forward_``, and ``close()``.
    """

    def __init__(self, stack: TrianglePairStack, world: int, rank: int, stage_ops=None,
                 trimul_exchange: str = "auto", exchange: str = "nccl", k1_direct: bool = False,
                 push: str = "kernel", fused_transpose: bool = True, fused_x: bool = True):
        if trimul_exchange not in ("auto", "gather", "channels"):
            raise ValueError(f"trimul_exchange must be auto, gather or channels, not {trimul_exchange!r}")
        if exchange not in ("nccl", "peer"):
            raise ValueError(f"exchange must be nccl or peer, not {exchange!r}")
        self.stack = stack
        self.world, self.rank = world, rank
        self.stage_ops = stage_ops
        self.exchange = exchange
        # peer mode, channel shards: K1 stores each channel group straight into its owner's
        # buffer (no push pass). Measured slower on 8 B200s (14.7 vs 14.1 ms per step): the
        # epilogue's 32-byte stores spread over the peers use NVLink less well than one bulk
        # push, so it is off by default.
        self.k1_direct = k1_direct
        self.push = push  # slab pushes of the default stage ops: "kernel" or "dma" (CudaStageOps)
        # peer mode: the attention blocks' K4e writes its output transposed straight into the
        # peers' shards (one kernel instead of K4e + a transpose push), when each rank's rows
        # are a multiple of 128
        self.fused_transpose = fused_transpose
        # peer mode, channel shards: K2 stores the x tiles straight into their row owners'
        # planes (one kernel instead of K2 + the x push), when each rank's rows are a
        # multiple of 128
        self.fused_x = fused_x
        # "auto" is settled once N is known (the buffers are sized); until then the byte rule
        self._trimul_request = trimul_exchange
        self.trimul_exchange = self._resolve_trimul_exchange(None) if trimul_exchange == "auto" else trimul_exchange
        self._key = None
        self._buf: Dict[str, Tensor] = {}
        self._peer: Dict[str, PeerBuffer] = {}
        self._ipc_own: List[int] = []     # allocations made here (peer_alloc)
        self._ipc_open: List[int] = []    # peer mappings opened here
        self._epoch = 0

    def _resolve_trimul_exchange(self, N: Optional[int]) -> str:
        """The multiplicative update's exchange for "auto" (N = None: not known yet).

        Bytes each rank moves per update outside the kernels: the gather (P-1) planes (+
        (P-1)/P for the incoming a), the channel shards 3 (P-1)/P -- the gather wins for
        P <= 3. With the peer exchange and a multiple of 128 rows per rank, the channel
        shards' x exchange is fused into the contraction's stores, leaving 2 (P-1)/P planes
        of pushes, fewer than the gather's at every P: 33.0-33.3 against 33.6 ms per step on
        2 B200s at N = 1024, both bitwise equal to the one-GPU result."""
        fused = self.exchange == "peer" and self.fused_x and N is not None and (N // self.world) % 128 == 0
        if fused:
            return "channels"
        return "gather" if self.world <= 3 else "channels"

    # ---------------------------------------------------------------- buffers
    def _sizes(self, spec: ShardSpec):
        """(local buffers, buffers other ranks write into), name -> bytes."""
        B, N, R = spec.B, spec.N, spec.R
        if self._trimul_request == "auto":
            self.trimul_exchange = self._resolve_trimul_exchange(N)
        plane = B * R * C * N * 2          # one rank's planes, fp16, pitch N (row or channel shard)
        lay = self.stage_ops.triatt_layout(B, R, N)
        pair_loc = B * R * N * PAIR_BYTES  # one row shard of the pair tensor, fp32
        local = {"a": plane, "b": plane}
        recv = {"tri": lay["total"], "zT": pair_loc}
        if self.trimul_exchange == "channels":
            local["x_ch"] = plane                                   # [B][N][C/P][N]
            recv.update({"a_ch": plane, "b_ch": plane, "x": plane})
        else:
            local["x"] = plane
            recv["a_recv"] = plane                                  # [B][N][C][R]
            if self.exchange == "nccl":
                recv["b_all"] = B * N * C * N * 2                  # [B][N][C][N]
            else:
                # two copies: a push for the incoming update must not land in the buffer the
                # outgoing contraction of a slower rank may still be reading (no barrier
                # separates them in this exchange)
                recv["b_all0"] = recv["b_all1"] = B * N * C * N * 2
        if self.exchange == "nccl":
            local.update({"send": plane, "x_recv": plane, "bias_send": R * B * H * N * 2,
                          "t_send": pair_loc, "t_recv": pair_loc})
            local.update(recv)
            recv = {}
        else:
            recv.update({"zs": pair_loc, "flags": 256})   # the residual stream; barrier flags
        return local, recv, lay

    def prepare(self, B: int, N: int, device: torch.device) -> ShardSpec:
        spec = ShardSpec(B, N, self.world, self.rank)
        if self.stage_ops is None:
            self.stage_ops = CudaStageOps(device, push=self.push)
        if self._key == (B, N):
            return spec
        if self.exchange == "peer":
            raise RuntimeError("ShardedTrianglePairStack(exchange='peer'): call connect() (or connect_emulated) "
                               "before running")
        local, recv, lay = self._sizes(spec)
        so = self.stage_ops
        self._buf = {k: so.alloc(_round256(v)) for k, v in local.items()}
        self._lay = lay
        self._key = (B, N)
        self._pack_weights(device)
        return spec

    def _pack_weights(self, device):
        so = self.stage_ops
        if isinstance(so, CudaStageOps) or isinstance(getattr(so, "inner", None), CudaStageOps):
            for layer in self.stack.layers:
                for name in OP_NAMES:
                    getattr(layer, name).packed_weights(device)

    @torch.no_grad()
    def connect(self, group, B: int, N: int, device: torch.device) -> None:
        """Peer mode, one process per GPU: allocate the receive buffers in IPC-shareable
        memory, exchange their handles over ``group`` and map the peers' buffers. A
        collective: every rank calls it with the same B and N."""
        import torch.distributed as dist
        if self.exchange != "peer":
            raise RuntimeError("connect() is for exchange='peer'")
        spec = ShardSpec(B, N, self.world, self.rank)
        if self.stage_ops is None:
            self.stage_ops = CudaStageOps(device, push=self.push)
        self.close()
        local, recv, lay = self._sizes(spec)
        lib = ops._lib.load()
        so = self.stage_ops
        self._buf = {k: so.alloc(_round256(v)) for k, v in local.items()}
        handles = {}
        for name, nbytes in recv.items():
            nbytes = _round256(nbytes)
            ptr = ctypes.c_void_p()
            h = ctypes.create_string_buffer(64)
            ops._lib.check(lib.gtk_peer_alloc(nbytes, ctypes.byref(ptr), h), "gtk_peer_alloc")
            self._ipc_own.append(ptr.value)
            self._buf[name] = torch.as_tensor(_CudaArray(ptr.value, nbytes), device=device)
            handles[name] = (h.raw, nbytes)
        gathered = [None] * self.world
        dist.all_gather_object(gathered, handles, group=group)
        for name in recv:
            addrs = []
            for q in range(self.world):
                if q == self.rank:
                    addrs.append(self._buf[name].data_ptr())
                    continue
                ptr = ctypes.c_void_p()
                ops._lib.check(lib.gtk_peer_open(gathered[q][name][0], ctypes.byref(ptr)), "gtk_peer_open")
                self._ipc_open.append(ptr.value)
                addrs.append(ptr.value)
            self._peer[name] = PeerBuffer(self._buf[name], addrs, device)
        self._lay = lay
        self._key = (B, N)
        self._epoch = 0
        self._pack_weights(device)
        dist.barrier(group=group)

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's IPC allocations (peer mode)."""
        if not (self._ipc_open or self._ipc_own):
            return
        lib = ops._lib.load()
        torch.cuda.synchronize()
        for p in self._ipc_open:
            lib.gtk_peer_close(ctypes.c_void_p(p))
        self._peer.clear()
        self._buf.clear()
        for p in self._ipc_own:
            lib.gtk_peer_free(ctypes.c_void_p(p))
        self._ipc_open, self._ipc_own = [], []
        self._key = None

    # ---------------------------------------------------------------- the per-rank program
    def steps(self, z: Tensor, mask: Optional[Tensor], z_in: Optional[Tensor] = None
              ) -> Generator[Request, None, None]:
        """This rank's stack as a generator of exchange requests (see module docstring).
        ``z`` is updated in place; with ``z_in`` the first block reads ``z_in`` instead and
        writes ``z`` (``z_in`` is left unchanged)."""
        B, R, N = z.shape[0], z.shape[1], z.shape[2]
        spec = self.prepare(B, N, z.device) if self.exchange == "nccl" else ShardSpec(B, N, self.world, self.rank)
        if self._key != (B, N):
            raise RuntimeError("ShardedTrianglePairStack: connect() was made for other sizes")
        if R != spec.R:
            raise ValueError(f"z_local has {R} rows; rank {self.rank} of {self.world} owns {spec.R}")
        if self.exchange == "peer":
            yield from self._steps_peer(z, mask, z_in, spec)
        else:
            yield from self._steps_nccl(z, mask, z_in, spec)

    def _common(self, z, mask, spec):
        B, N, R = spec.B, spec.N, spec.R
        mask_loc = mask_t = None
        if mask is not None:
            mask_loc = mask[:, spec.rows()].contiguous()
            mask_t = mask.transpose(1, 2).contiguous()
        tri = self._buf["tri"]
        lay = self._lay
        bias_all = tri[lay["bias"]:lay["bias"] + N * B * H * N * 2]
        bias_mine = bias_all[spec.row0 * B * H * N * 2:(spec.row0 + R) * B * H * N * 2]
        zT = self._buf["zT"][:B * R * N * PAIR_BYTES].view(torch.float32).view(B, R, N, C)
        return mask_loc, mask_t, tri, bias_all, bias_mine, zT

    def _steps_nccl(self, z, mask, z_in, spec):
        so, buf = self.stage_ops, self._buf
        B, N, R, P, row0 = spec.B, spec.N, spec.R, self.world, spec.row0
        CP = C // P
        src = z if z_in is None else z_in
        mask_loc, mask_t, tri, bias_all, bias_mine, zT = self._common(z, mask, spec)
        xs = 1.0 / N
        plane_b = R * C * N * 2            # bytes of one batch element's planes (row or channel shard)
        chunk = R * CP * N * 2             # one peer's share of them
        pair_chunk = B * R * R * PAIR_BYTES  # one peer's chunk of a pair-grid transpose
        t_send, t_recv = buf["t_send"], buf["t_recv"]

        def to_channels(rows_planes, ch_planes):
            # rows [R] x channels [C] -> all N rows x this rank's channel group [C/P]
            for bb in range(B):
                so.copy_3d(buf["send"], CP * N * 2, chunk, rows_planes[bb * plane_b:], C * N * 2, CP * N * 2,
                           CP * N * 2, R, P)
                yield ("all_to_all", ch_planes[bb * plane_b:(bb + 1) * plane_b], buf["send"][:plane_b])

        def to_rows(ch_planes, rows_planes):
            for bb in range(B):
                yield ("all_to_all", buf["x_recv"][:plane_b], ch_planes[bb * plane_b:(bb + 1) * plane_b])
                so.copy_3d(rows_planes[bb * plane_b:], C * N * 2, CP * N * 2, buf["x_recv"], CP * N * 2, chunk,
                           CP * N * 2, R, P)

        def multiply_channels(mod, outgoing, zz):
            so.trimul_project(mod, zz, mask_loc, buf["a"], buf["b"], B, R, N)
            yield from to_channels(buf["a"], buf["a_ch"])
            yield from to_channels(buf["b"], buf["b_ch"])
            # full N x N contractions for this rank's C/P channels
            so.trimul_contract(outgoing, buf["a_ch"], buf["b_ch"], buf["x_ch"], B, N, N, N, N, N, N, xs, CP)
            yield from to_rows(buf["x_ch"], buf["x"])
            so.trimul_finish(mod, zz, buf["x"], N, xs, B, R, N, z)

        def gather_b():
            for bb in range(B):
                yield ("all_gather", buf["b_all"][bb * N * C * N * 2:(bb + 1) * N * C * N * 2],
                       buf["b"][bb * plane_b:(bb + 1) * plane_b])

        def multiply_gather(mod, outgoing, zz):
            so.trimul_project(mod, zz, mask_loc, buf["a"], buf["b"], B, R, N)
            if outgoing:
                # x[i, j] for local rows i against all rows j of b
                yield from gather_b()
                so.trimul_contract(True, buf["a"], buf["b_all"], buf["x"], B, R, N, N, N, N, N, xs)
            else:
                # x[i, j] = sum_k a[k, i] b[k, j]: this rank's columns i of every row k of a
                for bb in range(B):
                    so.copy_3d(buf["send"], R * 2, R * C * R * 2, buf["a"][bb * plane_b:], N * 2, R * 2, R * 2, R * C,
                               P)
                    yield ("all_to_all", buf["a_recv"][bb * plane_b:(bb + 1) * plane_b], buf["send"][:plane_b])
                yield from gather_b()
                so.trimul_contract(False, buf["a_recv"], buf["b_all"], buf["x"], B, R, N, N, R, N, N, xs)
            so.trimul_finish(mod, zz, buf["x"], N, xs, B, R, N, z)

        multiply = multiply_channels if self.trimul_exchange == "channels" else multiply_gather

        def attention(mod, zz, mm):
            so.triatt_project(mod, zz, tri, B, R, N, row0)
            so.copy_2d(buf["bias_send"], bias_mine.numel(), bias_mine, bias_mine.numel(), bias_mine.numel(), 1)
            yield ("all_gather", bias_all, buf["bias_send"][:bias_mine.numel()])
            so.triatt_core(mod, mm, tri, B, R, N, row0)
            so.triatt_finish(mod, zz, tri, B, R, N)

        def transpose(src_pairs, dst_pairs):
            # dst = the transposed shard of the pair grid whose row shard is src
            so.pair_transpose_pack(src_pairs, t_send, B, R, N, P)
            yield ("all_to_all", t_recv[:P * pair_chunk], t_send[:P * pair_chunk])
            so.copy_3d(_bytes(dst_pairs), N * PAIR_BYTES, R * PAIR_BYTES, t_recv, R * PAIR_BYTES, pair_chunk,
                       R * PAIR_BYTES, B * R, P)

        for layer in self.stack.layers:
            yield from multiply(layer.tri_mul_out, True, src)
            yield from multiply(layer.tri_mul_in, False, z)
            yield from attention(layer.tri_att_start, z, mask)
            # TriAttEnd = Start(z^T, mask^T)^T, the residual added on the transposed shard
            yield from transpose(z, zT)
            yield from attention(layer.tri_att_end, zT, mask_t)
            yield from transpose(zT, z)
            src = z

    def _steps_peer(self, z_user, mask, z_in, spec):
        """Peer-memory exchanges. A push may overwrite a peer's receive buffer only once every
        rank has finished reading its previous contents; each exchange ends with a barrier
        that every rank enters after its own consumers of the previous exchange have run
        (stream order), so one barrier per exchange suffices for every buffer except the
        gathered b planes, whose outgoing and incoming uses follow each other with a single
        barrier in between and therefore alternate between two copies."""
        so, buf, peer = self.stage_ops, self._buf, self._peer
        B, N, R, P, row0, me = spec.B, spec.N, spec.R, self.world, spec.row0, self.rank
        CP = C // P
        mask_loc, mask_t, tri, bias_all, bias_mine, zT = self._common(z_user, mask, spec)
        # the residual stream lives in peer memory (the transposed-back updates land there)
        z = buf["zs"][:B * R * N * PAIR_BYTES].view(torch.float32).view(B, R, N, C)
        src = z
        if z_in is not None:
            src = z_in
        else:
            so.copy_2d(_bytes(z), z.numel() * 4, _bytes(z_user), z.numel() * 4, z.numel() * 4, 1)
        xs = 1.0 / N
        plane_b = R * C * N * 2
        tri_bias = self._lay["bias"]

        def multiply_channels(mod, outgoing, zz):
            if self.k1_direct:
                # K1 writes channel group q of my rows straight into rank q's channel shard
                so.trimul_project_to(mod, zz, mask_loc, peer["a_ch"], peer["b_ch"], B, R, N, row0)
            else:
                so.trimul_project(mod, zz, mask_loc, buf["a"], buf["b"], B, R, N)
                for bb in range(B):
                    # my rows, channel group q -> rows row0.. of rank q's channel shard
                    for name, planes in (("a_ch", buf["a"]), ("b_ch", buf["b"])):
                        so.push_3d(peer[name], (bb * N + row0) * CP * N * 2, CP * N * 2, planes[bb * plane_b:],
                                   C * N * 2, CP * N * 2, CP * N * 2, R)
            yield ("barrier",)
            if self.fused_x and R % 128 == 0 and hasattr(so, "trimul_contract_to"):
                # x tiles of peer p's rows straight into channel group `me` of p's x planes
                so.trimul_contract_to(outgoing, buf["a_ch"], buf["b_ch"], B, N, N, N, N, N, xs, CP, peer["x"],
                                      me * CP, N)
            else:
                so.trimul_contract(outgoing, buf["a_ch"], buf["b_ch"], buf["x_ch"], B, N, N, N, N, N, N, xs, CP)
                for bb in range(B):
                    # rows of peer p, my channel group -> channel group `me` of peer p's x rows
                    so.push_3d(peer["x"], (bb * R * C + me * CP) * N * 2, C * N * 2, buf["x_ch"][bb * plane_b:],
                               CP * N * 2, R * CP * N * 2, CP * N * 2, R)
            yield ("barrier",)
            so.trimul_finish(mod, zz, buf["x"], N, xs, B, R, N, z)

        def multiply_gather(mod, outgoing, zz):
            so.trimul_project(mod, zz, mask_loc, buf["a"], buf["b"], B, R, N)
            b_all = "b_all0" if outgoing else "b_all1"
            for bb in range(B):
                so.push_3d(peer[b_all], (bb * N + row0) * C * N * 2, plane_b, buf["b"][bb * plane_b:], plane_b, 0,
                           plane_b, 1)
                if not outgoing:
                    # columns i of peer q, every local row k and channel -> rows row0.. of q's a
                    so.push_3d(peer["a_recv"], (bb * N + row0) * C * R * 2, R * 2, buf["a"][bb * plane_b:], N * 2,
                               R * 2, R * 2, R * C)
            yield ("barrier",)
            if outgoing:
                so.trimul_contract(True, buf["a"], buf[b_all], buf["x"], B, R, N, N, N, N, N, xs)
            else:
                so.trimul_contract(False, buf["a_recv"], buf[b_all], buf["x"], B, R, N, N, R, N, N, xs)
            so.trimul_finish(mod, zz, buf["x"], N, xs, B, R, N, z)

        multiply = multiply_channels if self.trimul_exchange == "channels" else multiply_gather

        fuse = self.fused_transpose and R % 128 == 0 and hasattr(so, "triatt_finish_to")

        def attention(mod, zz, mm, dst_name=None):
            so.triatt_project(mod, zz, tri, B, R, N, row0)
            w = bias_mine.numel()
            so.push_3d(peer["tri"], tri_bias + row0 * B * H * N * 2, w, bias_mine, w, 0, w, 1)
            yield ("barrier",)
            so.triatt_core(mod, mm, tri, B, R, N, row0)
            if dst_name is None:
                so.triatt_finish(mod, zz, tri, B, R, N)
            else:
                # zz + update, transposed, straight into every rank's `dst_name` shard
                so.triatt_finish_to(mod, zz, tri, B, R, N, row0, peer[dst_name])
                yield ("barrier",)

        def transpose(src_pairs, dst_name):
            so.push_pair_transpose(src_pairs, peer[dst_name], B, R, N, P, N, row0)
            yield ("barrier",)

        for layer in self.stack.layers:
            yield from multiply(layer.tri_mul_out, True, src)
            yield from multiply(layer.tri_mul_in, False, z)
            # TriAttEnd = Start(z^T, mask^T)^T, the residual added on the transposed shard
            if fuse:
                yield from attention(layer.tri_att_start, z, mask, "zT")
                yield from attention(layer.tri_att_end, zT, mask_t, "zs")
            else:
                yield from attention(layer.tri_att_start, z, mask)
                yield from transpose(z, "zT")
                yield from attention(layer.tri_att_end, zT, mask_t)
                yield from transpose(zT, "zs")
            src = z
        so.copy_2d(_bytes(z_user), z.numel() * 4, _bytes(z), z.numel() * 4, z.numel() * 4, 1)

    # ---------------------------------------------------------------- runners
    @torch.no_grad()
    def forward_(self, z_local: Tensor, mask: Optional[Tensor] = None, group=None,
                 z_in: Optional[Tensor] = None, hook=None) -> Tensor:
        """Run this rank's share of the stack in place on ``z_local`` (reading ``z_in`` in
        the first block when given); exchanges over ``group``. ``hook(label)`` is called
        before and after (label "end") every exchange step."""
        import torch.distributed as dist
        if dist.get_world_size(group) != self.world or dist.get_rank(group) != self.rank:
            raise RuntimeError("ShardedTrianglePairStack: world/rank differ from the process group")
        _check_local(z_local, mask)
        if z_in is not None:
            _check_local(z_in, mask)
        h = hook or (lambda label: None)
        lib = ops._lib.load() if self.exchange == "peer" else None
        for req in self.steps(z_local, mask, z_in):
            kind = req[0]
            if kind == "barrier":
                h("peer_barrier")
                self._epoch += 1
                so = self.stage_ops
                dev = z_local.device
                ops._lib.check(lib.gtk_peer_barrier(ops._ptr(self._peer["flags"].ptrs), self.rank, self.world,
                                                    self._epoch, ops._ptr(ops.status_buffer(dev)), ops._stream(dev)),
                               "gtk_peer_barrier")
                if hasattr(so, "launches"):
                    so.launches += 1
            else:
                h("nccl_" + kind)
                _, out, inp = req
                if kind == "all_gather":
                    dist.all_gather_into_tensor(out, inp, group=group)
                elif kind == "all_to_all":
                    dist.all_to_all_single(out, inp, group=group)
                else:
                    raise RuntimeError(f"unknown exchange {kind}")
            h("end")
        return z_local


def connect_emulated(shards: List["ShardedTrianglePairStack"], B: int, N: int, device: torch.device) -> None:
    """Peer mode for P ranks emulated in one process: each shard's receive buffers are
    ordinary local allocations and every shard's pointer tables list all P of them."""
    P = len(shards)
    spec0 = None
    for s in shards:
        if s.exchange != "peer":
            raise RuntimeError("connect_emulated needs exchange='peer'")
        spec = ShardSpec(B, N, P, s.rank)
        spec0 = spec0 or spec
        if s.stage_ops is None:
            s.stage_ops = CudaStageOps(device, push=s.push)
        local, recv, lay = s._sizes(spec)
        so = s.stage_ops
        s._buf = {k: so.alloc(_round256(v)) for k, v in {**local, **recv}.items()}
        s._lay = lay
        s._recv_names = list(recv)
        s._key = (B, N)
        s._pack_weights(device)
    for name in shards[0]._recv_names:
        tensors = [s._buf[name] for s in shards]
        addrs = [t.data_ptr() for t in tensors]
        for s in shards:
            s._peer[name] = PeerBuffer(s._buf[name], addrs, tensors[0].device, tensors)


class TimedStageOps:
    """Wraps a stage-ops object and calls ``hook(name)`` before and ``hook("end")`` after
    every stage call (per-kernel timing with events) and counts the kernel launches."""

    KERNELS = ("trimul_project", "trimul_project_to", "trimul_contract", "trimul_finish", "triatt_project",
               "triatt_core",
               "triatt_finish", "triatt_finish_to", "trimul_contract_to", "copy_2d", "copy_3d", "pair_transpose_pack", "push_3d", "push_pair_transpose")

    def __init__(self, inner, hook=None):
        self.inner = inner
        self.hook = hook
        self.launches = 0

    def __getattr__(self, name):
        fn = getattr(self.inner, name)
        if name not in self.KERNELS:
            return fn

        def wrapped(*a, **k):
            if not (name == "push_3d" and getattr(self.inner, "push", "kernel") == "dma"):
                self.launches += 1  # copy-engine pushes launch no kernel
            if self.hook:
                self.hook(name)
            r = fn(*a, **k)
            if self.hook:
                self.hook("end")
            return r
        return wrapped


def _bytes(t: Tensor) -> Tensor:
    return t.view(-1).view(torch.uint8)


def _check_local(z: Tensor, mask: Optional[Tensor]) -> None:
    if not (z.dtype == torch.float32 and z.is_contiguous() and z.dim() == 4 and z.shape[-1] == C):
        raise RuntimeError("z_local must be a contiguous fp32 [B, N/P, N, 128] tensor")
    if mask is not None and (mask.dtype != torch.float32 or tuple(mask.shape) != (z.shape[0], z.shape[2], z.shape[2])):
        raise RuntimeError("mask must be the whole fp32 [B, N, N] mask")


@torch.no_grad()
def run_emulated(shards: List[ShardedTrianglePairStack], z_locals: List[Tensor], mask: Optional[Tensor],
                 z_ins: Optional[List[Tensor]] = None) -> None:
    """Run P ranks' programs in one process, in lockstep, performing each collective by
    copying between the ranks' buffers (all on one device). Updates ``z_locals`` in place
    (reading ``z_ins`` in the first block when given)."""
    for z in z_locals:
        _check_local(z, mask)
    z_ins = z_ins or [None] * len(z_locals)
    _drive([s.steps(z, mask, zi) for s, z, zi in zip(shards, z_locals, z_ins)], len(shards))


def _drive(gens, P: int) -> None:
    """Step P rank generators in lockstep; every round all of them must request the same
    collective, which is then carried out by copies."""
    while True:
        reqs = []
        for g in gens:
            try:
                reqs.append(next(g))
            except StopIteration:
                reqs.append(None)
        if all(r is None for r in reqs):
            return
        if any(r is None for r in reqs) or len({r[0] for r in reqs}) != 1:
            raise RuntimeError("ranks diverged: " + str([None if r is None else r[0] for r in reqs]))
        kind = reqs[0][0]
        if kind == "barrier":
            continue  # the ranks run in lockstep on one stream: every push before it is done
        if kind == "all_gather":
            ins = [r[2].clone() for r in reqs]
            for r in reqs:
                r[1].copy_(torch.cat(ins))
        elif kind == "all_to_all":
            chunks = [r[2].clone().chunk(P) for r in reqs]
            for q, r in enumerate(reqs):
                r[1].copy_(torch.cat([chunks[p][q] for p in range(P)]))
        else:
            raise RuntimeError(f"unknown collective {kind}")
