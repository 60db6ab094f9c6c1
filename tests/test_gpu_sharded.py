"""The row-sharded stack on B200: the exchange kernels against their definitions
(bit-exact), P ranks emulated on one GPU with the real stage kernels against the
unsharded stack and the oracle, and, when the box has two GPUs, two NCCL ranks."""

import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from gpu_util import assert_parity, assert_status_clean, require_gpu
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


def test_copy_2d_matches_strided_copy():
    dev = require_gpu()
    from genie_tk import _lib, ops
    lib = _lib.load()
    src = torch.randint(0, 255, (37 * 4096 + 64,), dtype=torch.uint8, device=dev)
    dst = torch.zeros(37 * 2048 + 512, dtype=torch.uint8, device=dev)
    # 37 rows of 1520 bytes: from pitch 4096 at offset 48 to pitch 2048 at offset 32
    rc = lib.gtk_copy_2d(ops._ptr(dst[32:]), 2048, ops._ptr(src[48:]), 4096, 1520, 37, ops._stream(dev))
    assert rc == 0, lib.gtk_last_error_string()
    ref = torch.zeros_like(dst)
    ref[32:32 + 37 * 2048].view(37, 2048)[:, :1520] = src[48:48 + 37 * 4096].view(37, 4096)[:, :1520]
    torch.cuda.synchronize()
    assert torch.equal(dst, ref)
    assert lib.gtk_copy_2d(ops._ptr(dst), 2048, ops._ptr(src), 4096, 1000, 2, ops._stream(dev)) == -3


def test_copy_3d_matches_strided_copy():
    dev = require_gpu()
    from genie_tk import _lib, ops
    lib = _lib.load()
    # 3 slabs of 5 rows of 96 bytes: source slabs 1024 apart with row pitch 160,
    # destination slabs 512 apart with row pitch 96 (packed rows)
    src = torch.randint(0, 255, (4096,), dtype=torch.uint8, device=dev)
    dst = torch.zeros(2048, dtype=torch.uint8, device=dev)
    rc = lib.gtk_copy_3d(ops._ptr(dst), 96, 512, ops._ptr(src), 160, 1024, 96, 5, 3, ops._stream(dev))
    assert rc == 0, lib.gtk_last_error_string()
    ref = torch.zeros_like(dst)
    for k in range(3):
        for r in range(5):
            ref[k * 512 + r * 96:k * 512 + r * 96 + 96] = src[k * 1024 + r * 160:k * 1024 + r * 160 + 96]
    torch.cuda.synchronize()
    assert torch.equal(dst, ref)


@pytest.mark.parametrize("B,R,Cn,P", [(1, 16, 64, 4), (2, 8, 48, 3), (1, 128, 1024, 8)])
def test_pair_transpose_pack_matches_permute(B, R, Cn, P):
    dev = require_gpu()
    from genie_tk import _lib, ops
    lib = _lib.load()
    src = torch.randn(B, R, Cn, 128, device=dev)
    dst = torch.empty(P, B, Cn // P, R, 128, device=dev)
    rc = lib.gtk_pair_transpose_pack(ops._ptr(src), ops._ptr(dst), B, R, Cn, P, ops._stream(dev))
    assert rc == 0, lib.gtk_last_error_string()
    ref = src.view(B, R, P, Cn // P, 128).permute(2, 0, 3, 1, 4)
    torch.cuda.synchronize()
    assert torch.equal(dst, ref)


def test_push_kernels_match_their_definitions():
    dev = require_gpu()
    from genie_tk import _lib, ops
    lib = _lib.load()
    st = ops._stream(dev)
    P = 3
    # push_3d: slab k of src -> destination k at an offset, with its own row pitch
    src = torch.randint(0, 255, (P * 4096,), dtype=torch.uint8, device=dev)
    dsts = [torch.zeros(8192, dtype=torch.uint8, device=dev) for _ in range(P)]
    ptrs = torch.tensor([d.data_ptr() for d in dsts], dtype=torch.int64, device=dev)
    assert lib.gtk_push_3d(ops._ptr(ptrs), P, 256, 512, ops._ptr(src), 1024, 4096, 160, 4, st) == 0
    torch.cuda.synchronize()
    for k in range(P):
        ref = torch.zeros(8192, dtype=torch.uint8, device=dev)
        for r in range(4):
            ref[256 + r * 512:256 + r * 512 + 160] = src[k * 4096 + r * 1024:k * 4096 + r * 1024 + 160]
        assert torch.equal(dsts[k], ref)
    # push_pair_transpose: pair (b, y, q*CP + x) -> dsts[q] at (b, x, row0 + y) of [B][CP][ndst][128]
    B, R, Cn, ndst, row0 = 2, 8, 24, 40, 16
    CP = Cn // P
    zsrc = torch.randn(B, R, Cn, 128, device=dev)
    outs = [torch.zeros(B, CP, ndst, 128, device=dev) for _ in range(P)]
    ptrs = torch.tensor([o.data_ptr() for o in outs], dtype=torch.int64, device=dev)
    assert lib.gtk_push_pair_transpose(ops._ptr(zsrc), ops._ptr(ptrs), B, R, Cn, P, ndst, row0, st) == 0
    torch.cuda.synchronize()
    for q in range(P):
        ref = torch.zeros_like(outs[q])
        ref[:, :, row0:row0 + R] = zsrc.view(B, R, P, CP, 128)[:, :, q].permute(0, 2, 1, 3)
        assert torch.equal(outs[q], ref)


def test_peer_barrier_passes_and_times_out_cleanly():
    """One rank alone passes; a barrier waiting for a peer that never arrives gives up after
    its bounded wait, sets GTK_STATUS_TIMEOUT_PEER and leaves the device usable."""
    dev = require_gpu()
    from genie_tk import _lib, ops
    lib = _lib.load()
    st = ops._stream(dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    flags = torch.zeros(64, dtype=torch.int32, device=dev)
    one = torch.tensor([flags.data_ptr()], dtype=torch.int64, device=dev)
    assert lib.gtk_peer_barrier(ops._ptr(one), 0, 1, 1, ops._ptr(status), st) == 0
    torch.cuda.synchronize()
    assert int(status.item()) == 0 and int(flags[0].item()) == 1
    other = torch.zeros(64, dtype=torch.int32, device=dev)   # a "peer" that never signals
    two = torch.tensor([flags.data_ptr(), other.data_ptr()], dtype=torch.int64, device=dev)
    assert lib.gtk_peer_barrier(ops._ptr(two), 0, 2, 2, ops._ptr(status), st) == 0
    torch.cuda.synchronize()
    assert int(status.item()) & 0x20
    assert int(other[0].item()) == 2          # this rank still published its arrival
    assert torch.equal(torch.ones(4, device=dev) * 2, torch.ones(4, device=dev) + 1)


def _problem(N, layers, seed=21):
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(1, N, N, 128, generator=gen)
    mask = torch.ones(1, N, N)
    mask[0, -7:, :] = 0
    mask[0, :, -5:] = 0
    params = []
    for _ in range(layers):
        params.append({
            "tri_mul_out": O.make_trimul_params(128, 128, gen, gate_bias=1.0, ln_random=True, bias_random=True),
            "tri_mul_in": O.make_trimul_params(128, 128, gen, gate_bias=1.0, ln_random=True, bias_random=True),
            "tri_att_start": O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0, ln_random=True,
                                                  bias_random=True),
            "tri_att_end": O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0, ln_random=True, bias_random=True),
        })
    return z, mask, params


def _stack(params, dev):
    import genie_tk
    st = genie_tk.TrianglePairStack(len(params)).to(dev)
    st.load_layer_params([{k: {n: t.to(dev) for n, t in v.items()} for k, v in lp.items()} for lp in params])
    return st


@pytest.mark.parametrize("N,P,layers,exchange", [(128, 2, 1, "gather"), (128, 2, 1, "channels"),
                                                 (128, 4, 2, "channels"), (128, 4, 1, "gather"),
                                                 (256, 8, 1, "channels")])
def test_emulated_shards_match_unsharded(N, P, layers, exchange):
    dev = require_gpu()
    from genie_tk.sharded import ShardedTrianglePairStack, run_emulated
    z, mask, params = _problem(N, layers)
    st = _stack(params, dev)
    zd, md = z.to(dev), mask.to(dev)
    full = st.forward(zd, md)
    R = N // P
    shards = [ShardedTrianglePairStack(st, P, r, trimul_exchange=exchange) for r in range(P)]
    zin = [zd[:, r * R:(r + 1) * R].clone() for r in range(P)]
    out = [torch.empty_like(t) for t in zin]
    run_emulated(shards, out, md, zin)
    got = torch.cat(out, dim=1)
    torch.cuda.synchronize()
    assert torch.equal(torch.cat(zin, 1), zd), "the input shards must be left unchanged"
    # same kernels, same per-element summation order: the sharding adds no error of its own
    assert float((got - full).abs().max()) <= 1e-3
    ref = O.stack_forward(z, mask, params, no_heads=4)
    assert_parity(got, ref, what=f"sharded P={P}")
    assert_status_clean(dev)


@pytest.mark.parametrize("N,P,exchange,k1_direct", [(128, 2, "gather", False), (128, 4, "channels", False),
                                                     (256, 8, "channels", False), (256, 8, "channels", True)])
def test_emulated_peer_exchange_matches_unsharded(N, P, exchange, k1_direct):
    dev = require_gpu()
    from genie_tk.sharded import ShardedTrianglePairStack, connect_emulated, run_emulated
    z, mask, params = _problem(N, 1)
    st = _stack(params, dev)
    zd, md = z.to(dev), mask.to(dev)
    full = st.forward(zd, md)
    R = N // P
    shards = [ShardedTrianglePairStack(st, P, r, trimul_exchange=exchange, exchange="peer", k1_direct=k1_direct)
              for r in range(P)]
    connect_emulated(shards, 1, N, dev)
    zl = [zd[:, r * R:(r + 1) * R].clone() for r in range(P)]
    run_emulated(shards, zl, md)
    got = torch.cat(zl, dim=1)
    torch.cuda.synchronize()
    assert float((got - full).abs().max()) <= 1e-3
    assert_status_clean(dev)


@pytest.mark.parametrize("N,P,exchange", [(256, 2, "gather"), (512, 4, "channels"), (1024, 8, "channels")])
def test_emulated_fused_stores_equal_separate_pushes(N, P, exchange):
    """With 128 rows per rank the attention blocks' K4e stores its output transposed straight
    into the ranks' shards, and (channel shards) K2 stores each x tile straight into its row
    owner's planes: TMA stores through per-rank tensor maps (emulated ranks on one GPU, so the
    shards are local allocations). Same arithmetic as the kernels followed by the pushes: the
    results are bitwise equal."""
    dev = require_gpu()
    from genie_tk.sharded import ShardedTrianglePairStack, connect_emulated, run_emulated
    z, mask, params = _problem(N, 1)
    st = _stack(params, dev)
    zd, md = z.to(dev), mask.to(dev)
    R = N // P
    res = []
    for fused in (True, False):
        shards = [ShardedTrianglePairStack(st, P, r, trimul_exchange=exchange, exchange="peer",
                                           fused_transpose=fused, fused_x=fused) for r in range(P)]
        connect_emulated(shards, 1, N, dev)
        zl = [zd[:, r * R:(r + 1) * R].clone() for r in range(P)]
        run_emulated(shards, zl, md)
        res.append(torch.cat(zl, dim=1))
    torch.cuda.synchronize()
    assert torch.equal(res[0], res[1])
    assert float((res[0] - st.forward(zd, md)).abs().max()) <= 1e-3
    assert_status_clean(dev)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_rank(rank, world, port, z, mask, params, q, exchange="nccl", trimul_exchange="auto", k1_direct=False,
               push="kernel"):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                            device_id=dev)
    try:
        from genie_tk.sharded import ShardedTrianglePairStack
        N = z.shape[1]
        R = N // world
        zl = z[:, rank * R:(rank + 1) * R].contiguous().to(dev)
        sh = ShardedTrianglePairStack(_stack(params, dev), world, rank, exchange=exchange,
                                      trimul_exchange=trimul_exchange, k1_direct=k1_direct, push=push)
        if exchange == "peer":
            sh.connect(None, 1, N, dev)
        sh.forward_(zl, mask.to(dev))
        torch.cuda.synchronize()
        from genie_tk import ops
        q.put((rank, zl.cpu(), ops.check_status(dev)))
        dist.barrier()
        sh.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange,trimul_exchange,k1_direct,push", [
    ("nccl", "auto", False, "kernel"), ("peer", "auto", False, "kernel"), ("peer", "channels", False, "kernel"),
    ("peer", "channels", True, "kernel"), ("peer", "auto", False, "dma"), ("peer", "channels", False, "dma")])
def test_two_ranks_match_single_gpu(exchange, trimul_exchange, k1_direct, push):
    require_gpu()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    z, mask, params = _problem(256, 1, seed=5)
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_nccl_rank, args=(r, world, port, z, mask, params, q, exchange, trimul_exchange,
                                                  k1_direct, push))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert all(r[2] == 0 for r in res), "a kernel or barrier timed out"
    parts = {r[0]: r[1] for r in res}
    got = torch.cat([parts[r] for r in range(world)], dim=1)
    dev = torch.device("cuda", 0)
    full = _stack(params, dev).forward(z.to(dev), mask.to(dev)).cpu()
    assert float((got - full).abs().max()) <= 1e-3
    ref = O.stack_forward(z, mask, params, no_heads=4)
    assert_parity(got, ref, what="two NCCL ranks")


def test_dma_push_matches_push_kernel():
    """The copy-engine slab push writes exactly what the push kernel writes (ranks emulated
    on one GPU: the destination buffers are local allocations)."""
    dev = require_gpu()
    from genie_tk.sharded import CudaStageOps, PeerBuffer
    P, height, width, spitch, dpitch, doff = 3, 20, 96, 160, 128, 64
    sslab = height * spitch
    gen = torch.Generator().manual_seed(2)
    src = torch.randint(0, 256, (P * sslab,), generator=gen, dtype=torch.uint8).to(dev)
    outs = {}
    for mode in ("kernel", "dma"):
        bufs = [torch.zeros(doff + height * dpitch, dtype=torch.uint8, device=dev) for _ in range(P)]
        peer = PeerBuffer(bufs[0], [b.data_ptr() for b in bufs], dev, bufs)
        CudaStageOps(dev, push=mode).push_3d(peer, doff, dpitch, src, spitch, sslab, width, height)
        torch.cuda.synchronize()
        outs[mode] = torch.stack(bufs).cpu()
    assert torch.equal(outs["kernel"], outs["dma"])
    ref = src.cpu().view(P, height, spitch)[:, :, :width]
    assert torch.equal(outs["dma"][:, doff:].view(P, height, dpitch)[:, :, :width], ref)
