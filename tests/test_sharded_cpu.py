"""The row-sharded stack's host logic on CPU: P ranks emulated in one process and two
real ``gloo`` ranks, with the stage computations done by the CPU stand-ins of
``shard_cpu_ops`` (the oracle's math in the kernels' byte layouts). Checked against
the unsharded oracle stack and against an unsharded (P = 1) run of the same program."""


import pytest
import torch
import torch.multiprocessing as mp

from oracle import triangle_oracle as O
from shard_cpu_ops import CpuStageOps

MAX_ABS, MEAN_ABS = 2e-2, 2e-3


def _problem(B, N, layers, seed=11, masked=True):
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(B, N, N, 128, generator=gen)
    mask = torch.ones(B, N, N)
    if masked:
        mask[-1, -5:, :] = 0
        mask[-1, :, -3:] = 0
        mask[0, 2, :] = 0
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


def _stack(params):
    import genie_tk
    st = genie_tk.TrianglePairStack(len(params))
    st.load_layer_params(params)
    return st


def _run_emulated(z, mask, params, P, exchange="auto"):
    from genie_tk.sharded import ShardedTrianglePairStack, run_emulated
    st = _stack(params)
    N = z.shape[1]
    R = N // P
    shards = [ShardedTrianglePairStack(st, P, r, stage_ops=CpuStageOps(), trimul_exchange=exchange)
              for r in range(P)]
    zl = [z[:, r * R:(r + 1) * R].clone() for r in range(P)]
    run_emulated(shards, zl, mask)
    return torch.cat(zl, dim=1)


@pytest.mark.parametrize("B,N,P,layers,exchange", [(1, 32, 2, 1, "auto"), (1, 32, 4, 2, "auto"),
                                                   (1, 64, 8, 1, "auto"), (2, 32, 2, 1, "auto"),
                                                   (1, 32, 2, 1, "channels"), (1, 32, 4, 1, "gather"),
                                                   (2, 32, 4, 1, "channels"), (2, 32, 2, 1, "gather")])
def test_emulated_ranks_match_oracle(B, N, P, layers, exchange):
    z, mask, params = _problem(B, N, layers)
    ref = O.stack_forward(z, mask, params, no_heads=4)
    got = _run_emulated(z, mask, params, P, exchange)
    err = (got - ref).abs()
    assert float(err.max()) <= MAX_ABS and float(err.mean()) <= MEAN_ABS, (float(err.max()), float(err.mean()))
    # the sharding itself is exact up to summation order: compare with the unsharded program
    one = _run_emulated(z, mask, params, 1)
    assert float((got - one).abs().max()) <= 2e-4


def test_out_of_place_first_block():
    from genie_tk.sharded import ShardedTrianglePairStack, run_emulated
    z, mask, params = _problem(1, 32, 1)
    st = _stack(params)
    ref = _run_emulated(z, mask, params, 2)
    sh = [ShardedTrianglePairStack(st, 2, r, stage_ops=CpuStageOps()) for r in range(2)]
    zin = [z[:, r * 16:(r + 1) * 16].clone() for r in range(2)]
    keep = [t.clone() for t in zin]
    out = [torch.full_like(t, float("nan")) for t in zin]
    run_emulated(sh, out, mask, zin)
    assert all(torch.equal(a, b) for a, b in zip(zin, keep))
    assert float((torch.cat(out, 1) - ref).abs().max()) == 0.0


def _run_emulated_peer(z, mask, params, P, exchange="auto", k1_direct=False, fused_transpose=True, fused_x=True):
    from genie_tk.sharded import ShardedTrianglePairStack, connect_emulated, run_emulated
    st = _stack(params)
    B, N = z.shape[0], z.shape[1]
    R = N // P
    shards = [ShardedTrianglePairStack(st, P, r, stage_ops=CpuStageOps(), trimul_exchange=exchange, exchange="peer",
                                       k1_direct=k1_direct, fused_transpose=fused_transpose, fused_x=fused_x)
              for r in range(P)]
    connect_emulated(shards, B, N, z.device)
    zl = [z[:, r * R:(r + 1) * R].clone() for r in range(P)]
    run_emulated(shards, zl, mask)
    return torch.cat(zl, dim=1)


@pytest.mark.parametrize("B,N,P,exchange,k1_direct", [(1, 32, 2, "auto", False), (1, 32, 4, "auto", False),
                                                       (1, 64, 8, "auto", False), (2, 32, 2, "channels", False),
                                                       (2, 32, 4, "gather", False), (2, 32, 4, "channels", True),
                                                       (1, 64, 8, "channels", True)])
def test_peer_exchange_matches_collectives(B, N, P, exchange, k1_direct):
    """Pushing every rank's share straight into the peers' buffers gives the same stack
    as the collective exchanges (and the oracle)."""
    z, mask, params = _problem(B, N, 1)
    got = _run_emulated_peer(z, mask, params, P, exchange, k1_direct)
    ref = _run_emulated(z, mask, params, P, exchange)
    assert float((got - ref).abs().max()) <= 1e-5
    err = (got - O.stack_forward(z, mask, params, no_heads=4)).abs()
    assert float(err.max()) <= MAX_ABS and float(err.mean()) <= MEAN_ABS


def test_fused_attention_transpose_matches_separate_pushes():
    """With 128 rows per rank the attention blocks' output goes transposed straight into the
    peers' shards (gtk_triatt_finish_to_peers); the result equals the separate K4e + transpose
    push program and the oracle."""
    z, mask, params = _problem(1, 256, 1)
    got = _run_emulated_peer(z, mask, params, 2, "gather")
    sep = _run_emulated_peer(z, mask, params, 2, "gather", fused_transpose=False)
    assert float((got - sep).abs().max()) <= 1e-5
    err = (got - O.stack_forward(z, mask, params, no_heads=4)).abs()
    assert float(err.max()) <= MAX_ABS and float(err.mean()) <= MEAN_ABS


def test_fused_x_scatter_matches_separate_push():
    """Channel shards with 128 rows per rank: K2 stores each x tile straight into its row
    owner's planes (gtk_trimul_contract_to_peers); equal to K2 + the x push, and the oracle."""
    z, mask, params = _problem(1, 256, 1)  # two ranks of 128 rows (the smallest fused case)
    got = _run_emulated_peer(z, mask, params, 2, "channels")
    sep = _run_emulated_peer(z, mask, params, 2, "channels", fused_transpose=False, fused_x=False)
    assert float((got - sep).abs().max()) <= 1e-5
    err = (got - O.stack_forward(z, mask, params, no_heads=4)).abs()
    assert float(err.max()) <= MAX_ABS and float(err.mean()) <= MEAN_ABS


def test_unmasked_and_no_mask_agree():
    z, mask, params = _problem(1, 32, 1, masked=False)
    a = _run_emulated(z, mask, params, 2)
    b = _run_emulated(z, None, params, 2)
    assert float((a - b).abs().max()) <= 1e-5


def test_shard_spec_validation():
    from genie_tk.sharded import ShardSpec
    s = ShardSpec(1, 1024, 8, 3)
    assert (s.R, s.row0) == (128, 384)
    with pytest.raises(ValueError):
        ShardSpec(1, 100, 8, 0)      # not divisible
    with pytest.raises(ValueError):
        ShardSpec(1, 36, 3, 0)       # 12 rows per rank: not a multiple of 8
    with pytest.raises(ValueError):
        ShardSpec(1, 64, 4, 4)       # rank out of range


def _gloo_rank(rank, world, store_file, z, mask, params, out_q):
    import torch.distributed as dist
    from genie_tk.sharded import ShardedTrianglePairStack
    # a file store: no TCP port to pick, so no race with other processes for a free port
    dist.init_process_group("gloo", init_method=f"file://{store_file}", rank=rank, world_size=world)
    try:
        N = z.shape[1]
        R = N // world
        zl = z[:, rank * R:(rank + 1) * R].clone()
        sh = ShardedTrianglePairStack(_stack(params), world, rank, stage_ops=CpuStageOps())
        sh.forward_(zl, mask)
        out_q.put((rank, zl))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_match_emulation(tmp_path):
    z, mask, params = _problem(1, 32, 1)
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    store = str(tmp_path / "gloo_store")
    procs = [ctx.Process(target=_gloo_rank, args=(r, world, store, z, mask, params, q)) for r in range(world)]
    for p in procs:
        p.start()
    parts = dict(q.get(timeout=240) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got = torch.cat([parts[r] for r in range(world)], dim=1)
    emu = _run_emulated(z, mask, params, world)
    assert float((got - emu).abs().max()) <= 1e-5
    ref = O.stack_forward(z, mask, params, no_heads=4)
    err = (got - ref).abs()
    assert float(err.max()) <= MAX_ABS and float(err.mean()) <= MEAN_ABS


def test_auto_trimul_exchange_prefers_fused_channel_shards():
    """"auto": the channel shards whenever their x exchange is fused into the contraction's
    stores (peer exchange, a multiple of 128 rows per rank); otherwise the exchange that
    moves fewer bytes (the gather for P <= 3)."""
    import genie_tk
    from genie_tk.sharded import ShardedTrianglePairStack
    st = genie_tk.TrianglePairStack(1)
    peer = ShardedTrianglePairStack(st, 2, 0, exchange="peer")
    assert peer._resolve_trimul_exchange(1024) == "channels"      # 512 rows per rank
    assert peer._resolve_trimul_exchange(200) == "gather"         # 100 rows: no fused stores
    assert ShardedTrianglePairStack(st, 2, 0, exchange="peer", fused_x=False)._resolve_trimul_exchange(1024) == "gather"
    assert ShardedTrianglePairStack(st, 2, 0, exchange="nccl")._resolve_trimul_exchange(1024) == "gather"
    assert ShardedTrianglePairStack(st, 8, 0, exchange="nccl")._resolve_trimul_exchange(1024) == "channels"
    assert ShardedTrianglePairStack(st, 2, 0, exchange="peer", trimul_exchange="gather").trimul_exchange == "gather"
