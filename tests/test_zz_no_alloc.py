"""The workspace-free TriMul entry point (gtk_trimul_forward_noalloc).

Some callers cannot allocate device memory at all: plugin hosts that own every device
allocation and hand their plugins no allocator, services that run under a fixed memory
budget, and latency paths that must not call cudaMalloc (it can synchronise the device).
For them the library provides a variant of gtk_trimul_forward that uses a built-in
scratch array instead of a caller workspace. These tests call both entry points through
the C ABI and check that the variant gives the same update, bit for bit, on calls in a
row: first at the largest size the scratch holds (B = 2, N = 128: B * N * round_up(N, 8)
= 32768), then at a smaller ragged size (N = 100, pitch 104) whose pitch padding would
show any bytes left over from the previous call. The ragged call is also checked against
the fp32 oracle. Sizes beyond the scratch are refused before any launch.

This file is collected last on purpose, so that a run stopping at the first failure has
already run every other test.
"""

import pytest
import torch

from gpu_util import assert_parity, assert_status_clean, require_gpu, to_dev
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


def _inputs(seed, B, N, dev):
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = torch.ones(B, N, N, device=dev)
    mask[-1, -5:, :] = 0
    params = to_dev(O.make_trimul_params(128, 128, gen, gate_bias=1.0, ln_random=True, bias_random=True), dev)
    return z, mask, params


@pytest.mark.parametrize("outgoing", [True, False])
def test_noalloc_matches_workspace_entry_point(outgoing):
    dev = require_gpu()
    from genie_tk import _lib, ops
    lib = _lib.load()
    P = ops._ptr
    stream = ops._stream(dev)
    status = ops.status_buffer(dev)
    for call, (seed, B, N) in enumerate(((101, 2, 128), (202, 1, 100), (303, 2, 128))):
        assert B * N * ops.plane_pitch(N) <= 32768
        z, mask, params = _inputs(seed, B, N, dev)
        packed = ops.pack_trimul(params, dev)
        ws = torch.empty(lib.gtk_trimul_workspace_bytes(B, N, 128, 128), dtype=torch.uint8, device=dev)
        ref = torch.empty_like(z)
        rc = lib.gtk_trimul_forward(int(outgoing), P(z), P(mask), P(packed), P(ref), 0, P(ws), ws.numel(), B, N,
                                    128, 128, P(status), stream)
        assert rc == _lib.GTK_OK, lib.gtk_last_error_string()
        got = torch.full_like(z, float("nan"))
        rc = lib.gtk_trimul_forward_noalloc(int(outgoing), P(z), P(mask), P(packed), P(got), 0, B, N, 128, 128,
                                            P(status), stream)
        assert rc == _lib.GTK_OK, lib.gtk_last_error_string()
        torch.cuda.synchronize()
        assert_status_clean(dev)
        # same kernels on the same inputs: the results must be identical
        assert torch.equal(got, ref), f"noalloc call {call} (B={B}, N={N}) differs from gtk_trimul_forward"
        if N % 8:
            assert_parity(got, O.trimul_forward(z, mask, params, outgoing=outgoing), what=f"noalloc N={N}")


def test_noalloc_rejects_sizes_beyond_its_scratch():
    """One past the limit (B = 2, N = 129: pitch 136) is refused with GTK_ERR_WORKSPACE before
    any launch. Real device tensors are passed, so nothing could read a made-up address even
    if the size check were to change."""
    dev = require_gpu()
    from genie_tk import _lib, ops
    lib = _lib.load()
    P = ops._ptr
    B, N = 2, 129
    z = torch.zeros(B, N, N, 128, device=dev)
    out = torch.zeros_like(z)
    packed = torch.zeros(lib.gtk_trimul_packed_bytes(128, 128), dtype=torch.uint8, device=dev)
    rc = lib.gtk_trimul_forward_noalloc(1, P(z), None, P(packed), P(out), 0, B, N, 128, 128, None,
                                        ops._stream(dev))
    assert rc == _lib.GTK_ERR_WORKSPACE
    msg = lib.gtk_last_error_string().decode()
    assert "scratch" in msg and "32768" in msg
    torch.cuda.synchronize()
    assert torch.count_nonzero(out) == 0
