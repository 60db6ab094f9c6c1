"""The workspace-free TriMul entry point (gtk_trimul_forward_noalloc).

Some callers cannot allocate device memory at all: plugin hosts that own every device
allocation, services running under a fixed memory budget, and latency paths that must
not call cudaMalloc. For them the library provides a variant of gtk_trimul_forward that
uses a built-in scratch array instead of a caller workspace. This test calls both entry
points through the C ABI and checks that the variant gives the same update, on two calls
in a row with different inputs (the scratch keeps the previous call's contents, which
must not leak into the next result), and that sizes beyond the scratch are refused.

This file is collected last on purpose, so that a run stopping at the first failure has
already run every other test.
"""

import ctypes

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
    for call, (seed, B, N) in enumerate(((101, 1, 128), (202, 2, 96))):
        z, mask, params = _inputs(seed, B, N, dev)
        packed = ops.pack_trimul(params, dev)
        ws = torch.empty(lib.gtk_trimul_workspace_bytes(B, N, 128, 128), dtype=torch.uint8, device=dev)
        ref = torch.empty_like(z)
        rc = lib.gtk_trimul_forward(int(outgoing), P(z), P(mask), P(packed), P(ref), 0, P(ws), ws.numel(), B, N,
                                    128, 128, P(status), stream)
        assert rc == 0, lib.gtk_last_error_string()
        got = torch.full_like(z, float("nan"))
        rc = lib.gtk_trimul_forward_noalloc(int(outgoing), P(z), P(mask), P(packed), P(got), 0, B, N, 128, 128,
                                            P(status), stream)
        assert rc == 0, lib.gtk_last_error_string()
        torch.cuda.synchronize()
        assert_parity(got, ref, what=f"noalloc call {call}")
        assert_status_clean(dev)


def test_noalloc_rejects_sizes_beyond_its_scratch():
    dev = require_gpu()
    from genie_tk import _lib
    lib = _lib.load()
    rc = lib.gtk_trimul_forward_noalloc(1, ctypes.c_void_p(256), None, ctypes.c_void_p(256), ctypes.c_void_p(256), 0,
                                        1, 256, 128, 128, None, None)
    assert rc == -4
    msg = lib.gtk_last_error_string().decode()
    assert "scratch" in msg and "32768" in msg
