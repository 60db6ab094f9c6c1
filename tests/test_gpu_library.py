"""GPU checks of the torch.ops.genie_tk.* operators: torch.library.opcheck (schema, fake
tensor and AOT dispatch against the real kernels), the in-place residual variants, and
CUDA-graph capture of a module forward that goes through the operators."""

import pytest
import torch

import genie_tk
from gpu_util import assert_status_clean, require_gpu

pytestmark = pytest.mark.gpu


def _inputs(dev, N=48, B=1, seed=11):
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(B, N, N, 128, generator=gen).to(dev)
    mask = torch.ones(B, N, N)
    mask[:, -5:, :] = 0
    return z, mask.to(dev)


def _modules(dev):
    torch.manual_seed(5)
    tm = genie_tk.TriangleMultiplicationIncoming(128, 128).to(dev)
    ta = genie_tk.TriangleAttentionEndingNode(128, 128, 4).to(dev)
    with torch.no_grad():  # non-trivial gates and output weights (the reference inits some to zero)
        for mod in (tm, ta):
            for name, p in mod.named_parameters():
                if p.dim() == 2:
                    p.copy_(torch.randn(p.shape) / p.shape[1] ** 0.5)
                elif name.endswith("bias"):
                    p.copy_(0.1 * torch.randn(p.shape))
    return tm, ta


def test_opcheck():
    dev = require_gpu()
    z, mask = _inputs(dev)
    tm, ta = _modules(dev)
    torch.library.opcheck(torch.ops.genie_tk.trimul_forward.default, (z, mask, tm.packed_weights(dev), False))
    torch.library.opcheck(torch.ops.genie_tk.triatt_forward.default, (z, mask, ta.packed_weights(dev), False, 1e9))
    torch.library.opcheck(torch.ops.genie_tk.trimul_forward.default, (z, None, tm.packed_weights(dev), True))
    assert_status_clean(dev)


def test_residual_ops_match_functional():
    dev = require_gpu()
    z, mask = _inputs(dev, N=72, B=2)
    tm, ta = _modules(dev)
    for res_op, fwd_op, extra, packed in (
            (torch.ops.genie_tk.trimul_residual_, torch.ops.genie_tk.trimul_forward, (False,), tm.packed_weights(dev)),
            (torch.ops.genie_tk.triatt_residual_, torch.ops.genie_tk.triatt_forward, (False, 1e9),
             ta.packed_weights(dev))):
        upd = fwd_op(z, mask, packed, *extra)
        zz = z.clone()
        res_op(zz, mask, packed, *extra)
        torch.cuda.synchronize()
        assert float((zz - (z + upd)).abs().max()) <= 1e-5
    assert_status_clean(dev)


def test_module_forward_in_cuda_graph():
    dev = require_gpu()
    z, mask = _inputs(dev, N=64)
    tm, ta = _modules(dev)
    eager = ta(tm(z, mask) + z, mask)  # packs the weights and sizes the workspace outside capture
    torch.cuda.synchronize()
    static_z = z.clone()
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream(dev))
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            out = ta(tm(static_z, mask) + static_z, mask)
    torch.cuda.current_stream(dev).wait_stream(s)
    static_z.copy_(z)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert_status_clean(dev)
