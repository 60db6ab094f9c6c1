"""GPU parity of the fused triangle pair stack (in-place fp32 residual stream)."""

import pytest
import torch

from golden_util import load_stack
from gpu_util import assert_parity, assert_status_clean, require_gpu, to_dev
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


def _stack(layers, dev):
    import genie_tk
    st = genie_tk.TrianglePairStack(len(layers)).to(dev)
    st.load_layer_params(layers)
    return st


def test_stack_matches_reference_golden():
    dev = require_gpu()
    z, mask, layers, out = load_stack()
    st = _stack(layers, dev)
    got = st(z.to(dev), mask.to(dev))
    torch.cuda.synchronize()
    assert_parity(got, out, what="stack2 golden")
    assert_status_clean(dev)


@pytest.mark.parametrize("N,n_layers", [(64, 2), (200, 1)])
def test_stack_matches_oracle_and_graph_replay(N, n_layers):
    dev = require_gpu()
    z, mask, params = O.config_inputs(5, N=N)
    layers = params[:n_layers]
    st = _stack(layers, dev)
    zd, md = z.to(dev), mask.to(dev)
    ref = O.stack_forward(zd, md, [{k: to_dev(v, dev) for k, v in lp.items()} for lp in layers], no_heads=4,
                          chunk_rows=64)
    out = torch.empty_like(zd)
    st.forward_into(zd, out, md)
    assert_parity(out, ref, max_abs=2e-2 * n_layers, mean_abs=2e-3 * n_layers, what=f"stack N={N}")
    out2 = torch.zeros_like(zd)
    g = st.capture_graph(zd, out2, md)
    g.replay()
    g.replay()  # the input is left unchanged, so replays are idempotent
    torch.cuda.synchronize()
    assert torch.equal(out2, out)
    assert_status_clean(dev)


def test_bench_layer_at_full_size_matches_oracle():
    """The benchmark's workload at its real size: the first layer of the cfg5 stack (B = 1,
    N = 1024, seeded weights and input of BASELINE config 5) against the fp32 oracle
    (run on the GPU with fp32 matmuls)."""
    dev = require_gpu()
    z, mask, params = O.config_inputs(5, N=1024)
    layers = params[:1]
    st = _stack(layers, dev)
    zd, md = z.to(dev), mask.to(dev)
    out = torch.empty_like(zd)
    st.forward_into(zd, out, md)
    torch.cuda.synchronize()
    assert_status_clean(dev)
    ref = O.stack_forward(zd, md, [{k: to_dev(v, dev) for k, v in lp.items()} for lp in layers], no_heads=4,
                          chunk_rows=32)
    assert_parity(out, ref, what="cfg5 layer N=1024")
