"""CPU checks of the drop-in Python API (no kernels run): class names, constructor
arguments, parameter names compatible with the reference's state dicts, and the
no-CPU-path contract."""

import numpy as np
import pytest
import torch

from golden_util import GOLDEN, SINGLE_CASES, load_case
from oracle import triangle_oracle as O


def test_public_names_match_the_reference():
    import genie_tk
    for name in ("TriangleMultiplicativeUpdate", "TriangleMultiplicationOutgoing", "TriangleMultiplicationIncoming",
                 "TriangleAttention", "TriangleAttentionStartingNode", "TriangleAttentionEndingNode",
                 "PairTransformLayer", "PairTransformNet", "has_cuda_kernels", "get_device_info"):
        assert hasattr(genie_tk, name), name
        assert name in genie_tk.__all__


@pytest.mark.parametrize("name", SINGLE_CASES)
def test_state_dict_keys_match_reference_modules(name):
    """The golden files record the reference modules' state_dict keys."""
    import genie_tk
    d = np.load(f"{GOLDEN}/{name}.npz")
    ref_keys = sorted(str(k) for k in d["param_keys"])
    op, c_z, c, H = str(d["op"]), int(d["c_z"]), int(d["c_hidden"]), int(d["heads"])
    cls = {"trimul_out": genie_tk.TriangleMultiplicationOutgoing, "trimul_in": genie_tk.TriangleMultiplicationIncoming,
           "triatt_start": genie_tk.TriangleAttentionStartingNode,
           "triatt_end": genie_tk.TriangleAttentionEndingNode}[op]
    mod = cls(c_z, c) if op.startswith("trimul") else cls(c_z, c, H)
    assert sorted(mod.state_dict().keys()) == ref_keys
    _, _, _, _, params, _ = load_case(name)
    mod.load_state_dict(params)  # reference parameters load unchanged


def test_constructor_signatures_and_defaults():
    import genie_tk
    m = genie_tk.TriangleMultiplicationOutgoing(c_z=128, c_hidden=128, use_fused_kernel=True)
    assert m._outgoing and m.c_z == 128
    a = genie_tk.TriangleAttentionEndingNode(c_in=128, c_hidden=128, no_heads=4, inf=1e9)
    assert not a.starting and a.mha.head_dim == 32 and a.inf == 1e9
    # AF2 initialisers: gating -> W=0, b=1; final -> zeros
    assert torch.all(m.linear_a_g.weight == 0) and torch.all(m.linear_a_g.bias == 1)
    assert torch.all(m.linear_z.weight == 0)
    layer = genie_tk.PairTransformLayer(c_p=128, c_hidden_mul=128, c_hidden_tri_att=128, n_head_tri=4,
                                        tri_dropout=0.0)
    assert hasattr(layer, "pair_transition") and hasattr(layer, "tri_att_end")
    net = genie_tk.PairTransformNet(c_p=128, n_layers=2, c_hidden_tri_att=128)
    assert len(net.layers) == 2


def test_cpu_tensors_are_rejected():
    """The package has no CPU path: the fused kernels are the only implementation."""
    import genie_tk
    z = torch.randn(1, 8, 8, 128)
    for mod in (genie_tk.TriangleMultiplicationOutgoing(128, 128), genie_tk.TriangleAttentionStartingNode(128, 128, 4),
                genie_tk.TrianglePairStack(1)):
        with pytest.raises(RuntimeError, match="CUDA"):
            mod(z)


def test_stack_loads_oracle_parameters():
    import genie_tk
    _, _, params = O.config_inputs(5, N=8)
    st = genie_tk.TrianglePairStack(2)
    st.load_layer_params(params[:2])
    torch.testing.assert_close(st.layers[1].tri_att_end.mha.linear_q.weight,
                               params[1]["tri_att_end"]["mha.linear_q.weight"])


def test_utils_match_torch():
    from genie_tk.utils import chunk_layer, flatten_final_dims, permute_final_dims
    x = torch.randn(2, 3, 4, 5)
    assert torch.equal(permute_final_dims(x, 2, 0, 1), x.permute(0, 3, 1, 2))
    assert flatten_final_dims(x, 2).shape == (2, 3, 20)
    out = chunk_layer(lambda t: t * 2, {"t": x}, chunk_size=2, no_batch_dims=2)
    assert torch.equal(out, x * 2)
