"""The pair-embedding oracle against the reference's own operations (examples/basic_usage.py:
188-196: expand, torch.cat, nn.Linear(2 c_s, c_p), mask outer product), and the module's
state-dict compatibility with that nn.Linear (no GPU)."""

import torch

import genie_tk
from oracle import triangle_oracle as O


def test_oracle_matches_reference_ops():
    gen = torch.Generator().manual_seed(3)
    B, L, c_s, c_p = 2, 7, 24, 128
    s = torch.randn(B, L, c_s, generator=gen)
    mask = (torch.rand(B, L, generator=gen) > 0.3).float()
    lin = torch.nn.Linear(c_s * 2, c_p)
    with torch.no_grad():
        s_i = s.unsqueeze(2).expand(-1, -1, L, -1)
        s_j = s.unsqueeze(1).expand(-1, L, -1, -1)
        ref = lin(torch.cat([s_i, s_j], dim=-1))
    ref_mask = mask.unsqueeze(1) * mask.unsqueeze(2)
    p, pm = O.pair_embed(s, mask, {"weight": lin.weight.detach(), "bias": lin.bias.detach()})
    torch.testing.assert_close(p, ref, rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(pm, ref_mask)
    # the identity the kernels use: p_ij = W_a s_i + W_b s_j + b
    W = lin.weight.detach()
    u = s @ W[:, :c_s].t()
    v = s @ W[:, c_s:].t() + lin.bias.detach()
    torch.testing.assert_close(p, u.unsqueeze(2) + v.unsqueeze(1), rtol=1e-5, atol=1e-5)


def test_module_state_dict_matches_linear():
    emb = genie_tk.PairEmbedding(c_s=24, c_p=128)
    lin = torch.nn.Linear(48, 128)
    assert set(emb.state_dict()) == set(lin.state_dict()) == {"weight", "bias"}
    emb.load_state_dict(lin.state_dict())
    assert torch.equal(emb.weight, lin.weight)
