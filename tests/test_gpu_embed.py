"""GPU parity of the pair-embedding kernels (gtk_pair_embed) against the fp32 oracle, whole
grids and row shards."""

import pytest
import torch

import genie_tk
from gpu_util import require_gpu
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,N,c_s", [(1, 1, 8), (2, 37, 24), (1, 130, 384), (1, 257, 100)])
def test_pair_embed_matches_oracle(B, N, c_s):
    dev = require_gpu()
    from genie_tk import ops
    gen = torch.Generator().manual_seed(N + c_s)
    s = torch.randn(B, N, c_s, generator=gen)
    mask = (torch.rand(B, N, generator=gen) > 0.2).float()
    w = torch.randn(128, 2 * c_s, generator=gen) / (2 * c_s) ** 0.5
    b = 0.1 * torch.randn(128, generator=gen)
    ref, ref_mask = O.pair_embed(s, mask, {"weight": w, "bias": b})
    p, pm = ops.pair_embed(s.to(dev), mask.to(dev), w.to(dev), b.to(dev))
    torch.cuda.synchronize()
    torch.testing.assert_close(p.cpu(), ref, rtol=1e-4, atol=1e-4)  # fp32 throughout
    assert torch.equal(pm.cpu(), ref_mask)
    # a row shard lands in its own [B, rows, N, 128] buffer
    if N >= 4:
        r0, rows = N // 4, N // 2
        ps, pms = ops.pair_embed(s.to(dev), mask.to(dev), w.to(dev), b.to(dev), rows=rows, row0=r0)
        torch.testing.assert_close(ps.cpu(), ref[:, r0:r0 + rows], rtol=1e-4, atol=1e-4)
        assert torch.equal(pms.cpu(), ref_mask[:, r0:r0 + rows])


def test_module_forward():
    dev = require_gpu()
    torch.manual_seed(0)
    emb = genie_tk.PairEmbedding(c_s=64, c_p=128).to(dev)
    s = torch.randn(1, 40, 64, device=dev)
    mask = torch.ones(1, 40, device=dev)
    p, pm = emb(s, mask)
    ref, ref_mask = O.pair_embed(s.cpu(), mask.cpu(), {"weight": emb.weight.detach().cpu(), "bias": emb.bias.detach().cpu()})
    torch.testing.assert_close(p.cpu(), ref, rtol=1e-4, atol=1e-4)
    p2, pm2 = emb(s)
    assert pm2 is None and torch.equal(p2, p)
