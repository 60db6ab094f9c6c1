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


@pytest.mark.parametrize("c_p,c_s", [(64, 32), (256, 48), (96, 16), (130, 20), (7, 9)])
def test_pair_embed_other_widths(c_p, c_s):
    """c_p other than 128: several 128-output chunks (256), a partial chunk (96, 130), and
    widths that are not a multiple of 4 (130, 7: the single-float path), with a row shard."""
    dev = require_gpu()
    from genie_tk import ops
    B, N = 2, 45
    gen = torch.Generator().manual_seed(c_p * 3 + c_s)
    s = torch.randn(B, N, c_s, generator=gen)
    mask = (torch.rand(B, N, generator=gen) > 0.2).float()
    w = torch.randn(c_p, 2 * c_s, generator=gen) / (2 * c_s) ** 0.5
    b = 0.1 * torch.randn(c_p, generator=gen)
    ref, ref_mask = O.pair_embed(s, mask, {"weight": w, "bias": b})
    p, pm = ops.pair_embed(s.to(dev), mask.to(dev), w.to(dev), b.to(dev))
    ps, _ = ops.pair_embed(s.to(dev), mask.to(dev), w.to(dev), None, rows=11, row0=30, with_mask=False)
    torch.cuda.synchronize()
    assert p.shape == (B, N, N, c_p)
    torch.testing.assert_close(p.cpu(), ref, rtol=1e-4, atol=1e-4)
    assert torch.equal(pm.cpu(), ref_mask)
    torch.testing.assert_close(ps.cpu(), (ref - b)[:, 30:41], rtol=1e-4, atol=1e-4)
    emb = genie_tk.PairEmbedding(c_s=c_s, c_p=c_p).to(dev)
    with torch.no_grad():
        emb.weight.copy_(w)
        emb.bias.copy_(b)
    pe, _ = emb(s.to(dev), mask.to(dev))
    assert torch.equal(pe, p)
