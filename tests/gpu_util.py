"""Helpers for the GPU parity tests."""

from __future__ import annotations

import pytest
import torch

# Parity bar of the benchmark configurations (bf16 compute vs the fp32 reference path).
MAX_ABS = 2e-2
MEAN_ABS = 2e-3


def require_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import genie_tk._lib as L
    L.load()  # raises if the library is missing: the GPU tests never run without it
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    return torch.device("cuda", 0)


def assert_parity(got: torch.Tensor, ref: torch.Tensor, max_abs: float = MAX_ABS, mean_abs: float = MEAN_ABS,
                  what: str = ""):
    got = got.detach().float()
    ref = ref.detach().float().to(got.device)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert torch.isfinite(got).all(), f"{what}: non-finite values"
    d = (got - ref).abs()
    mx, mn = float(d.max()), float(d.mean())
    assert mx <= max_abs and mn <= mean_abs, f"{what}: max-abs {mx:.3e} (<= {max_abs}), mean-abs {mn:.3e} (<= {mean_abs})"
    return mx, mn


def assert_status_clean(device):
    from genie_tk import ops
    st = ops.check_status(device)
    assert st == 0, f"a kernel reported a bounded-wait timeout (status 0x{st:x})"


def to_dev(params, device):
    return {k: v.to(device) for k, v in params.items()}
