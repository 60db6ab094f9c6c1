"""The reference's PyTorch path on the same B200, as the GPU baseline of the library.

The reference publishes per-op forward times of its PyTorch path against its own kernels
(README.md:333-337: TriMulOut / TriMulIn / TriAttStart / TriAttEnd at N = 256 and 512, bf16,
on an H100). These tests time the same reference math -- the oracle's restatement of
``_forward_pytorch`` (triangle_mul.py:103-132, triangle_attention.py:100-143), evaluated in
bf16 on cuBLAS with every row at once, as the reference does -- against the library's
kernels on the same GPU, per op at those sizes and for one cfg5 layer at N = 1024, and
require the library to be faster. Each timing is printed and, when the environment variable
GTK_TIMING_JSON names a file, appended to it as one JSON line.
"""

import json
import os

import pytest
import torch

from gpu_util import require_gpu
from oracle import triangle_oracle as O

pytestmark = pytest.mark.gpu

OPS = ("trimul_out", "trimul_in", "triatt_start", "triatt_end")


def _time_ms(fn, warm: int = 1, reps: int = 3) -> float:
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(reps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn()
        b.record()
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b))
    return sorted(times)[len(times) // 2]


def _record(row: dict) -> None:
    print(json.dumps(row))
    path = os.environ.get("GTK_TIMING_JSON")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(row) + "\n")


def _op_params(op, gen):
    if op.startswith("trimul"):
        return O.make_trimul_params(128, 128, gen, gate_bias=1.0)
    return O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0)


def _reference_update(op, z, mask, p, dtype):
    if op.startswith("trimul"):
        return O.trimul_forward(z, mask, p, outgoing=(op == "trimul_out"), dtype=dtype)
    return O.triatt_forward(z, mask, p, starting=(op == "triatt_start"), no_heads=4, dtype=dtype)


@pytest.mark.parametrize("op", OPS)
@pytest.mark.parametrize("N", [256, 512])
def test_op_beats_reference_pytorch_on_the_same_gpu(op, N):
    dev = require_gpu()
    from genie_tk import ops
    gen = torch.Generator().manual_seed(N + len(op))
    z = torch.randn(1, N, N, 128, generator=gen).to(dev)
    mask = torch.ones(1, N, N, device=dev)
    p = {k: v.to(dev) for k, v in _op_params(op, gen).items()}
    if op.startswith("trimul"):
        packed = ops.pack_trimul(p, dev)
        ours = lambda: ops.trimul_forward(z, mask, packed, op == "trimul_out")  # noqa: E731
    else:
        packed = ops.pack_triatt(p, dev, 4)
        ours = lambda: ops.triatt_forward(z, mask, packed, op == "triatt_start")  # noqa: E731
    p16 = {k: v.to(torch.bfloat16) for k, v in p.items()}
    z16, m16 = z.to(torch.bfloat16), mask.to(torch.bfloat16)
    with torch.no_grad():
        t_ref = _time_ms(lambda: _reference_update(op, z16, m16, p16, torch.bfloat16))
    t_ours = _time_ms(ours)
    _record({"case": f"{op} N={N} B=1", "reference_pytorch_bf16_ms": round(t_ref, 4), "genie_tk_b200_ms": round(t_ours, 4),
             "speedup": round(t_ref / t_ours, 2)})
    assert t_ours < t_ref


def test_cfg5_layer_beats_reference_pytorch_on_the_same_gpu():
    dev = require_gpu()
    import genie_tk
    z, mask, params = O.config_inputs(5, N=1024)
    layers = params[:1]
    st = genie_tk.TrianglePairStack(1).to(dev)
    st.load_layer_params(layers)
    zd, md = z.to(dev), mask.to(dev)
    out = torch.empty_like(zd)
    t_ours = _time_ms(lambda: st.forward_into(zd, out, md))
    l16 = [{blk: {k: v.to(dev, torch.bfloat16) for k, v in p.items()} for blk, p in lp.items()} for lp in layers]
    z16, m16 = zd.to(torch.bfloat16), md.to(torch.bfloat16)
    with torch.no_grad():
        t_ref = _time_ms(lambda: O.stack_forward(z16, m16, l16, no_heads=4, dtype=torch.bfloat16), warm=1, reps=2)
    _record({"case": "cfg5 one layer N=1024 B=1", "reference_pytorch_bf16_ms": round(t_ref, 3),
             "genie_tk_b200_ms": round(t_ours, 3), "speedup": round(t_ref / t_ours, 1)})
    assert t_ours < t_ref


def test_cfg5_layer_training_step_against_reference_pytorch_on_the_same_gpu():
    """Forward + backward of one cfg5 layer's four residual blocks at N = 1024: the library
    (kernel forwards, backward through the recompute with kernel contractions) against the
    reference's bf16 PyTorch autograd on the same GPU. Recorded, and required to finish;
    not required to be faster (the attention backward is a PyTorch recompute)."""
    dev = require_gpu()
    import genie_tk
    z, mask, params = O.config_inputs(5, N=1024)
    lp = params[0]
    zd, md = z.to(dev), mask.to(dev)
    w = torch.randn(zd.shape, generator=torch.Generator().manual_seed(1)).to(dev)
    mods = [genie_tk.TriangleMultiplicationOutgoing(128, 128), genie_tk.TriangleMultiplicationIncoming(128, 128),
            genie_tk.TriangleAttentionStartingNode(128, 128, 4), genie_tk.TriangleAttentionEndingNode(128, 128, 4)]
    for m, blk in zip(mods, O.STACK_OPS):
        m.to(dev).load_state_dict(lp[blk])

    def ours():
        x = zd.clone().requires_grad_(True)
        y = x
        for m in mods:
            y = y + m(y, md)
        (y * w).sum().backward()

    l16 = [{blk: {k: v.to(dev, torch.bfloat16).requires_grad_(True) for k, v in p.items()} for blk, p in lp.items()}]
    z16, m16, w16 = zd.to(torch.bfloat16), md.to(torch.bfloat16), w.to(torch.bfloat16)

    def reference():
        x = z16.clone().requires_grad_(True)
        (O.stack_forward(x, m16, l16, no_heads=4, dtype=torch.bfloat16) * w16).sum().backward()

    l32 = [{blk: {k: v.to(dev).requires_grad_(True) for k, v in p.items()} for blk, p in lp.items()}]

    def reference_fp32():
        x = zd.clone().requires_grad_(True)
        (O.stack_forward(x, md, l32, no_heads=4) * w).sum().backward()

    t_ours = _time_ms(ours, warm=1, reps=2)
    t_ref = _time_ms(reference, warm=1, reps=2)
    torch.cuda.empty_cache()
    t_ref32 = _time_ms(reference_fp32, warm=1, reps=2)
    _record({"case": "cfg5 one layer N=1024 B=1, forward + backward", "reference_pytorch_bf16_ms": round(t_ref, 2),
             "reference_pytorch_fp32_ms": round(t_ref32, 2), "genie_tk_b200_ms": round(t_ours, 2),
             "speedup_vs_bf16": round(t_ref / t_ours, 2), "speedup_vs_fp32": round(t_ref32 / t_ours, 2)})
    assert all(p.grad is not None and torch.isfinite(p.grad).all() for m in mods for p in m.parameters())


@pytest.mark.parametrize("op", ["trimul_out", "triatt_start"])
def test_peak_memory_against_reference_pytorch(op):
    """Peak device memory of one forward at B = 1, N = 512 (the reference's README.md:343-344
    reports 4.2 GB / 3.8 GB for its PyTorch path and 1.1 / 0.9 GB for its kernels, on an
    H100): the bytes allocated above the inputs and parameters during the call, for the
    library (its workspace included) and for the reference math in bf16."""
    dev = require_gpu()
    from genie_tk import ops
    N = 512
    gen = torch.Generator().manual_seed(N + 1)
    z = torch.randn(1, N, N, 128, generator=gen).to(dev)
    mask = torch.ones(1, N, N, device=dev)
    p = {k: v.to(dev) for k, v in _op_params(op, gen).items()}
    packed = ops.pack_trimul(p, dev) if op.startswith("trimul") else ops.pack_triatt(p, dev, 4)
    p16 = {k: v.to(torch.bfloat16) for k, v in p.items()}
    z16, m16 = z.to(torch.bfloat16), mask.to(torch.bfloat16)

    def peak(fn):
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        base = torch.cuda.memory_allocated(dev)
        torch.cuda.reset_peak_memory_stats(dev)
        out = fn()
        torch.cuda.synchronize()
        used = torch.cuda.max_memory_allocated(dev) - base
        del out
        return used

    ops.release_workspaces()
    if op.startswith("trimul"):
        ours = peak(lambda: ops.trimul_forward(z, mask, packed, True))
    else:
        ours = peak(lambda: ops.triatt_forward(z, mask, packed, True))
    with torch.no_grad():
        ref = peak(lambda: _reference_update(op, z16, m16, p16, torch.bfloat16))
    _record({"case": f"{op} N={N} B=1 peak memory", "reference_pytorch_bf16_GB": round(ref / 1e9, 3),
             "genie_tk_b200_GB": round(ours / 1e9, 3)})
    assert ours < ref
