"""CPU/fp32 restatement of the Genie-TK triangle hot path -- TEST INFRASTRUCTURE ONLY.

This module is the parity oracle. Only ``tests/``, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of ``bench.py`` may import it, and only as the checker (or, for
the baseline, as the timed CPU implementation). The product path in
``genie-tk_b200/genie_tk`` never imports it.

It restates, in plain fp32 PyTorch tensor algebra, the math of the reference's only
working implementation (the PyTorch path of northws/Genie-TK). Every function cites
the reference lines it follows (paths relative to the reference project root).

Pinning: the restatement is checked against golden vectors produced by the
reference's own modules (``tests/golden/make_golden.py`` imports the reference's
``src/genie_tk`` after a mechanical docstring repair and records inputs, weights
and outputs); ``tests/test_oracle_golden.py`` asserts agreement.

Parameters are plain ``dict[str, Tensor]`` keyed exactly like the reference modules'
``state_dict`` (``linear_a_p.weight``, ``mha.linear_q.weight``, ...), so a state dict
can be moved between the reference, this oracle and the B200 package unchanged.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional

import torch

Params = Dict[str, torch.Tensor]

LN_EPS = 1e-5  # nn.LayerNorm default, used at triangle_mul.py:72-73, triangle_attention.py:70


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float = LN_EPS) -> torch.Tensor:
    """LayerNorm over the last axis with the biased variance (what nn.LayerNorm computes)."""
    mu = x.mean(dim=-1, keepdim=True)
    var = (x - mu).square().mean(dim=-1, keepdim=True)
    return (x - mu) * torch.rsqrt(var + eps) * weight + bias


def linear(x: torch.Tensor, p: Params, name: str) -> torch.Tensor:
    """``nn.Linear`` with weight ``[out, in]`` (primitives.py:43-62)."""
    y = x @ p[name + ".weight"].t()
    b = p.get(name + ".bias")
    return y if b is None else y + b


# --------------------------------------------------------------------------------------
# Triangle multiplicative update -- src/genie_tk/triangle_mul.py:103-132
# --------------------------------------------------------------------------------------

def trimul_prepare(z: torch.Tensor, mask: Optional[torch.Tensor], p: Params, dtype: torch.dtype = torch.float32):
    """Row-independent part: default mask (triangle_mul.py:105-106), LN_in (:111) and the
    gated, masked projections a, b for every pair (:114-117). ``dtype`` is the compute
    type (fp32 for parity; bf16 with bf16 params times the reference's bf16 GPU path)."""
    z = z.to(dtype)
    if mask is None:
        mask = torch.ones(z.shape[:-1], dtype=z.dtype, device=z.device)
    m = mask.to(z.dtype).unsqueeze(-1)
    zn = layer_norm(z, p["layer_norm_in.weight"], p["layer_norm_in.bias"])
    a = linear(zn, p, "linear_a_p") * torch.sigmoid(linear(zn, p, "linear_a_g")) * m
    b = linear(zn, p, "linear_b_p") * torch.sigmoid(linear(zn, p, "linear_b_g")) * m
    return zn, a, b


def trimul_rows(zn: torch.Tensor, a: torch.Tensor, b: torch.Tensor, p: Params, outgoing: bool,
                r0: int = 0, r1: Optional[int] = None) -> torch.Tensor:
    """Output rows [r0, r1): the contraction, outgoing ``x[b,i,j,c] = sum_k a[b,i,k,c] b[b,j,k,c]``
    (triangle_mul.py:77-89) or incoming ``x[b,i,j,c] = sum_k a[b,k,i,c] b[b,k,j,c]`` (:91-101),
    then LN_out and linear_z (:126-127) and the output gate (:130-132)."""
    r1 = zn.shape[1] if r1 is None else r1
    if outgoing:
        x = torch.einsum("bikc,bjkc->bijc", a[:, r0:r1], b)
    else:
        x = torch.einsum("bkic,bkjc->bijc", a[:, :, r0:r1], b)
    x = layer_norm(x, p["layer_norm_out.weight"], p["layer_norm_out.bias"])
    x = linear(x, p, "linear_z")
    g = torch.sigmoid(linear(zn[:, r0:r1], p, "linear_g"))
    return x * g


def trimul_forward(z: torch.Tensor, mask: Optional[torch.Tensor], p: Params, outgoing: bool,
                   dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Update (not z + update) of the triangle multiplicative block (triangle_mul.py:103-132)."""
    zn, a, b = trimul_prepare(z, mask, p, dtype)
    return trimul_rows(zn, a, b, p, outgoing)


# --------------------------------------------------------------------------------------
# Triangle attention -- src/genie_tk/triangle_attention.py:100-143 and
# src/genie_tk/primitives.py:114-178
# --------------------------------------------------------------------------------------

def triatt_prepare(z: torch.Tensor, mask: Optional[torch.Tensor], p: Params, starting: bool,
                   dtype: torch.dtype = torch.float32):
    """Row-independent part: default mask (:106-107); ending node transposes x and mask
    (:110-112); LN (:115); triangle bias ``linear(x)`` permuted to ``[*,H,J,K]`` (query j,
    key k), shared by every row i (:121-129). ``dtype`` as in ``trimul_prepare``."""
    x = z.to(dtype)
    if mask is None:
        mask = torch.ones(x.shape[:-1], dtype=x.dtype, device=x.device)
    mask = mask.to(x.dtype)
    if not starting:
        x = x.transpose(-2, -3)
        mask = mask.transpose(-1, -2)
    x = layer_norm(x, p["layer_norm.weight"], p["layer_norm.bias"])
    tri = linear(x, p, "linear").permute(0, 3, 1, 2)
    return x, mask, tri


def triatt_rows(x: torch.Tensor, mask: torch.Tensor, tri: torch.Tensor, p: Params, no_heads: int,
                inf: float = 1e9, r0: int = 0, r1: Optional[int] = None) -> torch.Tensor:
    """Rows [r0, r1) of the gated multi-head attention (primitives.py:134-176): q,k,v
    without bias, scores ``q k^T / sqrt(d)`` then ``+ inf*(mask-1)`` on keys (:118) and
    ``+ tri_bias``, in that order; softmax over keys; ``@ v``; gate
    ``sigmoid(linear_g(x))``; ``linear_o``. Result in the problem orientation."""
    r1 = x.shape[1] if r1 is None else r1
    hd = p["mha.linear_q.weight"].shape[0]
    d = hd // no_heads
    scale = 1.0 / math.sqrt(d)
    B, N = x.shape[0], x.shape[2]
    xs = x[:, r0:r1]
    R = xs.shape[1]
    q = linear(xs, p, "mha.linear_q").view(B, R, N, no_heads, d).transpose(-2, -3)
    k = linear(xs, p, "mha.linear_k").view(B, R, N, no_heads, d).transpose(-2, -3)
    v = linear(xs, p, "mha.linear_v").view(B, R, N, no_heads, d).transpose(-2, -3)
    s = torch.matmul(q, k.transpose(-1, -2)) * scale          # [B, R, H, J, K]
    s = s + (inf * (mask[:, r0:r1] - 1.0))[:, :, None, None, :]
    s = s + tri[:, None]
    a = torch.softmax(s, dim=-1)
    o = torch.matmul(a, v).transpose(-2, -3).reshape(B, R, N, hd)
    o = o * torch.sigmoid(linear(xs, p, "mha.linear_g"))
    return linear(o, p, "mha.linear_o")


def triatt_forward(z: torch.Tensor, mask: Optional[torch.Tensor], p: Params, starting: bool,
                   no_heads: int, inf: float = 1e9, chunk_rows: int = 0,
                   dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Update of the triangle attention block around the starting (or ending) node
    (triangle_attention.py:100-143). ``chunk_rows`` > 0 evaluates the rows i in chunks
    to bound memory (rows are independent); 0 evaluates all rows at once like the
    reference. The ending node transposes back (:140-141)."""
    x, m, tri = triatt_prepare(z, mask, p, starting, dtype)
    N = x.shape[1]
    step = N if chunk_rows <= 0 else chunk_rows
    out = torch.cat([triatt_rows(x, m, tri, p, no_heads, inf, r0, min(N, r0 + step))
                     for r0 in range(0, N, step)], dim=1)
    if not starting:
        out = out.transpose(-2, -3)
    return out


# --------------------------------------------------------------------------------------
# The pair stack -- the explicit residual chain of examples/basic_usage.py:44-78, which
# equals PairTransformLayer.forward (pair_transform.py:162-195) minus PairTransition
# and the final mask multiply.
# --------------------------------------------------------------------------------------

STACK_OPS = ("tri_mul_out", "tri_mul_in", "tri_att_start", "tri_att_end")


def stack_forward(z: torch.Tensor, mask: Optional[torch.Tensor], layers: List[Dict[str, Params]],
                  no_heads: int, chunk_rows: int = 0, dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """``z += TriMulOut(z); z += TriMulIn(z); z += TriAttStart(z); z += TriAttEnd(z)`` per layer,
    computed in ``dtype`` (the parameters must be of that type)."""
    z = z.to(dtype).clone()
    for lp in layers:
        z = z + trimul_forward(z, mask, lp["tri_mul_out"], outgoing=True, dtype=dtype)
        z = z + trimul_forward(z, mask, lp["tri_mul_in"], outgoing=False, dtype=dtype)
        z = z + triatt_forward(z, mask, lp["tri_att_start"], starting=True, no_heads=no_heads,
                               chunk_rows=chunk_rows, dtype=dtype)
        z = z + triatt_forward(z, mask, lp["tri_att_end"], starting=False, no_heads=no_heads,
                               chunk_rows=chunk_rows, dtype=dtype)
    return z


# --------------------------------------------------------------------------------------
# Pair transition -- src/genie_tk/pair_transform.py:64-84, and the tail of
# PairTransformLayer.forward (:190-193)
# --------------------------------------------------------------------------------------

def transition_forward(z: torch.Tensor, p: Params) -> torch.Tensor:
    """PairTransition.forward (pair_transform.py:78-84): LN -> linear_1 -> ReLU -> linear_2.
    The reference ignores its mask argument here."""
    x = layer_norm(z.float(), p["layer_norm.weight"], p["layer_norm.bias"])
    return linear(torch.relu(linear(x, p, "linear_1")), p, "linear_2")


def layer_tail(z: torch.Tensor, mask: torch.Tensor, p: Params) -> torch.Tensor:
    """The last two statements of PairTransformLayer.forward (pair_transform.py:190-193):
    p = p + pair_transition(p, p_mask); p = p * p_mask.unsqueeze(-1)."""
    z = z.float()
    return (z + transition_forward(z, p)) * mask.float().unsqueeze(-1)


# --------------------------------------------------------------------------------------
# Seeded parameters and inputs of the benchmark configurations.
# Weights ~ N(0, 1/fan_in) in the reference layout [out, in]; biases 0 unless a gate
# bias of 1 is requested; LayerNorm gamma=1, beta=0 unless ``ln_random``.
# --------------------------------------------------------------------------------------

def _w(gen: torch.Generator, out_f: int, in_f: int) -> torch.Tensor:
    return torch.randn(out_f, in_f, generator=gen) / math.sqrt(in_f)


def make_trimul_params(c_z: int, c: int, gen: torch.Generator, gate_bias: float = 0.0,
                       ln_random: bool = False, bias_random: bool = False) -> Params:
    """Parameters of TriangleMultiplicativeUpdate (triangle_mul.py:64-73), in module order."""
    p: Params = {}
    for name, (o, i), gate in (("linear_a_p", (c, c_z), False), ("linear_a_g", (c, c_z), True),
                               ("linear_b_p", (c, c_z), False), ("linear_b_g", (c, c_z), True),
                               ("linear_g", (c_z, c_z), True), ("linear_z", (c_z, c), False)):
        p[name + ".weight"] = _w(gen, o, i)
        if bias_random:
            p[name + ".bias"] = 0.1 * torch.randn(o, generator=gen)
        else:
            p[name + ".bias"] = torch.full((o,), gate_bias if gate else 0.0)
    for name, n in (("layer_norm_in", c_z), ("layer_norm_out", c)):
        if ln_random:
            p[name + ".weight"] = 1.0 + 0.1 * torch.randn(n, generator=gen)
            p[name + ".bias"] = 0.1 * torch.randn(n, generator=gen)
        else:
            p[name + ".weight"] = torch.ones(n)
            p[name + ".bias"] = torch.zeros(n)
    return p


def make_triatt_params(c_in: int, c_hidden: int, no_heads: int, gen: torch.Generator,
                       gate_bias: float = 0.0, ln_random: bool = False,
                       bias_random: bool = False) -> Params:
    """Parameters of TriangleAttention (triangle_attention.py:70-82, primitives.py:319-328)."""
    p: Params = {}
    if ln_random:
        p["layer_norm.weight"] = 1.0 + 0.1 * torch.randn(c_in, generator=gen)
        p["layer_norm.bias"] = 0.1 * torch.randn(c_in, generator=gen)
    else:
        p["layer_norm.weight"] = torch.ones(c_in)
        p["layer_norm.bias"] = torch.zeros(c_in)
    p["linear.weight"] = _w(gen, no_heads, c_in)
    p["mha.linear_q.weight"] = _w(gen, c_hidden, c_in)
    p["mha.linear_k.weight"] = _w(gen, c_hidden, c_in)
    p["mha.linear_v.weight"] = _w(gen, c_hidden, c_in)
    p["mha.linear_o.weight"] = _w(gen, c_in, c_hidden)
    p["mha.linear_o.bias"] = 0.1 * torch.randn(c_in, generator=gen) if bias_random else torch.zeros(c_in)
    p["mha.linear_g.weight"] = _w(gen, c_hidden, c_in)
    p["mha.linear_g.bias"] = (0.1 * torch.randn(c_hidden, generator=gen) if bias_random
                              else torch.full((c_hidden,), gate_bias))
    return p


def pair_embed(s: torch.Tensor, mask: Optional[torch.Tensor], p: Params):
    """The pair embedding of examples/basic_usage.py:188-196: p_ij = Linear([s_i ; s_j]) over
    the concatenation (nn.Linear(2 c_s, c_p), keys ``weight`` / ``bias``) and
    p_mask = mask_i * mask_j (None without a mask)."""
    B, L, _ = s.shape
    s = s.float()
    s_i = s.unsqueeze(2).expand(-1, -1, L, -1)
    s_j = s.unsqueeze(1).expand(-1, L, -1, -1)
    pair = torch.cat([s_i, s_j], dim=-1) @ p["weight"].t()
    if p.get("bias") is not None:
        pair = pair + p["bias"]
    pm = None if mask is None else mask.float().unsqueeze(1) * mask.float().unsqueeze(2)
    return pair, pm


def make_transition_params(c_p: int, n: int, gen: torch.Generator, ln_random: bool = True,
                           bias_random: bool = True) -> Params:
    """Parameters of PairTransition (pair_transform.py:72-76), in module order. linear_2 is
    drawn like linear_1 rather than the reference's zero "final" init, so that the update
    is not identically zero."""
    p: Params = {}
    if ln_random:
        p["layer_norm.weight"] = 1.0 + 0.1 * torch.randn(c_p, generator=gen)
        p["layer_norm.bias"] = 0.1 * torch.randn(c_p, generator=gen)
    else:
        p["layer_norm.weight"] = torch.ones(c_p)
        p["layer_norm.bias"] = torch.zeros(c_p)
    for name, (o, i) in (("linear_1", (c_p * n, c_p)), ("linear_2", (c_p, c_p * n))):
        p[name + ".weight"] = _w(gen, o, i)
        p[name + ".bias"] = 0.1 * torch.randn(o, generator=gen) if bias_random else torch.zeros(o)
    return p


def make_pair(B: int, N: int, c_z: int, seed: int) -> torch.Tensor:
    """Pair tensor z ~ N(0, 1) from ``torch.manual_seed(seed)`` semantics (own generator)."""
    gen = torch.Generator().manual_seed(seed)
    return torch.randn(B, N, N, c_z, generator=gen)


def config_inputs(cfg: int, N: Optional[int] = None, B: Optional[int] = None):
    """Inputs, mask and parameters of benchmark configuration ``cfg`` (1..5).

    ``N``/``B`` override the size (for small parity cases with the same recipe).
    The z tensor uses seed ``cfg-1``; weights come from a generator seeded with
    ``1000 + cfg`` (drawn in module order).
    """
    defaults = {1: (1, 128), 2: (2, 384), 3: (1, 512), 4: (1, 768), 5: (1, 1024)}
    b0, n0 = defaults[cfg]
    B = b0 if B is None else B
    N = n0 if N is None else N
    z = make_pair(B, N, 128, seed=cfg - 1)
    mask = torch.ones(B, N, N)
    gen = torch.Generator().manual_seed(1000 + cfg)
    if cfg == 1:
        params = make_trimul_params(128, 128, gen)
    elif cfg == 2:
        if B > 1:
            pad = min(64, N // 2)
            mask[1, -pad:, :] = 0
            mask[1, :, -pad:] = 0
        params = make_trimul_params(128, 128, gen, gate_bias=1.0)
    elif cfg in (3, 4):
        if cfg == 3:
            pad = min(32, N // 4)
            mask[:, -pad:, :] = 0
            mask[:, :, -pad:] = 0
        params = make_triatt_params(128, 128, 4, gen, gate_bias=1.0)
    else:
        params = []
        for _ in range(8):
            params.append({
                "tri_mul_out": make_trimul_params(128, 128, gen, gate_bias=1.0),
                "tri_mul_in": make_trimul_params(128, 128, gen, gate_bias=1.0),
                "tri_att_start": make_triatt_params(128, 128, 4, gen, gate_bias=1.0),
                "tri_att_end": make_triatt_params(128, 128, 4, gen, gate_bias=1.0),
            })
    return z, mask, params


def flops_per_pair(op: str, N: int, c_z: int = 128, c: int = 128, H: int = 4, d: int = 32) -> float:
    """Algorithmic FLOPs per pair (i, j) of one op (reference math, multiply-add = 2)."""
    if op == "trimul":
        return 2.0 * N * c + 2.0 * c_z * (4 * c + c_z) + 2.0 * c * c_z
    if op == "triatt":
        hd = H * d
        return 4.0 * N * H * d + 2.0 * (3 * c_z * hd + c_z * hd + hd * c_z + c_z * H)
    if op == "layer":
        return 2 * flops_per_pair("trimul", N, c_z, c, H, d) + 2 * flops_per_pair("triatt", N, c_z, c, H, d)
    raise ValueError(op)


def time_layer_sample(z: torch.Tensor, mask: Optional[torch.Tensor], lp: Dict[str, Params], no_heads: int,
                      rows: int):
    """Wall-clock estimate of one full stack layer on this host, from a row sample.

    Each op is timed in two measured parts: its row-independent part (``*_prepare``:
    LayerNorm, the a/b projections or the triangle bias over all N^2 pairs) and the
    per-row part for ``rows`` output rows (``*_rows``). The per-row cost is linear in
    the number of rows, so the layer time is ``sum(t_prepare + t_rows * N / rows)``.
    Returns (estimated layer seconds, {op: (t_prepare, t_rows)}, measured seconds).
    """
    import time
    N = z.shape[1]
    parts = {}
    total = 0.0
    with torch.no_grad():
        for name in STACK_OPS:
            p = lp[name]
            t0 = time.perf_counter()
            if name.startswith("tri_mul"):
                zn, a, b = trimul_prepare(z, mask, p)
                t1 = time.perf_counter()
                trimul_rows(zn, a, b, p, name == "tri_mul_out", 0, rows)
            else:
                x, m, tri = triatt_prepare(z, mask, p, name == "tri_att_start")
                t1 = time.perf_counter()
                triatt_rows(x, m, tri, p, no_heads, 1e9, 0, rows)
            t2 = time.perf_counter()
            parts[name] = (t1 - t0, t2 - t1)
            total += t2 - t0
    est = sum(f + r * N / rows for f, r in parts.values())
    return est, parts, total
