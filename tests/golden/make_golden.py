"""Generate the golden vectors in this directory from the reference's own modules.

Run where the reference is mounted (its root is ``$GTK_REFERENCE_ROOT``, defaulting to
the mount point named in ``oracle/reference_copy.py``)::

    python tests/golden/make_golden.py              # triangle blocks and the 2-layer stack
    python tests/golden/make_golden.py transition   # the pair transition
    python tests/golden/make_golden.py general      # the reference's default / example / test shapes

The reference package is imported from a repaired copy (``oracle/reference_copy.py``:
mechanical docstring repair only). For every case the script builds the reference
module, loads seeded parameters (``oracle.triangle_oracle.make_*_params``) into it
with ``load_state_dict``, runs ``module(z, mask)`` in fp32 on the CPU and stores
inputs, outputs and (for small channel counts) the parameters themselves. For the
128-channel cases the parameters are regenerated from their seed by the tests and
pinned by a stored checksum, which keeps the fixtures small.
"""

from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle import triangle_oracle as O  # noqa: E402
from oracle.reference_copy import import_reference  # noqa: E402


def param_checksum(p):
    keys = sorted(p)
    return np.array([[float(p[k].double().sum()), float(p[k].double().square().sum())] for k in keys])


# name -> (op, B, N, c_z, c_hidden, heads, seed, store_params, mask_kind, param_kwargs)
CASES = {
    "trimul_out_small": ("trimul_out", 2, 12, 32, 16, 0, 11, True, "ragged", dict(ln_random=True, bias_random=True)),
    "trimul_in_small": ("trimul_in", 2, 12, 32, 16, 0, 12, True, "ragged", dict(ln_random=True, bias_random=True)),
    "triatt_start_small": ("triatt_start", 2, 10, 32, 16, 4, 13, True, "rowdead", dict(ln_random=True, bias_random=True)),
    "triatt_end_small": ("triatt_end", 2, 10, 32, 16, 4, 14, True, "rowdead", dict(ln_random=True, bias_random=True)),
    "trimul_out_c128": ("trimul_out", 1, 16, 128, 128, 0, 21, False, "ones", dict(ln_random=True, bias_random=True)),
    "trimul_in_c128": ("trimul_in", 2, 16, 128, 128, 0, 22, False, "pad", dict(gate_bias=1.0)),
    "triatt_start_c128": ("triatt_start", 1, 16, 128, 128, 4, 23, False, "pad", dict(ln_random=True, bias_random=True)),
    "triatt_end_c128": ("triatt_end", 1, 16, 128, 128, 4, 24, False, "rowdead", dict(gate_bias=1.0)),
}


def make_mask(kind, B, N, gen):
    m = torch.ones(B, N, N)
    if kind == "ragged":
        m = (torch.rand(B, N, N, generator=gen) > 0.2).float()
    elif kind == "pad":
        m[-1, -3:, :] = 0
        m[-1, :, -3:] = 0
    elif kind == "rowdead":
        m[:, 2, :] = 0           # a fully masked row (uniform softmax in the reference)
        m[:, :, N - 1] = 0       # and a masked key column
    return m


def build_params(op, c_z, c, H, seed, kw):
    gen = torch.Generator().manual_seed(seed)
    if op.startswith("trimul"):
        return O.make_trimul_params(c_z, c, gen, **kw)
    return O.make_triatt_params(c_z, c, H, gen, **kw)


def main():
    ref = import_reference()
    torch.set_grad_enabled(False)
    for name, (op, B, N, c_z, c, H, seed, store_params, mkind, kw) in CASES.items():
        gen = torch.Generator().manual_seed(seed)
        z = torch.randn(B, N, N, c_z, generator=gen)
        mask = make_mask(mkind, B, N, gen)
        p = build_params(op, c_z, c, H, seed + 100, kw)
        if op == "trimul_out":
            mod = ref.TriangleMultiplicationOutgoing(c_z, c, use_fused_kernel=False)
        elif op == "trimul_in":
            mod = ref.TriangleMultiplicationIncoming(c_z, c, use_fused_kernel=False)
        elif op == "triatt_start":
            mod = ref.TriangleAttentionStartingNode(c_z, c, H, use_fused_kernel=False)
        else:
            mod = ref.TriangleAttentionEndingNode(c_z, c, H, use_fused_kernel=False)
        missing = set(mod.state_dict()) ^ set(p)
        assert not missing, missing
        mod.load_state_dict(p)
        mod.eval()
        out = mod(z, mask)
        rec = dict(op=np.array(op), B=B, N=N, c_z=c_z, c_hidden=c, heads=H, param_seed=seed + 100,
                   z=z.numpy(), mask=mask.numpy(), out=out.numpy(),
                   param_keys=np.array(sorted(p)), param_checksum=param_checksum(p),
                   param_kwargs=np.array(repr(kw)))
        if store_params:
            for k, v in p.items():
                rec["p:" + k] = v.numpy()
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
        print(f"{name}: out |max| {out.abs().max():.4f}")

    # A 2-layer stack (the explicit 4-op residual chain) at c_z = 128, N = 8.
    B, N = 1, 8
    gen = torch.Generator().manual_seed(31)
    z0 = torch.randn(B, N, N, 128, generator=gen)
    mask = torch.ones(B, N, N)
    pgen = torch.Generator().manual_seed(131)
    layers = []
    for _ in range(2):
        layers.append({
            "tri_mul_out": O.make_trimul_params(128, 128, pgen, gate_bias=1.0),
            "tri_mul_in": O.make_trimul_params(128, 128, pgen, gate_bias=1.0),
            "tri_att_start": O.make_triatt_params(128, 128, 4, pgen, gate_bias=1.0),
            "tri_att_end": O.make_triatt_params(128, 128, 4, pgen, gate_bias=1.0),
        })
    z = z0.clone()
    for lp in layers:
        mods = [ref.TriangleMultiplicationOutgoing(128, 128, use_fused_kernel=False),
                ref.TriangleMultiplicationIncoming(128, 128, use_fused_kernel=False),
                ref.TriangleAttentionStartingNode(128, 128, 4, use_fused_kernel=False),
                ref.TriangleAttentionEndingNode(128, 128, 4, use_fused_kernel=False)]
        for m, key in zip(mods, O.STACK_OPS):
            m.load_state_dict(lp[key])
            z = z + m(z, mask)
    cks = np.concatenate([param_checksum(lp[k]) for lp in layers for k in O.STACK_OPS])
    np.savez_compressed(os.path.join(HERE, "stack2_c128.npz"), z=z0.numpy(), mask=mask.numpy(), out=z.numpy(),
                        param_seed=131, n_layers=2, param_checksum=cks)
    print(f"stack2_c128: out |max| {z.abs().max():.4f}")


def main_transition():
    """Golden vectors of the reference's PairTransition (pair_transform.py:64-84), c_p = 128,
    n = 4, with seeded parameters (regenerated by the tests, pinned by checksum)."""
    ref = import_reference()
    torch.set_grad_enabled(False)
    for name, (B, N, seed) in {"transition_c128": (2, 8, 41)}.items():
        gen = torch.Generator().manual_seed(seed)
        z = torch.randn(B, N, N, 128, generator=gen)
        mask = make_mask("ragged", B, N, gen)
        p = O.make_transition_params(128, 4, torch.Generator().manual_seed(seed + 100))
        mod = ref.pair_transform.PairTransition(128, 4) if hasattr(ref, "pair_transform") else ref.PairTransition(128, 4)
        missing = set(mod.state_dict()) ^ set(p)
        assert not missing, missing
        mod.load_state_dict(p)
        mod.eval()
        upd = mod(z, mask)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), op=np.array("transition"), B=B, N=N, c_z=128,
                            c_hidden=512, heads=0, param_seed=seed + 100, z=z.numpy(), mask=mask.numpy(),
                            out=upd.numpy(), param_keys=np.array(sorted(p)),
                            param_checksum=param_checksum(p), param_kwargs=np.array(repr({})))
        print(f"{name}: out |max| {upd.abs().max():.4f}")


# The shapes the reference's own defaults, examples and tests use (pair_transform.py:113-119:
# c_hidden_mul 128, c_hidden_tri_att 32 with 4 heads, i.e. head_dim 8; examples/basic_usage.py:
# 140-142: c_hidden_mul 64, c_hidden_tri_att 16; tests/test_triangle_mul.py:37 and
# tests/test_triangle_attention.py:36,74,127-137: c_z 64 / 32, c_hidden 32 / 16, 4 or 2 heads).
# name -> (op, B, N, c_z, c_hidden, heads, seed, mask_kind, param_kwargs); parameters regenerated
# from their seed by the tests and pinned by checksum.
GENERAL_CASES = {
    "gen_trimul_out_c64_h32": ("trimul_out", 2, 24, 64, 32, 0, 51, "ragged", dict(ln_random=True, bias_random=True)),
    "gen_trimul_in_c128_h64": ("trimul_in", 1, 20, 128, 64, 0, 52, "pad", dict(gate_bias=1.0)),
    "gen_trimul_in_c32_h16": ("trimul_in", 2, 15, 32, 16, 0, 53, "ragged", dict(ln_random=True, bias_random=True)),
    "gen_triatt_start_c128_h32x4": ("triatt_start", 1, 20, 128, 32, 4, 54, "rowdead",
                                    dict(ln_random=True, bias_random=True)),
    "gen_triatt_end_c64_h32x4": ("triatt_end", 2, 18, 64, 32, 4, 55, "pad", dict(gate_bias=1.0)),
    "gen_triatt_start_c32_h16x2": ("triatt_start", 2, 13, 32, 16, 2, 56, "ragged",
                                   dict(ln_random=True, bias_random=True)),
    "gen_triatt_end_c128_h16x4": ("triatt_end", 1, 17, 128, 16, 4, 57, "rowdead", dict(ln_random=True,
                                                                                       bias_random=True)),
}

# PairTransformLayer cases: name -> (B, N, c_p, c_hidden_mul, c_hidden_tri_att, n_head_tri, seed)
LAYER_CASES = {
    "gen_layer_c64_default_test": (1, 16, 64, 32, 16, 4, 61),   # tests/test_triangle_attention.py:127-137
    "gen_layer_c128_defaults": (1, 12, 128, 128, 32, 4, 62),     # pair_transform.py:113-119 defaults
}


def layer_params(c_p, c_mul, c_att, heads, gen):
    """Seeded parameters of PairTransformLayer in module order, keyed like its state_dict."""
    p = {}
    for name, kind in (("tri_mul_out", "mul"), ("tri_mul_in", "mul"), ("tri_att_start", "att"),
                       ("tri_att_end", "att")):
        sub = (O.make_trimul_params(c_p, c_mul, gen, ln_random=True, bias_random=True) if kind == "mul"
               else O.make_triatt_params(c_p, c_att, heads, gen, ln_random=True, bias_random=True))
        p.update({f"{name}.{k}": v for k, v in sub.items()})
    p.update({f"pair_transition.{k}": v for k, v in O.make_transition_params(c_p, 4, gen).items()})
    return p


def main_general():
    ref = import_reference()
    torch.set_grad_enabled(False)
    for name, (op, B, N, c_z, c, H, seed, mkind, kw) in GENERAL_CASES.items():
        gen = torch.Generator().manual_seed(seed)
        z = torch.randn(B, N, N, c_z, generator=gen)
        mask = make_mask(mkind, B, N, gen)
        p = build_params(op, c_z, c, H, seed + 100, kw)
        if op == "trimul_out":
            mod = ref.TriangleMultiplicationOutgoing(c_z, c, use_fused_kernel=False)
        elif op == "trimul_in":
            mod = ref.TriangleMultiplicationIncoming(c_z, c, use_fused_kernel=False)
        elif op == "triatt_start":
            mod = ref.TriangleAttentionStartingNode(c_z, c, H, use_fused_kernel=False)
        else:
            mod = ref.TriangleAttentionEndingNode(c_z, c, H, use_fused_kernel=False)
        missing = set(mod.state_dict()) ^ set(p)
        assert not missing, missing
        mod.load_state_dict(p)
        mod.eval()
        out = mod(z, mask)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), op=np.array(op), B=B, N=N, c_z=c_z, c_hidden=c,
                            heads=H, param_seed=seed + 100, z=z.numpy(), mask=mask.numpy(), out=out.numpy(),
                            param_keys=np.array(sorted(p)), param_checksum=param_checksum(p),
                            param_kwargs=np.array(repr(kw)))
        print(f"{name}: out |max| {out.abs().max():.4f}")

    # the pair transition at c_p = 64 (reference test width), n = 4
    B, N, seed = 2, 10, 58
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(B, N, N, 64, generator=gen)
    mask = make_mask("ragged", B, N, gen)
    p = O.make_transition_params(64, 4, torch.Generator().manual_seed(seed + 100))
    mod = ref.pair_transform.PairTransition(64, 4) if hasattr(ref, "pair_transform") else ref.PairTransition(64, 4)
    mod.load_state_dict(p)
    mod.eval()
    upd = mod(z, mask)
    np.savez_compressed(os.path.join(HERE, "gen_transition_c64.npz"), op=np.array("transition"), B=B, N=N, c_z=64,
                        c_hidden=256, heads=0, param_seed=seed + 100, z=z.numpy(), mask=mask.numpy(),
                        out=upd.numpy(), param_keys=np.array(sorted(p)), param_checksum=param_checksum(p),
                        param_kwargs=np.array(repr({})))
    print(f"gen_transition_c64: out |max| {upd.abs().max():.4f}")

    # whole PairTransformLayers in eval mode (dropout off), with a ragged pair mask
    for name, (B, N, c_p, c_mul, c_att, heads, seed) in LAYER_CASES.items():
        gen = torch.Generator().manual_seed(seed)
        z = torch.randn(B, N, N, c_p, generator=gen)
        mask = make_mask("pad", B, N, gen)
        p = layer_params(c_p, c_mul, c_att, heads, torch.Generator().manual_seed(seed + 100))
        mod = ref.PairTransformLayer(c_p=c_p, c_hidden_mul=c_mul, c_hidden_tri_att=c_att, n_head_tri=heads,
                                     use_fused_kernel=False)
        missing = set(mod.state_dict()) ^ set(p)
        assert not missing, missing
        mod.load_state_dict(p)
        mod.eval()
        out, _ = mod((z, mask))
        np.savez_compressed(os.path.join(HERE, name + ".npz"), B=B, N=N, c_p=c_p, c_mul=c_mul, c_att=c_att,
                            heads=heads, param_seed=seed + 100, z=z.numpy(), mask=mask.numpy(), out=out.numpy(),
                            param_keys=np.array(sorted(p)), param_checksum=param_checksum(p))
        print(f"{name}: out |max| {out.abs().max():.4f}")


if __name__ == "__main__":
    if sys.argv[1:] == ["transition"]:
        main_transition()
    elif sys.argv[1:] == ["general"]:
        main_general()
    else:
        main()
