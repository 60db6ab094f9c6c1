"""Loading helpers for the golden fixtures (tests only)."""

from __future__ import annotations

import ast
import os

import numpy as np
import torch

from oracle import triangle_oracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")

SINGLE_CASES = ["trimul_out_small", "trimul_in_small", "triatt_start_small", "triatt_end_small",
                "trimul_out_c128", "trimul_in_c128", "triatt_start_c128", "triatt_end_c128"]


def _checksum(p):
    return np.array([[float(p[k].double().sum()), float(p[k].double().square().sum())] for k in sorted(p)])


def load_case(name):
    """Return (op, dims, z, mask, params, out) for a golden case; params are regenerated and pinned."""
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    op = str(d["op"])
    dims = dict(B=int(d["B"]), N=int(d["N"]), c_z=int(d["c_z"]), c_hidden=int(d["c_hidden"]),
                heads=int(d["heads"]))
    keys = [str(k) for k in d["param_keys"]]
    if ("p:" + keys[0]) in d.files:
        params = {k: torch.from_numpy(d["p:" + k]) for k in keys}
    else:
        kw = ast.literal_eval(str(d["param_kwargs"]))
        gen = torch.Generator().manual_seed(int(d["param_seed"]))
        if op.startswith("trimul"):
            params = O.make_trimul_params(dims["c_z"], dims["c_hidden"], gen, **kw)
        else:
            params = O.make_triatt_params(dims["c_z"], dims["c_hidden"], dims["heads"], gen, **kw)
        np.testing.assert_allclose(_checksum(params), d["param_checksum"], rtol=1e-6, atol=1e-6)
    return op, dims, torch.from_numpy(d["z"]), torch.from_numpy(d["mask"]), params, torch.from_numpy(d["out"])


def load_transition(name="transition_c128"):
    """(z, mask, params, out) of a pair-transition golden case; params regenerated and pinned."""
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    params = O.make_transition_params(int(d["c_z"]), int(d["c_hidden"]) // int(d["c_z"]),
                                      torch.Generator().manual_seed(int(d["param_seed"])))
    np.testing.assert_allclose(_checksum(params), d["param_checksum"], rtol=1e-6, atol=1e-6)
    return torch.from_numpy(d["z"]), torch.from_numpy(d["mask"]), params, torch.from_numpy(d["out"])


def load_stack():
    d = np.load(os.path.join(GOLDEN, "stack2_c128.npz"))
    gen = torch.Generator().manual_seed(int(d["param_seed"]))
    layers = []
    for _ in range(int(d["n_layers"])):
        layers.append({
            "tri_mul_out": O.make_trimul_params(128, 128, gen, gate_bias=1.0),
            "tri_mul_in": O.make_trimul_params(128, 128, gen, gate_bias=1.0),
            "tri_att_start": O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0),
            "tri_att_end": O.make_triatt_params(128, 128, 4, gen, gate_bias=1.0),
        })
    cks = np.concatenate([_checksum(lp[k]) for lp in layers for k in O.STACK_OPS])
    np.testing.assert_allclose(cks, d["param_checksum"], rtol=1e-6, atol=1e-6)
    return torch.from_numpy(d["z"]), torch.from_numpy(d["mask"]), layers, torch.from_numpy(d["out"])


def oracle_run(op, dims, z, mask, params, chunk_rows=0):
    if op == "trimul_out":
        return O.trimul_forward(z, mask, params, outgoing=True)
    if op == "trimul_in":
        return O.trimul_forward(z, mask, params, outgoing=False)
    if op == "triatt_start":
        return O.triatt_forward(z, mask, params, starting=True, no_heads=dims["heads"], chunk_rows=chunk_rows)
    return O.triatt_forward(z, mask, params, starting=False, no_heads=dims["heads"], chunk_rows=chunk_rows)


GENERAL_CASES = ["gen_trimul_out_c64_h32", "gen_trimul_in_c128_h64", "gen_trimul_in_c32_h16",
                 "gen_triatt_start_c128_h32x4", "gen_triatt_end_c64_h32x4", "gen_triatt_start_c32_h16x2",
                 "gen_triatt_end_c128_h16x4"]
LAYER_CASES = ["gen_layer_c64_default_test", "gen_layer_c128_defaults"]


def layer_params(c_p, c_mul, c_att, heads, gen):
    """Seeded PairTransformLayer parameters in module order (as tests/golden/make_golden.py draws them),
    as {block: state_dict} with the transition under "pair_transition"."""
    out = {}
    for name, kind in (("tri_mul_out", "mul"), ("tri_mul_in", "mul"), ("tri_att_start", "att"),
                       ("tri_att_end", "att")):
        out[name] = (O.make_trimul_params(c_p, c_mul, gen, ln_random=True, bias_random=True) if kind == "mul"
                     else O.make_triatt_params(c_p, c_att, heads, gen, ln_random=True, bias_random=True))
    out["pair_transition"] = O.make_transition_params(c_p, 4, gen)
    return out


def load_layer(name):
    """(dims, z, mask, {block: params}, out) of a PairTransformLayer golden case; params regenerated
    from their seed and pinned by the stored checksum."""
    d = np.load(os.path.join(GOLDEN, name + ".npz"))
    dims = dict(B=int(d["B"]), N=int(d["N"]), c_p=int(d["c_p"]), c_mul=int(d["c_mul"]), c_att=int(d["c_att"]),
                heads=int(d["heads"]))
    blocks = layer_params(dims["c_p"], dims["c_mul"], dims["c_att"], dims["heads"],
                          torch.Generator().manual_seed(int(d["param_seed"])))
    flat = {f"{b}.{k}": v for b, p in blocks.items() for k, v in p.items()}
    np.testing.assert_allclose(_checksum(flat), d["param_checksum"], rtol=1e-6, atol=1e-6)
    return dims, torch.from_numpy(d["z"]), torch.from_numpy(d["mask"]), blocks, torch.from_numpy(d["out"])


def oracle_layer(z, mask, blocks, heads, chunk_rows=0):
    """PairTransformLayer.forward in eval mode (pair_transform.py:162-195) on the oracle."""
    z = O.stack_forward(z, mask, [{k: blocks[k] for k in O.STACK_OPS}], no_heads=heads, chunk_rows=chunk_rows)
    return O.layer_tail(z, mask, blocks["pair_transition"])
