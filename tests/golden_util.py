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
