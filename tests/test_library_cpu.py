"""The torch.ops.genie_tk.* operators: registration, schemas and shape propagation (no GPU)."""

import torch

import genie_tk  # noqa: F401  (registers the operators)


def _meta(*shape, dtype=torch.float32):
    return torch.empty(*shape, dtype=dtype, device="meta")


def test_operators_registered_with_schemas():
    for name, args in (("trimul_forward", "Tensor z, Tensor? mask, Tensor packed, bool outgoing"),
                       ("triatt_forward", "Tensor z, Tensor? mask, Tensor packed, bool starting, float inf"),
                       ("trimul_residual_", "Tensor(a0!) z, Tensor? mask, Tensor packed, bool outgoing"),
                       ("triatt_residual_", "Tensor(a0!) z, Tensor? mask, Tensor packed, bool starting, float inf"),
                       ("transition_forward", "Tensor z, Tensor packed"),
                       ("transition_residual_", "Tensor(a0!) z, Tensor? mask, Tensor packed")):
        op = getattr(torch.ops.genie_tk, name).default
        assert args in str(op._schema), str(op._schema)


def test_fake_implementations_propagate_shapes():
    z, m, p = _meta(2, 24, 24, 128), _meta(2, 24, 24), _meta(4096, dtype=torch.uint8)
    u = torch.ops.genie_tk.trimul_forward(z, m, p, True)
    assert u.shape == z.shape and u.dtype == torch.float32 and u.device.type == "meta"
    v = torch.ops.genie_tk.triatt_forward(z.to(torch.bfloat16), None, p, False, 1e9)
    assert v.shape == z.shape and v.dtype == torch.float32
    assert torch.ops.genie_tk.trimul_residual_(z, m, p, False) is None
    assert torch.ops.genie_tk.triatt_residual_(z, None, p, True, 1e9) is None
    t = torch.ops.genie_tk.transition_forward(z.half(), p)
    assert t.shape == z.shape and t.dtype == torch.float32
    assert torch.ops.genie_tk.transition_residual_(z, m, p) is None


def test_operators_refuse_cpu_tensors():
    from genie_tk import ops
    packed = torch.zeros(16, dtype=torch.uint8)
    for call in (lambda: torch.ops.genie_tk.trimul_forward(torch.zeros(1, 4, 4, 128), None, packed, True),
                 lambda: torch.ops.genie_tk.triatt_forward(torch.zeros(1, 4, 4, 128), None, packed, True, 1e9)):
        try:
            call()
        except (RuntimeError, OSError) as exc:  # no CPU path (and no GPU library load on CPU)
            assert "CUDA" in str(exc) or "cuda" in str(exc) or "lib" in str(exc).lower()
        else:
            raise AssertionError("a CPU tensor must be refused")
    assert ops.SUPPORTED_C == 128
