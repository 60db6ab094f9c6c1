"""CPU checks of ``genie_tk._C``, the counterpart of the reference's native module: the same
six functions with the same argument names and defaults as kernels/bindings.cpp:69-101,
CUDA-only behaviour (RuntimeError, like the reference's TORCH_CHECKs), and the argument
validation of the LayerNorm entry point of the C ABI. No kernel is launched here."""

import inspect
import os

import pytest
import torch

# name -> parameters, as bound in kernels/bindings.cpp:73-99 (py::arg names and defaults)
REFERENCE_C = {
    "triangle_mul_outgoing": ["a", "b", "mask"],
    "triangle_mul_incoming": ["a", "b", "mask"],
    "triangle_attention_starting": ["q", "k", "v", "bias", "mask", "scale"],
    "triangle_attention_ending": ["q", "k", "v", "bias", "mask", "scale"],
    "layernorm": ["x", "gamma", "beta", "eps=1e-05"],
    "fused_layernorm_linear": ["x", "gamma", "beta", "weight", "bias=None", "eps=1e-05"],
}


def _params(fn):
    out = []
    for p in inspect.signature(fn).parameters.values():
        out.append(p.name if p.default is inspect.Parameter.empty else f"{p.name}={p.default!r}")
    return out


def test_module_has_the_reference_functions_and_signatures():
    from genie_tk import _C
    public = sorted(n for n in dir(_C) if not n.startswith("_") and callable(getattr(_C, n))
                    and getattr(getattr(_C, n), "__module__", "") == _C.__name__)
    assert public == sorted(REFERENCE_C)
    for name, params in REFERENCE_C.items():
        assert _params(getattr(_C, name)) == params, name


def test_cpu_tensors_raise_runtime_error():
    from genie_tk import _C
    a = torch.zeros(1, 4, 4, 128)
    m = torch.ones(1, 4, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.triangle_mul_outgoing(a, a, m)
    q = torch.zeros(1, 4, 4, 4, 32)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.triangle_attention_starting(q, q, q, torch.zeros(1, 4, 4, 4), m, 32 ** -0.5)
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.layernorm(torch.zeros(3, 8), torch.ones(8), torch.zeros(8))
    with pytest.raises(RuntimeError, match="CUDA"):
        _C.fused_layernorm_linear(torch.zeros(3, 8), torch.ones(8), torch.zeros(8), torch.zeros(8, 4))


@pytest.fixture(scope="module")
def lib():
    import genie_tk._lib as L
    if not os.path.exists(L.LIB_PATH):
        import __graft_entry__ as g
        g.build()
    return L.load()


def test_layernorm_entry_point_validates_arguments(lib):
    fake = 1 << 20  # never dereferenced: every call below fails validation first
    assert lib.gtk_layernorm(fake, fake, fake, fake, 0, 128, 1e-5, None) == -1
    assert lib.gtk_layernorm(fake, fake, fake, fake, 4, 0, 1e-5, None) == -1
    assert lib.gtk_layernorm(fake, fake, fake, fake, 4, 128, -1.0, None) == -1
    assert lib.gtk_layernorm(None, fake, fake, fake, 4, 128, 1e-5, None) == -1
    assert lib.gtk_layernorm(fake + 2, fake, fake, fake, 4, 128, 1e-5, None) == -3
    assert "layernorm" in lib.gtk_last_error_string().decode() or "misaligned" in lib.gtk_last_error_string().decode()
