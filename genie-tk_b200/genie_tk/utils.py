"""Utility functions with the reference's names (src/genie_tk/utils.py)."""

from __future__ import annotations

from typing import Any, Callable, Dict

import torch
from torch import Tensor

from . import _lib


def has_cuda_kernels() -> bool:
    """True when the B200 kernel library loads and a CUDA device is present (utils.py:12-18)."""
    return _lib.available() and torch.cuda.is_available()


def get_device_info() -> Dict[str, Any]:
    """Device summary (utils.py:21-42), plus the library version."""
    info: Dict[str, Any] = {
        "cuda_available": torch.cuda.is_available(),
        "cuda_kernels_available": has_cuda_kernels(),
        "device_count": 0,
        "devices": [],
        "library": _lib.LIB_PATH,
        "library_version": _lib.load().gtk_version() if _lib.available() else None,
    }
    if torch.cuda.is_available():
        info["device_count"] = torch.cuda.device_count()
        for i in range(info["device_count"]):
            props = torch.cuda.get_device_properties(i)
            info["devices"].append({
                "name": props.name,
                "total_memory": props.total_memory,
                "major": props.major,
                "minor": props.minor,
                "multi_processor_count": props.multi_processor_count,
            })
    return info


def permute_final_dims(tensor: Tensor, *dims: int) -> Tensor:
    """Permute the trailing ``len(dims)`` axes (utils.py:45-60)."""
    lead = tensor.dim() - len(dims)
    return tensor.permute(list(range(lead)) + [lead + d for d in dims])


def flatten_final_dims(tensor: Tensor, num_dims: int) -> Tensor:
    """Flatten the trailing ``num_dims`` axes (utils.py:63-75)."""
    return tensor.reshape(tensor.shape[:-num_dims] + (-1,))


def chunk_layer(layer: Callable, inputs: Dict[str, Tensor], chunk_size: int, no_batch_dims: int) -> Tensor:
    """Apply ``layer`` over the flattened leading batch axes in chunks (utils.py:78-123)."""
    first = next(iter(inputs.values()))
    batch_shape = first.shape[:no_batch_dims]
    flat = {k: v.reshape((-1,) + v.shape[no_batch_dims:]) for k, v in inputs.items()}
    total = next(iter(flat.values())).shape[0]
    outs = [layer(**{k: v[s:s + chunk_size] for k, v in flat.items()}) for s in range(0, total, chunk_size)]
    out = torch.cat(outs, dim=0)
    return out.reshape(batch_shape + out.shape[1:])
