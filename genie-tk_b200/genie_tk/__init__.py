"""genie_tk (B200): drop-in triangle hot path of northws/Genie-TK on hand-written sm_100a kernels.

Public API as in the reference's src/genie_tk/__init__.py:13-50, plus the fused
``TrianglePairStack``, the ``ops`` module (thin wrappers over the C ABI) and the
``torch.ops.genie_tk.*`` operators registered by ``genie_tk.library``.
"""

__version__ = "0.1.0"

from .triangle_mul import (  # noqa: F401
    TriangleMultiplicativeUpdate,
    TriangleMultiplicationOutgoing,
    TriangleMultiplicationIncoming,
)
from .triangle_attention import (  # noqa: F401
    TriangleAttention,
    TriangleAttentionStartingNode,
    TriangleAttentionEndingNode,
)
from .pair_transform import PairEmbedding, PairTransformLayer, PairTransformNet  # noqa: F401
from .stack import TrianglePairStack  # noqa: F401
from .utils import has_cuda_kernels, get_device_info  # noqa: F401
from . import library  # noqa: F401  (registers torch.ops.genie_tk.*)

__all__ = [
    "TriangleMultiplicativeUpdate",
    "TriangleMultiplicationOutgoing",
    "TriangleMultiplicationIncoming",
    "TriangleAttention",
    "TriangleAttentionStartingNode",
    "TriangleAttentionEndingNode",
    "PairTransformLayer",
    "PairTransformNet",
    "PairEmbedding",
    "TrianglePairStack",
    "has_cuda_kernels",
    "get_device_info",
]
