"""B200-native (sm_100a) pre-norm causal Transformer forward.

Drop-in for the hot path of gwenlim89/GPU-kernel-for-transformer:
``UserOptimizedTransformer(config)(x, valid_token_mask)`` with the
reference's config, parameter names and forward contract, computed by
hand-written CUDA kernels (tcgen05/TMEM GEMMs, flash attention, fused
LayerNorm) behind the C ABI in ``include/tfx.h``.

The directory name is not a Python identifier; import it with
``importlib.import_module("gpu-kernel-for-transformer_b200")``.
"""

from . import _lib, ops, sharding  # noqa: F401
from .graph import FixedInputCUDAGraph, ForwardGraph, maybe_cuda_graph  # noqa: F401
from .streaming import StreamingForward  # noqa: F401
from .model import (  # noqa: F401
    OFFICIAL_BENCHMARK_SHAPES,
    BaselineTransformer,
    ShapeExecutionPlan,
    TransformerConfig,
    UserOptimizedTransformer,
)

__all__ = [
    "TransformerConfig",
    "OFFICIAL_BENCHMARK_SHAPES",
    "BaselineTransformer",
    "UserOptimizedTransformer",
    "ShapeExecutionPlan",
    "FixedInputCUDAGraph",
    "ForwardGraph",
    "maybe_cuda_graph",
    "StreamingForward",
    "ops",
    "sharding",
]


def library_path():
    """Path of the C-ABI shared library this package drives."""
    return _lib.LIB_PATH
