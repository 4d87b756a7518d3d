"""g4b -- B200 (sm_100a) int4/int8 quantized-weight matmuls for gemma4-adreno.

Host side of the drop-in for the engine's quantized-weight dispatches
(src/vk_engine.py): ``pack`` restates the engine's weight packing, ``ops``
calls the CUDA library through its C ABI (include/g4b.h) on torch tensors, and
``engine_surface`` mirrors the engine's per-op call surface
(gemv_ds/gemv/gemm_ds/gmm).
"""
from . import pack  # noqa: F401
from .pack import BLK, FP8, PREFILL_I8, PackedWeight, quant  # noqa: F401


def quant_device(*args, **kwargs):
    """GPU packing, see g4b.quant_gpu.quant_device (imports torch lazily)."""
    from .quant_gpu import quant_device as _qd
    return _qd(*args, **kwargs)

__version__ = "0.1.0"
