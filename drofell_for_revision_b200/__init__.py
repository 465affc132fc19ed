"""B200-native (sm_100a) GPTQ W4A16 quantized linear for DROFELL.

Drop-in for the reference's quantized-linear hot path:
  * ``real_quant``  - ``QuantLinear`` / ``QuantLinearMaker`` (operators/core/linear/real_quant.py)
  * ``exllama``     - ``make_q4``, ``Q4MatrixV2``, ``CacheV2``, ``TuningParams`` and the v2
                      kernel entry points (cuda_extends/exllama.py)
  * ``sharded``     - N-column-sharded linear over 1..8 GPUs with an NCCL all-gather
  * ``_capi``       - ctypes binding of the C ABI (include/drofell_w4a16.h)
"""
from . import _capi  # noqa: F401

__all__ = ["_capi"]
__version__ = "0.1.0"
