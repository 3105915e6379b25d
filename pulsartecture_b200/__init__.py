"""pulsartecture_b200: Ultra-RWKA's FA-KLA (causal temperature-modulated
kernelized linear attention) on NVIDIA B200, sm_100a.

Layout:
  csrc/        CUDA kernels (tcgen05 phi GEMM, tcgen05 chunk scan, decode,
               CUDA-core fp32 paths) and the C ABI (include/fakla.h)
  _lib.py      ctypes binding of lib/libfakla.so
  backend/     torch-tensor front end (reference: ultra_rwka.backend.interface)
  kernels/     FeatureMap / LearnablePositiveMap (reference: ultra_rwka.kernels)
  components/  LinearProjection (reference: ultra_rwka.components.projections)
  attention/   TMLinKernelAttn, TemperatureFunction, fa_kla, fa_kla_host, fa_kla_decode
               (reference: ultra_rwka.attention)
"""
__version__ = "0.1.0"

from .attention import TemperatureFunction, TMLinKernelAttn, fa_kla, fa_kla_decode, fa_kla_host  # noqa: F401,E402
from .backend import fa_kla_attention  # noqa: F401,E402
from .kernels import FeatureMap, LearnablePositiveMap  # noqa: F401,E402
