"""otf_llm -- B200-native (sm_100a) drop-in for OTF-LLM's quantized-decode hot path.

The module paths and class/function surfaces mirror the reference package
(GT-Labs-AI/otf-llm-engine, ``otf_llm``) so existing runners keep working:

* ``otf_llm.symmetric_2bit_engine``: SymmetricOTF2BitLinear, Symmetric2BitQuantizer,
  QuantizedEmbedding, QuantizedLinearHead, LLOYD_MAX_SYMMETRIC_CENTROIDS
* ``otf_llm.otf_2bit_quantizer``: OTF2BitQuantizer, OTF2BitLinear
* ``otf_llm.otf_triton_2bit_kernel``: triton_symmetric_2bit_gemm, triton_2bit_gemm

Every forward runs hand-written CUDA kernels from ``_lib/libotfb200.so`` through a C
ABI; there is no CPU, Triton or LUT fallback on that path.
"""
__version__ = "4.1.0+b200.1"

from .otf_2bit_quantizer import OTF2BitLinear, OTF2BitQuantizer  # noqa: F401
from .otf_triton_2bit_kernel import HAS_TRITON, triton_2bit_gemm, triton_symmetric_2bit_gemm  # noqa: F401
from .symmetric_2bit_engine import (  # noqa: F401
    LLOYD_MAX_SYMMETRIC_CENTROIDS,
    QuantizedEmbedding,
    QuantizedLinearHead,
    Symmetric2BitQuantizer,
    SymmetricOTF2BitLinear,
)

__all__ = [
    "OTF2BitQuantizer",
    "OTF2BitLinear",
    "triton_2bit_gemm",
    "triton_symmetric_2bit_gemm",
    "HAS_TRITON",
    "LLOYD_MAX_SYMMETRIC_CENTROIDS",
    "QuantizedEmbedding",
    "QuantizedLinearHead",
    "Symmetric2BitQuantizer",
    "SymmetricOTF2BitLinear",
]
