"""Function surface of the reference's kernel module, backed by the sm_100a library.

Mirrors ``otf_llm/otf_triton_2bit_kernel.py`` of the reference: the same names and
arguments, minus the inline ``load_inline`` JIT, the warp kernel and the 256-entry
LUT fallback, which are all replaced by one fused native call (``otf2b_linear``).

Two deliberate differences, both toward the reference's documented intent:
* ``group_size`` is honoured on every path (the reference's M==1 CUDA kernel
  assumed 32, otf_llm/otf_triton_2bit_kernel.py:49);
* ``triton_2bit_gemm`` applies ``zeros`` and the caller's codebook (the reference
  forwarded neither, :197-212), i.e. it computes the dequantisation of
  ``OTF2BitQuantizer.unpack_2bit_uint8`` (otf_llm/otf_2bit_quantizer.py:46-71).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _native

# The name is kept for callers that test it; it means "the fused decode kernel is
# present", which is always true for this package (no Triton is involved).
HAS_TRITON = True
LLOYD_MAX_SYMMETRIC_CENTROIDS = [-1.52, -0.45, 0.45, 1.52]


def _mask_fp16(outlier_mask: Optional[torch.Tensor], K: int) -> Optional[torch.Tensor]:
    if outlier_mask is None:
        return None
    m = outlier_mask.reshape(-1)
    if m.numel() != K:
        raise ValueError(f"outlier_mask has {m.numel()} entries, expected {K}")
    return m.to(torch.float16).contiguous()


def triton_symmetric_2bit_gemm(
    x: torch.Tensor,
    packed_uint8: torch.Tensor,
    scales: torch.Tensor,
    codebook: Optional[torch.Tensor] = None,
    group_size: int = 32,
    outlier_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """y = clamp((x * outlier_mask) @ dequant(packed, scales).T) as fp16 [..., N].

    Reference: otf_llm/otf_triton_2bit_kernel.py:164-194.  ``codebook`` defaults to the
    fp16 Lloyd-Max constant the reference always used.
    """
    orig_shape = x.shape
    K = packed_uint8.shape[1] * 4
    x2d = x.reshape(-1, orig_shape[-1]).to(torch.float16).contiguous()
    y = _native.linear_2bit(x2d, packed_uint8, scales.to(torch.float16), group_size, codebook,
                            mask=_mask_fp16(outlier_mask, K), clamp=True)
    return y.view(*orig_shape[:-1], packed_uint8.shape[0])


def triton_2bit_gemm(
    x: torch.Tensor,
    packed_uint8: torch.Tensor,
    scales: torch.Tensor,
    zeros: Optional[torch.Tensor] = None,
    codebook: Optional[torch.Tensor] = None,
    group_size: int = 32,
    outlier_mask: Optional[torch.Tensor] = None,
) -> torch.Tensor:
    """Asymmetric surface: w = codebook[q] * scale + zero, then the same fused GEMV.

    Reference signature: otf_llm/otf_triton_2bit_kernel.py:197-212.
    """
    orig_shape = x.shape
    K = packed_uint8.shape[1] * 4
    x2d = x.reshape(-1, orig_shape[-1]).to(torch.float16).contiguous()
    z = None if zeros is None else zeros.to(torch.float16).contiguous()
    y = _native.linear_2bit(x2d, packed_uint8, scales.to(torch.float16).contiguous(), group_size, codebook,
                            zeros=z, mask=_mask_fp16(outlier_mask, K), clamp=True)
    return y.view(*orig_shape[:-1], packed_uint8.shape[0])
