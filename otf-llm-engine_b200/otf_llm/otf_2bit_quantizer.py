"""Asymmetric 2-bit surface: OTF2BitQuantizer and OTF2BitLinear.

Mirrors ``otf_llm/otf_2bit_quantizer.py`` of the reference (same names, buffers and
arguments).  The layer's forward runs the fused sm_100a kernel with the zero point
applied, i.e. it computes exactly the dequantisation of ``unpack_2bit_uint8``
(w = scale * codebook[q] + zero, reference :46-71).  The reference's own forward
routed through a function that dropped ``zeros`` (otf_llm/otf_triton_2bit_kernel.py:
197-212); this package does not reproduce that defect.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import _native

# Reference constant (otf_llm/otf_2bit_quantizer.py:18), held in fp32 by this surface.
LLOYD_MAX_2BIT_CENTROIDS = [-1.52, -0.45, 0.45, 1.52]


class OTF2BitQuantizer:
    """Group quantizer with per-group scale and zero point (reference :22-141).

    Same algorithm as the reference, but it follows W's device instead of
    requiring CUDA.  Outliers: top-k columns by ||W[:, c]|| * act[c], kept in fp16.
    Groups: zero = mean, scale = rms(W - mean) / 0.95, then five rounds of nearest
    centroid on (W - zero) / scale and the closed-form regression of W on c_q.
    """

    def __init__(self, group_size: int = 32, outlier_ratio: float = 0.035):
        self.group_size = group_size
        self.outlier_ratio = outlier_ratio
        self.codebook = torch.tensor(LLOYD_MAX_2BIT_CENTROIDS, dtype=torch.float32)

    @torch.no_grad()
    def pack_2bit_uint8(self, q_indices: torch.Tensor) -> torch.Tensor:
        if q_indices.shape[1] % 4:
            raise ValueError("d_in must be divisible by 4 for 2-bit packing")
        q = q_indices.to(torch.uint8)
        rows, cols = q.shape
        quads = q.reshape(rows, cols // 4, 4)
        return quads[..., 0] | (quads[..., 1] << 2) | (quads[..., 2] << 4) | (quads[..., 3] << 6)

    @torch.no_grad()
    def unpack_2bit_uint8(self, packed: torch.Tensor, scales: torch.Tensor, zeros: torch.Tensor,
                          d_in: int) -> torch.Tensor:
        """fp16 [N, d_in] weights: scale * codebook[q] + zero in fp32, then fp16."""
        rows = packed.shape[0]
        cb = self.codebook.to(packed.device)
        shifts = torch.tensor([0, 2, 4, 6], dtype=torch.uint8, device=packed.device)
        q = ((packed.unsqueeze(-1) >> shifts) & 3).reshape(rows, d_in).to(torch.long)
        w = cb[q].view(rows, -1, self.group_size) * scales.unsqueeze(-1) + zeros.unsqueeze(-1)
        return w.view(rows, d_in).to(torch.float16)

    @torch.no_grad()
    def quantize_tensor(self, W: torch.Tensor, activation_profile: Optional[torch.Tensor] = None):
        dev = W.device
        Wf = W.detach().to(torch.float32)
        d_out, d_in = Wf.shape
        cb = self.codebook.to(dev)
        outliers_fp16 = outlier_indices = None
        if self.outlier_ratio > 0.0:
            impact = torch.norm(Wf, dim=0)
            if activation_profile is not None:
                impact = impact * activation_profile.detach().to(device=dev, dtype=torch.float32)
            k = max(1, int(d_in * self.outlier_ratio))
            outlier_indices = torch.topk(impact, k=k).indices
            outliers_fp16 = Wf[:, outlier_indices].to(torch.float16)
            Wf = Wf.clone()
            Wf[:, outlier_indices] = 0.0
        w = Wf.view(d_out, d_in // self.group_size, self.group_size)
        zeros = w.mean(dim=-1)
        scales = torch.sqrt(((w - zeros.unsqueeze(-1)) ** 2).mean(dim=-1) + 1e-8) / 0.95
        codes = None
        for _ in range(5):
            z = (w - zeros.unsqueeze(-1)) / scales.clamp(min=1e-8).unsqueeze(-1)
            codes = (z.unsqueeze(-1) - cb).abs().argmin(dim=-1)
            cq = cb[codes]
            cq_mean = cq.mean(dim=-1, keepdim=True)
            w_mean = w.mean(dim=-1, keepdim=True)
            dc = cq - cq_mean
            scales = ((dc * (w - w_mean)).sum(dim=-1) / (dc * dc).sum(dim=-1).clamp(min=1e-8)).clamp(min=1e-8)
            zeros = (w_mean - scales.unsqueeze(-1) * cq_mean).squeeze(-1)
        packed = self.pack_2bit_uint8(codes.view(d_out, d_in))
        return packed, scales.to(torch.float16), zeros.to(torch.float16), outliers_fp16, outlier_indices


class OTF2BitLinear(nn.Module):
    """Asymmetric 2-bit linear layer (reference :144-221); forward is one fused kernel."""

    def __init__(
        self,
        packed_uint8: torch.Tensor,
        scales: torch.Tensor,
        zeros: torch.Tensor,
        d_in: int,
        group_size: int = 32,
        outliers_fp16: Optional[torch.Tensor] = None,
        outlier_indices: Optional[torch.Tensor] = None,
        bias: Optional[torch.Tensor] = None,
    ):
        super().__init__()
        self.d_in = d_in
        self.group_size = group_size
        self.quantizer = OTF2BitQuantizer(group_size=group_size)
        self.register_buffer("packed_uint8", packed_uint8)
        self.register_buffer("scales", scales)
        self.register_buffer("zeros", zeros)
        self.register_buffer("codebook", torch.tensor(LLOYD_MAX_2BIT_CENTROIDS, dtype=torch.float32))
        if bias is not None:
            self.register_buffer("bias", bias.to(dtype=torch.float16))
            self.has_bias = True
        else:
            self.bias = None
            self.has_bias = False
        if outliers_fp16 is not None and outlier_indices is not None:
            idx = outlier_indices.to(dtype=torch.long)
            if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= d_in):
                raise ValueError("outlier_indices must lie in [0, d_in)")
            self.register_buffer("outliers_fp16", outliers_fp16.to(dtype=torch.float16))
            self.register_buffer("outlier_indices", idx)
            # on the packed codes' device (the reference builds it on the CPU), so a module made
            # from CUDA tensors runs without a .to()
            keep = torch.ones(d_in, dtype=torch.float16, device=packed_uint8.device)
            keep[idx.to(keep.device)] = 0.0
            self.register_buffer("outlier_mask_vector", keep)
            self.has_outliers = True
        else:
            self.outliers_fp16 = None
            self.outlier_indices = None
            self.outlier_mask_vector = None
            self.has_outliers = False

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig_dtype = x.dtype
        orig_shape = x.shape
        x2d = x.reshape(-1, orig_shape[-1]).to(torch.float16).contiguous()
        y = _native.linear_2bit(
            x2d, self.packed_uint8.contiguous(), self.scales.to(torch.float16).contiguous(), self.group_size,
            self.codebook, zeros=self.zeros.to(torch.float16).contiguous(),
            mask=self.outlier_mask_vector if self.has_outliers else None,
            outlier_idx=self.outlier_indices if self.has_outliers else None,
            outlier_vals=self.outliers_fp16.contiguous() if self.has_outliers else None,
            bias=self.bias if self.has_bias else None, clamp=False)
        y = y.view(*orig_shape[:-1], self.packed_uint8.shape[0])
        return y if y.dtype == orig_dtype else y.to(orig_dtype)
