"""Symmetric zero-free 2-bit layers and the INT8 shared-vocabulary embedding/head.

Same classes, constructor arguments, buffer names, dtypes and shapes as the
reference module ``otf_llm/symmetric_2bit_engine.py`` (GT-Labs-AI/otf-llm-engine),
so checkpoints, ``state_dict`` round trips and runner injection code carry over.
The forwards run one fused sm_100a kernel each; the offline quantizers are plain
torch code that follows the tensor's device.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from . import _native

# Same constant as the reference (otf_llm/symmetric_2bit_engine.py:14): the layer
# format stores codes against these four centroids.
LLOYD_MAX_SYMMETRIC_CENTROIDS = [-1.52, -0.45, 0.45, 1.52]


def _rowwise_int8(fp16_weight: torch.Tensor, chunk_size: int) -> Tuple[torch.Tensor, torch.Tensor]:
    """Row absmax/127 INT8 quantisation (otf_llm/symmetric_2bit_engine.py:26-39).

    scale = max(|w|max / 127, 1e-8) in fp32, q = clamp(round_half_even(w / scale), +-127),
    stored scale = fp16(scale).  Processed in row chunks to bound temporary memory.
    """
    rows, cols = fp16_weight.shape
    q = torch.empty((rows, cols), dtype=torch.int8, device="cpu")
    s = torch.empty((rows, 1), dtype=torch.float16, device="cpu")
    for lo in range(0, rows, chunk_size):
        hi = min(lo + chunk_size, rows)
        blk = fp16_weight[lo:hi].to(torch.float32)
        step = blk.abs().amax(dim=1, keepdim=True).div(127.0).clamp_min(1e-8)
        q[lo:hi] = blk.div(step).round().clamp(-127, 127).to(torch.int8).cpu()
        s[lo:hi] = step.to(torch.float16).cpu()
    return q, s


class QuantizedEmbedding(nn.Module):
    """INT8 token embedding with one fp16 scale per row (reference :17-47)."""

    def __init__(self, num_embeddings: int, embedding_dim: int):
        super().__init__()
        self.num_embeddings = num_embeddings
        self.embedding_dim = embedding_dim
        self.register_buffer("weight_int8", torch.zeros((num_embeddings, embedding_dim), dtype=torch.int8))
        self.register_buffer("scales", torch.ones((num_embeddings, 1), dtype=torch.float16))

    @torch.no_grad()
    def quantize_from_fp16(self, fp16_weight: torch.Tensor, chunk_size: int = 8192):
        self.weight_int8, self.scales = _rowwise_int8(fp16_weight, chunk_size)

    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        dev = input_ids.device
        w = self.weight_int8 if self.weight_int8.device == dev else self.weight_int8.to(dev)
        s = self.scales if self.scales.device == dev else self.scales.to(dev)
        # Ids outside [0, V) raise, as F.embedding does (reference :44).  The kernel flags them
        # on the device; reading the flag needs a host sync, which a CUDA graph capture cannot
        # take, so a captured call writes zero rows for them instead.
        capturing = torch.cuda.is_current_stream_capturing()
        flag = None if capturing else torch.zeros(1, dtype=torch.int32, device=dev)
        rows = _native.i8_embed(input_ids, w.contiguous(), s.contiguous(), flag)
        if flag is not None and int(flag.item()):
            raise IndexError("index out of range in self")
        return rows.view(*input_ids.shape, self.embedding_dim)


class QuantizedLinearHead(nn.Module):
    """INT8 LM head returning fp32 logits (reference :50-91).

    The weight may be the embedding's own buffer (tied head: the runner assigns
    ``head.weight_int8 = emb.weight_int8``); the kernel reads it in place.
    """

    def __init__(self, in_features: int, out_features: int):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("weight_int8", torch.zeros((out_features, in_features), dtype=torch.int8))
        self.register_buffer("scales", torch.ones((out_features, 1), dtype=torch.float16))

    @torch.no_grad()
    def quantize_from_fp16(self, fp16_weight: torch.Tensor, chunk_size: int = 8192):
        self.weight_int8, self.scales = _rowwise_int8(fp16_weight, chunk_size)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig_shape = x.shape
        x2d = x.reshape(-1, orig_shape[-1]).to(torch.float16).contiguous()
        logits = _native.i8_head(x2d, self.weight_int8, self.scales)
        return logits.view(*orig_shape[:-1], self.out_features)


class Symmetric2BitQuantizer:
    """Offline profile-guided symmetric 2-bit quantizer (reference :94-169).

    Produces the layer format: packed codes uint8 [N, K/4], fp16 group scales
    [N, K/G], fp16 outlier columns [N, k] and their int64 indices [k].  Steps:
    column impact ||W[:, c]||_2 * act[c] -> top-k outlier columns (k = max(1,
    int(K * ratio))) kept exactly in fp16 and zeroed in W; per group a masked RMS
    start s = rms / 0.95, then five rounds of nearest-centroid assignment and the
    closed-form least-squares scale s = <W, c_q> / <c_q, c_q>.  Rows are processed
    in chunks so the [rows, groups, G, 4] distance tensor stays bounded.
    """

    def __init__(self, group_size: int = 32, outlier_ratio: float = 0.035):
        self.group_size = group_size
        self.outlier_ratio = outlier_ratio
        self.codebook = torch.tensor(LLOYD_MAX_SYMMETRIC_CENTROIDS, dtype=torch.float32)

    @torch.no_grad()
    def pack_2bit_uint8(self, q_indices: torch.Tensor) -> torch.Tensor:
        """Four codes per byte, code k at bits 2*(k%4) of byte k/4 (reference :100-107)."""
        q = q_indices.to(torch.uint8)
        rows, cols = q.shape
        quads = q.reshape(rows, cols // 4, 4)
        return (quads[..., 0] | (quads[..., 1] << 2) | (quads[..., 2] << 4) | (quads[..., 3] << 6)).contiguous()

    @torch.no_grad()
    def _fit_groups(self, w: torch.Tensor, keep: torch.Tensor, cb: torch.Tensor):
        """Nearest-centroid codes and least-squares scales for a row chunk; w: [r, g, G] fp32."""
        keep_f = keep.to(torch.float32)
        n_active = keep_f.sum(dim=-1).clamp(min=1.0)
        s = torch.sqrt((w * w).sum(dim=-1) / n_active + 1e-8).div(0.95).clamp(min=1e-8)
        codes = None
        for _ in range(5):
            z = w / s.clamp(min=1e-8).unsqueeze(-1)
            codes = (z.unsqueeze(-1) - cb).abs().argmin(dim=-1)
            cq = cb[codes] * keep_f
            num = (w * cq).sum(dim=-1)
            den = (cq * cq).sum(dim=-1)
            s = (num / den.clamp(min=1e-8)).clamp(min=1e-8)
        return codes, s

    @torch.no_grad()
    def quantize_tensor(self, W: torch.Tensor, activation_profile: Optional[torch.Tensor] = None,
                        row_chunk: int = 2048):
        """Quantise W on its device.  CUDA tensors go through one native launch sequence
        (otf2b_quantize: column impact, anchor ranking, anchor gather, group fit; no [N, K/G, G, 4]
        temporaries); CPU tensors run the reference's torch ops, row-chunked."""
        if W.is_cuda:
            from . import _native
            k = max(1, int(W.shape[1] * self.outlier_ratio)) if self.outlier_ratio > 0.0 else 0
            return _native.quantize_2b(W.detach(), self.group_size, k, activation_profile,
                                       [float(v) for v in self.codebook.tolist()])
        dev = W.device
        Wf = W.detach().to(torch.float32)
        d_out, d_in = Wf.shape
        G = self.group_size
        if d_in % G or d_in % 4:
            raise ValueError(f"d_in={d_in} must be a multiple of group_size={G} and of 4")
        cb = self.codebook.to(dev)
        keep = torch.ones((1, d_in), dtype=torch.bool, device=dev)
        outliers_fp16 = outlier_indices = None
        if self.outlier_ratio > 0.0:
            impact = torch.norm(Wf, dim=0)
            if activation_profile is not None:
                impact = impact * activation_profile.detach().to(device=dev, dtype=torch.float32)
            k = max(1, int(d_in * self.outlier_ratio))
            outlier_indices = torch.topk(impact, k=k).indices
            outliers_fp16 = Wf[:, outlier_indices].to(torch.float16).contiguous()
            Wf = Wf.clone()
            Wf[:, outlier_indices] = 0.0
            keep[:, outlier_indices] = False
        ng = d_in // G
        keep_g = keep.view(1, ng, G)
        packed = torch.empty((d_out, d_in // 4), dtype=torch.uint8, device=dev)
        scales = torch.empty((d_out, ng), dtype=torch.float16, device=dev)
        for lo in range(0, d_out, row_chunk):
            hi = min(lo + row_chunk, d_out)
            w = Wf[lo:hi].view(hi - lo, ng, G)
            codes, s = self._fit_groups(w, keep_g.expand(hi - lo, -1, -1), cb)
            packed[lo:hi] = self.pack_2bit_uint8(codes.view(hi - lo, d_in))
            scales[lo:hi] = s.to(torch.float16)
        return packed, scales, outliers_fp16, outlier_indices


class SymmetricOTF2BitLinear(nn.Module):
    """Drop-in 2-bit linear layer (reference :172-235); forward is one fused kernel.

    y = clamp(GEMV(x * outlier_mask) + bias + x[..., outlier_indices] @ outliers_fp16.T)
    with fp32 accumulation, returned in x's dtype.
    """

    def __init__(
        self,
        packed_uint8: torch.Tensor,
        scales: torch.Tensor,
        d_in: int,
        group_size: int = 32,
        outliers_fp16: Optional[torch.Tensor] = None,
        outlier_indices: Optional[torch.Tensor] = None,
        bias: Optional[torch.Tensor] = None,
    ):
        super().__init__()
        if packed_uint8.shape[1] * 4 != d_in:
            raise ValueError(f"packed_uint8 has {packed_uint8.shape[1]} bytes per row; d_in={d_in} needs {d_in // 4}")
        if d_in % group_size:
            raise ValueError(f"d_in={d_in} is not a multiple of group_size={group_size}")
        self.d_in = d_in
        self.group_size = group_size
        self.out_features = packed_uint8.shape[0]
        dev = packed_uint8.device
        self.register_buffer("packed_uint8", packed_uint8.contiguous())
        self.register_buffer("scales", scales.to(device=dev, dtype=torch.float16).contiguous())
        self.register_buffer("codebook", torch.tensor(LLOYD_MAX_SYMMETRIC_CENTROIDS, dtype=torch.float16, device=dev))
        if bias is not None:
            self.register_buffer("bias", bias.to(device=dev, dtype=torch.float16).contiguous())
            self.has_bias = True
        else:
            self.bias = None
            self.has_bias = False
        if outliers_fp16 is not None and outlier_indices is not None:
            idx = outlier_indices.to(device=dev, dtype=torch.long)
            if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= d_in):
                raise ValueError("outlier_indices must lie in [0, d_in)")
            self.register_buffer("outliers_fp16", outliers_fp16.to(device=dev, dtype=torch.float16).contiguous())
            self.register_buffer("outlier_indices", idx)
            keep = torch.ones(d_in, dtype=torch.float16, device=dev)
            keep[idx] = 0.0
            self.register_buffer("outlier_mask_vector", keep.contiguous())
            self.has_outliers = True
        else:
            self.outliers_fp16 = None
            self.outlier_indices = None
            self.outlier_mask_vector = None
            self.has_outliers = False

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        orig_shape = x.shape
        x2d = x.reshape(-1, orig_shape[-1]).to(torch.float16).contiguous()
        y = _native.linear_2bit(
            x2d, self.packed_uint8, self.scales, self.group_size, self.codebook,
            mask=self.outlier_mask_vector if self.has_outliers else None,
            outlier_idx=self.outlier_indices if self.has_outliers else None,
            outlier_vals=self.outliers_fp16 if self.has_outliers else None,
            bias=self.bias if self.has_bias else None, clamp=True)
        return y.view(*orig_shape[:-1], self.out_features).to(x.dtype)
