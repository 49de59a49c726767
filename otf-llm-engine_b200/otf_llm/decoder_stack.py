"""Llama-shaped 2-bit decoder linear stack: one decode token through every projection.

This is the workload the reference's runner drives per generated token
(otf_llm/run_symmetric_2bit.py:150-187 injects one SymmetricOTF2BitLinear per
q/k/v/o/gate/up/down projection of every layer; HF's LlamaDecoderLayer calls them).
Attention is a single-position pass-through (softmax over one key returns V), so a
token's step is, per layer:

    x = rmsnorm(h); q, k, v = Wq x, Wk x, Wv x; h = h + Wo v
    x = rmsnorm(h); h = h + Wd (silu(Wg x) * Wu x)

The residual adds are fused into the o/down kernels' epilogue, RMSNorm and the SiLU
gate are small native kernels, and a whole step can be captured as one CUDA graph.
Tensor-parallel ranks hold column shards of q/k/v/gate/up and row shards of o/down
(anchor columns split by shard and re-based), with one all-reduce after o and down.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, List, Optional

import torch
import torch.nn as nn

from . import _native
from .symmetric_2bit_engine import Symmetric2BitQuantizer, SymmetricOTF2BitLinear

PROJECTIONS = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


@dataclass
class StackConfig:
    layers: int = 32
    hidden: int = 4096
    intermediate: int = 11008
    heads: int = 32
    kv_heads: int = 32
    head_dim: int = 128
    group_size: int = 64
    outlier_ratio: float = 0.005
    weight_std: float = 0.02
    rms_eps: float = 1e-5

    def shapes(self) -> Dict[str, tuple]:
        """(out_features N, in_features K) per projection."""
        h, i = self.hidden, self.intermediate
        q, kv = self.heads * self.head_dim, self.kv_heads * self.head_dim
        return {"q_proj": (q, h), "k_proj": (kv, h), "v_proj": (kv, h), "o_proj": (h, q),
                "gate_proj": (i, h), "up_proj": (i, h), "down_proj": (h, i)}


LLAMA2_7B = StackConfig()


def linear_bytes(N: int, K: int, G: int, n_out: int, batch: int = 1) -> int:
    """Algorithmic bytes of one 2-bit linear: codes + scales + anchors (+ indices) + x + y."""
    return N * K // 4 + N * (K // G) * 2 + N * n_out * 2 + n_out * 8 + batch * K * 2 + batch * N * 2


def activation_profile(K: int, gen: torch.Generator, device) -> torch.Tensor:
    """|N(0,1)| per input channel with 1% of the channels (at least one) scaled by 20."""
    p = torch.randn(K, generator=gen, device=device).abs()
    hot = torch.randperm(K, generator=gen, device=device)[: max(1, K // 100)]
    p[hot] *= 20.0
    return p


def random_quantized_linear(N: int, K: int, cfg: StackConfig, seed: int, device) -> SymmetricOTF2BitLinear:
    """W ~ N(0, std^2) from a per-layer seed, quantised with the layer's own scheme."""
    gen = torch.Generator(device=device).manual_seed(seed)
    W = torch.randn(N, K, generator=gen, device=device) * cfg.weight_std
    act = activation_profile(K, gen, device)
    q = Symmetric2BitQuantizer(group_size=cfg.group_size, outlier_ratio=cfg.outlier_ratio)
    packed, scales, ov, oi = q.quantize_tensor(W, act)
    return SymmetricOTF2BitLinear(packed, scales, K, cfg.group_size, ov, oi)


def shard_linear(lay: SymmetricOTF2BitLinear, rank: int, world: int, dim: str) -> SymmetricOTF2BitLinear:
    """Column (dim='out') or row (dim='in') shard of a 2-bit layer for tensor parallelism.

    Row shards cut K at group boundaries; the anchor columns falling inside a shard keep
    their values and are re-based to shard-local indices (a shard may have none).
    """
    N, K, G = lay.out_features, lay.d_in, lay.group_size
    if dim == "out":
        if N % world:
            raise ValueError(f"out_features {N} not divisible by {world}")
        n0, n1 = rank * N // world, (rank + 1) * N // world
        ov = lay.outliers_fp16[n0:n1] if lay.has_outliers else None
        oi = lay.outlier_indices if lay.has_outliers else None
        return SymmetricOTF2BitLinear(lay.packed_uint8[n0:n1].contiguous(), lay.scales[n0:n1].contiguous(), K, G,
                                      None if ov is None else ov.contiguous(), oi)
    if K % (world * G):
        raise ValueError(f"in_features {K} not divisible into {world} shards of whole groups of {G}")
    k0, k1 = rank * K // world, (rank + 1) * K // world
    packed = lay.packed_uint8[:, k0 // 4:k1 // 4].contiguous()
    scales = lay.scales[:, k0 // G:k1 // G].contiguous()
    ov = oi = None
    if lay.has_outliers:
        sel = (lay.outlier_indices >= k0) & (lay.outlier_indices < k1)
        if bool(sel.any()):
            oi = (lay.outlier_indices[sel] - k0).contiguous()
            ov = lay.outliers_fp16[:, sel].contiguous()
    return SymmetricOTF2BitLinear(packed, scales, k1 - k0, G, ov, oi)


class Llama2BitLinearStack(nn.Module):
    """Random-init, 2-bit quantized decoder linear stack (batch-1 decode step)."""

    def __init__(self, cfg: StackConfig = LLAMA2_7B, device="cuda", seed: int = 0, rank: int = 0, world: int = 1,
                 process_group=None, fused: bool = True):
        super().__init__()
        self.cfg = cfg
        self.fused = fused
        self.rank, self.world, self.pg = rank, world, process_group
        dev = torch.device(device)
        shapes = cfg.shapes()
        self.layers = nn.ModuleList()
        for li in range(cfg.layers):
            mods = {}
            for pi, name in enumerate(PROJECTIONS):
                N, K = shapes[name]
                full = random_quantized_linear(N, K, cfg, seed * 100003 + li * 7 + pi, dev)
                if world > 1:
                    full = shard_linear(full, rank, world, "in" if name in ("o_proj", "down_proj") else "out")
                mods[name] = full
            self.layers.append(nn.ModuleDict(mods))
            torch.cuda.synchronize(dev)
        h = cfg.hidden
        self.norm_w = torch.ones(h, dtype=torch.float16, device=dev)
        sh = {n: (m.out_features, m.d_in) for n, m in self.layers[0].items()}
        self._buf = {
            "xn": torch.empty(1, h, dtype=torch.float16, device=dev),
            "q": torch.empty(1, sh["q_proj"][0], dtype=torch.float16, device=dev),
            "k": torch.empty(1, sh["k_proj"][0], dtype=torch.float16, device=dev),
            "v": torch.empty(1, sh["v_proj"][0], dtype=torch.float16, device=dev),
            "attn": torch.empty(1, sh["o_proj"][1], dtype=torch.float16, device=dev),
            "g": torch.empty(1, sh["gate_proj"][0], dtype=torch.float16, device=dev),
            "u": torch.empty(1, sh["up_proj"][0], dtype=torch.float16, device=dev),
            "a": torch.empty(1, sh["gate_proj"][0], dtype=torch.float16, device=dev),
            "h1": torch.empty(1, h, dtype=torch.float16, device=dev),
            "h2": torch.empty(1, h, dtype=torch.float16, device=dev),
        }

    # -- accounting -----------------------------------------------------------------
    def bytes_per_token(self) -> int:
        """Algorithmic bytes this rank's linears read/write for one token."""
        total = 0
        for layer in self.layers:
            for m in layer.values():
                n_out = m.outlier_indices.numel() if m.has_outliers else 0
                total += linear_bytes(m.out_features, m.d_in, m.group_size, n_out)
        return total

    def linear_bytes_list(self) -> List[int]:
        return [linear_bytes(m.out_features, m.d_in, m.group_size,
                             m.outlier_indices.numel() if m.has_outliers else 0)
                for layer in self.layers for m in layer.values()]

    def launches_per_token(self) -> int:
        return (4 if self.fused else 10) * len(self.layers)

    # -- forward ----------------------------------------------------------------------
    def _lin(self, m: SymmetricOTF2BitLinear, x: torch.Tensor, out: torch.Tensor,
             residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        return _native.linear_2bit(
            x, m.packed_uint8, m.scales, m.group_size, m.codebook,
            mask=m.outlier_mask_vector if m.has_outliers else None,
            outlier_idx=m.outlier_indices if m.has_outliers else None,
            outlier_vals=m.outliers_fp16 if m.has_outliers else None,
            residual=residual, clamp=True, out=out)

    def _attn_passthrough(self, v: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        rep = cfg.heads // cfg.kv_heads
        if rep == 1:
            return v
        hd = cfg.head_dim
        out.view(-1, rep, hd).copy_(v.view(-1, 1, hd).expand(-1, rep, hd))
        return out

    def _forward_fused(self, h: torch.Tensor) -> torch.Tensor:
        """Four launches per layer: [rmsnorm + q/k/v], [o + residual], [rmsnorm + gate/up],
        [silu gate + down + residual] (the norms and the gate run inside the GEMV prologue)."""
        b = self._buf
        cfg = self.cfg
        tp = self.world > 1
        G = _native.GroupItem
        cur = h
        for layer in self.layers:
            _native.linear_group([G(layer[n], cur, b[o], x_op=_native.OTF_XOP_RMSNORM, x_aux=self.norm_w,
                                    eps=cfg.rms_eps) for n, o in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"))])
            attn = self._attn_passthrough(b["v"], b["attn"])
            _native.linear_group([G(layer["o_proj"], attn, b["h1"], residual=None if (tp and self.rank) else cur)])
            if tp:
                torch.distributed.all_reduce(b["h1"], group=self.pg)
            _native.linear_group([G(layer[n], b["h1"], b[o], x_op=_native.OTF_XOP_RMSNORM, x_aux=self.norm_w,
                                    eps=cfg.rms_eps) for n, o in (("gate_proj", "g"), ("up_proj", "u"))])
            _native.linear_group([G(layer["down_proj"], b["g"], b["h2"], residual=None if (tp and self.rank) else b["h1"],
                                    x_op=_native.OTF_XOP_SILU_MUL, x_aux=b["u"])])
            if tp:
                torch.distributed.all_reduce(b["h2"], group=self.pg)
            cur = b["h2"]
        return cur

    def forward(self, h: torch.Tensor, linears_only: bool = False, collectives: bool = True) -> torch.Tensor:
        """One decode step for h [1, hidden] fp16; returns the new residual stream.

        linears_only drops RMSNorm and SiLU (the 2-bit projections alone, for the roofline);
        collectives=False also drops the tensor-parallel all-reduces (per-rank kernel time)."""
        if self.fused and not linears_only:
            return self._forward_fused(h)
        b = self._buf
        cur = h
        for li, layer in enumerate(self.layers):
            xn = cur if linears_only else _native.rmsnorm(cur, self.norm_w, self.cfg.rms_eps, out=b["xn"])
            self._lin(layer["q_proj"], xn, b["q"])
            self._lin(layer["k_proj"], xn, b["k"])
            v = self._lin(layer["v_proj"], xn, b["v"])
            attn = self._attn_passthrough(v, b["attn"])
            tp = self.world > 1
            h1 = self._lin(layer["o_proj"], attn, b["h1"], residual=None if (tp and self.rank) else cur)
            if tp and collectives:
                torch.distributed.all_reduce(h1, group=self.pg)
            xn = h1 if linears_only else _native.rmsnorm(h1, self.norm_w, self.cfg.rms_eps, out=b["xn"])
            g = self._lin(layer["gate_proj"], xn, b["g"])
            u = self._lin(layer["up_proj"], xn, b["u"])
            a = g if linears_only else _native.silu_mul(g, u, out=b["a"])
            h2 = self._lin(layer["down_proj"], a, b["h2"], residual=None if (tp and self.rank) else h1)
            if tp and collectives:
                torch.distributed.all_reduce(h2, group=self.pg)
            cur = h2
        return cur


class DecodeGraph:
    """One decode step of a stack captured as a CUDA graph with static input/output."""

    def __init__(self, stack: Llama2BitLinearStack, linears_only: bool = False, collectives: bool = True):
        dev = stack.norm_w.device
        self.stack = stack
        self.x = torch.zeros(1, stack.cfg.hidden, dtype=torch.float16, device=dev)
        self.y = torch.zeros_like(self.x)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.y.copy_(stack(self.x, linears_only, collectives))
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.y.copy_(stack(self.x, linears_only, collectives))
        torch.cuda.synchronize(dev)

    def replay(self) -> None:
        self.graph.replay()

    def step_host(self, x_host: torch.Tensor, y_host: torch.Tensor) -> None:
        """Host -> device input, one graph replay, device -> host output (all async)."""
        self.x.copy_(x_host, non_blocking=True)
        self.graph.replay()
        y_host.copy_(self.y, non_blocking=True)
