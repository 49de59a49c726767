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
from typing import Dict, List, Optional, Tuple

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
    return even_scale_rows(SymmetricOTF2BitLinear(packed, scales, K, cfg.group_size, ov, oi))


def split_bounds(n: int, rank: int, world: int, align: int = 1):
    """[lo, hi) of rank's part of n items cut at multiples of align, as evenly as the
    alignment allows (parts differ by at most one align-block)."""
    if n % align:
        raise ValueError(f"{n} is not a multiple of {align}")
    units = n // align
    if units < world:
        raise ValueError(f"{n} items in blocks of {align} cannot be split over {world} ranks")
    return rank * units // world * align, (rank + 1) * units // world * align


def even_scale_rows(m: SymmetricOTF2BitLinear) -> SymmetricOTF2BitLinear:
    """Give the scale rows a 16-byte row stride (a multiple of 8 groups; padding columns are
    zero), so the GEMV kernels can copy scales in 4-byte pieces and the decode-step kernel
    in 16-byte TMA boxes.  The buffer keeps its [N, K/G] shape; only its storage grows."""
    N, ng = m.scales.shape
    if m.scales.stride(0) % 8:
        padded = torch.zeros(N, (ng + 7) // 8 * 8, dtype=m.scales.dtype, device=m.scales.device)
        padded[:, :ng] = m.scales
        m.scales = padded[:, :ng]
    return m


def shard_linear(lay: SymmetricOTF2BitLinear, rank: int, world: int, dim: str, align: int = 1) -> SymmetricOTF2BitLinear:
    """Column (dim='out') or row (dim='in') shard of a 2-bit layer for tensor parallelism.

    Row shards cut K at group boundaries (balanced over ranks when the group count does
    not divide evenly); the anchor columns falling inside a shard keep their values and are
    re-based to shard-local indices (a shard may have none); a bias stays on rank 0 (it is
    added once, before the partial sums are reduced).  Column shards cut N at multiples of
    ``align`` -- the consuming row-parallel layer's group size for gate/up, so that each
    rank's slice of the intermediate activation is exactly its down_proj's K slice; the
    head size for q/k/v.
    """
    N, K, G = lay.out_features, lay.d_in, lay.group_size
    if dim == "out":
        n0, n1 = split_bounds(N, rank, world, align)
        ov = lay.outliers_fp16[n0:n1] if lay.has_outliers else None
        oi = lay.outlier_indices if lay.has_outliers else None
        bias = lay.bias[n0:n1].contiguous() if lay.has_bias else None
        return SymmetricOTF2BitLinear(lay.packed_uint8[n0:n1].contiguous(), lay.scales[n0:n1].contiguous(), K, G,
                                      None if ov is None else ov.contiguous(), oi, bias)
    k0, k1 = split_bounds(K, rank, world, G)
    packed = lay.packed_uint8[:, k0 // 4:k1 // 4].contiguous()
    scales = lay.scales[:, k0 // G:k1 // G].contiguous()
    ov = oi = None
    if lay.has_outliers:
        sel = (lay.outlier_indices >= k0) & (lay.outlier_indices < k1)
        if bool(sel.any()):
            oi = (lay.outlier_indices[sel] - k0).contiguous()
            ov = lay.outliers_fp16[:, sel].contiguous()
    bias = lay.bias if (lay.has_bias and rank == 0) else None
    return even_scale_rows(SymmetricOTF2BitLinear(packed, scales, k1 - k0, G, ov, oi, bias))


class Llama2BitLinearStack(nn.Module):
    """Random-init, 2-bit quantized decoder linear stack (batch-1 decode step)."""

    def __init__(self, cfg: StackConfig = LLAMA2_7B, device="cuda", seed: int = 0, rank: int = 0, world: int = 1,
                 process_group=None, fused: bool = True,
                 layers: Optional[List[Dict[str, SymmetricOTF2BitLinear]]] = None,
                 norms: Optional[List[Tuple[torch.Tensor, torch.Tensor]]] = None, peer_ar=None,
                 persistent: bool = False):
        """Random-init layers from ``cfg`` and ``seed``, or the given (already sharded)
        ``layers`` keyed by q_proj ... down_proj with per-layer (input, post-attention)
        RMSNorm weights ``norms`` (default: all ones).  Under tensor parallelism ``peer_ar``
        (otf_llm.tp_allreduce.PeerAllReduce) replaces the NCCL all-reduces of the fused step
        by the exchange fused into the o/down and following grouped launches.  ``persistent``
        runs a whole single-GPU step as one launch (``_native.DecodeStep``) when the shapes
        allow it (else the grouped launches)."""
        super().__init__()
        self.cfg = cfg
        self.fused = fused
        self.rank, self.world, self.pg = rank, world, process_group
        self.peer_ar = peer_ar
        dev = torch.device(device)
        shapes = cfg.shapes()
        self.layers = nn.ModuleList()
        if layers is not None:
            for mods in layers:
                missing = [n for n in PROJECTIONS if n not in mods]
                if missing:
                    raise ValueError(f"decoder layer lacks {missing}")
                self.layers.append(nn.ModuleDict({n: mods[n] for n in PROJECTIONS}))
        else:
            for li in range(cfg.layers):
                mods = {}
                for pi, name in enumerate(PROJECTIONS):
                    N, K = shapes[name]
                    full = random_quantized_linear(N, K, cfg, seed * 100003 + li * 7 + pi, dev)
                    if world > 1:
                        if name in ("o_proj", "down_proj"):
                            full = shard_linear(full, rank, world, "in")
                        else:
                            full = shard_linear(full, rank, world, "out",
                                                cfg.group_size if name in ("gate_proj", "up_proj") else cfg.head_dim)
                    mods[name] = full
                self.layers.append(nn.ModuleDict(mods))
                torch.cuda.synchronize(dev)
        h = cfg.hidden
        self.norm_w = torch.ones(h, dtype=torch.float16, device=dev)
        if norms is None:
            norms = [(self.norm_w, self.norm_w)] * len(self.layers)
        if len(norms) != len(self.layers):
            raise ValueError(f"{len(norms)} norm pairs for {len(self.layers)} layers")
        self.in_norms = [a.to(device=dev, dtype=torch.float16).contiguous() for a, _ in norms]
        self.post_norms = [b.to(device=dev, dtype=torch.float16).contiguous() for _, b in norms]
        # The fused input transforms run only in the tensor-pipe GEMV; a layer outside its
        # layout rules runs the unfused sequence.  Every rank must take the same path (the
        # collectives differ), so the ranks agree on it.
        if self.fused and not all(_native.tensor_pipe_shape_ok(m) for layer in self.layers for m in layer.values()):
            self.fused = False
        self.mk = None
        if world == 1 and persistent and self.fused and dev.type == "cuda":
            try:
                cb = self.layers[0]["q_proj"].codebook
                self.mk = _native.DecodeStep(
                    [dict(layer) for layer in self.layers], list(zip(self.in_norms, self.post_norms)), cfg.hidden,
                    self.layers[0]["gate_proj"].out_features, cfg.heads, cfg.kv_heads, cfg.head_dim,
                    self.layers[0]["q_proj"].group_size, cfg.rms_eps, cb, dev)
            except (ValueError, RuntimeError):
                self.mk = None
        if world > 1 and process_group is not None and torch.distributed.is_initialized():
            flag = torch.tensor([1 if self.fused else 0], dtype=torch.int32,
                                device=dev if torch.distributed.get_backend(process_group) == "nccl" else "cpu")
            torch.distributed.all_reduce(flag, op=torch.distributed.ReduceOp.MIN, group=process_group)
            self.fused = bool(int(flag.item()))
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

    @classmethod
    def from_checkpoint(cls, ck, head_dim: int, rms_eps: float = 1e-5, process_group=None, fused: bool = True,
                        persistent: bool = False, peer_ar=None):
        """The stack of a loaded checkpoint (otf_llm.checkpoint.load_checkpoint), this rank's shard
        when the checkpoint was loaded tensor-parallel.  head_dim comes from the model config."""
        layers = [{p.split(".")[-1]: m for p, m in mods.items()} for mods in ck.layers]
        if not layers:
            raise ValueError("checkpoint has no decoder layers")
        l0, w = layers[0], ck.world
        hidden = l0["q_proj"].d_in
        cfg = StackConfig(layers=len(layers), hidden=hidden, intermediate=l0["gate_proj"].out_features * w,
                          heads=l0["q_proj"].out_features * w // head_dim,
                          kv_heads=l0["k_proj"].out_features * w // head_dim, head_dim=head_dim,
                          group_size=ck.group_size, rms_eps=rms_eps)
        ones = torch.ones(hidden, dtype=torch.float16)
        norms = [(n.get("input_layernorm", ones), n.get("post_attention_layernorm", ones)) for n in ck.layer_norms]
        return cls(cfg, device=l0["q_proj"].packed_uint8.device, rank=ck.rank, world=w, process_group=process_group,
                   fused=fused, layers=layers, norms=norms or None, persistent=persistent, peer_ar=peer_ar)

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
        if self.mk is not None:
            return 1
        n = (4 if self.fused else 10) * len(self.layers)
        return n + (1 if (self.fused and self.world > 1 and self.peer_ar is not None) else 0)

    # -- forward ----------------------------------------------------------------------
    def _lin(self, m: SymmetricOTF2BitLinear, x: torch.Tensor, out: torch.Tensor,
             residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        return _native.linear_2bit(
            x, m.packed_uint8, m.scales, m.group_size, m.codebook,
            mask=m.outlier_mask_vector if m.has_outliers else None,
            outlier_idx=m.outlier_indices if m.has_outliers else None,
            outlier_vals=m.outliers_fp16 if m.has_outliers else None,
            bias=m.bias if m.has_bias else None, residual=residual, clamp=True, out=out)

    def _attn_passthrough(self, v: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        rep = cfg.heads // cfg.kv_heads
        if rep == 1:
            return v
        hd = cfg.head_dim
        out.view(-1, rep, hd).copy_(v.view(-1, 1, hd).expand(-1, rep, hd))
        return out

    def _forward_fused_ar(self, h: torch.Tensor) -> torch.Tensor:
        """The fused step under tensor parallelism with the exchange inside the launches:
        o and down produce their rows into every rank's receive buffer (rank 0 adds the
        residual), and the next grouped launch consumes the sum while staging its input,
        writing the reduced hidden state once for the residual path.  One standalone
        finish ends the step."""
        b = self._buf
        cfg = self.cfg
        ar = self.peer_ar
        G = _native.GroupItem
        PROD, CONS = _native.OTF_AR_PRODUCE, _native.OTF_AR_CONSUME
        lead = self.rank == 0
        cur = h
        pending = None                       # buffer holding the previous down's rows
        for li, layer in enumerate(self.layers):
            if pending is None:
                items = [G(layer[n], cur, b[o], x_op=_native.OTF_XOP_RMSNORM, x_aux=self.in_norms[li], eps=cfg.rms_eps)
                         for n, o in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"))]
            else:
                items = [G(layer[n], b["h2"], b[o], x_op=_native.OTF_XOP_RMSNORM, x_aux=self.in_norms[li],
                           eps=cfg.rms_eps, ar=ar, ar_mode=CONS, ar_buf=pending,
                           ar_out=b["h2"].view(-1) if n == "q_proj" else None)
                         for n, o in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"))]
                cur = b["h2"]
            _native.linear_group(items)
            attn = self._attn_passthrough(b["v"], b["attn"])
            ob = ar.next_buffer()
            _native.linear_group([G(layer["o_proj"], attn, b["h1"], residual=cur if lead else None,
                                    ar=ar, ar_mode=PROD, ar_buf=ob)])
            _native.linear_group([G(layer[n], b["h1"], b[o], x_op=_native.OTF_XOP_RMSNORM, x_aux=self.post_norms[li],
                                    eps=cfg.rms_eps, ar=ar, ar_mode=CONS, ar_buf=ob,
                                    ar_out=b["h1"].view(-1) if n == "gate_proj" else None)
                                  for n, o in (("gate_proj", "g"), ("up_proj", "u"))])
            pending = ar.next_buffer()
            _native.linear_group([G(layer["down_proj"], b["g"], b["h2"], residual=b["h1"] if lead else None,
                                    x_op=_native.OTF_XOP_SILU_MUL, x_aux=b["u"], ar=ar, ar_mode=PROD, ar_buf=pending)])
        if pending is not None:
            ar.finish(b["h2"].view(-1), pending)
            return b["h2"]
        return cur

    def _forward_fused(self, h: torch.Tensor) -> torch.Tensor:
        """Four launches per layer: [rmsnorm + q/k/v], [o + residual], [rmsnorm + gate/up],
        [silu gate + down + residual] (the norms and the gate run inside the GEMV prologue)."""
        if self.world > 1 and self.peer_ar is not None:
            return self._forward_fused_ar(h)
        b = self._buf
        cfg = self.cfg
        tp = self.world > 1
        G = _native.GroupItem
        cur = h
        for li, layer in enumerate(self.layers):
            _native.linear_group([G(layer[n], cur, b[o], x_op=_native.OTF_XOP_RMSNORM, x_aux=self.in_norms[li],
                                    eps=cfg.rms_eps) for n, o in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"))])
            attn = self._attn_passthrough(b["v"], b["attn"])
            _native.linear_group([G(layer["o_proj"], attn, b["h1"], residual=None if (tp and self.rank) else cur)])
            if tp:
                torch.distributed.all_reduce(b["h1"], group=self.pg)
            _native.linear_group([G(layer[n], b["h1"], b[o], x_op=_native.OTF_XOP_RMSNORM, x_aux=self.post_norms[li],
                                    eps=cfg.rms_eps) for n, o in (("gate_proj", "g"), ("up_proj", "u"))])
            _native.linear_group([G(layer["down_proj"], b["g"], b["h2"], residual=None if (tp and self.rank) else b["h1"],
                                    x_op=_native.OTF_XOP_SILU_MUL, x_aux=b["u"])])
            if tp:
                torch.distributed.all_reduce(b["h2"], group=self.pg)
            cur = b["h2"]
        return cur

    def forward(self, h: torch.Tensor) -> torch.Tensor:
        """One decode step for h [1, hidden] fp16; returns the new residual stream."""
        if self.mk is not None:
            return self.mk(h)
        if self.fused:
            return self._forward_fused(h)
        b = self._buf
        cur = h
        for li, layer in enumerate(self.layers):
            xn = _native.rmsnorm(cur, self.in_norms[li], self.cfg.rms_eps, out=b["xn"])
            self._lin(layer["q_proj"], xn, b["q"])
            self._lin(layer["k_proj"], xn, b["k"])
            v = self._lin(layer["v_proj"], xn, b["v"])
            attn = self._attn_passthrough(v, b["attn"])
            tp = self.world > 1
            h1 = self._lin(layer["o_proj"], attn, b["h1"], residual=None if (tp and self.rank) else cur)
            if tp:
                torch.distributed.all_reduce(h1, group=self.pg)
            xn = _native.rmsnorm(h1, self.post_norms[li], self.cfg.rms_eps, out=b["xn"])
            g = self._lin(layer["gate_proj"], xn, b["g"])
            u = self._lin(layer["up_proj"], xn, b["u"])
            a = _native.silu_mul(g, u, out=b["a"])
            h2 = self._lin(layer["down_proj"], a, b["h2"], residual=None if (tp and self.rank) else h1)
            if tp:
                torch.distributed.all_reduce(h2, group=self.pg)
            cur = h2
        return cur


class DecodeGraph:
    """One decode step of a stack captured as a CUDA graph with static input/output."""

    def __init__(self, stack: Llama2BitLinearStack):
        dev = stack.norm_w.device
        self.stack = stack
        self.x = torch.zeros(1, stack.cfg.hidden, dtype=torch.float16, device=dev)
        self.y = torch.zeros_like(self.x)
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            for _ in range(2):
                self.y.copy_(stack(self.x))
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.y.copy_(stack(self.x))
        torch.cuda.synchronize(dev)

    def replay(self) -> None:
        self.graph.replay()

    def step_host(self, x_host: torch.Tensor, y_host: torch.Tensor) -> None:
        """Host -> device input, one graph replay, device -> host output (all async)."""
        self.x.copy_(x_host, non_blocking=True)
        self.graph.replay()
        y_host.copy_(self.y, non_blocking=True)


class CheckpointDecoder:
    """Greedy decode steps through a loaded checkpoint at batch 1: INT8 embedding row ->
    2-bit decoder stack (single-position attention) -> final RMSNorm -> INT8 head argmax.

    Under tensor parallelism the embedding is replicated, the stack all-reduces after o
    and down, and the head is vocabulary-parallel with one (max, index) exchange per step.
    """

    def __init__(self, ck, head_dim: int, rms_eps: float = 1e-5, process_group=None, fused: bool = True,
                 persistent: bool = False, peer_ar=None):
        if ck.embed is None or ck.head is None:
            raise ValueError("checkpoint was loaded without its embedding / head")
        self.ck = ck
        self.stack = Llama2BitLinearStack.from_checkpoint(ck, head_dim, rms_eps, process_group, fused, persistent,
                                                          peer_ar)
        dev = self.stack.norm_w.device
        fn = ck.final_norm if ck.final_norm is not None else self.stack.norm_w
        self.final_norm = fn.to(device=dev, dtype=torch.float16).contiguous()
        self.eps = rms_eps
        self.xn = torch.empty(1, self.stack.cfg.hidden, dtype=torch.float16, device=dev)

    def step(self, ids: torch.Tensor, logits: Optional[torch.Tensor] = None) -> torch.Tensor:
        """ids int64 [1] on the device -> next ids int64 [1]; fills ``logits`` (fp32 [1, V]
        on one device, this rank's [1, V/world] shard under tensor parallelism) when given."""
        h = self.ck.embed(ids.view(1)).view(1, -1)
        h = self.stack(h)
        xn = _native.rmsnorm(h, self.final_norm, self.eps, out=self.xn)
        head = self.ck.head
        if hasattr(head, "shard"):
            return head.argmax(xn, logits=logits)
        return _native.i8_head_argmax(xn, head.weight_int8, head.scales, logits=logits)

    def generate(self, prompt_last: int, steps: int) -> List[int]:
        """``steps`` greedy tokens after ``prompt_last`` (ids stay on the device until the end)."""
        dev = self.final_norm.device
        cur = torch.tensor([prompt_last], dtype=torch.int64, device=dev)
        out = []
        for _ in range(steps):
            cur = self.step(cur)
            out.append(cur)
        return [int(t) for t in torch.cat(out).cpu()] if out else []
