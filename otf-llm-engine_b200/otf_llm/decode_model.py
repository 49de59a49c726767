"""Greedy batch-1 decoding of a whole 2-bit Llama-shaped model on the native kernels.

Per token: INT8 embedding row -> per layer [RMSNorm + q/k/v] -> [RoPE + KV-cache write +
decode attention over the cache] -> [o + residual] -> [RMSNorm + gate/up] -> [SiLU gate +
down + residual] -> final RMSNorm -> INT8 head with fused argmax -> position + 1.  The token
id, the position and the KV caches live in device memory, so one token step is one CUDA
graph replay (prompt tokens are fed by overwriting the id before a replay).

This is what the reference's runner does for one generated token with HF's
LlamaForCausalLM around the injected modules (otf_llm/run_symmetric_2bit.py:150-215):
the projections are SymmetricOTF2BitLinear, the embedding / head QuantizedEmbedding /
QuantizedLinearHead, attention and norms HF's.  Here every step is a native kernel.

Tensor parallelism (world > 1, one process per GPU): q/k/v/gate/up are column shards (whole
heads; gate/up cut at down_proj's group boundaries), o/down row shards, so each rank attends
over its own heads with its own KV cache; the partial sums of o and down are exchanged either
inside the GEMV launches (peer stores over NVLink, ``peer_ar``) or by NCCL all-reduce; the
embedding is replicated and the INT8 head vocabulary-parallel, with one (max, index) pair per
rank exchanged for the greedy pick.  ``shard_layers`` cuts a full model into one rank's part.
"""
from __future__ import annotations

import ctypes
import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _native
from .decoder_stack import shard_linear
from .symmetric_2bit_engine import QuantizedEmbedding, QuantizedLinearHead, SymmetricOTF2BitLinear

PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")


@dataclass
class ModelConfig:
    layers: int
    hidden: int
    intermediate: int
    heads: int
    kv_heads: int
    head_dim: int
    vocab: int
    rope_theta: float = 500000.0
    rms_eps: float = 1e-5
    max_pos: int = 2048


LLAMA32_3B = ModelConfig(layers=28, hidden=3072, intermediate=8192, heads=24, kv_heads=8, head_dim=128,
                         vocab=128256, rope_theta=500000.0)


LLAMA3_70B = ModelConfig(layers=80, hidden=8192, intermediate=28672, heads=64, kv_heads=8, head_dim=128,
                         vocab=128256, rope_theta=500000.0)


def shard_layers(layers: Sequence[Dict[str, SymmetricOTF2BitLinear]], cfg: ModelConfig, rank: int, world: int
                 ) -> List[Dict[str, SymmetricOTF2BitLinear]]:
    """Rank ``rank``'s tensor-parallel part of full decoder layers: q/k/v by whole query / KV
    heads (the head counts must divide by world), gate/up by rows at multiples of down_proj's
    group size, o/down by input columns at group boundaries (anchors re-based, bias on rank 0)."""
    if cfg.heads % world or cfg.kv_heads % world:
        raise ValueError(f"{cfg.heads} query / {cfg.kv_heads} KV heads do not split over {world} ranks")
    out = []
    for l in layers:
        G = l["down_proj"].group_size
        out.append({"q_proj": shard_linear(l["q_proj"], rank, world, "out", cfg.head_dim),
                    "k_proj": shard_linear(l["k_proj"], rank, world, "out", cfg.head_dim),
                    "v_proj": shard_linear(l["v_proj"], rank, world, "out", cfg.head_dim),
                    "o_proj": shard_linear(l["o_proj"], rank, world, "in"),
                    "gate_proj": shard_linear(l["gate_proj"], rank, world, "out", G),
                    "up_proj": shard_linear(l["up_proj"], rank, world, "out", G),
                    "down_proj": shard_linear(l["down_proj"], rank, world, "in")})
    return out


def rope_table(cfg: ModelConfig, device) -> torch.Tensor:
    """fp16 [max_pos, 2, head_dim]: HF's default rotary cos and sin rows (fp32 angles
    pos * theta^(-2i/d), both halves duplicated, rounded to fp16 as HF casts them)."""
    d = cfg.head_dim
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(0, d, 2, dtype=torch.int64, device=device).float() / d))
    pos = torch.arange(cfg.max_pos, device=device, dtype=torch.float32)
    freqs = pos[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return torch.stack((emb.cos(), emb.sin()), dim=1).to(torch.float16).contiguous()


class GreedyDecoder:
    """Batch-1 greedy decoding through native kernels (see module docstring)."""

    def __init__(self, cfg: ModelConfig, layers: Sequence[Dict[str, SymmetricOTF2BitLinear]],
                 norms: Sequence[Tuple[torch.Tensor, torch.Tensor]], embed: QuantizedEmbedding,
                 head: QuantizedLinearHead, final_norm: Optional[torch.Tensor], device, *, rank: int = 0,
                 world: int = 1, process_group=None, peer_ar=None, head_row0: int = 0):
        """``layers``: this rank's modules (``shard_layers`` under tensor parallelism);
        ``head``: this rank's rows of the INT8 head, which start at vocabulary row
        ``head_row0``; ``peer_ar``: an otf_llm.tp_allreduce.PeerAllReduce for the exchange fused
        into the o/down launches (else NCCL all-reduce over ``process_group``)."""
        dev = torch.device(device)
        self.cfg, self.device = cfg, dev
        self.rank, self.world, self.pg, self.ar = rank, world, process_group, peer_ar
        self.head_row0 = int(head_row0)
        self.layers = [dict(l) for l in layers]
        for l in self.layers:
            missing = [n for n in PROJ if n not in l]
            if missing:
                raise ValueError(f"decoder layer lacks {missing}")
        l0 = self.layers[0]
        self.heads = l0["q_proj"].out_features // cfg.head_dim      # this rank's query / KV heads
        self.kv_heads = l0["k_proj"].out_features // cfg.head_dim
        if world == 1 and (self.heads, self.kv_heads) != (cfg.heads, cfg.kv_heads):
            raise ValueError("q/k projections do not match the configured head counts")
        if peer_ar is not None and world > 1:
            if not all(_native.tensor_pipe_shape_ok(m) for l in self.layers for m in l.values()):
                raise ValueError("the fused peer exchange needs every projection on the tensor-pipe GEMV")
        f16 = dict(dtype=torch.float16, device=dev)
        self.in_norms = [a.to(**f16).contiguous() for a, _ in norms]
        self.post_norms = [b.to(**f16).contiguous() for _, b in norms]
        self.embed, self.head = embed, head
        self.final_norm = (final_norm if final_norm is not None else torch.ones(cfg.hidden)).to(**f16).contiguous()
        qd, kvd = self.heads * cfg.head_dim, self.kv_heads * cfg.head_dim
        inter = l0["gate_proj"].out_features
        self.kc = [torch.zeros(cfg.max_pos, kvd, **f16) for _ in self.layers]
        self.vc = [torch.zeros(cfg.max_pos, kvd, **f16) for _ in self.layers]
        self.cos_sin = rope_table(cfg, dev)
        self.pos = torch.zeros(1, dtype=torch.int32, device=dev)
        self.ids = torch.zeros(1, dtype=torch.int64, device=dev)
        n = _native.lib().otf_attn_workspace_bytes(self.kv_heads, cfg.head_dim, cfg.max_pos)
        self.attn_ws = torch.zeros(int(n), dtype=torch.uint8, device=dev)
        self.b = {"h": torch.zeros(1, cfg.hidden, **f16), "h1": torch.zeros(1, cfg.hidden, **f16),
                  "h2": torch.zeros(1, cfg.hidden, **f16), "q": torch.zeros(1, qd, **f16),
                  "k": torch.zeros(1, kvd, **f16), "v": torch.zeros(1, kvd, **f16),
                  "attn": torch.zeros(1, qd, **f16), "g": torch.zeros(1, inter, **f16),
                  "u": torch.zeros(1, inter, **f16), "xn": torch.zeros(1, cfg.hidden, **f16)}
        self.logits = torch.zeros(1, head.weight_int8.shape[0], dtype=torch.float32, device=dev)
        if world > 1:
            self.loc_idx = torch.zeros(1, dtype=torch.int64, device=dev)
            self.pairs = torch.zeros(world, 2, dtype=torch.float64, device=dev)
        self.graph = None
        self._pf_graphs: Dict[int, Tuple[torch.cuda.CUDAGraph, torch.Tensor]] = {}

    # -- one token step (capturable) ----------------------------------------------------
    def _attention(self, li: int) -> None:
        """RoPE, KV-cache write and attention over this rank's heads in one launch."""
        cfg, b = self.cfg, self.b
        _native._check(_native.lib().otf_attn_rope_decode(
            b["q"].data_ptr(), b["k"].data_ptr(), b["v"].data_ptr(), self.cos_sin.data_ptr(), self.pos.data_ptr(),
            self.kc[li].data_ptr(), self.vc[li].data_ptr(), b["attn"].data_ptr(), 1.0 / math.sqrt(cfg.head_dim),
            self.heads, self.kv_heads, cfg.head_dim, cfg.max_pos, self.attn_ws.data_ptr(), self.attn_ws.numel(),
            _native._stream(self.device)), "otf_attn_rope_decode")

    def _layers_tp(self, cur: torch.Tensor) -> torch.Tensor:
        """The decoder layers under tensor parallelism; returns the reduced residual stream.
        NCCL: o / down write partial sums (rank 0 adds the residual), all-reduced in place.
        Peer: o / down store their partials into every rank's receive buffer and the next
        grouped launch sums them while staging its input (the q or gate item also writes the
        sum back for the residual path); one standalone finish closes the last layer."""
        cfg, b, G = self.cfg, self.b, _native.GroupItem
        lead = self.rank == 0
        RMS = _native.OTF_XOP_RMSNORM
        if self.ar is None:
            for li, layer in enumerate(self.layers):
                _native.linear_group([G(layer[n], cur, b[o], x_op=RMS, x_aux=self.in_norms[li], eps=cfg.rms_eps)
                                      for n, o in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"))])
                self._attention(li)
                _native.linear_group([G(layer["o_proj"], b["attn"], b["h1"], residual=cur if lead else None)])
                torch.distributed.all_reduce(b["h1"], group=self.pg)
                _native.linear_group([G(layer[n], b["h1"], b[o], x_op=RMS, x_aux=self.post_norms[li], eps=cfg.rms_eps)
                                      for n, o in (("gate_proj", "g"), ("up_proj", "u"))])
                _native.linear_group([G(layer["down_proj"], b["g"], b["h2"], residual=b["h1"] if lead else None,
                                        x_op=_native.OTF_XOP_SILU_MUL, x_aux=b["u"])])
                torch.distributed.all_reduce(b["h2"], group=self.pg)
                cur = b["h2"]
            return cur
        ar = self.ar
        PROD, CONS = _native.OTF_AR_PRODUCE, _native.OTF_AR_CONSUME
        pending = None
        for li, layer in enumerate(self.layers):
            if pending is None:
                items = [G(layer[n], cur, b[o], x_op=RMS, x_aux=self.in_norms[li], eps=cfg.rms_eps)
                         for n, o in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"))]
            else:
                items = [G(layer[n], b["h2"], b[o], x_op=RMS, x_aux=self.in_norms[li], eps=cfg.rms_eps, ar=ar,
                           ar_mode=CONS, ar_buf=pending, ar_out=b["h2"].view(-1) if n == "q_proj" else None)
                         for n, o in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"))]
                cur = b["h2"]
            _native.linear_group(items)
            self._attention(li)
            ob = ar.next_buffer()
            _native.linear_group([G(layer["o_proj"], b["attn"], b["h1"], residual=cur if lead else None, ar=ar,
                                    ar_mode=PROD, ar_buf=ob)])
            _native.linear_group([G(layer[n], b["h1"], b[o], x_op=RMS, x_aux=self.post_norms[li], eps=cfg.rms_eps,
                                    ar=ar, ar_mode=CONS, ar_buf=ob, ar_out=b["h1"].view(-1) if n == "gate_proj" else None)
                                  for n, o in (("gate_proj", "g"), ("up_proj", "u"))])
            pending = ar.next_buffer()
            _native.linear_group([G(layer["down_proj"], b["g"], b["h2"], residual=b["h1"] if lead else None,
                                    x_op=_native.OTF_XOP_SILU_MUL, x_aux=b["u"], ar=ar, ar_mode=PROD, ar_buf=pending)])
        ar.finish(b["h2"].view(-1), pending)
        return b["h2"]

    def _step(self) -> None:
        cfg, b, L = self.cfg, self.b, _native.lib()
        G = _native.GroupItem
        st = _native._stream(self.device)
        _embed_into(self.embed, self.ids.view(1), b["h"].view(1, -1))
        if self.world > 1:
            cur = self._layers_tp(b["h"])
            xn = _native.rmsnorm(cur, self.final_norm, cfg.rms_eps, out=b["xn"])
            self._argmax(xn)
            _native._check(L.otf_pos_advance(self.pos.data_ptr(), st), "otf_pos_advance")
            return
        cur = b["h"]
        for li, layer in enumerate(self.layers):
            _native.linear_group([G(layer[n], cur, b[o], x_op=_native.OTF_XOP_RMSNORM, x_aux=self.in_norms[li],
                                    eps=cfg.rms_eps) for n, o in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"))])
            self._attention(li)
            _native.linear_group([G(layer["o_proj"], b["attn"], b["h1"], residual=cur)])
            _native.linear_group([G(layer[n], b["h1"], b[o], x_op=_native.OTF_XOP_RMSNORM, x_aux=self.post_norms[li],
                                    eps=cfg.rms_eps) for n, o in (("gate_proj", "g"), ("up_proj", "u"))])
            # down writes the residual stream in place: o (its only other reader) already ran
            _native.linear_group([G(layer["down_proj"], b["g"], b["h"], residual=b["h1"],
                                    x_op=_native.OTF_XOP_SILU_MUL, x_aux=b["u"])])
            cur = b["h"]
        xn = _native.rmsnorm(cur, self.final_norm, cfg.rms_eps, out=b["xn"])
        self._argmax(xn)
        _native._check(L.otf_pos_advance(self.pos.data_ptr(), st), "otf_pos_advance")

    def _argmax(self, xn: torch.Tensor) -> None:
        """Greedy id into self.ids: the fused INT8 head + argmax over this rank's rows; under
        tensor parallelism every rank's (max logit, global row) pair is all-gathered and the
        first rank holding the maximum wins (rows ascend with rank, so ties go to the lowest
        vocabulary index, as torch.argmax)."""
        hd = self.head
        w, s = hd.weight_int8, hd.scales.reshape(-1)
        L = _native.lib()
        dst = self.ids if self.world == 1 else self.loc_idx
        with torch.cuda.device(self.device):
            _native._check(L.otf_i8_head_argmax(xn.data_ptr(), xn.shape[1], w.data_ptr(), w.stride(0), s.data_ptr(),
                                                self.logits.data_ptr(), self.logits.shape[1], dst.data_ptr(), 1,
                                                w.shape[0], w.shape[1], _native._stream(self.device)),
                           "otf_i8_head_argmax")
        if self.world > 1:
            vmax = self.logits.gather(1, self.loc_idx.view(1, 1)).view(1).to(torch.float64)
            pair = torch.cat([vmax, (self.loc_idx + self.head_row0).to(torch.float64)]).view(1, 2)
            torch.distributed.all_gather_into_tensor(self.pairs, pair, group=self.pg)
            best = torch.argmax(self.pairs[:, 0]).view(1)
            self.ids.copy_(self.pairs.index_select(0, best)[:, 1].to(torch.int64))

    def capture(self) -> None:
        """Record one token step as a CUDA graph (warm-up steps run eagerly first, then the
        position is reset)."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        self.reset()

    def reset(self) -> None:
        self.pos.zero_()
        torch.cuda.synchronize(self.device)

    def step(self) -> None:
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step()

    def prefill(self, prompt: torch.Tensor) -> None:
        """The prompt's P tokens as one pass of P rows from the current position, as the
        reference runner's HF generate runs a prompt in one forward: every projection at M = P
        rows (the tensor-memory GEMM from 9 rows), RoPE + KV-cache write + causal attention of
        the P rows (``otf_attn_prefill``), the MLP at M = P, then the final norm and the greedy
        pick of the last row into ``ids`` (its logits in ``logits``); the position advances by
        P.  One GPU (the tensor-parallel decoder feeds prompts token by token).  A prompt that
        would run past the cache writes nothing and raises the otf_device_error flag."""
        if self.world > 1:
            raise NotImplementedError("prefill runs on one GPU; tensor-parallel decoders step the prompt")
        ids = prompt.reshape(-1).to(device=self.device, dtype=torch.int64)
        P = int(ids.numel())
        if P == 0:
            return
        if P > self.cfg.max_pos:
            raise ValueError(f"prompt of {P} tokens exceeds the cache of {self.cfg.max_pos} positions")
        rec = self._pf_graphs.get(P)
        if rec is not None:                  # recorded by capture_prefill for this length
            rec[1].copy_(ids)
            rec[0].replay()
            return
        self._prefill_rows(ids)

    def capture_prefill(self, P: int) -> None:
        """Record the prefill of P-token prompts as one CUDA graph, which ``prefill`` then
        replays for every prompt of that length (the ids are copied into the graph's input
        first); one eager pass runs before the capture, and the position is reset afterwards."""
        if self.world > 1:
            raise NotImplementedError("prefill runs on one GPU")
        if not 0 < P <= self.cfg.max_pos:
            raise ValueError(f"prompt length {P} outside 1..{self.cfg.max_pos}")
        ids = torch.zeros(P, dtype=torch.int64, device=self.device)
        cur = torch.cuda.current_stream(self.device)
        s = torch.cuda.Stream(self.device)
        s.wait_stream(cur)
        with torch.cuda.stream(s):
            self._prefill_rows(ids)
        cur.wait_stream(s)
        torch.cuda.synchronize(self.device)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self._prefill_rows(ids)
        self._pf_graphs[P] = (g, ids)
        self.reset()

    def _prefill_rows(self, ids: torch.Tensor) -> None:
        cfg, L = self.cfg, _native.lib()
        P = int(ids.numel())
        f16 = dict(dtype=torch.float16, device=self.device)
        qd, kvd = self.heads * cfg.head_dim, self.kv_heads * cfg.head_dim
        inter = self.layers[0]["gate_proj"].out_features
        h, h1, xn = (torch.empty(P, cfg.hidden, **f16) for _ in range(3))
        q, attn = torch.empty(P, qd, **f16), torch.empty(P, qd, **f16)
        k, v = torch.empty(P, kvd, **f16), torch.empty(P, kvd, **f16)
        g, u, a = (torch.empty(P, inter, **f16) for _ in range(3))
        st = _native._stream(self.device)
        lin = BatchedGreedyDecoder._lin
        _embed_into(self.embed, ids, h)
        for li, layer in enumerate(self.layers):
            _native.rmsnorm(h, self.in_norms[li], cfg.rms_eps, out=xn)
            for n, o in (("q_proj", q), ("k_proj", k), ("v_proj", v)):
                lin(layer[n], xn, o)
            _native._check(L.otf_attn_prefill(
                q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0), self.cos_sin.data_ptr(),
                self.pos.data_ptr(), self.kc[li].data_ptr(), self.vc[li].data_ptr(), attn.data_ptr(), attn.stride(0),
                1.0 / math.sqrt(cfg.head_dim), self.heads, self.kv_heads, cfg.head_dim, cfg.max_pos, P, st),
                "otf_attn_prefill")
            lin(layer["o_proj"], attn, h1, residual=h)
            _native.rmsnorm(h1, self.post_norms[li], cfg.rms_eps, out=xn)
            lin(layer["gate_proj"], xn, g)
            lin(layer["up_proj"], xn, u)
            _native.silu_mul(g, u, out=a)
            lin(layer["down_proj"], a, h, residual=h1)
        xl = self.b["xn"]
        _native.rmsnorm(h[P - 1:P], self.final_norm, cfg.rms_eps, out=xl)
        self._argmax(xl)
        self.pos.add_(P)

    def generate(self, prompt: torch.Tensor, new_tokens: int, logits_out: Optional[List[torch.Tensor]] = None,
                 prefill: Optional[bool] = None) -> torch.Tensor:
        """Greedy continuation of prompt (int64 ids on the device) by new_tokens tokens.  The
        prompt runs as one ``prefill`` pass on one GPU unless per-token logits are asked for
        (``logits_out``) or ``prefill=False``; otherwise token by token."""
        _check_prompt(prompt, self.embed.weight_int8.shape[0])
        if prefill is None:
            prefill = logits_out is None and self.world == 1
        self.reset()
        out = torch.empty(new_tokens, dtype=torch.int64, device=self.device)
        n = prompt.numel()
        if prefill and n:
            self.prefill(prompt)
            if logits_out is not None:
                logits_out.append(self.logits.clone())
            n = 0
        for i in range(n):
            self.ids.copy_(prompt[i:i + 1])
            self.step()
            if logits_out is not None:
                logits_out.append(self.logits.clone())
        for i in range(new_tokens):
            out[i:i + 1].copy_(self.ids)
            if i + 1 < new_tokens:
                self.step()
                if logits_out is not None:
                    logits_out.append(self.logits.clone())
        return out


def _embed_into(embed, ids: torch.Tensor, out: torch.Tensor) -> None:
    """The INT8 embedding rows of ids written straight into the residual stream buffer (no
    intermediate tensor, no copy launch).  Ids come from the head's argmax or from prompts
    checked by ``_check_prompt``."""
    _native.i8_embed(ids, embed.weight_int8, embed.scales.reshape(-1), None, out=out)


def _check_prompt(prompt: torch.Tensor, vocab: int) -> None:
    """Prompt ids outside [0, vocab) raise IndexError before any step, as the reference's
    F.embedding does (the token steps themselves run without a host sync)."""
    if prompt.numel() and (int(prompt.min()) < 0 or int(prompt.max()) >= vocab):
        raise IndexError("index out of range in self")


class BatchedGreedyDecoder:
    """Greedy decoding of ``batch`` independent sequences in lockstep on one GPU: one token step
    moves every sequence by one position.  Per layer: RMSNorm, q/k/v, batched RoPE + KV-cache
    write + attention (each sequence its own caches and position), o + residual, RMSNorm,
    gate/up, SiLU gate, down + residual; the 2-bit projections run with M = batch rows (the
    batched integer-MMA kernel up to 8 rows per weight pass, the tensor-memory tcgen05 GEMM
    from 9).  Under tensor parallelism (``world`` > 1, layers from ``shard_layers``) each rank
    runs its query / KV heads, gate/up rows and o/down K slices; o and down write partial sums
    (rank 0 adds the residual) that one NCCL all-reduce per projection sums, and the INT8 head
    is vocabulary-parallel (rows from ``head_row0``), each sequence's greedy pick one all-gather
    of (max logit, global row) pairs.  The reference has no batched decoder; HF's generate with a
    padded batch does the same math."""

    def __init__(self, cfg: ModelConfig, layers: Sequence[Dict[str, SymmetricOTF2BitLinear]],
                 norms: Sequence[Tuple[torch.Tensor, torch.Tensor]], embed: QuantizedEmbedding,
                 head: QuantizedLinearHead, final_norm: Optional[torch.Tensor], device, batch: int, *,
                 rank: int = 0, world: int = 1, process_group=None, head_row0: int = 0):
        dev = torch.device(device)
        B = int(batch)
        if B < 1:
            raise ValueError("batch must be >= 1")
        self.cfg, self.device, self.batch = cfg, dev, B
        self.rank, self.world, self.pg, self.head_row0 = rank, world, process_group, int(head_row0)
        self.layers = [dict(l) for l in layers]
        for l in self.layers:
            missing = [n for n in PROJ if n not in l]
            if missing:
                raise ValueError(f"decoder layer lacks {missing}")
        l0 = self.layers[0]
        self.heads = l0["q_proj"].out_features // cfg.head_dim      # this rank's query / KV heads
        self.kv_heads = l0["k_proj"].out_features // cfg.head_dim
        if world == 1 and (self.heads, self.kv_heads) != (cfg.heads, cfg.kv_heads):
            raise ValueError("q/k projections do not match the configured head counts")
        f16 = dict(dtype=torch.float16, device=dev)
        self.in_norms = [a.to(**f16).contiguous() for a, _ in norms]
        self.post_norms = [b.to(**f16).contiguous() for _, b in norms]
        self.embed, self.head = embed, head
        self.final_norm = (final_norm if final_norm is not None else torch.ones(cfg.hidden)).to(**f16).contiguous()
        qd, kvd = self.heads * cfg.head_dim, self.kv_heads * cfg.head_dim
        self.kc = [torch.zeros(B, cfg.max_pos, kvd, **f16) for _ in self.layers]
        self.vc = [torch.zeros(B, cfg.max_pos, kvd, **f16) for _ in self.layers]
        self.cos_sin = rope_table(cfg, dev)
        self.pos = torch.zeros(B, dtype=torch.int32, device=dev)
        self.ids = torch.zeros(B, dtype=torch.int64, device=dev)
        n = _native.lib().otf_attn_workspace_bytes_batch(self.kv_heads, cfg.head_dim, cfg.max_pos, B)
        self.attn_ws = torch.zeros(int(n), dtype=torch.uint8, device=dev)
        inter = self.layers[0]["gate_proj"].out_features
        self.b = {n_: torch.zeros(B, w, **f16) for n_, w in (("h", cfg.hidden), ("h1", cfg.hidden), ("xn", cfg.hidden),
                                                               ("q", qd), ("k", kvd), ("v", kvd), ("attn", qd),
                                                               ("g", inter), ("u", inter), ("a", inter))}
        self.logits = torch.zeros(B, head.weight_int8.shape[0], dtype=torch.float32, device=dev)
        if world > 1:
            self.loc_idx = torch.zeros(B, dtype=torch.int64, device=dev)
            self.pairs = torch.zeros(world * B, 2, dtype=torch.float64, device=dev)
            self.seq = torch.arange(B, device=dev)
        self.graph = None

    @staticmethod
    def _lin(m: SymmetricOTF2BitLinear, x: torch.Tensor, out: torch.Tensor, residual=None) -> None:
        _native.linear_2bit(x, m.packed_uint8, m.scales, m.group_size, m.codebook,
                            mask=m.outlier_mask_vector if m.has_outliers else None,
                            outlier_idx=m.outlier_indices if m.has_outliers else None,
                            outlier_vals=m.outliers_fp16 if m.has_outliers else None,
                            bias=m.bias if m.has_bias else None, residual=residual, clamp=True, out=out)

    def _step(self) -> None:
        cfg, b, L, B = self.cfg, self.b, _native.lib(), self.batch
        st = _native._stream(self.device)
        tp, lead = self.world > 1, self.rank == 0
        _embed_into(self.embed, self.ids.view(B), b["h"].view(B, -1))
        kvd = self.kv_heads * cfg.head_dim
        for li, layer in enumerate(self.layers):
            _native.rmsnorm(b["h"], self.in_norms[li], cfg.rms_eps, out=b["xn"])
            for n, o in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v")):
                self._lin(layer[n], b["xn"], b[o])
            _native._check(L.otf_attn_rope_decode_batch(
                b["q"].data_ptr(), b["q"].stride(0), b["k"].data_ptr(), b["v"].data_ptr(), b["k"].stride(0),
                self.cos_sin.data_ptr(), self.pos.data_ptr(), self.kc[li].data_ptr(), self.vc[li].data_ptr(),
                cfg.max_pos * kvd, b["attn"].data_ptr(), b["attn"].stride(0), 1.0 / math.sqrt(cfg.head_dim), self.heads,
                self.kv_heads, cfg.head_dim, cfg.max_pos, B, self.attn_ws.data_ptr(), self.attn_ws.numel(), st),
                "otf_attn_rope_decode_batch")
            # row-parallel o / down: partial sums, the residual on rank 0 only, then one all-reduce
            self._lin(layer["o_proj"], b["attn"], b["h1"], residual=b["h"] if lead else None)
            if tp:
                torch.distributed.all_reduce(b["h1"], group=self.pg)
            _native.rmsnorm(b["h1"], self.post_norms[li], cfg.rms_eps, out=b["xn"])
            self._lin(layer["gate_proj"], b["xn"], b["g"])
            self._lin(layer["up_proj"], b["xn"], b["u"])
            _native.silu_mul(b["g"], b["u"], out=b["a"])
            self._lin(layer["down_proj"], b["a"], b["h"], residual=b["h1"] if lead else None)
            if tp:
                torch.distributed.all_reduce(b["h"], group=self.pg)
        _native.rmsnorm(b["h"], self.final_norm, cfg.rms_eps, out=b["xn"])
        w, s = self.head.weight_int8, self.head.scales.reshape(-1)
        dst = self.loc_idx if tp else self.ids
        _native._check(L.otf_i8_head_argmax(b["xn"].data_ptr(), b["xn"].stride(0), w.data_ptr(), w.stride(0),
                                            s.data_ptr(), self.logits.data_ptr(), self.logits.shape[1],
                                            dst.data_ptr(), B, w.shape[0], w.shape[1], st), "otf_i8_head_argmax")
        if tp:
            # every rank's (max logit, global row) per sequence; the first rank holding the maximum
            # wins, i.e. the lowest vocabulary index on ties (rows ascend with rank), as torch.argmax
            vmax = self.logits.gather(1, self.loc_idx.view(B, 1)).to(torch.float64)
            pair = torch.cat([vmax, (self.loc_idx + self.head_row0).to(torch.float64).view(B, 1)], dim=1)
            torch.distributed.all_gather_into_tensor(self.pairs, pair, group=self.pg)
            pr = self.pairs.view(self.world, B, 2)
            best = torch.argmax(pr[:, :, 0], dim=0)
            self.ids.copy_(pr[best, self.seq, 1].to(torch.int64))
        _native._check(L.otf_pos_advance_batch(self.pos.data_ptr(), B, st), "otf_pos_advance_batch")

    def capture(self) -> None:
        """Record one token step (all sequences) as a CUDA graph; positions reset afterwards."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            for _ in range(2):
                self._step()
        torch.cuda.current_stream(self.device).wait_stream(s)
        torch.cuda.synchronize(self.device)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self._step()
        self.reset()

    def reset(self) -> None:
        self.pos.zero_()
        torch.cuda.synchronize(self.device)

    def step(self) -> None:
        if self.graph is not None:
            self.graph.replay()
        else:
            self._step()

    def prefill(self, prompts: torch.Tensor) -> None:
        """Every sequence's P prompt tokens as one pass of batch x P rows from the current
        positions (``GreedyDecoder.prefill`` for a batch): the projections at M = batch x P rows,
        ``otf_attn_prefill`` per sequence on its own caches, then the last row of each sequence
        through the final norm and the head + argmax into ``ids``; every position advances by
        P.  One GPU."""
        if self.world > 1:
            raise NotImplementedError("prefill runs on one GPU; tensor-parallel decoders step the prompt")
        if prompts.dim() != 2 or prompts.shape[0] != self.batch:
            raise ValueError(f"prompts must be [{self.batch}, P]")
        cfg, L, B = self.cfg, _native.lib(), self.batch
        P = int(prompts.shape[1])
        if P == 0:
            return
        if P > cfg.max_pos:
            raise ValueError(f"prompts of {P} tokens exceed the cache of {cfg.max_pos} positions")
        ids = prompts.reshape(-1).to(device=self.device, dtype=torch.int64)
        R = B * P
        f16 = dict(dtype=torch.float16, device=self.device)
        qd, kvd = self.heads * cfg.head_dim, self.kv_heads * cfg.head_dim
        inter = self.layers[0]["gate_proj"].out_features
        h, h1, xn = (torch.empty(R, cfg.hidden, **f16) for _ in range(3))
        q, attn = torch.empty(R, qd, **f16), torch.empty(R, qd, **f16)
        k, v = torch.empty(R, kvd, **f16), torch.empty(R, kvd, **f16)
        g, u, a = (torch.empty(R, inter, **f16) for _ in range(3))
        st = _native._stream(self.device)
        scale = 1.0 / math.sqrt(cfg.head_dim)
        _embed_into(self.embed, ids, h)
        for li, layer in enumerate(self.layers):
            _native.rmsnorm(h, self.in_norms[li], cfg.rms_eps, out=xn)
            for n, o in (("q_proj", q), ("k_proj", k), ("v_proj", v)):
                self._lin(layer[n], xn, o)
            for sb in range(B):
                r0 = sb * P
                _native._check(L.otf_attn_prefill(
                    q[r0].data_ptr(), q.stride(0), k[r0].data_ptr(), v[r0].data_ptr(), k.stride(0),
                    self.cos_sin.data_ptr(), self.pos[sb].data_ptr(), self.kc[li][sb].data_ptr(),
                    self.vc[li][sb].data_ptr(), attn[r0].data_ptr(), attn.stride(0), scale, self.heads,
                    self.kv_heads, cfg.head_dim, cfg.max_pos, P, st), "otf_attn_prefill")
            self._lin(layer["o_proj"], attn, h1, residual=h)
            _native.rmsnorm(h1, self.post_norms[li], cfg.rms_eps, out=xn)
            self._lin(layer["gate_proj"], xn, g)
            self._lin(layer["up_proj"], xn, u)
            _native.silu_mul(g, u, out=a)
            self._lin(layer["down_proj"], a, h, residual=h1)
        last = self.b["h"]
        last.copy_(h.view(B, P, cfg.hidden)[:, P - 1])
        _native.rmsnorm(last, self.final_norm, cfg.rms_eps, out=self.b["xn"])
        w, s = self.head.weight_int8, self.head.scales.reshape(-1)
        _native._check(L.otf_i8_head_argmax(self.b["xn"].data_ptr(), self.b["xn"].stride(0), w.data_ptr(), w.stride(0),
                                            s.data_ptr(), self.logits.data_ptr(), self.logits.shape[1],
                                            self.ids.data_ptr(), B, w.shape[0], w.shape[1], st), "otf_i8_head_argmax")
        self.pos.add_(P)

    def generate(self, prompts: torch.Tensor, new_tokens: int, logits_out: Optional[List[torch.Tensor]] = None,
                 prefill: Optional[bool] = None) -> torch.Tensor:
        """Greedy continuation of prompts (int64 [batch, P] on the device, equal lengths) by
        new_tokens tokens per sequence; returns int64 [batch, new_tokens].  On one GPU the
        prompts run as one ``prefill`` pass unless per-token logits are asked for
        (``logits_out``) or ``prefill=False``."""
        if prompts.dim() != 2 or prompts.shape[0] != self.batch:
            raise ValueError(f"prompts must be [{self.batch}, P]")
        _check_prompt(prompts, self.embed.weight_int8.shape[0])
        if prefill is None:
            prefill = logits_out is None and self.world == 1
        self.reset()
        out = torch.empty(self.batch, new_tokens, dtype=torch.int64, device=self.device)
        n = prompts.shape[1]
        if prefill and n:
            self.prefill(prompts)
            if logits_out is not None:
                logits_out.append(self.logits.clone())
            n = 0
        for i in range(n):
            self.ids.copy_(prompts[:, i])
            self.step()
            if logits_out is not None:
                logits_out.append(self.logits.clone())
        for i in range(new_tokens):
            out[:, i].copy_(self.ids)
            if i + 1 < new_tokens:
                self.step()
                if logits_out is not None:
                    logits_out.append(self.logits.clone())
        return out
