"""CPU restatement of the reference engine's batch-1 greedy decode step (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may import this
module, and only to check or time against it.

The reference decodes by running Hugging Face's ``LlamaForCausalLM`` with its own modules
put in place of the embedding, the seven projections of every layer and the head
(otf_llm/run_symmetric_2bit.py:88-189), on the KV-cache path of ``model.generate``
(:210-220).  One token step of that engine, as restated here:

  * embedding: ``QuantizedEmbedding.forward`` -- fp16(int8 row x fp16 scale)
    (otf_llm/symmetric_2bit_engine.py:41-47), ``oracle.i8_embed``;
  * per layer, HF's ``LlamaDecoderLayer``: RMSNorm (fp32 mean of squares, ``x * rsqrt``
    rounded to fp16, times the fp16 weight), q/k/v through ``SymmetricOTF2BitLinear`` (:214-235;
    on the CPU the whole weight is LUT-dequantised to fp16 and multiplied,
    otf_llm/otf_triton_2bit_kernel.py:188-194 -- ``oracle.lut_linear``), rotary embedding
    (fp16 ``x*cos + rotate_half(x)*sin`` on HF's default table), attention over the cached
    positions, o_proj, fp16 residual add, RMSNorm, gate/up, ``silu(gate) * up`` in fp16, down_proj,
    fp16 residual add;
  * final RMSNorm and ``QuantizedLinearHead.forward`` (:75-91), ``oracle.i8_head``; greedy
    argmax.

Attention is evaluated in fp32 from the fp16 q / cache rows with one fp16 rounding of the
output (HF's CPU scaled-dot-product attention accumulates in fp32 too).  The rotary table is
HF's default one (inv_freq = 1 / theta^(2i/d) in fp32, angles pos * inv_freq in fp32, cos and
sin rounded to fp16).  The reference's own ``fix_rotary_embeddings``
(otf_llm/run_symmetric_2bit.py:34-49) recomputes the same inv_freq from ``config.rope_theta``
and the module's ``dim``; under transformers 5 neither attribute exists any more (theta falls
back to 1e6 and dim to 128), so this restatement follows the table the rotary module builds
from its config, which is what that function recomputes under transformers 4.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import numpy as np

from . import oracle

PROJ = ("q_proj", "k_proj", "v_proj", "o_proj", "gate_proj", "up_proj", "down_proj")
F16, F32 = np.float16, np.float32


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """HF LlamaRMSNorm on fp16 input: weight * fp16(x * rsqrt(mean(x^2) + eps))."""
    xf = x.astype(F32)
    var = np.mean(xf * xf, axis=-1, keepdims=True, dtype=F32)
    y = (xf * (F32(1.0) / np.sqrt(var + F32(eps)))).astype(F16)
    return (w.astype(F32) * y.astype(F32)).astype(F16)


def rope_table(head_dim: int, theta: float, max_pos: int):
    """HF's default rotary cos / sin rows, fp16 [max_pos, head_dim] each.  Evaluated with
    torch's CPU pow / cos / sin, the functions HF's rotary module calls, so the table is HF's
    bit for bit (numpy's float32 pow and cos round differently in the last place)."""
    import torch
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, dtype=torch.int64).float() / head_dim))
    freqs = torch.arange(max_pos, dtype=torch.float32)[:, None] * inv[None, :]
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().half().numpy(), emb.sin().half().numpy()


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x [heads, d] fp16: fp16(fp16(x*cos) + fp16(rotate_half(x)*sin)), HF's apply_rotary_pos_emb."""
    h = x.shape[-1] // 2
    rot = np.concatenate((-x[..., h:].astype(F32), x[..., :h].astype(F32)), axis=-1).astype(F16)
    a = (x.astype(F32) * cos.astype(F32)).astype(F16)
    b = (rot.astype(F32) * sin.astype(F32)).astype(F16)
    return (a.astype(F32) + b.astype(F32)).astype(F16)


def attention(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, n_pos: int, heads: int, kv_heads: int,
              head_dim: int) -> np.ndarray:
    """softmax(q k^T / sqrt(d)) v over cache rows [0, n_pos) with grouped KV heads; fp16 [heads*d]."""
    rep = heads // kv_heads
    qf = q.reshape(kv_heads, rep, head_dim).astype(F32)
    k = kc[:n_pos].reshape(n_pos, kv_heads, head_dim).astype(F32)
    v = vc[:n_pos].reshape(n_pos, kv_heads, head_dim).astype(F32)
    s = np.einsum("grd,lgd->grl", qf, k) * F32(1.0 / np.sqrt(head_dim))
    s = np.exp(s - s.max(axis=-1, keepdims=True))
    p = s / s.sum(axis=-1, keepdims=True)
    return np.einsum("grl,lgd->grd", p, v).reshape(-1).astype(F16)


def silu_mul(g: np.ndarray, u: np.ndarray) -> np.ndarray:
    """HF LlamaMLP's act_fn(gate) * up on fp16: silu rounded to fp16, then the fp16 product."""
    gf = g.astype(F32)
    a = (gf / (F32(1.0) + np.exp(-gf))).astype(F16)
    return (a.astype(F32) * u.astype(F32)).astype(F16)


def _np(t) -> Optional[np.ndarray]:
    if t is None:
        return None
    if isinstance(t, np.ndarray):
        return t
    return t.detach().cpu().numpy()


def projection(packed, scales, group_size: int, *, mask=None, idx=None, ov=None, bias=None) -> Dict:
    """One projection's reference tensors (packed codes, scales, mask vector, anchor
    indices / values, bias) as contiguous numpy arrays."""
    return {"packed": np.ascontiguousarray(_np(packed)), "scales": np.ascontiguousarray(_np(scales)),
            "G": int(group_size), "mask": _np(mask), "idx": _np(idx), "ov": _np(ov), "bias": _np(bias)}


def projection_of(module) -> Dict:
    """``projection`` from an object with the reference module's buffers
    (SymmetricOTF2BitLinear's names, otf_llm/symmetric_2bit_engine.py:186-208)."""
    has = bool(getattr(module, "has_outliers", False))
    return projection(module.packed_uint8, module.scales, module.group_size,
                      mask=module.outlier_mask_vector if has else None,
                      idx=module.outlier_indices if has else None, ov=module.outliers_fp16 if has else None,
                      bias=getattr(module, "bias", None))


class Decoder:
    """The reference engine's batch-1 decode (module docstring), one token per ``step``."""

    def __init__(self, layers: Sequence[Dict[str, Dict]], norms: Sequence[tuple], final_norm, embed_w8,
                 embed_scales, head_w8, head_scales, *, heads: int, kv_heads: int, head_dim: int,
                 rope_theta: float = 500000.0, rms_eps: float = 1e-5, max_pos: int = 2048):
        self.layers = [dict(l) for l in layers]
        self.norms = [(_np(a).astype(F16), _np(b).astype(F16)) for a, b in norms]
        self.final_norm = _np(final_norm).astype(F16)
        self.emb_w, self.emb_s = np.ascontiguousarray(_np(embed_w8)), np.ascontiguousarray(_np(embed_scales))
        self.head_w, self.head_s = np.ascontiguousarray(_np(head_w8)), np.ascontiguousarray(_np(head_scales))
        self.heads, self.kv_heads, self.head_dim = heads, kv_heads, head_dim
        self.eps, self.max_pos = rms_eps, max_pos
        self.cos, self.sin = rope_table(head_dim, rope_theta, max_pos)
        kvd = kv_heads * head_dim
        self.kc = [np.zeros((max_pos, kvd), F16) for _ in self.layers]
        self.vc = [np.zeros((max_pos, kvd), F16) for _ in self.layers]
        biggest = max(p["packed"].shape[0] * p["packed"].shape[1] * 4 for l in self.layers for p in l.values())
        self.wbuf = np.empty(biggest, F16)

    def set_cache(self, layer: int, k_rows: np.ndarray, v_rows: np.ndarray, start: int = 0) -> None:
        """Fill cache rows [start, start + len) of one layer (e.g. a prompt another engine ran)."""
        n = k_rows.shape[0]
        self.kc[layer][start:start + n] = k_rows
        self.vc[layer][start:start + n] = v_rows

    def _lin(self, p: Dict, x: np.ndarray) -> np.ndarray:
        return oracle.lut_linear(x.reshape(1, -1), p["packed"], p["scales"], p["G"], mask=p["mask"],
                                 outlier_idx=p["idx"], outlier_vals=p["ov"], bias=p["bias"], wbuf=self.wbuf)[0]

    def hidden(self, token: int, pos: int) -> np.ndarray:
        """Final-normed hidden state (fp16 [hidden]) of ``token`` at position ``pos``; writes the
        layer caches at ``pos``."""
        if not 0 <= pos < self.max_pos:
            raise IndexError(f"position {pos} outside [0, {self.max_pos})")
        hd = self.head_dim
        h = oracle.i8_embed(np.array([token]), self.emb_w, self.emb_s)[0]
        for li, l in enumerate(self.layers):
            w_in, w_post = self.norms[li]
            xn = rmsnorm(h, w_in, self.eps)
            q = apply_rope(self._lin(l["q_proj"], xn).reshape(-1, hd), self.cos[pos], self.sin[pos])
            k = apply_rope(self._lin(l["k_proj"], xn).reshape(-1, hd), self.cos[pos], self.sin[pos])
            v = self._lin(l["v_proj"], xn)
            self.kc[li][pos] = k.reshape(-1)
            self.vc[li][pos] = v
            a = attention(q, self.kc[li], self.vc[li], pos + 1, self.heads, self.kv_heads, hd)
            h = (h.astype(F32) + self._lin(l["o_proj"], a).astype(F32)).astype(F16)
            xn = rmsnorm(h, w_post, self.eps)
            m = silu_mul(self._lin(l["gate_proj"], xn), self._lin(l["up_proj"], xn))
            h = (h.astype(F32) + self._lin(l["down_proj"], m).astype(F32)).astype(F16)
        return rmsnorm(h, self.final_norm, self.eps)

    def step(self, token: int, pos: int) -> np.ndarray:
        """fp32 logits [vocab] after ``token`` at ``pos``."""
        return oracle.i8_head(self.hidden(token, pos).reshape(1, -1), self.head_w, self.head_s)[0]

    def generate(self, prompt: Sequence[int], new_tokens: int, start: int = 0,
                 logits_out: Optional[List[np.ndarray]] = None) -> List[int]:
        """Greedy decoding: feed ``prompt`` from position ``start`` one token at a time, then
        ``new_tokens`` argmax picks; returns the picks."""
        out: List[int] = []
        pos = start
        lg = None
        for t in prompt:
            lg = self.step(int(t), pos)
            pos += 1
            if logits_out is not None:
                logits_out.append(lg)
        for _ in range(new_tokens):
            nxt = int(oracle.argmax_rows(lg)[0])
            out.append(nxt)
            if len(out) == new_tokens:
                break
            lg = self.step(nxt, pos)
            pos += 1
            if logits_out is not None:
                logits_out.append(lg)
        return out
