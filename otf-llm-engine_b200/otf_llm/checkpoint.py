"""The converted OTF 2-bit checkpoint directory: reader (with tensor-parallel shards),
writer/converter, and injection into a Hugging Face causal-LM skeleton.

On-disk format (written by otf_llm/convert_symmetric_2bit.py:97-207, read by
otf_llm/run_symmetric_2bit.py:70-187)::

    otf_2bit_config.json        {"group_size", "outlier_ratio", "num_layers", "projections", ...}
    otf_2bit_model.safetensors  model.layers.{i}.{proj}.packed_uint8     uint8 [N, K/4]
                                model.layers.{i}.{proj}.scales           fp16  [N, K/G]
                                model.layers.{i}.{proj}.outlier_deltas   fp16  [N, k]   optional
                                model.layers.{i}.{proj}.outlier_indices  int64 [k]      optional
                                model.layers.{i}.{proj}.bias             [N]            optional
    otf_2bit_base.safetensors   model.embed_tokens.weight_int8 int8 [V, D], .scales fp16 [V, 1]
                                lm_head.weight_int8 / lm_head.scales   (absent: head tied to the embedding)
                                model.norm.weight
                                model.layers.{i}.input_layernorm.weight
                                model.layers.{i}.post_attention_layernorm.weight

Reading follows the reference runner's rules: ``group_size`` defaults to 32 and
``projections`` to the seven Llama projections when the config omits them
(run_symmetric_2bit.py:75-77); a projection without ``packed_uint8`` is skipped
(:157-158); ``d_in = packed_uint8.shape[1] * 4`` (:172); a missing ``lm_head`` ties the
head to the embedding's int8 buffer and scales by reference, not by copy (:128-135).

Tensor-parallel loads read only this rank's part of each tensor (safetensors slices):
q/k/v/gate/up are split by output rows, o/down by input columns at group boundaries
(balanced when the group count does not divide evenly; gate/up rows are cut at the same
points) with the anchor columns inside the slice re-based to slice-local indices and the
bias kept on rank 0 only (it must be added once before the all-reduce of the partial sums).
The INT8 head is split by vocabulary rows; a tied head's shard is a row view of the
replicated embedding.
"""
from __future__ import annotations

import json
import os
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch
import torch.nn as nn

from .symmetric_2bit_engine import (
    QuantizedEmbedding,
    QuantizedLinearHead,
    Symmetric2BitQuantizer,
    SymmetricOTF2BitLinear,
)

CONFIG_FILE = "otf_2bit_config.json"
MODEL_FILE = "otf_2bit_model.safetensors"
BASE_FILE = "otf_2bit_base.safetensors"

# otf_llm/run_symmetric_2bit.py:23-31 and otf_llm/convert_symmetric_2bit.py:30-38
DEFAULT_PROJECTIONS = [
    "self_attn.q_proj",
    "self_attn.k_proj",
    "self_attn.v_proj",
    "self_attn.o_proj",
    "mlp.gate_proj",
    "mlp.up_proj",
    "mlp.down_proj",
]
# Projections whose input dimension is split under tensor parallelism (their outputs are
# partial sums that an all-reduce completes); every other projection is split by rows.
ROW_PARALLEL = ("self_attn.o_proj", "mlp.down_proj")
FEEDS_ROW_PARALLEL_BY_GROUP = ("mlp.gate_proj", "mlp.up_proj")
LAYER_NORMS = ("input_layernorm", "post_attention_layernorm")
DEFAULT_GROUP_SIZE = 32


def read_config(model_dir: str) -> dict:
    """otf_2bit_config.json with the reference runner's defaults filled in."""
    with open(os.path.join(model_dir, CONFIG_FILE), "r", encoding="utf-8") as fh:
        cfg = json.load(fh)
    cfg.setdefault("group_size", DEFAULT_GROUP_SIZE)
    cfg.setdefault("projections", list(DEFAULT_PROJECTIONS))
    return cfg


def shard_bounds(n: int, rank: int, world: int, align: int = 1) -> Tuple[int, int]:
    """[lo, hi) of rank's part of n items cut at multiples of align, as evenly as the
    alignment allows (the split the decoder stack uses, decoder_stack.split_bounds)."""
    from .decoder_stack import split_bounds
    return split_bounds(n, rank, world, align)


def _get(f, key: str, rows: Optional[Tuple[int, int]] = None, cols: Optional[Tuple[int, int]] = None):
    """Read a tensor, or only rows/cols of it, from an open safetensors file."""
    if rows is None and cols is None:
        return f.get_tensor(key)
    sl = f.get_slice(key)
    r = slice(*rows) if rows is not None else slice(None)
    if cols is None:
        return sl[r]
    return sl[r, slice(*cols)]


@dataclass
class LinearShard:
    """Where a projection's tensor-parallel shard lies: dim 'out' (rows), 'in' (columns) or None."""
    dim: Optional[str] = None
    rank: int = 0
    world: int = 1
    align: int = 1          # column shards: cut rows at multiples of this


def load_linear(f, keys: set, prefix: str, group_size: int, device, shard: LinearShard = LinearShard()
                ) -> Optional[SymmetricOTF2BitLinear]:
    """One SymmetricOTF2BitLinear from the tensors under ``prefix`` (None if it has no codes)."""
    pk = f"{prefix}.packed_uint8"
    if pk not in keys:
        return None
    N, Kq = f.get_slice(pk).get_shape()
    K = Kq * 4
    G = group_size
    if K % G:
        raise ValueError(f"{pk}: d_in={K} is not a multiple of group_size={G}")
    sc_shape = tuple(f.get_slice(f"{prefix}.scales").get_shape())
    if sc_shape != (N, K // G):
        raise ValueError(f"{prefix}.scales has shape {sc_shape}; packed codes need ({N}, {K // G})")
    has_out = f"{prefix}.outlier_deltas" in keys and f"{prefix}.outlier_indices" in keys
    has_bias = f"{prefix}.bias" in keys
    rows = cols = None
    k0, k1 = 0, K
    if shard.world > 1 and shard.dim == "out":
        rows = shard_bounds(N, shard.rank, shard.world, shard.align)
    elif shard.world > 1 and shard.dim == "in":
        k0, k1 = shard_bounds(K, shard.rank, shard.world, G)
        cols = (k0, k1)
    elif shard.world > 1:
        raise ValueError(f"shard dim must be 'out' or 'in', got {shard.dim!r}")
    packed = _get(f, pk, rows, None if cols is None else (k0 // 4, k1 // 4))
    scales = _get(f, f"{prefix}.scales", rows, None if cols is None else (k0 // G, k1 // G))
    ov = oi = None
    if has_out:
        oi = f.get_tensor(f"{prefix}.outlier_indices").to(torch.long)
        ov = _get(f, f"{prefix}.outlier_deltas", rows)
        if cols is not None:
            sel = (oi >= k0) & (oi < k1)
            if bool(sel.any()):
                oi, ov = (oi[sel] - k0).contiguous(), ov[:, sel].contiguous()
            else:
                oi = ov = None
    bias = None
    if has_bias and not (cols is not None and shard.rank != 0):
        bias = _get(f, f"{prefix}.bias", rows)
    dev = torch.device(device)
    to = lambda t: None if t is None else t.contiguous().to(dev)  # noqa: E731
    from .decoder_stack import even_scale_rows
    return even_scale_rows(SymmetricOTF2BitLinear(to(packed), to(scales), k1 - k0, G, to(ov), to(oi), to(bias)))


@dataclass
class OTF2BitCheckpoint:
    """A loaded checkpoint (or this rank's shard of it), ready to run on the native kernels."""
    config: dict
    layers: List[Dict[str, SymmetricOTF2BitLinear]]
    embed: Optional[QuantizedEmbedding] = None
    head: Optional[nn.Module] = None            # QuantizedLinearHead, or VocabParallelHead when sharded
    head_tied: bool = False
    final_norm: Optional[torch.Tensor] = None
    layer_norms: List[Dict[str, torch.Tensor]] = field(default_factory=list)
    rank: int = 0
    world: int = 1

    @property
    def num_layers(self) -> int:
        return len(self.layers)

    @property
    def group_size(self) -> int:
        return int(self.config["group_size"])

    @property
    def projections(self) -> List[str]:
        return list(self.config["projections"])


def _layer_count(cfg: dict, model_keys: Sequence[str], num_layers: Optional[int]) -> int:
    if num_layers is not None:
        return int(num_layers)
    if "num_layers" in cfg:
        return int(cfg["num_layers"])
    idx = {int(k.split(".")[2]) for k in model_keys if k.startswith("model.layers.")}
    return (max(idx) + 1) if idx else 0


def load_checkpoint(model_dir: str, device="cuda", rank: int = 0, world: int = 1, group=None,
                    num_layers: Optional[int] = None, load_base: bool = True) -> OTF2BitCheckpoint:
    """Load a converted checkpoint directory onto ``device``, or rank ``rank`` of ``world`` shards.

    ``num_layers`` overrides the config's count (the reference falls back to the HF config's
    ``num_hidden_layers``, run_symmetric_2bit.py:74).  With ``world > 1`` the INT8 head is
    vocabulary-parallel (``VocabParallelHead`` over ``group``) and the embedding replicated.
    """
    from safetensors import safe_open

    cfg = read_config(model_dir)
    G = int(cfg["group_size"])
    projections = list(cfg["projections"])
    dev = torch.device(device)
    layers: List[Dict[str, SymmetricOTF2BitLinear]] = []
    with safe_open(os.path.join(model_dir, MODEL_FILE), framework="pt", device="cpu") as f:
        keys = set(f.keys())
        L = _layer_count(cfg, keys, num_layers)
        for i in range(L):
            mods: Dict[str, SymmetricOTF2BitLinear] = {}
            for proj in projections:
                # gate/up rows are cut at down_proj's group boundaries, so each rank's slice
                # of the intermediate activation is exactly its down_proj input slice
                align = G if proj in FEEDS_ROW_PARALLEL_BY_GROUP else 1
                shard = (LinearShard("in" if proj in ROW_PARALLEL else "out", rank, world, align) if world > 1
                         else LinearShard())
                m = load_linear(f, keys, f"model.layers.{i}.{proj}", G, dev, shard)
                if m is not None:
                    mods[proj] = m
            layers.append(mods)
    ck = OTF2BitCheckpoint(config=cfg, layers=layers, rank=rank, world=world)
    if load_base:
        _load_base(ck, os.path.join(model_dir, BASE_FILE), L, dev, rank, world, group)
    return ck


def _load_base(ck: OTF2BitCheckpoint, path: str, L: int, dev, rank: int, world: int, group) -> None:
    from safetensors import safe_open

    with safe_open(path, framework="pt", device="cpu") as f:
        keys = set(f.keys())
        if "model.embed_tokens.weight_int8" in keys:
            w = f.get_tensor("model.embed_tokens.weight_int8")
            with torch.device("meta"):                   # no placeholder allocation
                emb = QuantizedEmbedding(w.shape[0], w.shape[1])
            emb.weight_int8 = w.contiguous().to(dev)
            emb.scales = f.get_tensor("model.embed_tokens.scales").to(torch.float16).contiguous().to(dev)
            ck.embed = emb
        if "lm_head.weight_int8" in keys:
            V, D = f.get_slice("lm_head.weight_int8").get_shape()
            rows = shard_bounds(V, rank, world) if world > 1 else None
            with torch.device("meta"):
                head = QuantizedLinearHead(D, V if rows is None else rows[1] - rows[0])
            head.weight_int8 = _get(f, "lm_head.weight_int8", rows).contiguous().to(dev)
            head.scales = _get(f, "lm_head.scales", rows).to(torch.float16).contiguous().to(dev)
            ck.head_tied = False
        elif ck.embed is not None:
            V, D = ck.embed.weight_int8.shape
            rows = shard_bounds(V, rank, world) if world > 1 else (0, V)
            with torch.device("meta"):
                head = QuantizedLinearHead(D, rows[1] - rows[0])
            # Tied: the head reads the embedding's own buffers (a row view when sharded).
            head.weight_int8 = ck.embed.weight_int8[rows[0]:rows[1]]
            head.scales = ck.embed.scales[rows[0]:rows[1]]
            rows = rows if world > 1 else None
            ck.head_tied = True
        else:
            head, rows = None, None
        if head is not None and world > 1:
            from .vocab_parallel import VocabParallelHead
            head = VocabParallelHead(head, rows[0], V, group)
        ck.head = head
        if "model.norm.weight" in keys:
            ck.final_norm = f.get_tensor("model.norm.weight").to(dev)
        ck.layer_norms = []
        for i in range(L):
            norms = {}
            for ln in LAYER_NORMS:
                k = f"model.layers.{i}.{ln}.weight"
                if k in keys:
                    norms[ln] = f.get_tensor(k).to(dev)
            ck.layer_norms.append(norms)


# -- writing ---------------------------------------------------------------------------

FORMAT_NAME = "OTF-Engine-v4.1-Symmetric-2Bit"      # the "architecture" value of the format


def save_checkpoint(output_dir: str, quant_tensors: Dict[str, torch.Tensor], base_tensors: Dict[str, torch.Tensor],
                    group_size: int, outlier_ratio: float, num_layers: int,
                    projections: Sequence[str] = DEFAULT_PROJECTIONS, source_model: str = "") -> None:
    """Write the three files of the format from already-keyed host tensors."""
    import time

    from safetensors.torch import save_file

    os.makedirs(output_dir, exist_ok=True)
    cpu = lambda d: {k: v.detach().cpu().contiguous() for k, v in d.items()}  # noqa: E731
    save_file(cpu(base_tensors), os.path.join(output_dir, BASE_FILE))
    save_file(cpu(quant_tensors), os.path.join(output_dir, MODEL_FILE))
    cfg = {"architecture": FORMAT_NAME, "group_size": int(group_size), "outlier_ratio": float(outlier_ratio),
           "num_layers": int(num_layers), "projections": list(projections), "source_model": source_model,
           "created_by": "otf_llm b200", "timestamp": time.strftime("%Y-%m-%d %H:%M:%S")}
    with open(os.path.join(output_dir, CONFIG_FILE), "w", encoding="utf-8") as fh:
        json.dump(cfg, fh, indent=4)


def convert_symmetric_model(model_dir: str, output_dir: str, group_size: int = 32, outlier_ratio: float = 0.035,
                            profile_path: Optional[str] = None, act_profiles: Optional[Dict[str, torch.Tensor]] = None,
                            device=None) -> None:
    """Convert a local Hugging Face safetensors model directory to the 2-bit + INT8 format.

    Same products as otf_llm/convert_symmetric_2bit.py:51-207: INT8 embedding and (if the
    source has one) an independent INT8 head, the norms copied through, and every
    projection quantized by ``Symmetric2BitQuantizer(group_size, outlier_ratio)`` from its
    fp16 weight and its activation profile (``act_profiles["model.layers.{i}.{proj}"]``,
    or a ``torch.save``d dict of them at ``profile_path``; none means column norms only).
    Quantization runs on ``device`` (default: the first GPU when there is one).  Hub
    download and calibration-profile generation are outside this package.
    """
    from safetensors import safe_open

    if act_profiles is None and profile_path is not None:
        act_profiles = torch.load(profile_path, map_location="cpu")
    act_profiles = act_profiles or {}
    dev = torch.device(device if device is not None else ("cuda" if torch.cuda.is_available() else "cpu"))
    files = sorted(os.path.join(model_dir, n) for n in os.listdir(model_dir) if n.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {model_dir}")
    where: Dict[str, str] = {}
    for path in files:
        with safe_open(path, framework="pt", device="cpu") as f:
            for k in f.keys():
                where[k] = path

    def tensor(key: str) -> torch.Tensor:
        with safe_open(where[key], framework="pt", device="cpu") as f:
            return f.get_tensor(key)

    num_layers = len({int(k.split(".")[2]) for k in where if k.startswith("model.layers.")})
    base: Dict[str, torch.Tensor] = {}
    if "model.embed_tokens.weight" in where:
        w = tensor("model.embed_tokens.weight")
        with torch.device("meta"):
            emb = QuantizedEmbedding(w.shape[0], w.shape[1])
        emb.quantize_from_fp16(w)
        base["model.embed_tokens.weight_int8"], base["model.embed_tokens.scales"] = emb.weight_int8, emb.scales
    if "lm_head.weight" in where:
        w = tensor("lm_head.weight")
        with torch.device("meta"):
            head = QuantizedLinearHead(w.shape[1], w.shape[0])
        head.quantize_from_fp16(w)
        base["lm_head.weight_int8"], base["lm_head.scales"] = head.weight_int8, head.scales
    if "model.norm.weight" in where:
        base["model.norm.weight"] = tensor("model.norm.weight")
    for i in range(num_layers):
        for ln in LAYER_NORMS:
            k = f"model.layers.{i}.{ln}.weight"
            if k in where:
                base[k] = tensor(k)

    quantizer = Symmetric2BitQuantizer(group_size=group_size, outlier_ratio=outlier_ratio)
    quant: Dict[str, torch.Tensor] = {}
    for i in range(num_layers):
        for proj in DEFAULT_PROJECTIONS:
            pfx = f"model.layers.{i}.{proj}"
            if f"{pfx}.weight" not in where:
                continue
            W = tensor(f"{pfx}.weight").to(dev).to(torch.float16)
            if f"{pfx}.bias" in where:
                quant[f"{pfx}.bias"] = tensor(f"{pfx}.bias")
            prof = act_profiles.get(pfx)
            packed, scales, ov, oi = quantizer.quantize_tensor(W, activation_profile=None if prof is None else prof.to(dev))
            quant[f"{pfx}.packed_uint8"] = packed.cpu()
            quant[f"{pfx}.scales"] = scales.cpu()
            if ov is not None and oi is not None:
                quant[f"{pfx}.outlier_deltas"] = ov.cpu()
                quant[f"{pfx}.outlier_indices"] = oi.cpu()
            del W
    save_checkpoint(output_dir, quant, base, group_size, outlier_ratio, num_layers, DEFAULT_PROJECTIONS,
                    source_model=model_dir)


# -- Hugging Face injection ----------------------------------------------------------------

def _set_sub(root: nn.Module, path: str, module: nn.Module) -> None:
    parts = path.split(".")
    for p in parts[:-1]:
        root = getattr(root, p)
    setattr(root, parts[-1], module)


def inject_into_model(model: nn.Module, ck: OTF2BitCheckpoint) -> nn.Module:
    """Put a loaded checkpoint into a Hugging Face causal LM (``model.model.layers[i]``).

    Follows otf_llm/run_symmetric_2bit.py:112-187: the INT8 embedding replaces
    ``embed_tokens``, the INT8 head replaces ``lm_head`` (tied: it shares the embedding's
    buffers), the norm weights are copied in, and every projection with codes becomes a
    ``SymmetricOTF2BitLinear``.  Norms the checkpoint lacks are set to 1 (the reference
    leaves them as whatever ``to_empty`` allocated).
    """
    if ck.world > 1:
        raise ValueError("a tensor-parallel shard cannot be injected into a single-device model")
    inner = model.model
    if ck.embed is not None:
        inner.embed_tokens = ck.embed
    if ck.head is not None:
        model.lm_head = ck.head
    with torch.no_grad():
        if getattr(inner, "norm", None) is not None and getattr(inner.norm, "weight", None) is not None:
            if ck.final_norm is not None:
                inner.norm.weight.copy_(ck.final_norm.to(inner.norm.weight.device))
            else:
                inner.norm.weight.fill_(1.0)
        for i, layer in enumerate(inner.layers[: ck.num_layers]):
            norms = ck.layer_norms[i] if i < len(ck.layer_norms) else {}
            for ln in LAYER_NORMS:
                mod = getattr(layer, ln, None)
                if mod is None or getattr(mod, "weight", None) is None:
                    continue
                if ln in norms:
                    mod.weight.copy_(norms[ln].to(mod.weight.device))
                else:
                    mod.weight.fill_(1.0)
    for i, mods in enumerate(ck.layers):
        for proj, m in mods.items():
            _set_sub(inner.layers[i], proj, m)
    return model


def _rebuild_rotary(model: nn.Module, device) -> None:
    """Recreate rotary-embedding modules after ``to_empty`` left their inv_freq unset
    (the reference recomputes inv_freq in place, run_symmetric_2bit.py:34-49)."""
    found = [(n, m) for n, m in model.named_modules() if "RotaryEmbedding" in type(m).__name__]
    for name, mod in found:
        fresh = type(mod)(config=mod.config, device=device)
        _set_sub(model, name, fresh)


def build_hf_model(hf_config, model_dir: str, device="cuda", dtype=torch.float16) -> nn.Module:
    """A Hugging Face causal LM for ``hf_config`` running the checkpoint in ``model_dir``.

    The skeleton is built on the meta device, the modules the checkpoint supplies are
    replaced before anything is allocated, and the rest (norms, rotary tables) is
    materialised on ``device`` -- run_symmetric_2bit.py:81-110 and :187.
    """
    from transformers import AutoModelForCausalLM

    cfg = read_config(model_dir)
    with torch.device("meta"):
        model = AutoModelForCausalLM.from_config(hf_config, dtype=dtype)
    model.model.embed_tokens = nn.Identity()
    model.lm_head = nn.Identity()
    for layer in model.model.layers:
        for proj in cfg["projections"]:
            _set_sub(layer, proj, nn.Identity())
    model = model.to_empty(device=device)
    model.requires_grad_(False)
    ck = load_checkpoint(model_dir, device=device, num_layers=len(model.model.layers))
    inject_into_model(model, ck)
    _rebuild_rotary(model, device)
    return model.eval()
