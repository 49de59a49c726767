"""Generate ``engine_<ckpt>.npz``: the reference engine's per-token decode logits on the
converted-checkpoint fixtures ``ckpt_tied/`` and ``ckpt_untied/``.

The engine is assembled on the CPU the way the reference runner assembles it
(otf_llm/run_symmetric_2bit.py:88-189): a Hugging Face causal-LM skeleton on the meta
device, embedding / head / projections replaced by identities, ``to_empty``, then the
reference's own ``QuantizedEmbedding``, ``QuantizedLinearHead`` (tied to the embedding when
the base file has no ``lm_head`` rows) and ``SymmetricOTF2BitLinear`` modules filled from
the checkpoint, and the RMSNorm weights copied in.  The runner's ``fix_rotary_embeddings``
(:34-49) reads ``config.rope_theta`` and the rotary module's ``dim``, which transformers 5
no longer has (it would fall back to theta 1e6 and dim 128); the script instead rebuilds the
rotary module from the config, the table that function computes under transformers 4.

Decoding is greedy with a KV cache, one token per forward (the path ``model.generate``
takes): the prompt, then new tokens.  Saved per step: the fp32 logits; plus the prompt, the
picks, and the rotary theta / RMSNorm epsilon the config used.

    python tests/golden/make_engine_logits.py --reference /root/reference

The tests never import the reference; they read these files.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

import numpy as np
import torch
import torch.nn as nn

OUT = os.path.dirname(os.path.abspath(__file__))
# fixture -> (HF config class, prompt length, new tokens)
MODELS = {"ckpt_tied": ("Qwen2Config", 10, 6), "ckpt_untied": ("LlamaConfig", 10, 6)}


def _set_sub(root: nn.Module, path: str, mod: nn.Module) -> None:
    parts = path.split(".")
    for p in parts[:-1]:
        root = getattr(root, p)
    setattr(root, parts[-1], mod)


def build_engine(name: str, cls_name: str):
    import transformers
    from safetensors.torch import load_file
    from otf_llm.symmetric_2bit_engine import QuantizedEmbedding, QuantizedLinearHead, SymmetricOTF2BitLinear

    d = os.path.join(OUT, name)
    meta = json.load(open(os.path.join(d, "source.json")))
    qcfg = json.load(open(os.path.join(d, "otf_2bit_config.json")))
    cfg = getattr(transformers, cls_name)(
        vocab_size=meta["vocab"], hidden_size=meta["hidden"], intermediate_size=meta["intermediate"],
        num_hidden_layers=meta["layers"], num_attention_heads=meta["heads"], num_key_value_heads=meta["kv_heads"],
        max_position_embeddings=64, tie_word_embeddings=meta["tied"])
    with torch.device("meta"):
        model = transformers.AutoModelForCausalLM.from_config(cfg, dtype=torch.float16)
    model.model.embed_tokens = nn.Identity()
    model.lm_head = nn.Identity()
    for layer in model.model.layers:
        for proj in qcfg["projections"]:
            _set_sub(layer, proj, nn.Identity())
    model = model.to_empty(device="cpu")
    model.requires_grad_(False)
    base = load_file(os.path.join(d, "otf_2bit_base.safetensors"))
    quant = load_file(os.path.join(d, "otf_2bit_model.safetensors"))
    emb = QuantizedEmbedding(cfg.vocab_size, cfg.hidden_size)
    emb.weight_int8.copy_(base["model.embed_tokens.weight_int8"])
    emb.scales.copy_(base["model.embed_tokens.scales"])
    model.model.embed_tokens = emb
    head = QuantizedLinearHead(cfg.hidden_size, cfg.vocab_size)
    if "lm_head.weight_int8" in base:
        head.weight_int8.copy_(base["lm_head.weight_int8"])
        head.scales.copy_(base["lm_head.scales"])
    else:
        head.weight_int8, head.scales = emb.weight_int8, emb.scales
    model.lm_head = head
    model.model.norm.weight.copy_(base["model.norm.weight"])
    G = qcfg["group_size"]
    for i, layer in enumerate(model.model.layers):
        for ln in ("input_layernorm", "post_attention_layernorm"):
            getattr(layer, ln).weight.copy_(base[f"model.layers.{i}.{ln}.weight"])
        for proj in qcfg["projections"]:
            p = f"model.layers.{i}.{proj}"
            packed = quant[f"{p}.packed_uint8"]
            _set_sub(layer, proj, SymmetricOTF2BitLinear(packed, quant[f"{p}.scales"], packed.shape[1] * 4, G,
                                                         quant.get(f"{p}.outlier_deltas"),
                                                         quant.get(f"{p}.outlier_indices"), quant.get(f"{p}.bias")))
    model.model.rotary_emb = type(model.model.rotary_emb)(config=cfg, device="cpu")
    return model.eval(), cfg, meta


@torch.inference_mode()
def decode(model, ids, new_tokens):
    from transformers import DynamicCache
    cache = DynamicCache()
    feed = [int(t) for t in ids]
    logits, picks = [], []
    while len(picks) < new_tokens:
        step = len(logits)
        tok = feed[step] if step < len(feed) else picks[-1]
        out = model(input_ids=torch.tensor([[tok]]), past_key_values=cache, use_cache=True)
        lg = out.logits[0, -1].float()
        logits.append(lg.numpy().copy())
        if step + 1 >= len(feed):
            picks.append(int(lg.argmax()))
    return np.stack(logits), picks        # logits of the P prompt steps and the first T-1 picks


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("OTF_REFERENCE_DIR"),
                    help="directory holding the reference's otf_llm package (read-only)")
    ref = ap.parse_args(argv).reference
    if not ref or not os.path.isdir(os.path.join(ref, "otf_llm")):
        ap.error("give the reference's source tree with --reference or OTF_REFERENCE_DIR")
    sys.path.insert(0, ref)
    torch.manual_seed(0)
    for name, (cls_name, P, T) in MODELS.items():
        model, cfg, meta = build_engine(name, cls_name)
        prompt = np.random.default_rng(7).integers(0, meta["vocab"], P)
        logits, picks = decode(model, prompt, T)
        path = os.path.join(OUT, f"engine_{name}.npz")
        np.savez(path, prompt=prompt.astype(np.int64), logits=logits.astype(np.float32),
                 picks=np.array(picks, dtype=np.int64), rope_theta=float(cfg.rope_parameters["rope_theta"]),
                 rms_eps=float(cfg.rms_norm_eps), head_dim=int(meta["hidden"] // meta["heads"]),
                 source="HF %s + QuantizedEmbedding / SymmetricOTF2BitLinear / QuantizedLinearHead "
                        "(otf_llm v4.1.0), CPU, KV-cache greedy decode" % cls_name)
        print("wrote", path, "picks", picks)


if __name__ == "__main__":
    main()
