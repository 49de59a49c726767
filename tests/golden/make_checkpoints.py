"""Generate the converted-checkpoint fixtures ``ckpt_tied/`` and ``ckpt_untied/``.

Each fixture directory holds a tiny Llama-format source model (``source.safetensors``,
Hugging Face key names, fp16), the activation profile it was converted with
(``profile.safetensors``), and the three files the reference converter wrote for it:
``otf_2bit_config.json``, ``otf_2bit_model.safetensors`` and
``otf_2bit_base.safetensors``.

The outputs come from running the reference converter itself,
``otf_llm.convert_symmetric_2bit.convert_symmetric_model`` (GT-Labs-AI/otf-llm-engine,
otf_llm v4.1.0), unmodified, on CPU.  It moves each weight to the GPU with
``Tensor.cuda()`` (otf_llm/convert_symmetric_2bit.py:168, :177); this script makes that
call return the tensor itself, so the same quantizer arithmetic runs on the host.
Run where the reference's source tree is available (read-only), named by --reference or
the OTF_REFERENCE_DIR environment variable:

    python tests/golden/make_checkpoints.py --reference /root/reference

The tests never import the reference; they read these files.
"""
from __future__ import annotations

import argparse
import json
import os
import shutil
import sys
import tempfile

import torch
from safetensors.torch import save_file

OUT = os.path.dirname(os.path.abspath(__file__))

# name: (hidden, intermediate, layers, heads, kv_heads, vocab, tied, qkv_bias, group_size, outlier_ratio, seed)
FIXTURES = {
    "ckpt_tied": (64, 128, 2, 4, 2, 64, True, True, 32, 0.035, 11),
    "ckpt_untied": (128, 192, 1, 4, 2, 80, False, False, 64, 0.02, 12),
}

PROJ = ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
        "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj")


def source_model(hidden, inter, layers, heads, kv_heads, vocab, tied, qkv_bias, seed):
    """Seeded fp16 weights under Hugging Face Llama key names, plus per-projection profiles."""
    g = torch.Generator().manual_seed(seed)
    hd = hidden // heads
    shapes = {"self_attn.q_proj": (heads * hd, hidden), "self_attn.k_proj": (kv_heads * hd, hidden),
              "self_attn.v_proj": (kv_heads * hd, hidden), "self_attn.o_proj": (hidden, heads * hd),
              "mlp.gate_proj": (inter, hidden), "mlp.up_proj": (inter, hidden), "mlp.down_proj": (hidden, inter)}
    sd, prof = {}, {}
    sd["model.embed_tokens.weight"] = (torch.randn(vocab, hidden, generator=g) * 0.02).half()
    if not tied:
        sd["lm_head.weight"] = (torch.randn(vocab, hidden, generator=g) * 0.02).half()
    sd["model.norm.weight"] = (1.0 + 0.1 * torch.randn(hidden, generator=g)).half()
    for i in range(layers):
        for ln in ("input_layernorm", "post_attention_layernorm"):
            sd[f"model.layers.{i}.{ln}.weight"] = (1.0 + 0.1 * torch.randn(hidden, generator=g)).half()
        for p in PROJ:
            n, k = shapes[p]
            sd[f"model.layers.{i}.{p}.weight"] = (torch.randn(n, k, generator=g) * 0.02).half()
            if qkv_bias and p in PROJ[:3]:
                sd[f"model.layers.{i}.{p}.bias"] = (torch.randn(n, generator=g) * 0.01).half()
            a = torch.randn(k, generator=g).abs()
            a[torch.randperm(k, generator=g)[: max(1, k // 100)]] *= 20.0
            prof[f"model.layers.{i}.{p}"] = a.contiguous()
    return sd, prof


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("OTF_REFERENCE_DIR"),
                    help="directory holding the reference's otf_llm package (read-only)")
    ref = ap.parse_args(argv).reference
    if not ref or not os.path.isdir(os.path.join(ref, "otf_llm")):
        ap.error("give the reference's source tree with --reference or OTF_REFERENCE_DIR")
    sys.path.insert(0, ref)
    torch.Tensor.cuda = lambda self, *a, **k: self      # run the converter's quantizer on the host
    from otf_llm.convert_symmetric_2bit import convert_symmetric_model

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    for name, (h, i, L, nh, nkv, V, tied, qb, G, ratio, seed) in FIXTURES.items():
        sd, prof = source_model(h, i, L, nh, nkv, V, tied, qb, seed)
        dst = os.path.join(OUT, name)
        os.makedirs(dst, exist_ok=True)
        with tempfile.TemporaryDirectory() as tmp:
            src = os.path.join(tmp, "tiny_llama")
            os.makedirs(src)
            save_file(sd, os.path.join(src, "model.safetensors"))
            torch.save(prof, os.path.join(tmp, "profile.pt"))
            out = os.path.join(tmp, "out")
            cwd = os.getcwd()
            os.chdir(tmp)
            try:
                convert_symmetric_model("tiny_llama", out, group_size=G, outlier_ratio=ratio,
                                        profile_path=os.path.join(tmp, "profile.pt"))
            finally:
                os.chdir(cwd)
            for f in ("otf_2bit_config.json", "otf_2bit_model.safetensors", "otf_2bit_base.safetensors"):
                path = os.path.join(out, f)
                if not os.path.exists(path):
                    raise SystemExit(f"reference converter wrote no {f} for {name}")
                shutil.copyfile(path, os.path.join(dst, f))
        cfg_path = os.path.join(dst, "otf_2bit_config.json")
        with open(cfg_path) as fh:
            cfg = json.load(fh)
        cfg["timestamp"] = "fixture"                    # keep regenerated files byte-stable
        with open(cfg_path, "w") as fh:
            json.dump(cfg, fh, indent=4)
        save_file(sd, os.path.join(dst, "source.safetensors"))
        save_file(prof, os.path.join(dst, "profile.safetensors"))
        meta = {"hidden": h, "intermediate": i, "layers": L, "heads": nh, "kv_heads": nkv, "vocab": V,
                "tied": tied, "qkv_bias": qb, "group_size": G, "outlier_ratio": ratio, "seed": seed}
        with open(os.path.join(dst, "source.json"), "w") as fh:
            json.dump(meta, fh, indent=2)
        print("wrote", dst)


if __name__ == "__main__":
    main()
