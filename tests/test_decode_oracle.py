"""The oracle's restatement of the reference engine's decode step (oracle/decode.py) pinned
against the reference engine itself: per-token KV-cache decode logits and greedy picks the
reference's modules produced inside Hugging Face's model on the converted-checkpoint fixtures
(tests/golden/engine_ckpt_*.npz, written by tests/golden/make_engine_logits.py)."""
import json
import os

import numpy as np
import pytest

from conftest import GOLDEN, rel_err
from oracle import decode, oracle

safetensors_np = pytest.importorskip("safetensors.numpy")


def _decoder(name: str, fx, max_pos: int = 64) -> decode.Decoder:
    d = os.path.join(GOLDEN, name)
    meta = json.load(open(os.path.join(d, "source.json")))
    qcfg = json.load(open(os.path.join(d, "otf_2bit_config.json")))
    base = safetensors_np.load_file(os.path.join(d, "otf_2bit_base.safetensors"))
    quant = safetensors_np.load_file(os.path.join(d, "otf_2bit_model.safetensors"))
    layers, norms = [], []
    for i in range(meta["layers"]):
        l = {}
        for proj in qcfg["projections"]:
            p = f"model.layers.{i}.{proj}"
            K = quant[f"{p}.packed_uint8"].shape[1] * 4
            idx = quant.get(f"{p}.outlier_indices")
            mask = None
            if idx is not None:
                mask = np.ones(K, np.float16)
                mask[idx] = 0
            l[proj.split(".")[-1]] = decode.projection(quant[f"{p}.packed_uint8"], quant[f"{p}.scales"],
                                                       qcfg["group_size"], mask=mask, idx=idx,
                                                       ov=quant.get(f"{p}.outlier_deltas"),
                                                       bias=quant.get(f"{p}.bias"))
        layers.append(l)
        norms.append((base[f"model.layers.{i}.input_layernorm.weight"],
                      base[f"model.layers.{i}.post_attention_layernorm.weight"]))
    hw, hs = (base["lm_head.weight_int8"], base["lm_head.scales"]) if "lm_head.weight_int8" in base else \
        (base["model.embed_tokens.weight_int8"], base["model.embed_tokens.scales"])
    return decode.Decoder(layers, norms, base["model.norm.weight"], base["model.embed_tokens.weight_int8"],
                          base["model.embed_tokens.scales"], hw, hs, heads=meta["heads"], kv_heads=meta["kv_heads"],
                          head_dim=int(fx["head_dim"]), rope_theta=float(fx["rope_theta"]),
                          rms_eps=float(fx["rms_eps"]), max_pos=max_pos)


@pytest.mark.parametrize("name", ["ckpt_tied", "ckpt_untied"])
def test_decode_matches_reference_engine(name):
    fx = np.load(os.path.join(GOLDEN, f"engine_{name}.npz"))
    dec = _decoder(name, fx)
    prompt, picks, ref = fx["prompt"], fx["picks"], fx["logits"]
    got = []
    assert dec.generate(prompt, len(picks), logits_out=got) == picks.tolist()
    got = np.stack(got)
    assert got.shape == ref.shape
    err = rel_err(got, ref)
    print(f"{name}: decode logits rel err {err:.2e} over {len(got)} steps")
    # the reference's head multiplies in fp16 (symmetric_2bit_engine.py:84-88), the oracle's in fp32
    assert err < 5e-3


def test_rope_table_matches_hf():
    transformers = pytest.importorskip("transformers")
    torch = pytest.importorskip("torch")
    cfg = transformers.LlamaConfig(hidden_size=512, num_attention_heads=4, head_dim=128, rope_theta=500000.0,
                                   max_position_embeddings=600)
    rot = transformers.models.llama.modeling_llama.LlamaRotaryEmbedding(cfg, device="cpu")
    pos = torch.arange(600).view(1, -1)
    cos, sin = rot(torch.zeros(1, 1, 8, dtype=torch.float16), pos)
    c, s = decode.rope_table(128, 500000.0, 600)
    assert np.array_equal(cos[0].numpy(), c) and np.array_equal(sin[0].numpy(), s)


def test_decode_cache_handoff_and_bounds():
    """Decoding from a cache another run filled gives the same logits as running the prompt."""
    fx = np.load(os.path.join(GOLDEN, "engine_ckpt_untied.npz"))
    a = _decoder("ckpt_untied", fx)
    la = []
    a.generate(fx["prompt"], 3, logits_out=la)
    b = _decoder("ckpt_untied", fx)
    P = len(fx["prompt"])
    for li in range(len(b.layers)):
        b.set_cache(li, a.kc[li][:P - 1], a.vc[li][:P - 1])
    lb = []
    b.generate(fx["prompt"][P - 1:], 3, start=P - 1, logits_out=lb)
    assert all(np.array_equal(x, y) for x, y in zip(la[P - 1:], lb))
    with pytest.raises(IndexError):
        a.step(0, 64)
    assert oracle.argmax_rows(la[-1][None])[0] == int(np.argmax(la[-1]))
