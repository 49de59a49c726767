"""GPU runs of checkpoints the reference converter wrote (tests/golden/ckpt_*): every loaded
projection against the oracle, a Hugging Face model with the checkpoint injected against
the same model with dense dequantized weights, and greedy decode steps through the
checkpoint against a CPU restatement built on the oracle."""
import os

import numpy as np
import pytest
import torch

from conftest import GOLDEN, rel_err
from oracle import oracle

pytestmark = pytest.mark.gpu

# name -> (HF config class, head_dim)
MODELS = {"ckpt_tied": ("Qwen2Config", 16), "ckpt_untied": ("LlamaConfig", 32)}


def _np(t):
    return None if t is None else t.detach().cpu().numpy()


def _oracle_lin(m, x16):
    return oracle.linear_f32(x16, _np(m.packed_uint8), _np(m.scales), m.group_size,
                             mask=_np(m.outlier_mask_vector), outlier_idx=_np(m.outlier_indices),
                             outlier_vals=_np(m.outliers_fp16), bias=_np(m.bias) if m.has_bias else None)


def _dense_weight(m):
    """Dense fp32 [N, K]: the oracle's dequant of the codes, anchor columns from outliers_fp16."""
    eye = np.eye(m.d_in, dtype=np.float16)
    wt = oracle.linear_f32(eye, _np(m.packed_uint8), _np(m.scales), m.group_size, clamp=False)
    w = torch.from_numpy(wt.T.copy())
    if m.has_outliers:
        w[:, m.outlier_indices.cpu()] = m.outliers_fp16.cpu().float()
    return w


@pytest.mark.parametrize("name", list(MODELS))
def test_loaded_projections_match_oracle(name, cuda_dev):
    from otf_llm.checkpoint import load_checkpoint
    ck = load_checkpoint(os.path.join(GOLDEN, name), device=cuda_dev)
    rng = np.random.default_rng(3)
    for mods in ck.layers:
        for proj, m in mods.items():
            for M in (1, 3):
                x = rng.standard_normal((M, m.d_in)).astype(np.float16)
                y = m(torch.from_numpy(x).to(cuda_dev))
                assert rel_err(_np(y.float()), _oracle_lin(m, x)) < 1e-3, (proj, M)


def _hf_config(name, vocab, hidden, inter, layers, heads, kv_heads):
    import transformers
    cls = getattr(transformers, MODELS[name][0])
    return cls(vocab_size=vocab, hidden_size=hidden, intermediate_size=inter, num_hidden_layers=layers,
               num_attention_heads=heads, num_key_value_heads=kv_heads, max_position_embeddings=64,
               tie_word_embeddings=(name == "ckpt_tied"))


@pytest.mark.parametrize("name", list(MODELS))
def test_hf_model_with_checkpoint_matches_dense(name, cuda_dev):
    """Logits of the injected model vs the same architecture in fp32 with the checkpoint's
    dequantized weights.  Tolerance 2e-2 of max|logit|: the injected model runs the
    activations in fp16 (as the reference runner does), the dense one in fp32."""
    import json

    from transformers import AutoModelForCausalLM

    from otf_llm.checkpoint import build_hf_model, load_checkpoint
    d = os.path.join(GOLDEN, name)
    meta = json.load(open(os.path.join(d, "source.json")))
    cfg = _hf_config(name, meta["vocab"], meta["hidden"], meta["intermediate"], meta["layers"], meta["heads"],
                     meta["kv_heads"])
    model = build_hf_model(cfg, d, device=cuda_dev)
    ids = torch.from_numpy(np.random.default_rng(4).integers(0, meta["vocab"], (1, 12))).to(cuda_dev)
    with torch.inference_mode():
        got = model(ids).logits.float()

    ck = load_checkpoint(d, device="cpu")
    dense = AutoModelForCausalLM.from_config(cfg, dtype=torch.float32).eval()
    emb = ck.embed.weight_int8.float() * ck.embed.scales.float()
    with torch.no_grad():
        dense.model.embed_tokens.weight.copy_(emb)
        dense.lm_head.weight.copy_(ck.head.weight_int8.float() * ck.head.scales.float())
        dense.model.norm.weight.copy_(ck.final_norm.float())
        for i, layer in enumerate(dense.model.layers):
            layer.input_layernorm.weight.copy_(ck.layer_norms[i]["input_layernorm"].float())
            layer.post_attention_layernorm.weight.copy_(ck.layer_norms[i]["post_attention_layernorm"].float())
            for proj, m in ck.layers[i].items():
                lin = layer.get_submodule(proj)
                lin.weight.copy_(_dense_weight(m))
                if lin.bias is not None:
                    lin.bias.copy_(m.bias.float() if m.has_bias else torch.zeros_like(lin.bias))
    dense = dense.to(cuda_dev)
    with torch.inference_mode():
        ref = dense(ids).logits.float()
    assert got.shape == ref.shape
    assert rel_err(_np(got), _np(ref)) < 2e-2


def _cpu_decode_step(ck, tok, head_dim, eps=1e-5):
    """One single-position decode step on the CPU: oracle embedding / linears / head,
    HF-style RMSNorm (fp32 normalise, fp16 round, fp16 weight multiply), attention over
    one key = V repeated over each KV head's query heads."""
    def rms(x, w):
        v = x.float()
        v = (v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + eps)).half()
        return (w.cpu() * v).half()

    def lin(m, x):
        return torch.from_numpy(_oracle_lin(m, x.numpy()))

    h = torch.from_numpy(oracle.i8_embed(np.array([tok]), _np(ck.embed.weight_int8), _np(ck.embed.scales)))
    for i, mods in enumerate(ck.layers):
        nrm = ck.layer_norms[i]
        xn = rms(h, nrm["input_layernorm"])
        v = lin(mods["self_attn.v_proj"], xn).half()
        rep = mods["self_attn.q_proj"].out_features // mods["self_attn.k_proj"].out_features
        attn = v.view(-1, 1, head_dim).expand(-1, rep, head_dim).reshape(1, -1)
        h = (lin(mods["self_attn.o_proj"], attn) + h.float()).half()
        xn = rms(h, nrm["post_attention_layernorm"])
        g = lin(mods["mlp.gate_proj"], xn).half()
        u = lin(mods["mlp.up_proj"], xn).half()
        a = torch.nn.functional.silu(g.float()).half() * u
        h = (lin(mods["mlp.down_proj"], a) + h.float()).half()
    xn = rms(h, ck.final_norm)
    return oracle.i8_head(xn.numpy(), _np(ck.head.weight_int8), _np(ck.head.scales))


@pytest.mark.parametrize("persistent", [False, True])
@pytest.mark.parametrize("name", list(MODELS))
def test_checkpoint_decoder_matches_cpu_step(name, persistent, cuda_dev):
    from otf_llm.checkpoint import load_checkpoint
    from otf_llm.decoder_stack import CheckpointDecoder
    d = os.path.join(GOLDEN, name)
    hd = MODELS[name][1]
    ck = load_checkpoint(d, device=cuda_dev)
    dec = CheckpointDecoder(ck, head_dim=hd, persistent=persistent)
    assert (dec.stack.mk is not None) == persistent
    V = ck.head.out_features
    tok = 5
    for _ in range(3):
        logits = torch.empty(1, V, dtype=torch.float32, device=cuda_dev)
        nxt = dec.step(torch.tensor([tok], device=cuda_dev), logits=logits)
        ref = _cpu_decode_step(ck, tok, hd)
        assert rel_err(_np(logits), ref) < 3e-3
        assert int(nxt) == int(torch.argmax(logits[0]))
        tok = int(nxt)
