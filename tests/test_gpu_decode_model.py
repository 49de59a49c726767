"""Greedy decoding with a KV cache on the native kernels (otf_llm.decode_model): the RoPE +
cache-write kernel against HF's rotary arithmetic, the decode attention against an fp32
softmax(q k^T) v, and a whole small model against HF's LlamaForCausalLM running the same
2-bit / INT8 modules."""
import math

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _lib():
    from otf_llm import _native
    return _native


def test_rope_kv_matches_hf_rotary(cuda_dev):
    transformers = pytest.importorskip("transformers")
    from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
    from otf_llm.decode_model import ModelConfig, rope_table
    N = _lib()
    cfg = ModelConfig(layers=1, hidden=512, intermediate=512, heads=8, kv_heads=2, head_dim=64, vocab=16, max_pos=40)
    g = torch.Generator(device=cuda_dev).manual_seed(0)
    q = torch.randn(cfg.heads * cfg.head_dim, generator=g, device=cuda_dev).half()
    k = torch.randn(cfg.kv_heads * cfg.head_dim, generator=g, device=cuda_dev).half()
    v = torch.randn(cfg.kv_heads * cfg.head_dim, generator=g, device=cuda_dev).half()
    cs = rope_table(cfg, cuda_dev)
    kc = torch.zeros(cfg.max_pos, cfg.kv_heads * cfg.head_dim, dtype=torch.float16, device=cuda_dev)
    vc = torch.zeros_like(kc)
    p = 37
    pos = torch.tensor([p], dtype=torch.int32, device=cuda_dev)
    hcfg = transformers.LlamaConfig(hidden_size=512, num_attention_heads=8, num_key_value_heads=2, head_dim=64,
                                    rope_theta=cfg.rope_theta, max_position_embeddings=cfg.max_pos)
    # The table is HF's default rotary cos/sin (equal bit for bit when both are computed on the
    # CPU; HF's GPU path forms the angles with a matmul that may round differently), so the
    # kernel is checked against HF's rotary arithmetic on this same table.
    rot = transformers.models.llama.modeling_llama.LlamaRotaryEmbedding(hcfg, device="cpu")
    cos_c, sin_c = rot(torch.zeros(1, 1, 8, dtype=torch.float16), torch.tensor([[p]]))
    assert torch.equal(cos_c.view(-1), rope_table(cfg, "cpu")[p, 0]) and torch.equal(sin_c.view(-1), rope_table(cfg, "cpu")[p, 1])
    cos, sin = cs[p, 0].view(1, 1, -1), cs[p, 1].view(1, 1, -1)
    q_ref, k_ref = apply_rotary_pos_emb(q.view(1, cfg.heads, 1, cfg.head_dim), k.view(1, cfg.kv_heads, 1, cfg.head_dim),
                                        cos, sin)
    qq, kk = q.clone(), k.clone()
    N._check(N.lib().otf_rope_kv(qq.data_ptr(), kk.data_ptr(), v.data_ptr(), cs.data_ptr(), pos.data_ptr(),
                                 kc.data_ptr(), vc.data_ptr(), cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.max_pos,
                                 N._stream(cuda_dev)), "otf_rope_kv")
    torch.cuda.synchronize()
    assert torch.equal(qq, q_ref.reshape(-1)) and torch.equal(kk, k_ref.reshape(-1))
    assert torch.equal(kc[p], kk) and torch.equal(vc[p], v)
    assert int(kc[:p].abs().sum()) == 0


@pytest.mark.parametrize("hd,heads,kv,L", [(128, 24, 8, 1), (128, 24, 8, 300), (64, 8, 8, 64), (128, 8, 1, 1000)])
def test_attn_decode_matches_fp32_softmax(hd, heads, kv, L, cuda_dev):
    N = _lib()
    max_pos = 1024
    g = torch.Generator(device=cuda_dev).manual_seed(L)
    q = torch.randn(heads * hd, generator=g, device=cuda_dev).half()
    kc = torch.randn(max_pos, kv * hd, generator=g, device=cuda_dev).half()
    vc = torch.randn(max_pos, kv * hd, generator=g, device=cuda_dev).half()
    pos = torch.tensor([L - 1], dtype=torch.int32, device=cuda_dev)
    out = torch.empty(heads * hd, dtype=torch.float16, device=cuda_dev)
    ws = torch.zeros(int(N.lib().otf_attn_workspace_bytes(kv, hd, max_pos)), dtype=torch.uint8, device=cuda_dev)
    scale = 1.0 / math.sqrt(hd)
    for _ in range(2):   # the second call reuses the re-armed tickets
        N._check(N.lib().otf_attn_decode(q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), out.data_ptr(),
                                         scale, heads, kv, hd, max_pos, ws.data_ptr(), ws.numel(),
                                         N._stream(cuda_dev)), "otf_attn_decode")
    torch.cuda.synchronize()
    rep = heads // kv
    qf = q.float().view(heads, hd)
    kf = kc[:L].float().view(L, kv, hd).repeat_interleave(rep, dim=1)   # [L, heads, hd]
    vf = vc[:L].float().view(L, kv, hd).repeat_interleave(rep, dim=1)
    s = torch.einsum("hd,lhd->hl", qf, kf) * scale
    ref = torch.einsum("hl,lhd->hd", torch.softmax(s, dim=-1), vf).reshape(-1)
    assert rel_err(out.float().cpu().numpy(), ref.cpu().numpy()) < 2e-3


def _tiny_model(dev, seed=0, hidden=256, heads=4, kv_heads=2, head_dim=64, inter=512, vocab=512, max_pos=64):
    from otf_llm.decode_model import ModelConfig
    from otf_llm.symmetric_2bit_engine import (QuantizedEmbedding, QuantizedLinearHead, Symmetric2BitQuantizer,
                                                SymmetricOTF2BitLinear)
    cfg = ModelConfig(layers=2, hidden=hidden, intermediate=inter, heads=heads, kv_heads=kv_heads,
                      head_dim=head_dim, vocab=vocab, rope_theta=500000.0, max_pos=max_pos)
    g = torch.Generator(device=dev).manual_seed(seed)
    qd, kvd = heads * head_dim, kv_heads * head_dim
    shapes = {"q_proj": (qd, hidden), "k_proj": (kvd, hidden), "v_proj": (kvd, hidden), "o_proj": (hidden, qd),
              "gate_proj": (inter, hidden), "up_proj": (inter, hidden), "down_proj": (hidden, inter)}
    qz = Symmetric2BitQuantizer(group_size=64, outlier_ratio=0.01)
    layers, norms = [], []
    for _ in range(cfg.layers):
        mods = {}
        for n, (o, i) in shapes.items():
            W = torch.randn(o, i, generator=g, device=dev) * 0.05
            act = torch.randn(i, generator=g, device=dev).abs()
            packed, scales, ov, oi = qz.quantize_tensor(W, act)
            mods[n] = SymmetricOTF2BitLinear(packed, scales, i, 64, ov, oi)
        layers.append(mods)
        norms.append(((1 + 0.1 * torch.randn(hidden, generator=g, device=dev)).half(),
                      (1 + 0.1 * torch.randn(hidden, generator=g, device=dev)).half()))
    E = (torch.randn(cfg.vocab, hidden, generator=g, device=dev) * 0.5).half()
    emb = QuantizedEmbedding(cfg.vocab, hidden)
    emb.quantize_from_fp16(E)
    emb.weight_int8, emb.scales = emb.weight_int8.to(dev), emb.scales.to(dev)
    head = QuantizedLinearHead(hidden, cfg.vocab)
    head.weight_int8, head.scales = emb.weight_int8, emb.scales          # tied, as the 3B model
    fnorm = (1 + 0.1 * torch.randn(hidden, generator=g, device=dev)).half()
    return cfg, layers, norms, emb, head, fnorm


@pytest.mark.parametrize("graph", [False, True])
def test_greedy_decoder_matches_hf_model(graph, cuda_dev):
    """Teacher-forced logits of the native decoder vs HF's LlamaForCausalLM with the same
    2-bit / INT8 modules injected (HF attention, fp16).  Tolerance 2e-2 of max|logit|."""
    transformers = pytest.importorskip("transformers")
    from otf_llm.checkpoint import OTF2BitCheckpoint, inject_into_model
    from otf_llm.decode_model import GreedyDecoder
    cfg, layers, norms, emb, head, fnorm = _tiny_model(cuda_dev)
    dec = GreedyDecoder(cfg, layers, norms, emb, head, fnorm, cuda_dev)
    if graph:
        dec.capture()
    T = 12
    prompt = torch.from_numpy(np.random.default_rng(3).integers(0, cfg.vocab, T)).to(cuda_dev)
    got = []
    dec.generate(prompt, 1, logits_out=got)
    got = torch.cat(got).float()                                        # [T, V]

    hcfg = transformers.LlamaConfig(vocab_size=cfg.vocab, hidden_size=256, intermediate_size=512,
                                    num_hidden_layers=2, num_attention_heads=4, num_key_value_heads=2, head_dim=64,
                                    rope_theta=cfg.rope_theta, max_position_embeddings=cfg.max_pos,
                                    rms_norm_eps=cfg.rms_eps, tie_word_embeddings=True)
    hf = transformers.AutoModelForCausalLM.from_config(hcfg, dtype=torch.float16).to(cuda_dev).eval()
    proj = {"q_proj": "self_attn.q_proj", "k_proj": "self_attn.k_proj", "v_proj": "self_attn.v_proj",
            "o_proj": "self_attn.o_proj", "gate_proj": "mlp.gate_proj", "up_proj": "mlp.up_proj",
            "down_proj": "mlp.down_proj"}
    ck = OTF2BitCheckpoint(config={"group_size": 64, "projections": list(proj.values())},
                           layers=[{proj[n]: m for n, m in l.items()} for l in layers], embed=emb, head=head,
                           head_tied=True, final_norm=fnorm,
                           layer_norms=[{"input_layernorm": a, "post_attention_layernorm": b} for a, b in norms])
    inject_into_model(hf, ck)
    with torch.inference_mode():
        ref = hf(prompt.view(1, -1)).logits[0].float()                  # [T, V]
    assert got.shape == ref.shape
    assert rel_err(got.cpu().numpy(), ref.cpu().numpy()) < 2e-2
    # greedy picks agree wherever HF's top-2 margin is clear
    top2 = ref.topk(2, dim=-1).values
    clear = (top2[:, 0] - top2[:, 1]) > 0.05 * ref.abs().max()
    assert bool((got.argmax(-1) == ref.argmax(-1))[clear].all())
    assert _lib().device_error() == 0


@pytest.mark.parametrize("graph", [False, True])
def test_greedy_decoder_matches_oracle_decode(graph, cuda_dev):
    """The native decoder against the oracle's restatement of the reference engine's decode
    step (the CPU baseline bench.py times), at the 3B model's head shape (head_dim 128, 3 query
    heads per KV head): teacher-forced logits over 40 positions within 1e-2 of max|logit|, and
    the same greedy picks wherever the oracle's top-2 margin is clear."""
    from oracle import decode
    from otf_llm.decode_model import GreedyDecoder
    cfg, layers, norms, emb, head, fnorm = _tiny_model(cuda_dev, seed=9, hidden=768, heads=6, kv_heads=2,
                                                        head_dim=128, inter=1024, vocab=1000, max_pos=64)
    dec = GreedyDecoder(cfg, layers, norms, emb, head, fnorm, cuda_dev)
    if graph:
        dec.capture()
    T = 40
    prompt = np.random.default_rng(5).integers(0, cfg.vocab, T)
    got = []
    dec.generate(torch.from_numpy(prompt).to(cuda_dev), 1, logits_out=got)
    got = torch.cat(got).float().cpu().numpy()
    cpu = decode.Decoder([{n: decode.projection_of(m) for n, m in l.items()} for l in layers], norms, fnorm,
                         emb.weight_int8, emb.scales, head.weight_int8, head.scales, heads=cfg.heads,
                         kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, rope_theta=cfg.rope_theta,
                         rms_eps=cfg.rms_eps, max_pos=cfg.max_pos)
    ref = []
    cpu.generate(prompt, 1, logits_out=ref)
    ref = np.stack(ref)
    err = rel_err(got, ref)
    print(f"native decoder vs oracle decode: rel err {err:.2e}")
    assert err < 1e-2
    top2 = np.sort(ref, axis=-1)[:, -2:]
    clear = (top2[:, 1] - top2[:, 0]) > 0.02 * np.abs(ref).max()
    assert bool((got.argmax(-1) == ref.argmax(-1))[clear].all())
    assert _lib().device_error() == 0


@pytest.mark.parametrize("hd,heads,kv", [(128, 24, 8), (64, 8, 2)])
def test_fused_rope_attention_matches_two_launches(hd, heads, kv, cuda_dev):
    """otf_attn_rope_decode against otf_rope_kv + otf_attn_decode: the same cache rows and
    the same attention output, over a run of consecutive positions (splits of 64 crossed)."""
    from otf_llm.decode_model import ModelConfig, rope_table
    N = _lib()
    L_ = N.lib()
    cfg = ModelConfig(layers=1, hidden=heads * hd, intermediate=64, heads=heads, kv_heads=kv, head_dim=hd, vocab=16,
                      max_pos=160)
    cs = rope_table(cfg, cuda_dev)
    g = torch.Generator(device=cuda_dev).manual_seed(hd)
    f16 = dict(dtype=torch.float16, device=cuda_dev)
    kc_a, vc_a = torch.zeros(cfg.max_pos, kv * hd, **f16), torch.zeros(cfg.max_pos, kv * hd, **f16)
    kc_b, vc_b = kc_a.clone(), vc_a.clone()
    nb = int(L_.otf_attn_workspace_bytes(kv, hd, cfg.max_pos))
    ws_a = torch.zeros(nb, dtype=torch.uint8, device=cuda_dev)
    ws_b = torch.zeros_like(ws_a)
    scale = 1.0 / math.sqrt(hd)
    st = N._stream(cuda_dev)
    worst = 0.0
    for p in list(range(0, 70)) + [127, 128, 150]:
        q = torch.randn(heads * hd, generator=g, device=cuda_dev).half()
        k = torch.randn(kv * hd, generator=g, device=cuda_dev).half()
        v = torch.randn(kv * hd, generator=g, device=cuda_dev).half()
        pos = torch.tensor([p], dtype=torch.int32, device=cuda_dev)
        out_a = torch.empty(heads * hd, **f16)
        out_b = torch.empty_like(out_a)
        qa, ka = q.clone(), k.clone()
        N._check(L_.otf_rope_kv(qa.data_ptr(), ka.data_ptr(), v.data_ptr(), cs.data_ptr(), pos.data_ptr(),
                                kc_a.data_ptr(), vc_a.data_ptr(), heads, kv, hd, cfg.max_pos, st), "otf_rope_kv")
        N._check(L_.otf_attn_decode(qa.data_ptr(), kc_a.data_ptr(), vc_a.data_ptr(), pos.data_ptr(), out_a.data_ptr(),
                                    scale, heads, kv, hd, cfg.max_pos, ws_a.data_ptr(), nb, st), "otf_attn_decode")
        N._check(L_.otf_attn_rope_decode(q.data_ptr(), k.data_ptr(), v.data_ptr(), cs.data_ptr(), pos.data_ptr(),
                                         kc_b.data_ptr(), vc_b.data_ptr(), out_b.data_ptr(), scale, heads, kv, hd,
                                         cfg.max_pos, ws_b.data_ptr(), nb, st), "otf_attn_rope_decode")
        torch.cuda.synchronize()
        assert torch.equal(kc_a[p], kc_b[p]) and torch.equal(vc_a[p], vc_b[p])
        worst = max(worst, rel_err(out_b.float().cpu().numpy(), out_a.float().cpu().numpy()))
    assert worst < 2e-3
    assert _lib().device_error() == 0
