"""bench.py's CPU-baseline legs on the CPU: the decode-step restatement it times after an e2e
run (cpu_decode_sample, fed a decoder's KV cache and first token) and the per-layer LUT sample
of the stack (cpu_reference_sample) return the cpu_baseline fields the bench line carries."""
import numpy as np
import pytest
import torch

import bench


def _tiny_modules(seed=0):
    """A 2-layer model's projections as the reference module type, built on the CPU from the
    oracle's quantizer (the bench leg only reads their buffers)."""
    from oracle import oracle
    from otf_llm.decode_model import ModelConfig
    from otf_llm.symmetric_2bit_engine import SymmetricOTF2BitLinear
    cfg = ModelConfig(layers=2, hidden=128, intermediate=256, heads=2, kv_heads=1, head_dim=64, vocab=96,
                      rope_theta=500000.0, max_pos=40)
    rng = np.random.default_rng(seed)
    shapes = {"q_proj": (128, 128), "k_proj": (64, 128), "v_proj": (64, 128), "o_proj": (128, 128),
              "gate_proj": (256, 128), "up_proj": (256, 128), "down_proj": (128, 256)}
    layers = []
    for _ in range(cfg.layers):
        mods = {}
        for n, (N, K) in shapes.items():
            W = (rng.standard_normal((N, K)) * 0.05).astype(np.float32)
            packed, scales, ov, idx = oracle.quantize_2b(W, 64, 0.02)
            mods[n] = SymmetricOTF2BitLinear(torch.from_numpy(packed), torch.from_numpy(scales), K, 64,
                                             torch.from_numpy(ov), torch.from_numpy(idx))
        layers.append(mods)
    w = (rng.standard_normal((cfg.vocab, cfg.hidden)) * 0.02).astype(np.float16)
    w8, sc = oracle.i8_quantize(w)
    return cfg, layers, torch.from_numpy(w8), torch.from_numpy(sc)


class _FakeDecoder:
    def __init__(self, cfg, start):
        g = torch.Generator().manual_seed(1)
        kvd = cfg.kv_heads * cfg.head_dim
        self.kc = [(torch.randn(cfg.max_pos, kvd, generator=g) * 0.5).half() for _ in range(cfg.layers)]
        self.vc = [(torch.randn(cfg.max_pos, kvd, generator=g) * 0.5).half() for _ in range(cfg.layers)]


def test_cpu_decode_sample_fields():
    cfg, layers, w8, sc = _tiny_modules()
    start = 8
    dec = _FakeDecoder(cfg, start)
    tokens = list(range(5, 5 + 40))
    cpu = bench.cpu_decode_sample(dec, layers, cfg, w8, sc, start, tokens, target_s=0.2)
    assert cpu["kind"] == "port" and cpu["unit"] == "tokens/s"
    assert cpu["value"] > 0 and cpu["cores"] >= 1
    n = int(cpu["picks_equal_to_gpu"].split(" of ")[1])
    assert 1 <= n <= 64       # at most 64 steps per sample
    assert f"positions {start}.." in cpu["sample"]


def test_cpu_decode_sample_matches_oracle_decoder():
    """The leg's greedy picks are the oracle decoder's on the same cache and first token."""
    from oracle import decode, oracle
    cfg, layers, w8, sc = _tiny_modules(seed=2)
    start = 6
    dec = _FakeDecoder(cfg, start)
    ones = np.ones(cfg.hidden, np.float16)
    ref = decode.Decoder([{n: decode.projection_of(m) for n, m in l.items()} for l in layers],
                         [(ones, ones)] * cfg.layers, ones, w8.numpy(), sc.numpy(), w8.numpy(), sc.numpy(),
                         heads=cfg.heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, rope_theta=cfg.rope_theta,
                         rms_eps=cfg.rms_eps, max_pos=start + 65)
    for li in range(cfg.layers):
        ref.set_cache(li, dec.kc[li][:start].numpy(), dec.vc[li][:start].numpy())
    picks, tok = [], 7
    for i in range(4):
        tok = int(oracle.argmax_rows(ref.step(tok, start + i)[None])[0])
        picks.append(tok)
    tokens = [7] + picks + [0] * 40
    cpu = bench.cpu_decode_sample(dec, layers, cfg, w8, sc, start, tokens, target_s=0.0)
    assert cpu["picks_equal_to_gpu"].startswith("1 of 1")


def test_cpu_reference_sample_fields():
    from otf_llm.decoder_stack import StackConfig
    gbs, cores, sample, el = bench.cpu_reference_sample(StackConfig(layers=1, hidden=256, intermediate=512),
                                                         target_s=0.0)
    assert gbs > 0 and cores >= 1 and el > 0
    assert "7 projections" in sample
