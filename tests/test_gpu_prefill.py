"""Prompt prefill: otf_attn_prefill (RoPE + KV-cache write for P rows, then causal attention of
every row over the cache) against per-row otf_rope_kv and an fp32 causal softmax, and
GreedyDecoder.prefill (projections at M = P rows) against the same prompt decoded token by
token."""
import math

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _table(dev, hd, max_pos, theta=500000.0):
    ang = torch.arange(max_pos, device=dev).float()[:, None] * (
        1.0 / (theta ** (torch.arange(0, hd, 2, device=dev).float() / hd)))[None, :]
    e = torch.cat((ang, ang), dim=-1)
    return torch.stack((e.cos(), e.sin()), dim=1).half().contiguous()


@pytest.mark.parametrize("heads,kv,hd,start,P", [(24, 8, 128, 0, 37), (8, 8, 64, 5, 20), (64, 8, 128, 3, 70),
                                                  (10, 2, 128, 0, 1)])
def test_attn_prefill_matches_rows_and_fp32(heads, kv, hd, start, P, cuda_dev):
    from otf_llm import _native
    L = _native.lib()
    max_pos = start + P + 9
    g = torch.Generator(device=cuda_dev).manual_seed(heads + P)
    q = torch.randn(P, heads * hd, generator=g, device=cuda_dev).half()
    k = torch.randn(P, kv * hd, generator=g, device=cuda_dev).half()
    v = torch.randn(P, kv * hd, generator=g, device=cuda_dev).half()
    kc = (torch.randn(max_pos, kv * hd, generator=g, device=cuda_dev) * 0.5).half()
    vc = (torch.randn(max_pos, kv * hd, generator=g, device=cuda_dev) * 0.5).half()
    cs = _table(cuda_dev, hd, max_pos)
    # per-row reference: otf_rope_kv one position at a time on copies
    q1, k1, kc1, vc1 = q.clone(), k.clone(), kc.clone(), vc.clone()
    for r in range(P):
        pr = torch.tensor([start + r], dtype=torch.int32, device=cuda_dev)
        qr, kr = q1[r].clone(), k1[r].clone()
        _native._check(L.otf_rope_kv(qr.data_ptr(), kr.data_ptr(), v[r].data_ptr(), cs.data_ptr(), pr.data_ptr(),
                                     kc1.data_ptr(), vc1.data_ptr(), heads, kv, hd, max_pos,
                                     _native._stream(cuda_dev)), "otf_rope_kv")
        q1[r], k1[r] = qr, kr
    out = torch.full((P, heads * hd), 7.0, dtype=torch.float16, device=cuda_dev)
    pos = torch.tensor([start], dtype=torch.int32, device=cuda_dev)
    _native.device_error(clear=True)
    qp = torch.zeros(P, heads * hd + 8, dtype=torch.float16, device=cuda_dev)[:, :heads * hd]   # strided rows
    qp.copy_(q)
    kp = k.clone()
    _native._check(L.otf_attn_prefill(qp.data_ptr(), qp.stride(0), kp.data_ptr(), v.data_ptr(), kp.stride(0),
                                      cs.data_ptr(), pos.data_ptr(), kc.data_ptr(), vc.data_ptr(), out.data_ptr(),
                                      out.stride(0), 1.0 / math.sqrt(hd), heads, kv, hd, max_pos, P,
                                      _native._stream(cuda_dev)), "otf_attn_prefill")
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 0
    assert torch.equal(kc, kc1) and torch.equal(vc, vc1)          # rows written bit for bit, others kept
    assert torch.equal(qp, q1) and torch.equal(kp, k1)
    # causal attention in fp32 over the cache rows [0, start + r]
    rep = heads // kv
    kf = kc.float().view(max_pos, kv, hd)
    vf = vc.float().view(max_pos, kv, hd)
    qf = q1.float().view(P, heads, hd)
    ref = torch.empty(P, heads, hd, device=cuda_dev)
    for r in range(P):
        n = start + r + 1
        kk = kf[:n].repeat_interleave(rep, dim=1)                  # [n, heads, hd]
        vv = vf[:n].repeat_interleave(rep, dim=1)
        s = torch.einsum("hd,nhd->hn", qf[r], kk) / math.sqrt(hd)
        ref[r] = torch.einsum("hn,nhd->hd", torch.softmax(s, dim=-1), vv)
    assert rel_err(out.float().cpu().numpy(), ref.view(P, -1).cpu().numpy()) < 2e-3


def test_attn_prefill_past_cache_writes_nothing(cuda_dev):
    from otf_llm import _native
    L = _native.lib()
    heads, kv, hd, max_pos, P = 8, 2, 64, 40, 12
    g = torch.Generator(device=cuda_dev).manual_seed(9)
    q = torch.randn(P, heads * hd, generator=g, device=cuda_dev).half()
    k = torch.randn(P, kv * hd, generator=g, device=cuda_dev).half()
    v = torch.randn(P, kv * hd, generator=g, device=cuda_dev).half()
    kc = torch.randn(max_pos, kv * hd, generator=g, device=cuda_dev).half()
    vc = torch.randn(max_pos, kv * hd, generator=g, device=cuda_dev).half()
    kc0, vc0 = kc.clone(), vc.clone()
    out = torch.full((P, heads * hd), 7.0, dtype=torch.float16, device=cuda_dev)
    pos = torch.tensor([max_pos - 5], dtype=torch.int32, device=cuda_dev)   # rows 5.. fall past the cache
    _native.device_error(clear=True)
    _native._check(L.otf_attn_prefill(q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0),
                                      _table(cuda_dev, hd, max_pos).data_ptr(), pos.data_ptr(), kc.data_ptr(),
                                      vc.data_ptr(), out.data_ptr(), out.stride(0), 0.125, heads, kv, hd, max_pos, P,
                                      _native._stream(cuda_dev)), "otf_attn_prefill")
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 1
    assert torch.equal(kc[:max_pos - 5], kc0[:max_pos - 5]) and torch.equal(vc[:max_pos - 5], vc0[:max_pos - 5])
    assert bool((out[5:] == 7.0).all()) and not bool((out[:5] == 7.0).all())


@pytest.mark.parametrize("P", [1, 6, 23])
def test_decoder_prefill_matches_token_steps(P, cuda_dev):
    """The prompt as one pass of P rows (projections at M = P) gives the caches, the last
    row's logits and the continuation of the same prompt decoded token by token, within the
    whole-model tolerance (the tensor-memory GEMM and the batch-1 GEMV round differently)."""
    from test_gpu_decode_model import _tiny_model
    from otf_llm.decode_model import GreedyDecoder
    cfg, layers, norms, emb, head, fnorm = _tiny_model(cuda_dev, seed=4, max_pos=64)
    a = GreedyDecoder(cfg, layers, norms, emb, head, fnorm, cuda_dev)
    b = GreedyDecoder(cfg, layers, norms, emb, head, fnorm, cuda_dev)
    a.capture()
    prompt = torch.from_numpy(np.random.default_rng(P).integers(0, cfg.vocab, P)).to(cuda_dev)
    la = []
    a.generate(prompt, 1, logits_out=la, prefill=False)
    from otf_llm import _native
    _native.device_error(clear=True)
    b.prefill(prompt)
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 0
    assert int(b.pos.item()) == P
    for li in range(cfg.layers):
        assert rel_err(b.kc[li][:P].float().cpu().numpy(), a.kc[li][:P].float().cpu().numpy()) < 2e-2
        assert rel_err(b.vc[li][:P].float().cpu().numpy(), a.vc[li][:P].float().cpu().numpy()) < 2e-2
    assert rel_err(b.logits.cpu().numpy(), la[-1].cpu().numpy()) < 2e-2
    first = int(torch.argmax(b.logits[0]))
    assert int(b.ids[0]) == first
    # generate: prefill (the default on one GPU), then graph steps from the prefilled caches
    b.capture()
    tb = b.generate(prompt, 5)
    assert tb.shape == (5,) and int(tb[0]) == first
    lg = []
    tc = b.generate(prompt, 2, logits_out=lg, prefill=True)
    assert len(lg) == 2 and torch.equal(tc, tb[:2])
    assert rel_err(lg[0].cpu().numpy(), la[-1].cpu().numpy()) < 2e-2


@pytest.mark.parametrize("B,P", [(3, 7), (16, 5)])
def test_batched_prefill_matches_batch1_prefill(B, P, cuda_dev):
    """BatchedGreedyDecoder.prefill (projections at M = B x P rows, prefill attention per
    sequence on its own caches) against the batch-1 decoder's prefill of each sequence."""
    from test_gpu_decode_model import _tiny_model
    from otf_llm import _native
    from otf_llm.decode_model import BatchedGreedyDecoder, GreedyDecoder
    cfg, layers, norms, emb, head, fnorm = _tiny_model(cuda_dev, seed=6, max_pos=64)
    bat = BatchedGreedyDecoder(cfg, layers, norms, emb, head, fnorm, cuda_dev, B)
    one = GreedyDecoder(cfg, layers, norms, emb, head, fnorm, cuda_dev)
    prompts = torch.from_numpy(np.random.default_rng(B + P).integers(0, cfg.vocab, (B, P))).to(cuda_dev)
    _native.device_error(clear=True)
    bat.prefill(prompts)
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == 0
    assert bool((bat.pos == P).all())
    assert torch.equal(bat.ids, torch.argmax(bat.logits, dim=1))
    for s in (0, B // 2, B - 1):
        one.reset()
        one.prefill(prompts[s])
        assert rel_err(bat.logits[s].cpu().numpy(), one.logits[0].cpu().numpy()) < 2e-2, s
        for li in range(cfg.layers):
            assert rel_err(bat.kc[li][s][:P].float().cpu().numpy(), one.kc[li][:P].float().cpu().numpy()) < 2e-2
    bat.capture()
    out = bat.generate(prompts, 4)                  # prefill + graph steps
    assert out.shape == (B, 4) and bool((bat.pos == P + 3).all())


def test_prefill_graph_matches_eager(cuda_dev):
    """capture_prefill records the prefill of one prompt length as a CUDA graph; replays give
    the eager prefill's logits, pick, caches and position bit for bit, for any prompt of that
    length."""
    from test_gpu_decode_model import _tiny_model
    from otf_llm.decode_model import GreedyDecoder
    cfg, layers, norms, emb, head, fnorm = _tiny_model(cuda_dev, seed=8, max_pos=64)
    a = GreedyDecoder(cfg, layers, norms, emb, head, fnorm, cuda_dev)
    b = GreedyDecoder(cfg, layers, norms, emb, head, fnorm, cuda_dev)
    P = 11
    b.capture_prefill(P)
    assert int(b.pos.item()) == 0
    for seed in (1, 2):
        prompt = torch.from_numpy(np.random.default_rng(seed).integers(0, cfg.vocab, P)).to(cuda_dev)
        a.reset()
        b.reset()
        a.prefill(prompt)
        b.prefill(prompt)
        torch.cuda.synchronize()
        assert torch.equal(a.logits, b.logits) and torch.equal(a.ids, b.ids)
        assert int(b.pos.item()) == P
        for li in range(cfg.layers):
            assert torch.equal(a.kc[li][:P], b.kc[li][:P]) and torch.equal(a.vc[li][:P], b.vc[li][:P])
