"""Attention entry points with a device-side position outside [0, max_pos): the launch writes
nothing (no cache row, no output) and raises the otf_device_error flag; in a batch only the
sequence with the bad position is skipped.  Covers the cluster-merge form (1, 2, 3, 4 or 8
query heads per KV head), the ticket-merge form (other ratios, and batches) and the
separate attention kernel."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from otf_llm import _native
    return _native


def _case(dev, heads, kv, hd=128, max_pos=200, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    f16 = dict(dtype=torch.float16, device=dev)
    t = {"q": torch.randn(heads * hd, generator=g, device=dev).half(),
         "k": torch.randn(kv * hd, generator=g, device=dev).half(),
         "v": torch.randn(kv * hd, generator=g, device=dev).half(),
         "kc": torch.randn(max_pos, kv * hd, generator=g, device=dev).half(),
         "vc": torch.randn(max_pos, kv * hd, generator=g, device=dev).half(),
         "out": torch.full((heads * hd,), 7.0, **f16)}
    ang = torch.arange(max_pos, device=dev).float()[:, None] * (
        1.0 / (500000.0 ** (torch.arange(0, hd, 2, device=dev).float() / hd)))[None, :]
    e = torch.cat((ang, ang), dim=-1)
    t["cs"] = torch.stack((e.cos(), e.sin()), dim=1).half().contiguous()
    return t


@pytest.mark.parametrize("heads,kv", [(24, 8), (10, 2), (64, 8)])
@pytest.mark.parametrize("bad", [-1, 200, 1 << 20])
def test_fused_attention_skips_bad_position(heads, kv, bad, cuda_dev):
    N = _lib()
    L = N.lib()
    hd, max_pos = 128, 200
    t = _case(cuda_dev, heads, kv, hd, max_pos)
    kc0, vc0 = t["kc"].clone(), t["vc"].clone()
    pos = torch.tensor([bad], dtype=torch.int32, device=cuda_dev)
    nb = int(L.otf_attn_workspace_bytes(kv, hd, max_pos))
    ws = torch.zeros(nb, dtype=torch.uint8, device=cuda_dev)
    N.device_error(clear=True)
    N._check(L.otf_attn_rope_decode(t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(), t["cs"].data_ptr(),
                                    pos.data_ptr(), t["kc"].data_ptr(), t["vc"].data_ptr(), t["out"].data_ptr(),
                                    1.0 / math.sqrt(hd), heads, kv, hd, max_pos, ws.data_ptr(), nb,
                                    N._stream(cuda_dev)), "otf_attn_rope_decode")
    torch.cuda.synchronize()
    assert N.device_error(clear=True) == 1
    assert torch.equal(t["kc"], kc0) and torch.equal(t["vc"], vc0)
    assert bool((t["out"] == 7.0).all())
    # the next call with a good position runs normally (workspace and flag re-armed)
    pos.fill_(max_pos - 1)
    N._check(L.otf_attn_rope_decode(t["q"].data_ptr(), t["k"].data_ptr(), t["v"].data_ptr(), t["cs"].data_ptr(),
                                    pos.data_ptr(), t["kc"].data_ptr(), t["vc"].data_ptr(), t["out"].data_ptr(),
                                    1.0 / math.sqrt(hd), heads, kv, hd, max_pos, ws.data_ptr(), nb,
                                    N._stream(cuda_dev)), "otf_attn_rope_decode")
    torch.cuda.synchronize()
    assert N.device_error(clear=True) == 0
    assert bool(torch.isfinite(t["out"].float()).all()) and not bool((t["out"] == 7.0).all())


@pytest.mark.parametrize("bad", [-1, 300])
def test_attention_kernel_skips_bad_position(bad, cuda_dev):
    N = _lib()
    L = N.lib()
    heads, kv, hd, max_pos = 24, 8, 128, 300
    t = _case(cuda_dev, heads, kv, hd, max_pos)
    pos = torch.tensor([bad], dtype=torch.int32, device=cuda_dev)
    nb = int(L.otf_attn_workspace_bytes(kv, hd, max_pos))
    ws = torch.zeros(nb, dtype=torch.uint8, device=cuda_dev)
    N.device_error(clear=True)
    N._check(L.otf_attn_decode(t["q"].data_ptr(), t["kc"].data_ptr(), t["vc"].data_ptr(), pos.data_ptr(),
                               t["out"].data_ptr(), 1.0 / math.sqrt(hd), heads, kv, hd, max_pos, ws.data_ptr(), nb,
                               N._stream(cuda_dev)), "otf_attn_decode")
    torch.cuda.synchronize()
    assert N.device_error(clear=True) == 1
    assert bool((t["out"] == 7.0).all())


def test_batched_attention_skips_only_the_bad_sequence(cuda_dev):
    N = _lib()
    L = N.lib()
    heads, kv, hd, max_pos, B = 24, 8, 128, 150, 3
    g = torch.Generator(device=cuda_dev).manual_seed(5)
    f16 = dict(dtype=torch.float16, device=cuda_dev)
    q = torch.randn(B, heads * hd, generator=g, device=cuda_dev).half()
    k = torch.randn(B, kv * hd, generator=g, device=cuda_dev).half()
    v = torch.randn(B, kv * hd, generator=g, device=cuda_dev).half()
    kc = torch.randn(B, max_pos, kv * hd, generator=g, device=cuda_dev).half()
    vc = torch.randn(B, max_pos, kv * hd, generator=g, device=cuda_dev).half()
    kc0, vc0 = kc.clone(), vc.clone()
    out = torch.full((B, heads * hd), 7.0, **f16)
    cs = _case(cuda_dev, heads, kv, hd, max_pos)["cs"]
    pos = torch.tensor([40, max_pos, 99], dtype=torch.int32, device=cuda_dev)
    nb = int(L.otf_attn_workspace_bytes_batch(kv, hd, max_pos, B))
    ws = torch.zeros(nb, dtype=torch.uint8, device=cuda_dev)
    N.device_error(clear=True)
    N._check(L.otf_attn_rope_decode_batch(q.data_ptr(), q.stride(0), k.data_ptr(), v.data_ptr(), k.stride(0),
                                          cs.data_ptr(), pos.data_ptr(), kc.data_ptr(), vc.data_ptr(),
                                          max_pos * kv * hd, out.data_ptr(), out.stride(0), 1.0 / math.sqrt(hd),
                                          heads, kv, hd, max_pos, B, ws.data_ptr(), nb, N._stream(cuda_dev)),
             "otf_attn_rope_decode_batch")
    torch.cuda.synchronize()
    assert N.device_error(clear=True) == 1
    assert bool((out[1] == 7.0).all()) and torch.equal(kc[1], kc0[1]) and torch.equal(vc[1], vc0[1])
    for b, p in ((0, 40), (2, 99)):
        assert not bool((out[b] == 7.0).all())
        assert not torch.equal(kc[b, p], kc0[b, p])          # the good sequences wrote their row
        assert torch.equal(kc[b, :p], kc0[b, :p]) and torch.equal(vc[b, :p], vc0[b, :p])
