"""The GPU quantizer (otf2b_quantize via Symmetric2BitQuantizer.quantize_tensor on CUDA tensors).

* Bit-exact against the oracle (same summation order): packed codes, fp16 scales, anchor
  indices and anchor values, over group sizes 16..256, fp16 / bf16 / fp32 weights, strided
  weights, no anchors, no activation profile, several row chunks, and a 4096 x 4096 layer.
* Against the reference's own outputs (golden fixtures): codes, indices and anchors
  identical; scales identical or one fp16 ulp apart in at most 0.1% of the groups.
* The quantized layer's forward against the oracle linear (end to end).
"""
import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from oracle import oracle

pytestmark = pytest.mark.gpu


def _q(W, G, ratio, act=None):
    from otf_llm.symmetric_2bit_engine import Symmetric2BitQuantizer
    out = Symmetric2BitQuantizer(G, ratio).quantize_tensor(W, act)
    torch.cuda.synchronize()
    return [None if t is None else t.cpu().numpy() for t in out]


def _same(got, ref):
    for a, b, what in zip(got, ref, ("packed", "scales", "outliers", "indices")):
        if b is None:
            assert a is None, what
        else:
            assert a.shape == b.shape and a.dtype == b.dtype, what
            assert np.array_equal(a, b), f"{what}: {np.sum(a != b)} of {a.size} differ"


CASES = [  # N, K, G, ratio, dtype, seed
    (37, 192, 64, 0.005, torch.float16, 1),
    (64, 512, 32, 0.035, torch.float16, 2),
    (300, 1024, 16, 0.05, torch.float16, 3),
    (48, 1024, 128, 0.01, torch.bfloat16, 4),
    (33, 2048, 256, 0.01, torch.float32, 5),
    (513, 768, 64, 0.0, torch.float16, 6),
    (700, 4096, 64, 0.005, torch.float32, 7),
]


@pytest.mark.parametrize("N,K,G,ratio,dtype,seed", CASES)
@pytest.mark.parametrize("with_act", [True, False])
def test_quantize_matches_oracle(N, K, G, ratio, dtype, seed, with_act, cuda_dev):
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(N, K, generator=g) * 0.02).to(dtype)
    act = torch.randn(K, generator=g).abs() if with_act else None
    got = _q(W.to(cuda_dev), G, ratio, None if act is None else act.to(cuda_dev))
    ref = oracle.quantize_2b(W.float().numpy(), G, ratio, None if act is None else act.numpy())
    _same(got, ref)


def test_quantize_strided_weight(cuda_dev):
    g = torch.Generator().manual_seed(11)
    big = (torch.randn(96, 1100, generator=g) * 0.02).half()
    W = big[:, 12:12 + 1024]                       # row stride 1100, offset 12 elements (24 B)
    act = torch.randn(1024, generator=g).abs()
    got = _q(W.to(cuda_dev), 64, 0.01, act.to(cuda_dev))
    _same(got, oracle.quantize_2b(W.float().numpy(), 64, 0.01, act.numpy()))


def test_quantize_layer_4096(cuda_dev):
    g = torch.Generator().manual_seed(12)
    W = (torch.randn(4096, 4096, generator=g) * 0.02).half()
    act = torch.randn(4096, generator=g).abs()
    act[torch.randperm(4096, generator=g)[:40]] *= 20.0
    got = _q(W.to(cuda_dev), 64, 0.005, act.to(cuda_dev))
    _same(got, oracle.quantize_2b(W.float().numpy(), 64, 0.005, act.numpy()))


def test_quantize_edges(cuda_dev):
    """Zero rows, duplicate columns (impact ties: lower index first), a group made only of
    anchor columns (codes 1, scale 1e-8)."""
    rng = np.random.default_rng(0)
    W = (rng.standard_normal((8, 64)) * 0.02).astype(np.float32)
    W[3] = 0.0
    W[:, 7] *= 9.0
    W[:, 40] = W[:, 7]
    for ratio in (0.0, 2 / 64):
        _same(_q(torch.from_numpy(W).to(cuda_dev), 16, ratio), oracle.quantize_2b(W, 16, ratio))
    W3 = W.copy()
    W3[:, 16:32] *= 100.0
    got = _q(torch.from_numpy(W3).to(cuda_dev), 16, 16 / 64)
    _same(got, oracle.quantize_2b(W3, 16, 16 / 64))
    assert np.all(got[1][:, 1] == np.float16(1e-8))


def _ulps(a, b):
    return np.abs(a.view(np.int16).astype(np.int64) - b.view(np.int16).astype(np.int64))


@pytest.mark.parametrize("name", ["quant_g64", "sym_g64_small", "sym_g32_legacy", "sym_g128", "sym_g64_k4096"])
def test_quantize_matches_reference_fixture(name, cuda_dev):
    d = load_golden(name)
    if "W" in d:
        W, act = d["W"], d["act"]
    else:                                          # regenerated from make_golden.py's seed
        g = torch.Generator().manual_seed(2)
        W = (torch.randn(256, 4096, generator=g) * 0.02).numpy()
        p = torch.randn(4096, generator=g).abs()
        p[torch.randperm(4096, generator=g)[:40]] *= 20.0
        act = p.numpy()
        assert np.array_equal(act, d["act"])
    packed, scales, ov, idx = _q(torch.from_numpy(W).to(cuda_dev), int(d["G"]), float(d["ratio"]),
                                 torch.from_numpy(act).to(cuda_dev))
    assert np.array_equal(packed, d["packed"])
    assert np.array_equal(idx, d["outlier_idx"])
    assert np.array_equal(ov, d["outliers"])
    u = _ulps(scales, d["scales"])
    assert u.max() <= 1 and (u > 0).sum() <= scales.size // 1000


def test_quantized_layer_forward(cuda_dev):
    from otf_llm.symmetric_2bit_engine import Symmetric2BitQuantizer, SymmetricOTF2BitLinear
    g = torch.Generator().manual_seed(13)
    W = (torch.randn(1024, 2048, generator=g) * 0.02).half().to(cuda_dev)
    act = torch.randn(2048, generator=g).abs().to(cuda_dev)
    packed, scales, ov, oi = Symmetric2BitQuantizer(64, 0.005).quantize_tensor(W, act)
    lay = SymmetricOTF2BitLinear(packed, scales, 2048, 64, ov, oi).to(cuda_dev)
    x = torch.randn(3, 2048, generator=g).half()
    y = lay(x.to(cuda_dev)).float().cpu().numpy()
    ref = oracle.linear_f32(x.numpy(), packed.cpu().numpy(), scales.cpu().numpy(), 64,
                            mask=lay.outlier_mask_vector.cpu().numpy(), outlier_idx=oi.cpu().numpy(),
                            outlier_vals=ov.cpu().numpy())
    assert rel_err(y, ref) < 1e-3


def test_quantize_rejects_unsupported(cuda_dev):
    from otf_llm import _native
    W = torch.randn(16, 96, device=cuda_dev).half()
    with pytest.raises(RuntimeError):
        _native.quantize_2b(W, 48, 1)              # group size outside 16..256 powers of two
    with pytest.raises(ValueError):
        _native.quantize_2b(W, 64, 1)              # K not a multiple of G
