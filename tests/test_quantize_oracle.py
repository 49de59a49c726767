"""The quantizer oracle (oracle.quantize_2b, fixed summation order) against the reference's own
Symmetric2BitQuantizer.quantize_tensor outputs (tests/golden, made by make_golden.py).

Codes, anchor indices and anchor values must be identical.  Scales are identical on the small
fixtures; on the 256 x 4096 fixture the reference's vectorised fp32 sums and the oracle's fixed
order land on different sides of an fp16 rounding boundary for a handful of groups, which then
differ by exactly one fp16 ulp (bound below: 0.1% of the groups).
"""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import oracle


def _profile(K, g):
    """x_profile of make_golden.py: |N(0,1)| with 1% of the channels x 20."""
    p = torch.randn(K, generator=g).abs()
    hot = torch.randperm(K, generator=g)[: max(1, K // 100)]
    p[hot] *= 20.0
    return p


def _ulps(a, b):
    return np.abs(a.view(np.int16).astype(np.int64) - b.view(np.int16).astype(np.int64))


@pytest.mark.parametrize("name", ["quant_g64", "sym_g64_small", "sym_g32_legacy", "sym_g128"])
def test_oracle_quantizer_matches_reference_fixture(name):
    d = load_golden(name)
    packed, scales, ov, idx = oracle.quantize_2b(d["W"], int(d["G"]), float(d["ratio"]), d["act"])
    assert np.array_equal(packed, d["packed"])
    assert np.array_equal(idx, d["outlier_idx"])
    assert np.array_equal(ov, d["outliers"])
    assert np.array_equal(scales, d["scales"])


def test_oracle_quantizer_k4096_fixture():
    """W and the profile regenerated from make_golden.py's seeded torch generator (seed 2)."""
    d = load_golden("sym_g64_k4096")
    g = torch.Generator().manual_seed(2)
    W = (torch.randn(256, 4096, generator=g) * 0.02).numpy()
    act = _profile(4096, g).numpy()
    assert np.array_equal(act, d["act"]), "torch generator stream changed: W cannot be regenerated"
    packed, scales, ov, idx = oracle.quantize_2b(W, 64, 0.005, act)
    assert np.array_equal(packed, d["packed"])
    assert np.array_equal(idx, d["outlier_idx"])
    assert np.array_equal(ov, d["outliers"])
    u = _ulps(scales, d["scales"])
    assert u.max() <= 1
    assert (u > 0).sum() <= scales.size // 1000


def test_oracle_quantizer_edges():
    """No anchors (ratio 0), a group made only of anchor columns, all-zero rows, ties in impact."""
    rng = np.random.default_rng(0)
    W = (rng.standard_normal((8, 64)) * 0.02).astype(np.float32)
    W[3] = 0.0
    p, s, ov, idx = oracle.quantize_2b(W, 16, 0.0)
    assert ov is None and idx is None
    codes = oracle.unpack_codes(p, 64)
    assert np.all(codes[3] == 1)                   # w = 0: |0 - c1| == |0 - c2|, first index wins
    assert np.all(s[3] == np.float16(1e-8))        # <w, c> = 0 -> clamp(0, 1e-8)
    # duplicate columns tie in impact: the lower index ranks first
    W2 = W.copy()
    W2[:, 40] = W2[:, 7]
    W2[:, 7] *= 9.0
    W2[:, 40] = W2[:, 7]
    p, s, ov, idx = oracle.quantize_2b(W2, 16, 2 / 64)
    assert list(idx) == [7, 40]
    # 16 anchors out of 64 columns at G = 16: with the largest columns all in group 1 that
    # group is entirely anchors: codes 1, scale 1e-8
    W3 = W.copy()
    W3[:, 16:32] *= 100.0
    p, s, ov, idx = oracle.quantize_2b(W3, 16, 16 / 64)
    assert sorted(idx.tolist()) == list(range(16, 32))
    assert np.all(oracle.unpack_codes(p, 64)[:, 16:32] == 1)
    assert np.all(s[:, 1] == np.float16(1e-8))
    assert np.array_equal(ov, W3[:, idx].astype(np.float16))
