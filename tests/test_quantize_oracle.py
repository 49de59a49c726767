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


def _team_sum(v, G):
    """The summation order of otf2b_quantize / orc_quantize_2b, restated with numpy: TL =
    min(32, G/4) partial sums, partial l taking elements 4l..4l+3 of each slab of 4*TL in order
    (sequential fp32), then combined pairwise (l + TL/2, ..., l + 1)."""
    TL = min(32, G // 4)
    S = G // (4 * TL)
    a = v.reshape(*v.shape[:-1], S, TL, 4).swapaxes(-3, -2).reshape(*v.shape[:-1], TL, S * 4)
    a = np.cumsum(a, axis=-1, dtype=np.float32)[..., -1]
    o = TL // 2
    while o:
        a = (a[..., :o] + a[..., o:2 * o]).astype(np.float32)
        o //= 2
    return a[..., 0]


def _numpy_quantize(W, G, ratio, act):
    """Independent numpy restatement of the quantizer in the fixed order (column sums over
    256-row chunks, then chunk order)."""
    N, K = W.shape
    k = oracle.n_outliers(K, ratio)
    keep = np.ones(K, np.float32)
    idx = None
    if k:
        sq = (W * W).astype(np.float32)
        pad = (-N) % 256
        sq = np.concatenate([sq, np.zeros((pad, K), np.float32)]).reshape(-1, 256, K)
        part = np.cumsum(sq, axis=1, dtype=np.float32)[:, -1, :]
        imp = np.sqrt(np.cumsum(part, axis=0, dtype=np.float32)[-1]).astype(np.float32)
        if act is not None:
            imp = (imp * act).astype(np.float32)
        idx = np.array(sorted(range(K), key=lambda c: (-imp[c], c))[:k], dtype=np.int64)
        keep[idx] = 0
    w = (W * keep).reshape(N, K // G, G).astype(np.float32)
    kp = keep.reshape(1, K // G, G)
    cb = oracle.CB_F32
    cnt = np.maximum(kp.sum(-1), 1).astype(np.float32)
    s = np.maximum(np.sqrt(_team_sum(w * w, G) / cnt + np.float32(1e-8)) / np.float32(0.95),
                   np.float32(1e-8)).astype(np.float32)
    for _ in range(5):
        z = w / np.maximum(s, np.float32(1e-8))[..., None]
        q = np.abs(z[..., None] - cb).argmin(-1)
        cq = (cb[q] * kp).astype(np.float32)
        s = np.maximum(_team_sum(w * cq, G) / np.maximum(_team_sum(cq * cq, G), np.float32(1e-8)),
                       np.float32(1e-8)).astype(np.float32)
    codes = q.reshape(N, K).astype(np.uint8)
    packed = codes[:, 0::4] | (codes[:, 1::4] << 2) | (codes[:, 2::4] << 4) | (codes[:, 3::4] << 6)
    return packed, s.astype(np.float16), idx


@pytest.mark.parametrize("N,K,G,ratio,seed", [(64, 1024, 16, 0.05, 1), (300, 2048, 32, 0.035, 2),
                                              (50, 4096, 64, 0.005, 3), (40, 2048, 128, 0.01, 4),
                                              (33, 4096, 256, 0.01, 5), (7, 512, 64, 0.0, 6)])
def test_oracle_summation_order(N, K, G, ratio, seed):
    """orc_quantize_2b against an independent numpy restatement of the same fixed order: bit-exact
    codes, scales and anchor indices (fp16-valued weights, as the converter feeds them)."""
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16).astype(np.float32)
    act = np.abs(rng.standard_normal(K)).astype(np.float32)
    p, s, ov, idx = oracle.quantize_2b(W, G, ratio, act)
    rp, rs, ridx = _numpy_quantize(W, G, ratio, act)
    assert np.array_equal(p, rp) and np.array_equal(s, rs)
    if ratio:
        assert np.array_equal(idx, ridx)
    else:
        assert idx is None
