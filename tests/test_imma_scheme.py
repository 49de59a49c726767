"""CPU check of the decode kernel's integer-MMA scheme against the oracle.

The emulator (tests/imma_emulator.py) mirrors the kernel's per-lane fragments and
flush arithmetic; agreement here shows the bit-plane decomposition, the fixed-point
limbs and the lane/column mapping compute the reference's layer on real golden data.
"""
import numpy as np
import pytest

from conftest import load_golden, rel_err
import imma_emulator as emu
from oracle import oracle


def _ref_no_tail(gd, x, zeros=None, cb=oracle.CB_F16, clamp=True):
    return oracle.linear_f32(x, gd["packed"], gd["scales"], int(gd["G"]), codebook=cb, zeros=zeros,
                             mask=gd["mask"], clamp=clamp)[0]


@pytest.mark.parametrize("name,W", [("sym_g64_small", 4), ("sym_g64_k4096", 4), ("sym_g128", 4),
                                    ("sym_g32_legacy", 2)])
def test_scheme_symmetric(name, W):
    gd = load_golden(name)
    x = gd["x_m1"][0]
    N = gd["packed"].shape[0]
    ref = _ref_no_tail(gd, x[None])
    rows = list(range(min(N, 32)))
    got = []
    for r0 in range(0, len(rows), 16):
        got.extend(emu.tile_gemv(x, gd["packed"], gd["scales"], int(gd["G"]), oracle.CB_F16.astype(np.float32),
                                 mask16=gd["mask"], W=W, rows=range(r0, r0 + 16))[: max(0, min(16, N - r0))])
    got = np.array(got[: len(rows)])
    assert rel_err(got, ref[: len(rows)]) < 2e-4


def test_scheme_asymmetric_zeros():
    gd = load_golden("asym_g32")
    x = gd["x_m1"][0]
    ref = _ref_no_tail(gd, x[None], zeros=gd["zeros"], cb=oracle.CB_F32, clamp=False)
    got = emu.tile_gemv(x, gd["packed"], gd["scales"], int(gd["G"]), oracle.CB_F32, mask16=gd["mask"],
                        zeros=gd["zeros"], W=2, rows=range(16))
    assert rel_err(got, ref[:16]) < 2e-4
