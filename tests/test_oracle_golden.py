"""Pin the CPU oracle to the reference's own outputs (golden fixtures, no GPU)."""
import numpy as np
import pytest

from conftest import load_golden, rel_err
from oracle import oracle

SYM = ["sym_g64_small", "sym_g64_k4096", "sym_g32_legacy", "sym_g128"]


def _ms(gd):
    return sorted(int(k[3:]) for k in gd if k.startswith("x_m"))


@pytest.mark.parametrize("name", SYM)
def test_oracle_matches_reference_layer(name):
    gd = load_golden(name)
    for M in _ms(gd):
        y = oracle.linear_f32(gd[f"x_m{M}"], gd["packed"], gd["scales"], int(gd["G"]), mask=gd["mask"],
                              outlier_idx=gd["outlier_idx"], outlier_vals=gd["outliers"], bias=gd.get("bias"))
        # tight pin against the double-precision restatement of the reference dequant
        assert rel_err(y, gd[f"y_f64_m{M}"]) < 1e-6
        # the reference module itself computes in fp16: within the 1e-3 bar
        assert rel_err(y, gd[f"y_ref_m{M}"]) < 1e-3


@pytest.mark.parametrize("name", SYM)
def test_oracle_gemm_function(name):
    gd = load_golden(name)
    for M in _ms(gd):
        y = oracle.linear_f32(gd[f"x_m{M}"], gd["packed"], gd["scales"], int(gd["G"]), mask=gd["mask"])
        assert rel_err(y, gd[f"y_gemm_m{M}"]) < 1e-3


@pytest.mark.parametrize("name", SYM)
def test_lut_port_reproduces_reference(name):
    """The timed CPU baseline is a port of the reference's LUT path: it must agree with it."""
    gd = load_golden(name)
    for M in _ms(gd):
        y = oracle.lut_linear(gd[f"x_m{M}"], gd["packed"], gd["scales"], int(gd["G"]), mask=gd["mask"],
                              outlier_idx=gd["outlier_idx"], outlier_vals=gd["outliers"], bias=gd.get("bias"))
        assert rel_err(y, gd[f"y_ref_m{M}"]) < 5e-4


def test_oracle_asymmetric_matches_unpack():
    gd = load_golden("asym_g32")
    for M in (1, 3):
        y = oracle.linear_f32(gd[f"x_m{M}"], gd["packed"], gd["scales"], int(gd["G"]), codebook=oracle.CB_F32,
                              zeros=gd["zeros"], mask=gd["mask"], outlier_idx=gd["outlier_idx"],
                              outlier_vals=gd["outliers"], bias=gd["bias"], clamp=False)
        assert rel_err(y, gd[f"y_f64_m{M}"]) < 1e-6
        assert rel_err(y, gd[f"y_a7_m{M}"]) < 1e-3   # a7 rounds W to fp16 first


def test_code_unpack_bit_exact():
    gd = load_golden("codes_pack")
    K = gd["codes"].shape[1]
    assert np.array_equal(oracle.unpack_codes(gd["packed"], K), gd["codes"])
    assert np.array_equal(oracle.pack_codes(gd["codes"]), gd["packed"])


def test_int8_embedding_bit_exact():
    gd = load_golden("int8_v1000_d256")
    out = oracle.i8_embed(gd["ids"], gd["weight_int8"], gd["scales"])
    ref = gd["emb_out"].reshape(out.shape)
    assert np.array_equal(out.view(np.uint16), ref.view(np.uint16))


def test_int8_quantize_bit_exact():
    gd = load_golden("int8_v1000_d256")
    q, s = oracle.i8_quantize(gd["W_fp16"])
    assert np.array_equal(q, gd["weight_int8"])
    assert np.array_equal(s.view(np.uint16), gd["scales"].view(np.uint16))


def test_int8_head():
    gd = load_golden("int8_v1000_d256")
    for M in (1, 5):
        lg = oracle.i8_head(gd[f"x_m{M}"], gd["weight_int8"], gd["scales"])
        assert rel_err(lg, gd[f"logits_f64_m{M}"]) < 1e-6
        assert rel_err(lg, gd[f"logits_m{M}"]) < 1e-3
        assert np.array_equal(oracle.argmax_rows(lg), np.argmax(gd[f"logits_f64_m{M}"], axis=1))
