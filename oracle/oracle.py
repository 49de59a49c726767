"""Python face of the CPU oracle (test infrastructure only).

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline leg may
import this module, and only to check or time against it.  It wraps
``liboracle.so`` (built from ``otf_oracle.c`` by ``oracle/Makefile``) with numpy
arrays; every function names the reference code it restates.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

# Reference codebook constants: LLOYD_MAX_SYMMETRIC_CENTROIDS held as fp16 by the
# symmetric module (otf_llm/symmetric_2bit_engine.py:14,191) and as fp32 by the
# asymmetric one (otf_llm/otf_2bit_quantizer.py:18,169).
CB_F32 = np.array([-1.52, -0.45, 0.45, 1.52], dtype=np.float32)
CB_F16 = CB_F32.astype(np.float16)


def build() -> str:
    """Compile liboracle.so in place (gcc + OpenMP) and return its path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return os.path.join(_HERE, "liboracle.so")


def lib() -> ctypes.CDLL:
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            build()
        _LIB = ctypes.CDLL(path)
        i64, vp = ctypes.c_int64, ctypes.c_void_p
        _LIB.orc_linear_f32.argtypes = [vp, i64, vp, i64, vp, i64, vp, i64, vp, vp, vp, i64, vp, i64, vp, vp, i64,
                                        i64, i64, i64, i64, ctypes.c_int]
        _LIB.orc_lut_linear.argtypes = [vp, i64, vp, i64, vp, i64, vp, vp, vp, i64, vp, i64, vp, vp, i64,
                                        i64, i64, i64, i64, vp]
        _LIB.orc_unpack_codes.argtypes = [vp, i64, i64, i64, vp]
        _LIB.orc_pack_codes.argtypes = [vp, i64, i64, vp]
        _LIB.orc_i8_head.argtypes = [vp, i64, vp, i64, vp, vp, i64, i64, i64, i64]
        _LIB.orc_argmax_rows.argtypes = [vp, i64, i64, i64, vp]
        _LIB.orc_i8_embed.argtypes = [vp, i64, vp, i64, vp, vp, i64, i64, i64]
        _LIB.orc_i8_embed.restype = i64
        _LIB.orc_i8_quantize.argtypes = [vp, i64, i64, i64, vp, vp]
        _LIB.orc_quantize_2b.argtypes = [vp, i64, i64, i64, i64, vp, i64, vp, vp, vp, vp, vp]
        _LIB.orc_num_threads.restype = ctypes.c_int
        _LIB.orc_set_num_threads.argtypes = [ctypes.c_int]
    return _LIB


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dt):
    return None if a is None else np.ascontiguousarray(a, dtype=dt)


def num_threads() -> int:
    return lib().orc_num_threads()


def set_num_threads(n: int) -> None:
    lib().orc_set_num_threads(int(n))


def unpack_codes(packed: np.ndarray, K: int) -> np.ndarray:
    """Codes [N, K] from packed [N, K/4] (pack_2bit_uint8 inverse, otf_llm/symmetric_2bit_engine.py:100-107)."""
    packed = _c(packed, np.uint8)
    N = packed.shape[0]
    out = np.empty((N, K), dtype=np.uint8)
    lib().orc_unpack_codes(_p(packed), packed.shape[1], N, K, _p(out))
    return out


def pack_codes(codes: np.ndarray) -> np.ndarray:
    codes = _c(codes, np.uint8)
    N, K = codes.shape
    out = np.empty((N, K // 4), dtype=np.uint8)
    lib().orc_pack_codes(_p(codes), N, K, _p(out))
    return out


def linear_f32(x, packed, scales, group_size, *, codebook=CB_F16, zeros=None, mask=None, outlier_idx=None,
               outlier_vals=None, bias=None, clamp=True) -> np.ndarray:
    """fp32 restatement of the quantized linear (see orc_linear_f32). x: fp16 [M, K]; returns fp32 [M, N]."""
    x = _c(np.atleast_2d(x), np.float16)
    packed = _c(packed, np.uint8)
    scales = _c(scales, np.float16)
    zeros = _c(zeros, np.float16)
    mask = _c(mask, np.float16)
    M, K = x.shape
    N = packed.shape[0]
    cb = np.ascontiguousarray(np.asarray(codebook, dtype=np.float32))
    if outlier_idx is not None and len(outlier_idx) > 0:
        oidx = _c(outlier_idx, np.int64)
        ov = _c(outlier_vals, np.float16)
        nk, ldo = oidx.shape[0], ov.shape[1]
    else:
        oidx = ov = None
        nk, ldo = 0, 0
    bias = _c(bias, np.float16)
    y = np.empty((M, N), dtype=np.float32)
    lib().orc_linear_f32(_p(x), K, _p(packed), packed.shape[1], _p(scales), scales.shape[1], _p(zeros),
                         0 if zeros is None else zeros.shape[1], _p(cb), _p(mask), _p(oidx), nk, _p(ov), ldo,
                         _p(bias), _p(y), N, M, N, K, group_size, 1 if clamp else 0)
    return y


def lut_linear(x, packed, scales, group_size, *, mask=None, outlier_idx=None, outlier_vals=None, bias=None,
               wbuf=None) -> np.ndarray:
    """Port of the reference's CPU forward (LUT dequant to fp16 + matmul); returns fp16 [M, N]."""
    x = _c(np.atleast_2d(x), np.float16)
    packed = _c(packed, np.uint8)
    scales = _c(scales, np.float16)
    mask = _c(mask, np.float16)
    M, K = x.shape
    N = packed.shape[0]
    if outlier_idx is not None and len(outlier_idx) > 0:
        oidx = _c(outlier_idx, np.int64)
        ov = _c(outlier_vals, np.float16)
        nk, ldo = oidx.shape[0], ov.shape[1]
    else:
        oidx = ov = None
        nk, ldo = 0, 0
    bias = _c(bias, np.float16)
    if wbuf is None or wbuf.size < N * K:
        wbuf = np.empty(N * K, dtype=np.float16)
    y = np.empty((M, N), dtype=np.float16)
    lib().orc_lut_linear(_p(x), K, _p(packed), packed.shape[1], _p(scales), scales.shape[1], _p(CB_F16), _p(mask),
                         _p(oidx), nk, _p(ov), ldo, _p(bias), _p(y), N, M, N, K, group_size, _p(wbuf))
    return y


def i8_head(x, w_i8, scales) -> np.ndarray:
    """fp32 restatement of QuantizedLinearHead.forward (otf_llm/symmetric_2bit_engine.py:75-91)."""
    x = _c(np.atleast_2d(x), np.float16)
    w = _c(w_i8, np.int8)
    s = _c(np.asarray(scales).reshape(-1), np.float16)
    M, D = x.shape
    V = w.shape[0]
    out = np.empty((M, V), dtype=np.float32)
    lib().orc_i8_head(_p(x), D, _p(w), w.shape[1], _p(s), _p(out), V, M, V, D)
    return out


def argmax_rows(logits: np.ndarray) -> np.ndarray:
    lg = _c(np.atleast_2d(logits), np.float32)
    out = np.empty(lg.shape[0], dtype=np.int64)
    lib().orc_argmax_rows(_p(lg), lg.shape[1], lg.shape[0], lg.shape[1], _p(out))
    return out


def i8_embed(ids, w_i8, scales) -> np.ndarray:
    """QuantizedEmbedding.forward (otf_llm/symmetric_2bit_engine.py:41-47), bit-exact fp16."""
    ids = _c(np.asarray(ids).reshape(-1), np.int64)
    w = _c(w_i8, np.int8)
    s = _c(np.asarray(scales).reshape(-1), np.float16)
    V, D = w.shape
    out = np.zeros((ids.shape[0], D), dtype=np.float16)
    bad = lib().orc_i8_embed(_p(ids), ids.shape[0], _p(w), D, _p(s), _p(out), D, V, D)
    if bad:
        raise IndexError(f"{bad} ids outside [0, {V})")
    return out


def i8_quantize(w_f16):
    """quantize_from_fp16 (otf_llm/symmetric_2bit_engine.py:26-39): int8 [V, D] and fp16 scales [V, 1]."""
    w = _c(w_f16, np.float16)
    V, D = w.shape
    q = np.empty((V, D), dtype=np.int8)
    s = np.empty(V, dtype=np.float16)
    lib().orc_i8_quantize(_p(w), D, V, D, _p(q), _p(s))
    return q, s.reshape(V, 1)


def n_outliers(K: int, ratio: float) -> int:
    """Anchor column count of quantize_tensor: max(1, int(K * ratio)) when ratio > 0, else 0
    (otf_llm/symmetric_2bit_engine.py:132)."""
    return max(1, int(K * ratio)) if ratio > 0.0 else 0


def quantize_2b(W, group_size: int, ratio: float, act=None, codebook=CB_F32):
    """Symmetric2BitQuantizer.quantize_tensor (otf_llm/symmetric_2bit_engine.py:109-169) in
    the fixed summation order of orc_quantize_2b.  W: float array [N, K] (fp16/bf16 values are
    exact in fp32).  Returns (packed uint8 [N, K/4], scales fp16 [N, K/G], outliers fp16 [N, k]
    or None, indices int64 [k] or None)."""
    W = np.ascontiguousarray(W, dtype=np.float32)
    N, K = W.shape
    G = int(group_size)
    assert K % G == 0 and G % 4 == 0 and G <= 256
    k = n_outliers(K, ratio)
    a = None if act is None else _c(act, np.float32)
    cb = _c(codebook, np.float32)
    packed = np.empty((N, K // 4), np.uint8)
    scales = np.empty((N, K // G), np.float16)
    ov = np.empty((N, max(k, 1)), np.float16)
    idx = np.empty(max(k, 1), np.int64)
    lib().orc_quantize_2b(_p(W), K, N, K, G, _p(a), k, _p(cb), _p(packed), _p(scales), _p(ov), _p(idx))
    if k == 0:
        return packed, scales, None, None
    return packed, scales, ov, idx
