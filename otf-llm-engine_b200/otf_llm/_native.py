"""ctypes binding of libotfb200.so, the sm_100a kernels behind this package.

Every wrapper takes torch CUDA tensors, checks device, dtype, shape and strides,
passes raw pointers plus the current CUDA stream across the C ABI declared in
``include/otf_b200.h``, and turns a nonzero status into ``RuntimeError``.  There
is no CPU or pure-PyTorch fallback: a missing library or a non-CUDA tensor is an
error.
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import torch

_LIB_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_lib", "libotfb200.so")
_lib: Optional[ctypes.CDLL] = None

OTF_FLAG_CLAMP = 1
OTF_FLAG_FORCE_GENERIC = 2
OTF_XOP_NONE = 0
OTF_XOP_RMSNORM = 1
OTF_XOP_SILU_MUL = 2
OTF_AR_NONE = 0
OTF_AR_PRODUCE = 1
OTF_AR_CONSUME = 2
OTF_AR_HANDLE_BYTES = 64


class Layer(ctypes.Structure):
    """Mirror of `otf2b_layer` (include/otf_b200.h)."""
    _fields_ = [
        ("x", ctypes.c_void_p), ("ldx", ctypes.c_int64),
        ("packed", ctypes.c_void_p), ("ld_packed", ctypes.c_int64),
        ("scales", ctypes.c_void_p), ("ld_scales", ctypes.c_int64),
        ("zeros", ctypes.c_void_p), ("ld_zeros", ctypes.c_int64),
        ("codebook", ctypes.POINTER(ctypes.c_float)),
        ("mask", ctypes.c_void_p),
        ("outlier_idx", ctypes.c_void_p), ("n_outliers", ctypes.c_int64),
        ("outlier_vals", ctypes.c_void_p), ("ld_outlier_vals", ctypes.c_int64),
        ("bias", ctypes.c_void_p),
        ("residual", ctypes.c_void_p), ("ld_residual", ctypes.c_int64),
        ("y", ctypes.c_void_p), ("ldy", ctypes.c_int64),
        ("N", ctypes.c_int64), ("K", ctypes.c_int64), ("group_size", ctypes.c_int64),
        ("flags", ctypes.c_uint32),
        ("x_op", ctypes.c_int32),
        ("x_aux", ctypes.c_void_p),
        ("eps", ctypes.c_float),
        ("ar", ctypes.c_void_p), ("ar_mode", ctypes.c_int32), ("ar_buf", ctypes.c_int32),
        ("ar_out", ctypes.c_void_p),
    ]

class Proj(ctypes.Structure):
    """Mirror of `otf2b_proj` (include/otf_b200.h)."""
    _fields_ = [
        ("packed", ctypes.c_void_p), ("ld_packed", ctypes.c_int64),
        ("scales", ctypes.c_void_p), ("ld_scales", ctypes.c_int64),
        ("mask", ctypes.c_void_p),
        ("outlier_idx", ctypes.c_void_p), ("n_outliers", ctypes.c_int64),
        ("outlier_vals", ctypes.c_void_p), ("ld_outlier_vals", ctypes.c_int64),
        ("bias", ctypes.c_void_p),
        ("N", ctypes.c_int64), ("K", ctypes.c_int64),
    ]


class DecoderLayer(ctypes.Structure):
    """Mirror of `otf2b_decoder_layer`."""
    _fields_ = [(n, Proj) for n in ("q", "k", "v", "o", "gate", "up", "down")] + [
        ("input_norm", ctypes.c_void_p), ("post_norm", ctypes.c_void_p)]


class DecodeDims(ctypes.Structure):
    """Mirror of `otf2b_decode_dims`."""
    _fields_ = [("n_layers", ctypes.c_int64), ("hidden", ctypes.c_int64), ("intermediate", ctypes.c_int64),
                ("heads", ctypes.c_int64), ("kv_heads", ctypes.c_int64), ("head_dim", ctypes.c_int64),
                ("group_size", ctypes.c_int64), ("eps", ctypes.c_float), ("codebook", ctypes.c_float * 4)]


# Names exported by the library; kept in step with include/otf_b200.h.
EXPORTS = (
    "otf_version",
    "otf_status_string",
    "otf_last_cuda_error",
    "otf_device_error",
    "otf2b_linear",
    "otf2b_gemm_mma",
    "otf2b_linear_group",
    "otf2b_unpack_codes",
    "otf_i8_head",
    "otf_i8_head_argmax",
    "otf_i8_embed",
    "otf_rmsnorm",
    "otf_silu_mul",
    "otf_ar_create",
    "otf_ar_open",
    "otf_ar_destroy",
    "otf_ar_push",
    "otf_ar_finish",
    "otf2b_decode_workspace_bytes",
    "otf2b_decode_prepare",
    "otf2b_decode_step",
    "otf_rope_kv",
    "otf_attn_workspace_bytes",
    "otf_attn_decode",
    "otf_pos_advance",
    "otf_attn_decode_noalloc",
    "otf_attn_rope_decode",
    "otf2b_quantize_workspace_bytes",
    "otf2b_quantize",
    "otf_attn_workspace_bytes_batch",
    "otf_attn_rope_decode_batch",
    "otf_pos_advance_batch",
    "otf_attn_prefill",
)


def library_path() -> str:
    return _LIB_PATH


def lib() -> ctypes.CDLL:
    """Load the native library once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH):
        raise RuntimeError(
            f"libotfb200.so not found at {_LIB_PATH}; build it with `make -C otf-llm-engine_b200/csrc` "
            "(or __graft_entry__.build()). There is no fallback path.")
    L = ctypes.CDLL(_LIB_PATH)
    i64, vp, u32, i32 = ctypes.c_int64, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int
    L.otf_version.restype = i32
    L.otf_status_string.argtypes = [i32]
    L.otf_status_string.restype = ctypes.c_char_p
    L.otf_last_cuda_error.restype = i32
    L.otf_device_error.argtypes = [i32]
    L.otf_device_error.restype = i32
    L.otf2b_linear.argtypes = [vp, i64, vp, i64, vp, i64, vp, i64, vp, vp, vp, i64, vp, i64, vp, vp, i64, vp, i64,
                               i64, i64, i64, i64, u32, vp]
    L.otf2b_linear.restype = i32
    L.otf2b_gemm_mma.argtypes = L.otf2b_linear.argtypes
    L.otf2b_gemm_mma.restype = i32
    L.otf2b_linear_group.argtypes = [ctypes.POINTER(Layer), ctypes.c_int, vp]
    L.otf2b_linear_group.restype = i32
    L.otf2b_unpack_codes.argtypes = [vp, i64, i64, i64, vp, i64, vp]
    L.otf2b_unpack_codes.restype = i32
    L.otf_i8_head.argtypes = [vp, i64, vp, i64, vp, vp, i64, i64, i64, i64, vp]
    L.otf_i8_head_argmax.argtypes = [vp, i64, vp, i64, vp, vp, i64, vp, i64, i64, i64, vp]
    L.otf_i8_head_argmax.restype = i32
    L.otf_i8_head.restype = i32
    L.otf_i8_embed.argtypes = [vp, i64, vp, i64, vp, vp, i64, i64, i64, vp, vp]
    L.otf_i8_embed.restype = i32
    L.otf_rmsnorm.argtypes = [vp, i64, vp, ctypes.c_float, vp, i64, i64, i64, vp]
    L.otf_rmsnorm.restype = i32
    L.otf_silu_mul.argtypes = [vp, vp, vp, i64, vp]
    L.otf_silu_mul.restype = i32
    L.otf_ar_create.argtypes = [i32, i32, i64, vp, ctypes.POINTER(vp)]
    L.otf_ar_create.restype = i32
    L.otf_ar_open.argtypes = [vp, vp]
    L.otf_ar_open.restype = i32
    L.otf_ar_destroy.argtypes = [vp]
    L.otf_ar_destroy.restype = i32
    L.otf_ar_push.argtypes = [vp, i32, vp, i64, vp]
    L.otf_ar_push.restype = i32
    L.otf_ar_finish.argtypes = [vp, i32, vp, i64, vp]
    L.otf_ar_finish.restype = i32
    L.otf2b_decode_workspace_bytes.argtypes = [ctypes.POINTER(DecodeDims)]
    L.otf2b_decode_workspace_bytes.restype = i64
    L.otf2b_decode_prepare.argtypes = [ctypes.POINTER(DecoderLayer), ctypes.POINTER(DecodeDims), vp, i64]
    L.otf2b_decode_prepare.restype = i32
    L.otf2b_decode_step.argtypes = [ctypes.POINTER(DecodeDims), vp, vp, vp]
    L.otf2b_decode_step.restype = i32
    L.otf_rope_kv.argtypes = [vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, vp]
    L.otf_rope_kv.restype = i32
    L.otf_attn_workspace_bytes.argtypes = [i64, i64, i64]
    L.otf_attn_workspace_bytes.restype = i64
    L.otf_attn_decode.argtypes = [vp, vp, vp, vp, vp, ctypes.c_float, i64, i64, i64, i64, vp, i64, vp]
    L.otf_attn_decode.restype = i32
    L.otf_pos_advance.argtypes = [vp, vp]
    L.otf_pos_advance.restype = i32
    L.otf_attn_decode_noalloc.argtypes = [vp, vp, vp, vp, vp, ctypes.c_float, i64, i64, i64, i64, vp]
    L.otf_attn_decode_noalloc.restype = i32
    L.otf_attn_rope_decode.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, ctypes.c_float, i64, i64, i64, i64, vp, i64, vp]
    L.otf_attn_rope_decode.restype = i32
    L.otf_attn_workspace_bytes_batch.argtypes = [i64, i64, i64, i64]
    L.otf_attn_workspace_bytes_batch.restype = i64
    L.otf_attn_rope_decode_batch.argtypes = [vp, i64, vp, vp, i64, vp, vp, vp, vp, i64, vp, i64, ctypes.c_float, i64,
                                             i64, i64, i64, i64, vp, i64, vp]
    L.otf_attn_rope_decode_batch.restype = i32
    L.otf_pos_advance_batch.argtypes = [vp, i64, vp]
    L.otf_pos_advance_batch.restype = i32
    L.otf_attn_prefill.argtypes = [vp, i64, vp, vp, i64, vp, vp, vp, vp, vp, i64, ctypes.c_float, i64, i64, i64, i64,
                                   i64, vp]
    L.otf_attn_prefill.restype = i32
    L.otf2b_quantize_workspace_bytes.argtypes = [i64, i64]
    L.otf2b_quantize_workspace_bytes.restype = i64
    L.otf2b_quantize.argtypes = [vp, i32, i64, i64, i64, i64, vp, i64, vp, vp, i64, vp, i64, vp, i64, vp, i64, vp,
                                 vp]
    L.otf2b_quantize.restype = i32
    _lib = L
    return L


def _check(status: int, what: str) -> None:
    if status != 0:
        L = lib()
        msg = L.otf_status_string(status).decode()
        if status == 3:
            msg += f" (cudaError {L.otf_last_cuda_error()})"
        raise RuntimeError(f"{what} failed: {msg}")


def _stream(dev: torch.device) -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)


def _ptr(t: Optional[torch.Tensor]) -> Optional[ctypes.c_void_p]:
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _need_cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise RuntimeError(f"{name} must be a CUDA tensor: this package runs its hot path on B200 GPUs only "
                           "and has no CPU fallback")


def _rows(t: torch.Tensor, name: str, dtype: torch.dtype, cols: int) -> int:
    """Check a row-major 2-D tensor with unit inner stride; return its row stride."""
    if t.dtype != dtype:
        raise TypeError(f"{name} must be {dtype}, got {t.dtype}")
    if t.dim() != 2 or t.shape[1] != cols or t.stride(1) != 1:
        raise ValueError(f"{name} must be a row-major [*, {cols}] tensor with unit inner stride, got "
                         f"shape {tuple(t.shape)} strides {t.stride()}")
    return t.stride(0) if t.shape[0] > 1 else max(t.stride(0), cols)


_CB_CACHE: dict = {}


def codebook_floats(codebook) -> Sequence[float]:
    """The 4 codebook values as Python floats (the kernel takes them by value).

    Device tensors are read once per (storage, version) and cached, so steady-state
    calls neither synchronise nor copy (which also keeps forward graph-capturable).
    """
    if codebook is None:
        from .symmetric_2bit_engine import LLOYD_MAX_SYMMETRIC_CENTROIDS
        return [float(torch.tensor(c, dtype=torch.float16)) for c in LLOYD_MAX_SYMMETRIC_CENTROIDS]
    if isinstance(codebook, torch.Tensor):
        key = (codebook.data_ptr(), codebook._version, codebook.numel(), codebook.dtype, str(codebook.device))
        vals = _CB_CACHE.get(key)
        if vals is None:
            vals = [float(v) for v in codebook.detach().float().cpu().tolist()]
            if len(_CB_CACHE) > 4096:
                _CB_CACHE.clear()
            _CB_CACHE[key] = vals
    else:
        vals = [float(v) for v in codebook]
    if len(vals) != 4:
        raise ValueError("a 2-bit codebook has exactly 4 entries")
    return vals


def tensor_pipe_shape_ok(module) -> bool:
    """Whether a 2-bit module's batch-1 shapes meet the tensor-pipe GEMV's layout rules (the
    host-side half of fast_variant in gemv2b.cu): power-of-two group of 32..256, K a
    multiple of 8, even scale stride, packed row stride a multiple of 16 bytes, and an
    affine codebook (c3 - c2 == c1 - c0).  Pointer alignment is checked at launch.  Only
    layers that pass can take the fused RMSNorm / SiLU input transforms."""
    G, K = int(module.group_size), int(module.d_in)
    if G < 32 or G > 256 or G & (G - 1) or K % 8:
        return False
    if module.scales.stride(0) % 2 or module.packed_uint8.stride(0) % 16:
        return False
    c = codebook_floats(module.codebook)
    return abs((c[3] - c[2]) - (c[1] - c[0])) <= 1e-6 * max(1.0, abs(c[1] - c[0]))


def linear_2bit(x2d: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor, group_size: int, codebook4,
                *, zeros: Optional[torch.Tensor] = None, mask: Optional[torch.Tensor] = None,
                outlier_idx: Optional[torch.Tensor] = None, outlier_vals: Optional[torch.Tensor] = None,
                bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None, clamp: bool = True,
                out: Optional[torch.Tensor] = None, force_generic: bool = False,
                gemm_mma: bool = False) -> torch.Tensor:
    """y[M, N] fp16 = fused 2-bit linear over x2d [M, K] fp16 (see otf2b_linear).

    gemm_mma=True forces the tcgen05 dequant GEMM (otf2b_gemm_mma) whatever M is; otherwise
    the library picks the kernel (tcgen05 GEMM from 32 activation rows)."""
    _need_cuda(x2d, "x")
    dev = x2d.device
    M, K = x2d.shape
    N = packed.shape[0]
    if packed.shape[1] * 4 != K:
        raise ValueError(f"packed has {packed.shape[1]} bytes per row, expected K/4 = {K // 4}")
    if K % group_size:
        raise ValueError(f"K={K} is not a multiple of group_size={group_size}")
    for name, t in (("packed", packed), ("scales", scales), ("zeros", zeros), ("mask", mask),
                    ("outlier_idx", outlier_idx), ("outlier_vals", outlier_vals), ("bias", bias),
                    ("residual", residual)):
        if t is not None:
            _need_cuda(t, name)
            if t.device != dev:
                raise ValueError(f"{name} is on {t.device}, x on {dev}")
    ldx = _rows(x2d, "x", torch.float16, K)
    ldp = _rows(packed, "packed", torch.uint8, K // 4)
    lds = _rows(scales, "scales", torch.float16, K // group_size)
    ldz = _rows(zeros, "zeros", torch.float16, K // group_size) if zeros is not None else 0
    if mask is not None and (mask.dtype != torch.float16 or mask.numel() != K or not mask.is_contiguous()):
        raise ValueError("mask must be a contiguous fp16 vector of length K")
    n_out = 0
    ldo = 0
    if outlier_idx is not None and outlier_vals is not None and outlier_idx.numel() > 0:
        if outlier_idx.dtype != torch.int64 or not outlier_idx.is_contiguous():
            raise ValueError("outlier_idx must be a contiguous int64 vector")
        n_out = outlier_idx.numel()
        ldo = _rows(outlier_vals, "outlier_vals", torch.float16, n_out)
        if outlier_vals.shape[0] != N:
            raise ValueError("outlier_vals must have one row per output feature")
    else:
        outlier_idx = outlier_vals = None
    if bias is not None and (bias.dtype != torch.float16 or bias.numel() != N or not bias.is_contiguous()):
        raise ValueError("bias must be a contiguous fp16 vector of length N")
    ldr = 0
    if residual is not None:
        if residual.shape[0] != M:
            raise ValueError("residual must have one row per activation row")
        ldr = _rows(residual, "residual", torch.float16, N)
    if out is None:
        out = torch.empty((M, N), dtype=torch.float16, device=dev)
    ldy = _rows(out, "out", torch.float16, N)
    cb = (ctypes.c_float * 4)(*codebook_floats(codebook4))
    flags = (OTF_FLAG_CLAMP if clamp else 0) | (OTF_FLAG_FORCE_GENERIC if force_generic else 0)
    with torch.cuda.device(dev):
        fn = lib().otf2b_gemm_mma if gemm_mma else lib().otf2b_linear
        st = fn(_ptr(x2d), ldx, _ptr(packed), ldp, _ptr(scales), lds, _ptr(zeros), ldz, cb,
                _ptr(mask), _ptr(outlier_idx), n_out, _ptr(outlier_vals), ldo, _ptr(bias),
                _ptr(residual), ldr, _ptr(out), ldy, M, N, K, group_size, flags, _stream(dev))
    _check(st, "otf2b_gemm_mma" if gemm_mma else "otf2b_linear")
    return out


def unpack_codes(packed: torch.Tensor, K: int) -> torch.Tensor:
    """uint8 [N, K] codes in {0..3} from packed [N, K/4] (bit-exact unpack)."""
    _need_cuda(packed, "packed")
    ldp = _rows(packed, "packed", torch.uint8, K // 4)
    N = packed.shape[0]
    codes = torch.empty((N, K), dtype=torch.uint8, device=packed.device)
    with torch.cuda.device(packed.device):
        st = lib().otf2b_unpack_codes(_ptr(packed), ldp, N, K, _ptr(codes), K, _stream(packed.device))
    _check(st, "otf2b_unpack_codes")
    return codes


_QUANT_DTYPES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}


def quantize_2b(W: torch.Tensor, group_size: int, n_outliers: int, act: Optional[torch.Tensor] = None,
                codebook: Optional[Sequence[float]] = None):
    """Symmetric 2-bit quantisation of W [N, K] on its GPU (otf2b_quantize).

    Returns (packed uint8 [N, K/4], scales fp16 [N, K/G], outliers fp16 [N, k] or None,
    outlier indices int64 [k] or None), as Symmetric2BitQuantizer.quantize_tensor does.
    W may be fp16, bf16 or fp32 (other float types are converted to fp32 first)."""
    _need_cuda(W, "W")
    if W.dim() != 2:
        raise ValueError(f"W must be 2-D, got shape {tuple(W.shape)}")
    if W.dtype not in _QUANT_DTYPES:
        W = W.float()
    N, K = W.shape
    esize = W.element_size()
    if W.stride(1) != 1 or (W.stride(0) % 4 if N > 1 else 0) or W.data_ptr() % (4 * esize):
        W = W.contiguous()
    ldw = W.stride(0) if N > 1 else K
    G, k = int(group_size), int(n_outliers)
    if K % G or K % 4:
        raise ValueError(f"d_in={K} must be a multiple of group_size={G} and of 4")
    dev = W.device
    packed = torch.empty((N, K // 4), dtype=torch.uint8, device=dev)
    scales = torch.empty((N, K // G), dtype=torch.float16, device=dev)
    ov = idx = ws = a = None
    nws = 0
    if k > 0:
        ov = torch.empty((N, k), dtype=torch.float16, device=dev)
        idx = torch.empty(k, dtype=torch.int64, device=dev)
        nws = int(lib().otf2b_quantize_workspace_bytes(N, K))
        ws = torch.empty(nws, dtype=torch.uint8, device=dev)
        if act is not None:
            a = act.detach().to(device=dev, dtype=torch.float32).contiguous()
            if a.numel() != K:
                raise ValueError(f"activation profile has {a.numel()} entries, expected {K}")
    cb = None
    if codebook is not None:
        cb = (ctypes.c_float * 4)(*[float(v) for v in codebook])
    with torch.cuda.device(dev):
        st = lib().otf2b_quantize(_ptr(W), _QUANT_DTYPES[W.dtype], ldw, N, K, G, _ptr(a), k, cb, _ptr(ws), nws,
                                  _ptr(packed), K // 4, _ptr(scales), K // G, _ptr(ov), k, _ptr(idx), _stream(dev))
    _check(st, "otf2b_quantize")
    return packed, scales, ov, idx


def i8_head(x2d: torch.Tensor, w_i8: torch.Tensor, scales: torch.Tensor,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp32 logits [M, V] = (x2d @ w_i8.T) * scales (see otf_i8_head)."""
    _need_cuda(x2d, "x")
    M, D = x2d.shape
    V = w_i8.shape[0]
    ldx = _rows(x2d, "x", torch.float16, D)
    ldw = _rows(w_i8, "weight_int8", torch.int8, D)
    s = scales.reshape(-1)
    if s.dtype != torch.float16 or s.numel() != V or not s.is_contiguous():
        raise ValueError("scales must hold V contiguous fp16 values")
    for name, t in (("weight_int8", w_i8), ("scales", s)):
        _need_cuda(t, name)
    if out is None:
        out = torch.empty((M, V), dtype=torch.float32, device=x2d.device)
    ldl = _rows(out, "logits", torch.float32, V)
    with torch.cuda.device(x2d.device):
        st = lib().otf_i8_head(_ptr(x2d), ldx, _ptr(w_i8), ldw, _ptr(s), _ptr(out), ldl, M, V, D,
                               _stream(x2d.device))
    _check(st, "otf_i8_head")
    return out


def i8_head_argmax(x2d: torch.Tensor, w_i8: torch.Tensor, scales: torch.Tensor,
                   logits: Optional[torch.Tensor] = None):
    """Greedy step: int64 [M] first index of the largest logit per row (see otf_i8_head_argmax);
    also fills `logits` (fp32 [M, V]) when given."""
    _need_cuda(x2d, "x")
    M, D = x2d.shape
    V = w_i8.shape[0]
    ldx = _rows(x2d, "x", torch.float16, D)
    ldw = _rows(w_i8, "weight_int8", torch.int8, D)
    s = scales.reshape(-1)
    if s.dtype != torch.float16 or s.numel() != V or not s.is_contiguous():
        raise ValueError("scales must hold V contiguous fp16 values")
    for name, t in (("weight_int8", w_i8), ("scales", s)):
        _need_cuda(t, name)
    ldl = _rows(logits, "logits", torch.float32, V) if logits is not None else 0
    ids = torch.empty(M, dtype=torch.int64, device=x2d.device)
    with torch.cuda.device(x2d.device):
        st = lib().otf_i8_head_argmax(_ptr(x2d), ldx, _ptr(w_i8), ldw, _ptr(s), _ptr(logits), ldl, _ptr(ids), M, V, D,
                                      _stream(x2d.device))
    _check(st, "otf_i8_head_argmax")
    return ids


def i8_embed(ids: torch.Tensor, w_i8: torch.Tensor, scales: torch.Tensor,
             bad_flag: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp16 [n, D] rows of the INT8 embedding (bit-identical to the reference gather), into
    ``out`` (n rows of D fp16, row stride a multiple of 8 for the 16-byte-piece form) if given."""
    _need_cuda(ids, "input_ids")
    flat = ids.reshape(-1)
    if flat.dtype != torch.int64:
        flat = flat.to(torch.int64)
    flat = flat.contiguous()
    V, D = w_i8.shape
    ldw = _rows(w_i8, "weight_int8", torch.int8, D)
    s = scales.reshape(-1)
    if s.dtype != torch.float16 or s.numel() != V or not s.is_contiguous():
        raise ValueError("scales must hold V contiguous fp16 values")
    if w_i8.device != ids.device or s.device != ids.device:
        raise ValueError(f"weight_int8 and scales must be on {ids.device}")
    if out is None:
        out = torch.empty((flat.numel(), D), dtype=torch.float16, device=ids.device)
    elif out.dim() != 2 or out.shape[0] != flat.numel() or out.device != ids.device:
        raise ValueError(f"out must be [{flat.numel()}, {D}] on {ids.device}")
    ldo = _rows(out, "out", torch.float16, D)
    with torch.cuda.device(ids.device):
        st = lib().otf_i8_embed(_ptr(flat), flat.numel(), _ptr(w_i8), ldw, _ptr(s), _ptr(out), ldo, V, D,
                                _ptr(bad_flag), _stream(ids.device))
    _check(st, "otf_i8_embed")
    return out


def rmsnorm(x2d: torch.Tensor, weight: Optional[torch.Tensor], eps: float,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Llama RMSNorm over rows of x2d (fp16), see otf_rmsnorm."""
    _need_cuda(x2d, "x")
    M, K = x2d.shape
    ldx = _rows(x2d, "x", torch.float16, K)
    if weight is not None and (weight.dtype != torch.float16 or weight.numel() != K or not weight.is_contiguous()):
        raise ValueError("weight must be a contiguous fp16 vector of length K")
    if out is None:
        out = torch.empty_like(x2d)
    ldo = _rows(out, "out", torch.float16, K)
    with torch.cuda.device(x2d.device):
        st = lib().otf_rmsnorm(_ptr(x2d), ldx, _ptr(weight), float(eps), _ptr(out), ldo, M, K, _stream(x2d.device))
    _check(st, "otf_rmsnorm")
    return out


def silu_mul(g: torch.Tensor, u: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp16(silu(g)) * u elementwise (fp16), see otf_silu_mul."""
    _need_cuda(g, "gate")
    if g.shape != u.shape or g.dtype != torch.float16 or u.dtype != torch.float16:
        raise ValueError("gate and up must be fp16 tensors of the same shape")
    if not (g.is_contiguous() and u.is_contiguous()):
        raise ValueError("gate and up must be contiguous")
    if out is None:
        out = torch.empty_like(g)
    elif (out.dtype != torch.float16 or out.numel() != g.numel() or not out.is_contiguous()
          or out.device != g.device):
        raise ValueError("out must be a contiguous fp16 tensor with gate's element count on its device")
    with torch.cuda.device(g.device):
        st = lib().otf_silu_mul(_ptr(g), _ptr(u), _ptr(out), g.numel(), _stream(g.device))
    _check(st, "otf_silu_mul")
    return out


def device_error(clear: bool = True) -> int:
    """1 if a pipelined kernel gave up on a bounded wait since the last clear (synchronous)."""
    return int(lib().otf_device_error(1 if clear else 0))


class GroupItem:
    """One layer of `linear_group`: a SymmetricOTF2BitLinear-like module plus its input,
    output, optional residual and input transform (x_op with its aux vector and eps)."""

    def __init__(self, module, x: torch.Tensor, out: torch.Tensor, residual: Optional[torch.Tensor] = None,
                 x_op: int = OTF_XOP_NONE, x_aux: Optional[torch.Tensor] = None, eps: float = 0.0,
                 clamp: bool = True, ar=None, ar_mode: int = OTF_AR_NONE, ar_buf: int = 0,
                 ar_out: Optional[torch.Tensor] = None):
        self.m, self.x, self.out, self.residual = module, x, out, residual
        self.x_op, self.x_aux, self.eps, self.clamp = x_op, x_aux, eps, clamp
        # tensor-parallel exchange (otf_llm.tp_allreduce.PeerAllReduce): produce this layer's
        # rows into every rank's buffer ar_buf, or consume their sum as x (ar_out: its fp16 copy)
        self.ar, self.ar_mode, self.ar_buf, self.ar_out = ar, ar_mode, ar_buf, ar_out


def _layer_struct(it: GroupItem, keep: list) -> Layer:
    m = it.m
    K, N, G = m.d_in, m.out_features, m.group_size
    for name, t, dt, cols in (("x", it.x, torch.float16, K), ("out", it.out, torch.float16, N)):
        _need_cuda(t, name)
        _rows(t, name, dt, cols)
    if it.x.shape[0] != 1:
        raise ValueError("linear_group runs batch-1 decode steps")
    cb = (ctypes.c_float * 4)(*codebook_floats(m.codebook))
    keep.append(cb)
    has_o = getattr(m, "has_outliers", False)
    zeros = getattr(m, "zeros", None)
    L = Layer()
    L.x, L.ldx = it.x.data_ptr(), _rows(it.x, "x", torch.float16, K)
    L.packed, L.ld_packed = m.packed_uint8.data_ptr(), _rows(m.packed_uint8, "packed", torch.uint8, K // 4)
    L.scales, L.ld_scales = m.scales.data_ptr(), _rows(m.scales, "scales", torch.float16, K // G)
    if zeros is not None:
        L.zeros, L.ld_zeros = zeros.data_ptr(), _rows(zeros, "zeros", torch.float16, K // G)
    L.codebook = ctypes.cast(cb, ctypes.POINTER(ctypes.c_float))
    if has_o:
        L.mask = m.outlier_mask_vector.data_ptr()
        L.outlier_idx, L.n_outliers = m.outlier_indices.data_ptr(), m.outlier_indices.numel()
        L.outlier_vals = m.outliers_fp16.data_ptr()
        L.ld_outlier_vals = _rows(m.outliers_fp16, "outlier_vals", torch.float16, L.n_outliers)
    if getattr(m, "has_bias", False):
        L.bias = m.bias.data_ptr()
    if it.residual is not None:
        L.residual, L.ld_residual = it.residual.data_ptr(), _rows(it.residual, "residual", torch.float16, N)
    L.y, L.ldy = it.out.data_ptr(), _rows(it.out, "out", torch.float16, N)
    L.N, L.K, L.group_size = N, K, G
    L.flags = OTF_FLAG_CLAMP if it.clamp else 0
    L.x_op = it.x_op
    if it.x_aux is not None:
        if it.x_aux.dtype != torch.float16 or it.x_aux.numel() != K or not it.x_aux.is_contiguous():
            raise ValueError("x_aux must be a contiguous fp16 vector of length K")
        L.x_aux = it.x_aux.data_ptr()
    L.eps = float(it.eps)
    if it.ar is not None and it.ar_mode != OTF_AR_NONE:
        L.ar, L.ar_mode, L.ar_buf = it.ar.handle, int(it.ar_mode), int(it.ar_buf)
        if it.ar_out is not None:
            _need_cuda(it.ar_out, "ar_out")
            if it.ar_out.dtype != torch.float16 or it.ar_out.numel() != K or not it.ar_out.is_contiguous():
                raise ValueError("ar_out must be a contiguous fp16 vector of length K")
            L.ar_out = it.ar_out.data_ptr()
    return L


def linear_group(items: Sequence[GroupItem]) -> None:
    """Run up to 4 decode-step layers in one launch (see otf2b_linear_group)."""
    if not 1 <= len(items) <= 4:
        raise ValueError("linear_group takes 1 to 4 layers")
    dev = items[0].x.device
    keep: list = []
    arr = (Layer * len(items))(*[_layer_struct(it, keep) for it in items])
    with torch.cuda.device(dev):
        st = lib().otf2b_linear_group(arr, len(items), _stream(dev))
    _check(st, "otf2b_linear_group")


def proj_struct(m) -> Proj:
    """otf2b_proj view of a SymmetricOTF2BitLinear's buffers (pointers only; keep m alive)."""
    K, N, G = m.d_in, m.out_features, m.group_size
    p = Proj()
    p.packed, p.ld_packed = m.packed_uint8.data_ptr(), _rows(m.packed_uint8, "packed", torch.uint8, K // 4)
    p.scales, p.ld_scales = m.scales.data_ptr(), _rows(m.scales, "scales", torch.float16, K // G)
    if m.has_outliers:
        p.mask = m.outlier_mask_vector.data_ptr()
        p.outlier_idx, p.n_outliers = m.outlier_indices.data_ptr(), m.outlier_indices.numel()
        p.outlier_vals = m.outliers_fp16.data_ptr()
        p.ld_outlier_vals = _rows(m.outliers_fp16, "outlier_vals", torch.float16, p.n_outliers)
    if m.has_bias:
        p.bias = m.bias.data_ptr()
    p.N, p.K = N, K
    return p


class DecodeStep:
    """One persistent launch per decode step of a Llama-shaped 2-bit stack (otf2b_decode_step).

    layers: per decoder layer a mapping q_proj ... down_proj -> SymmetricOTF2BitLinear;
    norms: per layer (input, post-attention) RMSNorm weights (fp16 [hidden]).
    """

    def __init__(self, layers, norms, hidden: int, intermediate: int, heads: int, kv_heads: int, head_dim: int,
                 group_size: int, eps: float, codebook, device):
        self.device = torch.device(device)
        d = DecodeDims()
        d.n_layers, d.hidden, d.intermediate = len(layers), hidden, intermediate
        d.heads, d.kv_heads, d.head_dim, d.group_size, d.eps = heads, kv_heads, head_dim, group_size, float(eps)
        for i, c in enumerate(codebook_floats(codebook)):
            d.codebook[i] = c
        self.dims = d
        n = lib().otf2b_decode_workspace_bytes(ctypes.byref(d))
        if n < 0:
            raise ValueError("dimensions not supported by otf2b_decode_step")
        self.ws = torch.zeros(int(n), dtype=torch.uint8, device=self.device)
        arr = (DecoderLayer * len(layers))()
        keep = []
        for i, (mods, (wi, wp)) in enumerate(zip(layers, norms)):
            for name, field in (("q_proj", "q"), ("k_proj", "k"), ("v_proj", "v"), ("o_proj", "o"),
                                ("gate_proj", "gate"), ("up_proj", "up"), ("down_proj", "down")):
                setattr(arr[i], field, proj_struct(mods[name]))
            wi = wi.to(device=self.device, dtype=torch.float16).contiguous()
            wp = wp.to(device=self.device, dtype=torch.float16).contiguous()
            keep += [wi, wp]
            arr[i].input_norm, arr[i].post_norm = wi.data_ptr(), wp.data_ptr()
        self._keep = (keep, layers)
        with torch.cuda.device(self.device):
            _check(lib().otf2b_decode_prepare(arr, ctypes.byref(d), self.ws.data_ptr(), self.ws.numel()),
                   "otf2b_decode_prepare")
        self.h = torch.zeros(hidden, dtype=torch.float16, device=self.device)

    def __call__(self, h: torch.Tensor) -> torch.Tensor:
        """h fp16 [1, hidden] -> the residual stream after every layer ([1, hidden], an internal buffer)."""
        self.h.copy_(h.reshape(-1))
        with torch.cuda.device(self.device):
            _check(lib().otf2b_decode_step(ctypes.byref(self.dims), self.h.data_ptr(), self.ws.data_ptr(),
                                           _stream(self.device)), "otf2b_decode_step")
        return self.h.view(1, -1)
