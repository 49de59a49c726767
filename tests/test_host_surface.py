"""Host-side checks that need no GPU: the drop-in surface, quantizers, the C ABI."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from conftest import ROOT, load_golden


def test_native_library_exports_header_symbols():
    from otf_llm import _native
    hdr = open(os.path.join(ROOT, "include", "otf_b200.h")).read()
    declared = set(re.findall(r"OTF_API\s+[\w\s\*]+?\b(\w+)\s*\(", hdr))
    assert declared, "no OTF_API declarations parsed"
    assert declared == set(_native.EXPORTS)
    lib = ctypes.CDLL(_native.library_path())
    for name in declared:
        assert hasattr(lib, name), name
    L = _native.lib()
    assert L.otf_version() >= 100
    assert L.otf_status_string(0) == b"ok"


def test_no_cpu_fallback():
    from otf_llm.symmetric_2bit_engine import SymmetricOTF2BitLinear
    gd = load_golden("sym_g64_small")
    lay = SymmetricOTF2BitLinear(torch.from_numpy(gd["packed"]), torch.from_numpy(gd["scales"]), 192, 64,
                                 torch.from_numpy(gd["outliers"]), torch.from_numpy(gd["outlier_idx"]))
    with pytest.raises(RuntimeError, match="CUDA"):
        lay(torch.from_numpy(gd["x_m1"]))


def test_module_buffers_match_reference_layout():
    from otf_llm.otf_2bit_quantizer import OTF2BitLinear
    from otf_llm.symmetric_2bit_engine import QuantizedEmbedding, QuantizedLinearHead, SymmetricOTF2BitLinear
    gd = load_golden("sym_g64_small")
    lay = SymmetricOTF2BitLinear(torch.from_numpy(gd["packed"]), torch.from_numpy(gd["scales"]), 192, 64,
                                 torch.from_numpy(gd["outliers"]), torch.from_numpy(gd["outlier_idx"]),
                                 torch.from_numpy(gd["bias"]))
    sd = lay.state_dict()
    assert list(sd) == ["packed_uint8", "scales", "codebook", "bias", "outliers_fp16", "outlier_indices",
                        "outlier_mask_vector"]
    assert sd["codebook"].dtype == torch.float16 and sd["outlier_indices"].dtype == torch.int64
    assert np.array_equal(sd["outlier_mask_vector"].numpy(), gd["mask"])
    ga = load_golden("asym_g32")
    al = OTF2BitLinear(*(torch.from_numpy(ga[k]) for k in ("packed", "scales", "zeros")), 256, 32,
                       torch.from_numpy(ga["outliers"]), torch.from_numpy(ga["outlier_idx"]),
                       torch.from_numpy(ga["bias"]))
    assert list(al.state_dict()) == ["packed_uint8", "scales", "zeros", "codebook", "bias", "outliers_fp16",
                                     "outlier_indices", "outlier_mask_vector"]
    assert al.codebook.dtype == torch.float32
    emb, head = QuantizedEmbedding(10, 8), QuantizedLinearHead(8, 10)
    assert list(emb.state_dict()) == ["weight_int8", "scales"] == list(head.state_dict())
    head.weight_int8 = emb.weight_int8
    assert head.weight_int8.data_ptr() == emb.weight_int8.data_ptr()


@pytest.mark.parametrize("name", ["quant_g64", "sym_g64_small"])
def test_symmetric_quantizer_bit_exact(name):
    from otf_llm.symmetric_2bit_engine import Symmetric2BitQuantizer
    gd = load_golden(name)
    q = Symmetric2BitQuantizer(int(gd["G"]), float(gd["ratio"]))
    packed, scales, ov, oi = q.quantize_tensor(torch.from_numpy(gd["W"]), torch.from_numpy(gd["act"]), row_chunk=16)
    assert np.array_equal(oi.numpy(), gd["outlier_idx"])
    assert np.array_equal(ov.numpy().view(np.uint16), gd["outliers"].view(np.uint16))
    assert np.array_equal(packed.numpy(), gd["packed"])
    assert np.array_equal(scales.numpy().view(np.uint16), gd["scales"].view(np.uint16))


def test_asymmetric_unpack_bit_exact():
    from otf_llm.otf_2bit_quantizer import OTF2BitQuantizer
    gd = load_golden("asym_g32")
    w = OTF2BitQuantizer(group_size=32).unpack_2bit_uint8(torch.from_numpy(gd["packed"]),
                                                         torch.from_numpy(gd["scales"]),
                                                         torch.from_numpy(gd["zeros"]), 256)
    assert np.array_equal(w.numpy().view(np.uint16), gd["W_dequant"].view(np.uint16))


def test_int8_quantize_from_fp16_bit_exact():
    from otf_llm.symmetric_2bit_engine import QuantizedEmbedding
    gd = load_golden("int8_v1000_d256")
    emb = QuantizedEmbedding(*gd["W_fp16"].shape)
    emb.quantize_from_fp16(torch.from_numpy(gd["W_fp16"]), chunk_size=300)
    assert np.array_equal(emb.weight_int8.numpy(), gd["weight_int8"])
    assert np.array_equal(emb.scales.numpy().view(np.uint16), gd["scales"].view(np.uint16))


def test_pack_matches_reference_packing():
    from otf_llm.symmetric_2bit_engine import Symmetric2BitQuantizer
    gd = load_golden("codes_pack")
    got = Symmetric2BitQuantizer().pack_2bit_uint8(torch.from_numpy(gd["codes"]))
    assert np.array_equal(got.numpy(), gd["packed"])
    # the same buffer read as little-endian int32 holds 16 codes per word
    w32 = torch.from_numpy(gd["packed"]).view(torch.int32).numpy().astype(np.int64) & 0xFFFFFFFF
    k = np.arange(gd["codes"].shape[1])
    assert np.array_equal((w32[:, k // 16] >> (2 * (k % 16))) & 3, gd["codes"])


def test_gpu_quantizer_refuses_cpu_tensors():
    """The native quantizer entry point has no CPU path (the module-level quantize_tensor keeps
    the reference's torch ops for CPU tensors, checked against the fixtures above)."""
    from otf_llm import _native
    with pytest.raises(RuntimeError, match="CUDA"):
        _native.quantize_2b(torch.zeros(8, 64), 32, 1)


def test_quantize_abi_rejects_bad_arguments():
    """otf2b_quantize validates sizes, group sizes, strides and outlier counts before touching
    the device (no GPU needed for these checks)."""
    import ctypes

    from otf_llm import _native
    L = _native.lib()
    i64 = ctypes.c_int64
    nul = None
    OTF_ERR_INVALID, OTF_ERR_UNSUPPORTED = 1, 2

    def call(w, dtype, ldw, N, K, G, k, packed, ldp, scales, lds, ov=None, ldo=0, idx=None, ws=None, nws=0):
        return L.otf2b_quantize(w, dtype, ldw, N, K, G, nul, k, nul, ws, nws, packed, ldp, scales, lds, ov, ldo, idx,
                                nul)

    fake = ctypes.c_void_p(1 << 20)   # never dereferenced: every case fails validation first
    assert call(nul, 0, 64, 8, 64, 32, 0, fake, 16, fake, 2) == OTF_ERR_INVALID          # no weights
    assert call(fake, 0, 64, 8, 64, 48, 0, fake, 16, fake, 2) == OTF_ERR_UNSUPPORTED     # group size 48
    assert call(fake, 0, 64, 8, 96, 64, 0, fake, 24, fake, 2) == OTF_ERR_INVALID         # K % G
    assert call(fake, 0, 62, 8, 64, 32, 0, fake, 16, fake, 2) == OTF_ERR_INVALID         # ldw < K
    assert call(fake, 7, 64, 8, 64, 32, 0, fake, 16, fake, 2) == OTF_ERR_INVALID         # dtype
    assert call(fake, 0, 64, 8, 64, 32, 65, fake, 16, fake, 2) == OTF_ERR_INVALID        # k > K
    assert call(fake, 0, 64, 8, 64, 32, 2, fake, 16, fake, 2) == OTF_ERR_INVALID         # anchors, no buffers
    assert L.otf2b_quantize_workspace_bytes(300, 1024) == (2 * 1024 * 4) + 1024 * 4 + 256   # 2 row chunks
