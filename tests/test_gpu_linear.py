"""GPU parity of the 2-bit linear kernels against the oracle (bar: max rel err 1e-3)."""
import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-3
SYM = ["sym_g64_small", "sym_g64_k4096", "sym_g32_legacy", "sym_g128"]


def _t(a, dev, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    return t if dtype is None else t.to(dtype)


def _ms(gd):
    return sorted(int(k[3:]) for k in gd if k.startswith("x_m"))


@pytest.mark.parametrize("name", SYM)
def test_symmetric_module_golden(name, cuda_dev):
    from otf_llm.symmetric_2bit_engine import SymmetricOTF2BitLinear
    gd = load_golden(name)
    K = gd["packed"].shape[1] * 4
    lay = SymmetricOTF2BitLinear(_t(gd["packed"], cuda_dev), _t(gd["scales"], cuda_dev), K, int(gd["G"]),
                                 _t(gd["outliers"], cuda_dev), _t(gd["outlier_idx"], cuda_dev),
                                 _t(gd["bias"], cuda_dev) if "bias" in gd else None)
    for M in _ms(gd):
        x = gd[f"x_m{M}"]
        y = lay(_t(x, cuda_dev).view(1, M, K)).view(M, -1).cpu().numpy()
        ref = oracle.linear_f32(x, gd["packed"], gd["scales"], int(gd["G"]), mask=gd["mask"],
                                outlier_idx=gd["outlier_idx"], outlier_vals=gd["outliers"], bias=gd.get("bias"))
        assert y.dtype == np.float16
        assert rel_err(y, ref) < TOL, (name, M)
        assert rel_err(y, gd[f"y_ref_m{M}"]) < 1.5e-3   # vs the reference's own fp16 output


@pytest.mark.parametrize("name", SYM)
def test_gemm_function_golden(name, cuda_dev):
    from otf_llm.otf_triton_2bit_kernel import triton_symmetric_2bit_gemm
    gd = load_golden(name)
    for M in _ms(gd):
        y = triton_symmetric_2bit_gemm(_t(gd[f"x_m{M}"], cuda_dev), _t(gd["packed"], cuda_dev),
                                       _t(gd["scales"], cuda_dev), None, int(gd["G"]), _t(gd["mask"], cuda_dev))
        ref = oracle.linear_f32(gd[f"x_m{M}"], gd["packed"], gd["scales"], int(gd["G"]), mask=gd["mask"])
        assert rel_err(y.cpu().numpy(), ref) < TOL


def test_asymmetric_module_golden(cuda_dev):
    from otf_llm.otf_2bit_quantizer import OTF2BitLinear
    gd = load_golden("asym_g32")
    lay = OTF2BitLinear(*(_t(gd[k], cuda_dev) for k in ("packed", "scales", "zeros")), 256, 32,
                        _t(gd["outliers"], cuda_dev), _t(gd["outlier_idx"], cuda_dev), _t(gd["bias"], cuda_dev))
    lay = lay.to(cuda_dev)
    for M in (1, 3):
        y = lay(_t(gd[f"x_m{M}"], cuda_dev)).cpu().numpy()
        assert rel_err(y, gd[f"y_f64_m{M}"]) < TOL
        assert rel_err(y, gd[f"y_a7_m{M}"]) < 1.5e-3


def _random_layer(N, K, G, n_out, dev, seed, zeros=False, bias=False):
    g = torch.Generator(device="cpu").manual_seed(seed)
    packed = torch.randint(0, 256, (N, K // 4), generator=g, dtype=torch.int32).to(torch.uint8)
    scales = (torch.rand(N, K // G, generator=g) * 0.03 + 0.002).half()
    z = (torch.randn(N, K // G, generator=g) * 0.01).half() if zeros else None
    idx = torch.randperm(K, generator=g)[:n_out] if n_out else None
    ov = (torch.randn(N, n_out, generator=g) * 0.05).half() if n_out else None
    b = (torch.randn(N, generator=g) * 0.1).half() if bias else None
    mask = None
    if n_out:
        mask = torch.ones(K, dtype=torch.float16)
        mask[idx] = 0
    return packed, scales, z, idx, ov, b, mask


@pytest.mark.parametrize("N,K,G,M,n_out,zeros,bias", [
    (1, 64, 64, 1, 0, False, False),
    (17, 192, 64, 1, 1, False, True),
    (100, 256, 32, 1, 3, True, False),
    (1000, 4096, 64, 1, 20, False, False),
    (333, 1024, 128, 1, 5, False, True),
    (24, 512, 256, 1, 2, False, False),
    (37, 192, 64, 3, 1, False, True),
    (64, 4096, 64, 8, 20, True, True),
    (40, 96, 32, 2, 0, False, False),
    (8, 100, 4, 1, 0, False, False),
])
def test_random_layers(N, K, G, M, n_out, zeros, bias, cuda_dev):
    from otf_llm import _native
    packed, scales, z, idx, ov, b, mask = _random_layer(N, K, G, n_out, cuda_dev, seed=N * 7 + K)
    x = (torch.randn(M, K, generator=torch.Generator().manual_seed(K)) * 1.5).half()
    cb = oracle.CB_F32 if zeros else oracle.CB_F16.astype(np.float32)
    ref = oracle.linear_f32(x.numpy(), packed.numpy(), scales.numpy(), G, codebook=cb,
                            zeros=None if z is None else z.numpy(), mask=None if mask is None else mask.numpy(),
                            outlier_idx=None if idx is None else idx.numpy(),
                            outlier_vals=None if ov is None else ov.numpy(), bias=None if b is None else b.numpy())
    d = lambda t: None if t is None else t.to(cuda_dev)
    for generic in (False, True):
        y = _native.linear_2bit(x.to(cuda_dev), packed.to(cuda_dev), scales.to(cuda_dev), G, cb,
                                zeros=d(z), mask=d(mask), outlier_idx=d(idx), outlier_vals=d(ov), bias=d(b),
                                clamp=True, force_generic=generic)
        assert rel_err(y.cpu().numpy(), ref) < TOL, (generic,)


@pytest.mark.parametrize("N,K", [(11008, 4096), (4096, 11008), (4096, 4096), (1024, 3072), (8192, 28672)])
def test_full_size_shapes(N, K, cuda_dev):
    """Llama-2-7B, Llama-3.2-3B and Llama-3-70B projection shapes at G=64, 0.5% anchors."""
    from otf_llm import _native
    n_out = max(1, int(K * 0.005))
    packed, scales, _, idx, ov, _, mask = _random_layer(N, K, 64, n_out, cuda_dev, seed=K + N)
    x = torch.randn(1, K, generator=torch.Generator().manual_seed(N)).half()
    ref = oracle.linear_f32(x.numpy(), packed.numpy(), scales.numpy(), 64, mask=mask.numpy(),
                            outlier_idx=idx.numpy(), outlier_vals=ov.numpy())
    args = [t.to(cuda_dev) for t in (x, packed, scales)]
    y1 = _native.linear_2bit(*args, 64, None, mask=mask.to(cuda_dev), outlier_idx=idx.to(cuda_dev),
                             outlier_vals=ov.to(cuda_dev))
    y2 = _native.linear_2bit(*args, 64, None, mask=mask.to(cuda_dev), outlier_idx=idx.to(cuda_dev),
                             outlier_vals=ov.to(cuda_dev))
    assert rel_err(y1.cpu().numpy(), ref) < TOL
    assert torch.equal(y1, y2)  # deterministic
    assert _native.device_error() == 0  # no pipeline wait gave up


def test_unpack_codes_bit_exact(cuda_dev):
    from otf_llm import _native
    gd = load_golden("codes_pack")
    K = gd["codes"].shape[1]
    got = _native.unpack_codes(_t(gd["packed"], cuda_dev), K).cpu().numpy()
    assert np.array_equal(got, gd["codes"])
    big = torch.randint(0, 256, (4096, 1024), dtype=torch.int32).to(torch.uint8)
    got = _native.unpack_codes(big.to(cuda_dev), 4096).cpu().numpy()
    assert np.array_equal(got, oracle.unpack_codes(big.numpy(), 4096))


def test_outlier_columns_are_masked(cuda_dev):
    """Codes at anchor columns are nonzero (argmin tie -> code 1); the mask must remove them."""
    from otf_llm import _native
    gd = load_golden("sym_g64_k4096")
    x = gd["x_m1"]
    packed, scales = _t(gd["packed"], cuda_dev), _t(gd["scales"], cuda_dev)
    y_mask = _native.linear_2bit(_t(x, cuda_dev), packed, scales, 64, None, mask=_t(gd["mask"], cuda_dev))
    y_nomask = _native.linear_2bit(_t(x, cuda_dev), packed, scales, 64, None)
    ref = oracle.linear_f32(x, gd["packed"], gd["scales"], 64, mask=gd["mask"])
    assert rel_err(y_mask.cpu().numpy(), ref) < TOL
    assert rel_err(y_nomask.cpu().numpy(), ref) > 5 * TOL


def test_cuda_graph_capture(cuda_dev):
    from otf_llm.symmetric_2bit_engine import SymmetricOTF2BitLinear
    gd = load_golden("sym_g64_k4096")
    lay = SymmetricOTF2BitLinear(_t(gd["packed"], cuda_dev), _t(gd["scales"], cuda_dev), 4096, 64,
                                 _t(gd["outliers"], cuda_dev), _t(gd["outlier_idx"], cuda_dev))
    x = _t(gd["x_m1"], cuda_dev)
    y_eager = lay(x)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        lay(x)
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        y_graph = lay(x)
    graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(y_eager, y_graph)
