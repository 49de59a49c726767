"""GPU parity of the tcgen05 dequant GEMM (otf2b_gemm_mma; otf2b_linear from 16 rows) against
the oracle (bar: max rel err 1e-3), over group sizes, zero points, anchors, ragged M/N/K, a
non-affine codebook and the reference module's [B, T, K] input."""
import numpy as np
import pytest
import torch

from oracle import oracle
from conftest import rel_err
from test_gpu_linear import _random_layer

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _run(N, K, G, M, n_out, zeros, bias, dev, codebook=None, forced=False, residual=False, seed=0):
    from otf_llm import _native
    packed, scales, z, idx, ov, b, mask = _random_layer(N, K, G, n_out, dev, seed=seed + N * 3 + K + M, zeros=zeros,
                                                        bias=bias)
    x = (torch.randn(M, K, generator=torch.Generator().manual_seed(K + M)) * 1.5).half()
    res = torch.randn(M, N, generator=torch.Generator().manual_seed(7)).half() if residual else None
    if codebook is None:
        cb = oracle.CB_F32 if zeros else oracle.CB_F16.astype(np.float32)
    else:
        cb = np.asarray(codebook, dtype=np.float32)
    ref = oracle.linear_f32(x.numpy(), packed.numpy(), scales.numpy(), G, codebook=cb,
                            zeros=None if z is None else z.numpy(), mask=None if mask is None else mask.numpy(),
                            outlier_idx=None if idx is None else idx.numpy(),
                            outlier_vals=None if ov is None else ov.numpy(), bias=None if b is None else b.numpy())
    if res is not None:
        ref = ref + res.float().numpy()
    d = lambda t: None if t is None else t.to(dev)
    y = _native.linear_2bit(x.to(dev), packed.to(dev), scales.to(dev), G, cb, zeros=d(z), mask=d(mask),
                            outlier_idx=d(idx), outlier_vals=d(ov), bias=d(b), residual=d(res), clamp=True,
                            gemm_mma=forced)
    torch.cuda.synchronize()
    assert _native.device_error(True) == 0
    return y.cpu().numpy(), ref


@pytest.mark.parametrize("N,K,G,M,n_out,zeros,bias", [
    (256, 4096, 64, 16, 20, False, False),
    (1000, 4096, 64, 48, 20, False, True),
    (300, 1024, 128, 64, 5, True, True),
    (777, 2048, 32, 100, 10, False, False),
    (128, 512, 256, 130, 1, False, False),
    (4096, 8192, 64, 64, 40, False, False),
    (512, 11008, 64, 32, 55, False, False),
    (200, 4160, 32, 24, 20, True, False),     # 65 tiles of 64 codes (odd tile count)
    (129, 192, 32, 17, 0, False, True),
])
def test_tc_gemm(N, K, G, M, n_out, zeros, bias, cuda_dev):
    y, ref = _run(N, K, G, M, n_out, zeros, bias, cuda_dev, forced=True)
    assert rel_err(y, ref) < TOL, (N, K, G, M, rel_err(y, ref))


@pytest.mark.parametrize("M", [1, 3, 8])
def test_tc_gemm_forced_small_batch(M, cuda_dev):
    y, ref = _run(640, 4096, 64, M, 20, False, True, cuda_dev, forced=True, residual=True)
    assert rel_err(y, ref) < TOL


def test_tc_gemm_any_codebook(cuda_dev):
    # The table-lookup dequant needs no affine codebook (the integer-MMA GEMV does).
    y, ref = _run(384, 2048, 64, 32, 10, False, False, cuda_dev, codebook=[-1.0, -0.3, 0.5, 1.7], forced=True)
    assert rel_err(y, ref) < TOL


def test_tc_gemm_module_prefill(cuda_dev):
    from otf_llm.symmetric_2bit_engine import SymmetricOTF2BitLinear
    N, K, G = 1024, 4096, 64
    packed, scales, _, idx, ov, b, mask = _random_layer(N, K, G, 20, cuda_dev, seed=11, bias=True)
    lay = SymmetricOTF2BitLinear(packed.to(cuda_dev), scales.to(cuda_dev), K, G, ov.to(cuda_dev), idx.to(cuda_dev),
                                 b.to(cuda_dev))
    x = (torch.randn(2, 40, K, generator=torch.Generator().manual_seed(2))).half()
    ref = oracle.linear_f32(x.view(80, K).numpy(), packed.numpy(), scales.numpy(), G,
                            codebook=oracle.CB_F16.astype(np.float32), mask=mask.numpy(), outlier_idx=idx.numpy(),
                            outlier_vals=ov.numpy(), bias=b.numpy())
    y = lay(x.to(cuda_dev))
    assert y.shape == (2, 40, N)
    assert rel_err(y.view(80, N).cpu().numpy(), ref) < TOL


def test_tc_gemm_deterministic(cuda_dev):
    from otf_llm import _native
    N, K, G, M = 768, 4096, 64, 64
    packed, scales, _, idx, ov, _, mask = _random_layer(N, K, G, 20, cuda_dev, seed=4)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(1)).half().to(cuda_dev)
    args = (packed.to(cuda_dev), scales.to(cuda_dev), G, None)
    kw = dict(mask=mask.to(cuda_dev), outlier_idx=idx.to(cuda_dev), outlier_vals=ov.to(cuda_dev))
    assert torch.equal(_native.linear_2bit(x, *args, **kw), _native.linear_2bit(x, *args, **kw))


def test_tc_auto_route_matches_forced(cuda_dev):
    # otf2b_linear sends 64 rows to the tcgen05 GEMM by itself: same bits as the forced call.
    from otf_llm import _native
    N, K, G, M = 2048, 8192, 64, 64
    packed, scales, _, idx, ov, _, mask = _random_layer(N, K, G, 40, cuda_dev, seed=6)
    x = torch.randn(M, K, generator=torch.Generator().manual_seed(8)).half().to(cuda_dev)
    args = (packed.to(cuda_dev), scales.to(cuda_dev), G, None)
    kw = dict(mask=mask.to(cuda_dev), outlier_idx=idx.to(cuda_dev), outlier_vals=ov.to(cuda_dev))
    assert torch.equal(_native.linear_2bit(x, *args, **kw), _native.linear_2bit(x, *args, gemm_mma=True, **kw))
