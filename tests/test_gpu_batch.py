"""GPU parity of the batched (2 <= M <= 8 activation rows per launch) 2-bit linear path
against the oracle (bar: max rel err 1e-3), including slices of more than 8 rows, residual
rows, zero points and the reference module's [B, T, K] input."""
import numpy as np
import pytest
import torch

from oracle import oracle
from conftest import rel_err
from test_gpu_linear import _random_layer

pytestmark = pytest.mark.gpu
TOL = 1e-3


@pytest.mark.parametrize("N,K,G,M,n_out,zeros,bias", [
    (4096, 4096, 64, 2, 20, False, False),
    (4096, 4096, 64, 4, 20, False, True),
    (1000, 4096, 64, 5, 20, False, False),
    (1024, 8192, 64, 8, 40, False, True),
    (512, 11008, 64, 3, 55, False, False),
    (333, 1024, 128, 6, 5, True, True),
    (300, 2048, 256, 7, 10, False, False),
    (777, 4096, 64, 11, 20, False, False),     # 8 + 3 rows: two slices
    (48, 256, 64, 4, 1, False, False),
    (17, 192, 64, 2, 0, True, False),
])
def test_batched_layers(N, K, G, M, n_out, zeros, bias, cuda_dev):
    from otf_llm import _native
    packed, scales, z, idx, ov, b, mask = _random_layer(N, K, G, n_out, cuda_dev, seed=N * 13 + K + M)
    x = (torch.randn(M, K, generator=torch.Generator().manual_seed(K + M)) * 1.5).half()
    cb = oracle.CB_F32 if zeros else oracle.CB_F16.astype(np.float32)
    ref = oracle.linear_f32(x.numpy(), packed.numpy(), scales.numpy(), G, codebook=cb,
                            zeros=None if z is None else z.numpy(), mask=None if mask is None else mask.numpy(),
                            outlier_idx=None if idx is None else idx.numpy(),
                            outlier_vals=None if ov is None else ov.numpy(), bias=None if b is None else b.numpy())
    d = lambda t: None if t is None else t.to(cuda_dev)
    y = _native.linear_2bit(x.to(cuda_dev), packed.to(cuda_dev), scales.to(cuda_dev), G, cb, zeros=d(z),
                            mask=d(mask), outlier_idx=d(idx), outlier_vals=d(ov), bias=d(b), clamp=True)
    torch.cuda.synchronize()
    assert _native.device_error(True) == 0
    e = rel_err(y.cpu().numpy(), ref)
    assert e < TOL, (N, K, G, M, e)
    # every batch row on its own matches its row of the batched result's bar too
    for m in (0, M - 1):
        e1 = rel_err(y[m:m + 1].cpu().numpy(), ref[m:m + 1])
        assert e1 < TOL, (m, e1)


def test_batched_residual_and_module_shape(cuda_dev):
    from otf_llm import _native
    from otf_llm.symmetric_2bit_engine import SymmetricOTF2BitLinear
    N, K, G, M = 2048, 4096, 64, 6
    packed, scales, _, idx, ov, b, mask = _random_layer(N, K, G, 20, cuda_dev, seed=5, bias=True)
    x = (torch.randn(M, K, generator=torch.Generator().manual_seed(3)) * 1.5).half()
    res = (torch.randn(M, N, generator=torch.Generator().manual_seed(4))).half()
    cb = oracle.CB_F16.astype(np.float32)
    ref = oracle.linear_f32(x.numpy(), packed.numpy(), scales.numpy(), G, codebook=cb, mask=mask.numpy(),
                            outlier_idx=idx.numpy(), outlier_vals=ov.numpy(), bias=b.numpy())
    y = _native.linear_2bit(x.to(cuda_dev), packed.to(cuda_dev), scales.to(cuda_dev), G, cb, mask=mask.to(cuda_dev),
                            outlier_idx=idx.to(cuda_dev), outlier_vals=ov.to(cuda_dev), bias=b.to(cuda_dev),
                            residual=res.to(cuda_dev))
    assert rel_err(y.cpu().numpy(), ref + res.float().numpy()) < TOL
    # the reference module surface: x [B, T, K] -> y [B, T, N]
    lay = SymmetricOTF2BitLinear(packed.to(cuda_dev), scales.to(cuda_dev), K, G, ov.to(cuda_dev), idx.to(cuda_dev),
                                 b.to(cuda_dev))
    y3 = lay(x.to(cuda_dev).view(2, 3, K))
    assert y3.shape == (2, 3, N)
    assert rel_err(y3.reshape(M, N).cpu().numpy(), ref) < TOL


def test_batched_deterministic(cuda_dev):
    from otf_llm import _native
    N, K, G, M = 1536, 4096, 64, 8
    packed, scales, _, idx, ov, _, mask = _random_layer(N, K, G, 20, cuda_dev, seed=9)
    x = (torch.randn(M, K, generator=torch.Generator().manual_seed(1))).half().to(cuda_dev)
    args = (packed.to(cuda_dev), scales.to(cuda_dev), G, None)
    kw = dict(mask=mask.to(cuda_dev), outlier_idx=idx.to(cuda_dev), outlier_vals=ov.to(cuda_dev))
    y1 = _native.linear_2bit(x, *args, **kw)
    y2 = _native.linear_2bit(x, *args, **kw)
    assert torch.equal(y1, y2)
