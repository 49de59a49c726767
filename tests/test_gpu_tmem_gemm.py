"""GPU parity of the tensor-memory tcgen05 GEMM (k_gemm2b_tmem: otf2b_linear from 9
activation rows, otf2b_gemm_mma) against the oracle (bar: max rel err 1e-3).

The kernel takes symmetric layers with G 32 or 64 and 16-byte aligned code, scale and
activation rows; every case below has such rows (scale rows padded to a multiple of 8 groups
where K/G is not) and they cover ragged M, N and K, the split of K over a cluster, anchors,
bias, residual, a non-affine codebook, CUDA-graph replay and determinism."""
import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import oracle
from test_gpu_linear_shapes import _layer, _ref

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _run(L, x, residual=None, codebook=None, gemm_mma=False, out=None):
    from otf_llm import _native
    return _native.linear_2bit(x, L["packed"], L["scales"], L["G"], codebook, mask=L["mask"], outlier_idx=L["idx"],
                               outlier_vals=L["ov"], bias=L["bias"], residual=residual, clamp=True,
                               gemm_mma=gemm_mma, out=out)


@pytest.mark.parametrize("N,K,G,M,n_out,bias,res", [
    (256, 4096, 64, 9, 20, False, False),
    (256, 4096, 64, 16, 20, True, True),
    (1000, 4096, 64, 17, 20, False, True),
    (4100, 4096, 64, 31, 20, True, False),
    (333, 2048, 32, 64, 10, False, False),
    (256, 4160, 64, 48, 20, False, False),    # 65 groups: a last K tile and super-stage past K
    (4096, 11008, 64, 16, 55, False, True),   # 7B down_proj: split K over the cluster
    (11008, 4096, 64, 64, 20, False, False),
    (8192, 28672, 64, 16, 143, False, False), # 70B down_proj: three anchor tiles
    (28672, 8192, 64, 64, 40, False, False),
    (512, 8192, 32, 100, 40, True, True),     # NB 128
    (300, 4096, 64, 130, 20, False, True),    # NB 256
    (129, 1024, 64, 257, 5, True, False),     # two column blocks of 256
    (640, 4096, 64, 24, 0, False, False),     # no anchors
])
def test_tmem_gemm(N, K, G, M, n_out, bias, res, cuda_dev):
    from otf_llm import _native
    L = _layer(N, K, G, n_out, cuda_dev, seed=N + 3 * K + M)
    gen = torch.Generator().manual_seed(K + M)
    x = (torch.randn(M, K, generator=gen) * 1.5).half().to(cuda_dev)
    r = torch.randn(M, N, generator=gen).half().to(cuda_dev) if res else None
    ref = _ref(L, x, r)
    y = _run(L, x, r)
    y2 = _run(L, x, r, gemm_mma=True)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    err = rel_err(y.cpu().numpy(), ref)
    print(f"{N}x{K} G{G} M{M}: rel err {err:.2e}")
    assert err < TOL
    assert torch.equal(y, y2)  # same kernel either way, deterministic


def test_tmem_gemm_codebook_and_graph(cuda_dev):
    """A non-affine codebook (the dequant is a table lookup) and a captured launch."""
    L = _layer(1024, 4096, 64, 20, cuda_dev, seed=77)
    cb = np.array([-1.3, -0.2, 0.55, 1.7], dtype=np.float32)
    x = torch.randn(32, 4096, device=cuda_dev).half()
    p = lambda t: None if t is None else t.cpu().numpy()
    ref = oracle.linear_f32(p(x), p(L["packed"]), p(L["scales"]), 64, codebook=cb.astype(np.float16).astype(np.float32),
                            mask=p(L["mask"]), outlier_idx=p(L["idx"]), outlier_vals=p(L["ov"]))
    y = torch.empty(32, 1024, dtype=torch.float16, device=cuda_dev)
    _run(L, x, codebook=cb, out=y)
    assert rel_err(y.cpu().numpy(), ref) < TOL
    eager = y.clone()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        _run(L, x, codebook=cb, out=y)
    torch.cuda.current_stream().wait_stream(st)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        _run(L, x, codebook=cb, out=y)
    y.zero_()
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, eager)
