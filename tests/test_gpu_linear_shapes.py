"""GPU parity of the batch-1 GEMV on scale rows padded to 16 bytes (the decoder stacks'
layout) against the oracle (bar: max rel err 1e-3 against the fp32 oracle): ragged N, K
tails inside a 512-code chunk, anchors, bias, residual, the grouped launch with the RMSNorm
and SiLU prologues, CUDA-graph replay and the decode-step shapes of Llama-2-7B, Llama-3.2-3B
and Llama-3-70B."""
import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import oracle

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _padded_scales(scales):
    """Same values, rows 16-byte aligned (a multiple of 8 groups per row)."""
    N, ng = scales.shape
    buf = torch.zeros(N, (ng + 7) // 8 * 8, dtype=scales.dtype, device=scales.device)
    buf[:, :ng] = scales
    return buf[:, :ng]


def _layer(N, K, G, n_out, dev, seed, bias=False):
    g = torch.Generator().manual_seed(seed)
    packed = torch.randint(0, 256, (N, K // 4), generator=g, dtype=torch.int32).to(torch.uint8)
    scales = (torch.rand(N, K // G, generator=g) * 0.03 + 0.002).half()
    idx = torch.randperm(K, generator=g)[:n_out] if n_out else None
    ov = (torch.randn(N, n_out, generator=g) * 0.05).half() if n_out else None
    b = (torch.randn(N, generator=g) * 0.1).half() if bias else None
    mask = None
    if n_out:
        mask = torch.ones(K, dtype=torch.float16)
        mask[idx] = 0
    d = lambda t: None if t is None else t.to(dev)
    return dict(packed=d(packed), scales=_padded_scales(scales.to(dev)), idx=d(idx), ov=d(ov), bias=d(b),
                mask=d(mask), G=G, N=N, K=K)


def _ref(L, x, residual=None):
    p = lambda t: None if t is None else t.cpu().numpy()
    y = oracle.linear_f32(p(x), p(L["packed"]), p(L["scales"]), L["G"], mask=p(L["mask"]), outlier_idx=p(L["idx"]),
                          outlier_vals=p(L["ov"]), bias=p(L["bias"]))
    return y if residual is None else y + residual.float().cpu().numpy()


def _run(L, x, residual=None):
    from otf_llm import _native
    return _native.linear_2bit(x, L["packed"], L["scales"], L["G"], None, mask=L["mask"], outlier_idx=L["idx"],
                               outlier_vals=L["ov"], bias=L["bias"], residual=residual, clamp=True)


@pytest.mark.parametrize("N,K,G,n_out,bias,res", [
    (64, 512, 64, 2, False, False),
    (17, 1024, 64, 5, True, False),        # one partial row tile
    (1000, 4096, 64, 20, False, True),
    (4100, 4096, 64, 20, True, True),      # a last tile of 4 rows
    (333, 2048, 32, 10, False, False),
    (256, 4160, 64, 20, False, False),     # 65 groups: the last chunk is 1/8 full
    (4096, 11008, 64, 55, False, True),    # 7B down_proj (172 groups, padded scale rows)
    (11008, 4096, 64, 20, False, False),   # 7B gate/up
    (1024, 3072, 64, 15, True, False),     # 3B k/v
    (8192, 28672, 64, 143, False, True),   # 70B down_proj
    (28672, 8192, 64, 40, False, False),   # 70B gate/up
    (1536, 11008, 32, 55, False, False),
])
def test_padded_scale_rows(N, K, G, n_out, bias, res, cuda_dev):
    from otf_llm import _native
    L = _layer(N, K, G, n_out, cuda_dev, seed=N + K + G)
    gen = torch.Generator().manual_seed(K)
    x = (torch.randn(1, K, generator=gen) * 1.5).half().to(cuda_dev)
    r = (torch.randn(1, N, generator=gen)).half().to(cuda_dev) if res else None
    ref = _ref(L, x, r)
    y = _run(L, x, r)
    y2 = _run(L, x, r)
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    err = rel_err(y.cpu().numpy(), ref)
    print(f"{N}x{K} G{G}: rel err {err:.2e}")
    assert err < TOL
    assert torch.equal(y, y2)  # deterministic (fixed summation order)


def test_graph_replay(cuda_dev):
    """A captured launch replays exactly what the eager launch computed."""
    L = _layer(4096, 4096, 64, 20, cuda_dev, seed=9)
    x = torch.randn(1, 4096, device=cuda_dev).half()
    y = torch.empty(1, 4096, dtype=torch.float16, device=cuda_dev)
    from otf_llm import _native
    run = lambda: _native.linear_2bit(x, L["packed"], L["scales"], 64, None, mask=L["mask"], outlier_idx=L["idx"],
                                      outlier_vals=L["ov"], out=y)
    run()
    eager = y.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        run()
    torch.cuda.current_stream().wait_stream(s)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        run()
    y.zero_()
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(y, eager)


def _modules(dev, shapes, K, seed):
    from otf_llm.decoder_stack import StackConfig, random_quantized_linear
    cfg = StackConfig()
    return [random_quantized_linear(N, K, cfg, seed + i, dev) for i, N in enumerate(shapes)]


@pytest.mark.parametrize("xop", ["rmsnorm", "silu"])
def test_group_launch(xop, cuda_dev):
    """The grouped decode launch (q/k/v with the RMSNorm prologue; down with the SiLU gate)
    against the oracle."""
    from otf_llm import _native
    K = 4096
    shapes = (4096, 1024, 1024) if xop == "rmsnorm" else (4096,)
    mods = _modules(cuda_dev, shapes, K, seed=31)
    gen = torch.Generator().manual_seed(5)
    h = (torch.randn(1, K, generator=gen) * 3).half().to(cuda_dev)
    aux = ((torch.rand(K, generator=gen) + 0.5) if xop == "rmsnorm" else torch.randn(K, generator=gen)).half()
    aux = aux.to(cuda_dev)
    op = _native.OTF_XOP_RMSNORM if xop == "rmsnorm" else _native.OTF_XOP_SILU_MUL
    outs = [torch.empty(1, m.out_features, dtype=torch.float16, device=cuda_dev) for m in mods]
    _native.linear_group([_native.GroupItem(m, h, oo, x_op=op, x_aux=aux, eps=1e-5) for m, oo in zip(mods, outs)])
    xin = _native.rmsnorm(h, aux, 1e-5) if xop == "rmsnorm" else _native.silu_mul(h, aux.view(1, -1))
    for i, m in enumerate(mods):
        p = lambda t: t.cpu().numpy()
        ref = oracle.linear_f32(p(xin), p(m.packed_uint8), p(m.scales), 64, mask=p(m.outlier_mask_vector),
                                outlier_idx=p(m.outlier_indices), outlier_vals=p(m.outliers_fp16))
        assert rel_err(p(outs[i]), ref) < TOL, i
    assert _native.device_error() == 0
