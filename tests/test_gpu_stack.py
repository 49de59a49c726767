"""GPU checks of the decode-step fusions: grouped launches, fused RMSNorm / SiLU gate, and
a small decoder linear stack against a CPU restatement built on the oracle."""
import numpy as np
import pytest
import torch

from conftest import rel_err
from oracle import oracle

pytestmark = pytest.mark.gpu


def _layers(dev, shapes, K, seed=0):
    from otf_llm.decoder_stack import StackConfig, random_quantized_linear
    cfg = StackConfig()
    return [random_quantized_linear(N, K, cfg, seed + i, dev) for i, N in enumerate(shapes)]


def test_group_matches_single_launches(cuda_dev):
    from otf_llm import _native
    mods = _layers(cuda_dev, (1024, 256, 4096), 2048)
    x = torch.randn(1, 2048, device=cuda_dev).half()
    outs = [torch.empty(1, m.out_features, dtype=torch.float16, device=cuda_dev) for m in mods]
    _native.linear_group([_native.GroupItem(m, x, o) for m, o in zip(mods, outs)])
    for m, o in zip(mods, outs):
        ref = _native.linear_2bit(x, m.packed_uint8, m.scales, 64, m.codebook, mask=m.outlier_mask_vector,
                                  outlier_idx=m.outlier_indices, outlier_vals=m.outliers_fp16)
        assert torch.equal(o, ref)
    assert _native.device_error() == 0


def test_fused_rmsnorm_and_silu(cuda_dev):
    from otf_llm import _native
    K = 4096
    mods = _layers(cuda_dev, (2048, 1024), K, seed=7)
    h = (torch.randn(1, K, device=cuda_dev) * 3).half()
    w = (torch.rand(K, device=cuda_dev) + 0.5).half()
    outs = [torch.empty(1, m.out_features, dtype=torch.float16, device=cuda_dev) for m in mods]
    _native.linear_group([_native.GroupItem(m, h, o, x_op=_native.OTF_XOP_RMSNORM, x_aux=w, eps=1e-5)
                          for m, o in zip(mods, outs)])
    xn = _native.rmsnorm(h, w, 1e-5)
    for m, o in zip(mods, outs):
        ref = _native.linear_2bit(xn, m.packed_uint8, m.scales, 64, m.codebook, mask=m.outlier_mask_vector,
                                  outlier_idx=m.outlier_indices, outlier_vals=m.outliers_fp16)
        assert rel_err(o.float().cpu().numpy(), ref.float().cpu().numpy()) < 1e-3
    # SiLU gate fused into the staging of the next layer's input
    down = _layers(cuda_dev, (512,), K, seed=11)[0]
    g = torch.randn(1, K, device=cuda_dev).half()
    u = torch.randn(1, K, device=cuda_dev).half()
    out = torch.empty(1, 512, dtype=torch.float16, device=cuda_dev)
    _native.linear_group([_native.GroupItem(down, g, out, x_op=_native.OTF_XOP_SILU_MUL, x_aux=u.view(-1))])
    a = _native.silu_mul(g, u)
    ref = _native.linear_2bit(a, down.packed_uint8, down.scales, 64, down.codebook, mask=down.outlier_mask_vector,
                              outlier_idx=down.outlier_indices, outlier_vals=down.outliers_fp16)
    assert rel_err(out.float().cpu().numpy(), ref.float().cpu().numpy()) < 1e-3


@pytest.mark.parametrize("K", [3072, 4100, 8192, 16384, 20000])
def test_rmsnorm_widths(K, cuda_dev):
    """otf_rmsnorm at widths served by the register-held 16-byte pieces (K = 8k up to 16384)
    and by the strided form (4100, 20000), against HF's Llama RMSNorm in fp32."""
    from otf_llm import _native
    g = torch.Generator(device=cuda_dev).manual_seed(K)
    h = (torch.randn(3, K, generator=g, device=cuda_dev) * 2).half()
    h[1, 5] = 300.0
    w = (torch.rand(K, generator=g, device=cuda_dev) + 0.5).half()
    for weight in (w, None):
        got = _native.rmsnorm(h, weight, 1e-5).float().cpu().numpy()
        xf = h.float()
        ref = (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + 1e-5)).half()
        if weight is not None:
            ref = weight * ref
        assert rel_err(got, ref.float().cpu().numpy()) < 1e-3


def test_silu_mul_piece_and_strided_forms_agree(cuda_dev):
    """otf_silu_mul on 16-byte pieces (element count a multiple of 8) equals the per-element
    form bit for bit (an odd count takes that form), and both are within an fp16 ulp of torch's
    fp32 silu rounded to fp16 times up."""
    from otf_llm import _native
    g0 = torch.Generator(device=cuda_dev).manual_seed(3)
    n = 8 * 4001
    g = (torch.randn(n + 1, generator=g0, device=cuda_dev) * 4).half()
    u = torch.randn(n + 1, generator=g0, device=cuda_dev).half()
    odd = _native.silu_mul(g, u)
    vec = _native.silu_mul(g[:n].clone(), u[:n].clone())
    assert torch.equal(vec, odd[:n])
    ref = (torch.nn.functional.silu(g.float()).half() * u).float()
    assert rel_err(odd.float().cpu().numpy(), ref.cpu().numpy()) < 1e-3


def _cpu_step(stack, h):
    """The decode step restated on the CPU: HF RMSNorm / SiLU in torch, linears by the oracle."""
    def lin(m, x):
        p = lambda t: t.cpu().numpy()
        y = oracle.linear_f32(x.numpy(), p(m.packed_uint8), p(m.scales), m.group_size,
                              mask=p(m.outlier_mask_vector), outlier_idx=p(m.outlier_indices),
                              outlier_vals=p(m.outliers_fp16))
        return torch.from_numpy(y)

    def rms(x):
        v = x.float()
        v = v * torch.rsqrt(v.pow(2).mean(-1, keepdim=True) + stack.cfg.rms_eps)
        return v.half()

    cur = h.cpu()
    for layer in stack.layers:
        xn = rms(cur)
        v = lin(layer["v_proj"], xn).half()
        cur = (lin(layer["o_proj"], v) + cur.float()).half()
        xn = rms(cur)
        g = lin(layer["gate_proj"], xn).half()
        u = lin(layer["up_proj"], xn).half()
        a = (torch.nn.functional.silu(g.float()).half() * u)
        cur = (lin(layer["down_proj"], a) + cur.float()).half()
    return cur


@pytest.mark.parametrize("fused", [True, False])
def test_small_stack_matches_cpu_step(fused, cuda_dev):
    from otf_llm.decoder_stack import Llama2BitLinearStack, StackConfig
    cfg = StackConfig(layers=2, hidden=1024, intermediate=2816, heads=8, kv_heads=8, head_dim=128)
    stack = Llama2BitLinearStack(cfg, device=cuda_dev, seed=3, fused=fused)
    h = torch.randn(1, 1024, generator=torch.Generator().manual_seed(1)).half()
    out = stack(h.to(cuda_dev)).cpu()
    ref = _cpu_step(stack, h)
    assert rel_err(out.float().numpy(), ref.float().numpy()) < 3e-3
