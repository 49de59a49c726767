"""Generate the golden fixtures in this directory from the reference implementation.

Run where the reference's source tree is available (it is imported read-only from the
directory given by --reference, or by the OTF_REFERENCE_DIR environment variable):

    python tests/golden/make_golden.py --reference /root/reference

Each fixture is an .npz of seeded inputs and the reference's own outputs, produced by
the reference functions named in its ``source`` entry (GT-Labs-AI/otf-llm-engine,
otf_llm v4.1.0, run on CPU).  The tests never import the reference; they only read
these files.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np
import torch


def reference_dir(argv=None) -> str:
    """The reference's source tree: --reference DIR, else $OTF_REFERENCE_DIR."""
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--reference", default=os.environ.get("OTF_REFERENCE_DIR"),
                    help="directory holding the reference's otf_llm package")
    ref = ap.parse_args(argv).reference
    if not ref or not os.path.isdir(os.path.join(ref, "otf_llm")):
        ap.error("give the reference's source tree with --reference or OTF_REFERENCE_DIR")
    return ref


REF = reference_dir()
OUT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REF)

from otf_llm.otf_2bit_quantizer import OTF2BitLinear, OTF2BitQuantizer  # noqa: E402
from otf_llm.otf_triton_2bit_kernel import _get_byte_lut, triton_symmetric_2bit_gemm  # noqa: E402
from otf_llm.symmetric_2bit_engine import (  # noqa: E402
    QuantizedEmbedding,
    QuantizedLinearHead,
    Symmetric2BitQuantizer,
    SymmetricOTF2BitLinear,
)

torch.set_num_threads(max(1, os.cpu_count() or 1))


def profile(K: int, g: torch.Generator) -> torch.Tensor:
    """x_profile = |N(0,1)| with 1% of the channels (at least one) multiplied by 20."""
    p = torch.randn(K, generator=g).abs()
    hot = torch.randperm(K, generator=g)[: max(1, K // 100)]
    p[hot] *= 20.0
    return p


def fp64_linear(x16, packed, scales, G, mask=None, oidx=None, ovals=None, bias=None, zeros=None, cb16=True):
    """Double-precision restatement of the reference dequant (for a tight oracle pin)."""
    N, Kq = packed.shape
    K = Kq * 4
    if cb16:
        lut = _get_byte_lut(torch.device("cpu")).double()          # fp16 centroids, :149-161
        w = lut[packed.long()].view(N, -1, G) * scales.double().unsqueeze(-1)
    else:
        cb = torch.tensor([-1.52, -0.45, 0.45, 1.52], dtype=torch.float32).double()
        q = torch.stack([(packed >> s) & 3 for s in (0, 2, 4, 6)], dim=-1).view(N, K).long()
        w = cb[q].view(N, -1, G) * scales.double().unsqueeze(-1)
    if zeros is not None:
        w = w + zeros.double().unsqueeze(-1)
    w = w.view(N, K)
    xm = (x16 * mask).double() if mask is not None else x16.double()
    y = xm @ w.T
    if bias is not None:
        y = y + bias.double()
    if oidx is not None:
        y = y + x16.double()[:, oidx] @ ovals.double().T
    return y


def sym_case(name, N, K, G, ratio, Ms, seed, with_bias):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(N, K, generator=g) * 0.02
    act = profile(K, g)
    q = Symmetric2BitQuantizer(group_size=G, outlier_ratio=ratio)
    packed, scales, ovals, oidx = q.quantize_tensor(W, activation_profile=act)
    bias = (torch.randn(N, generator=g) * 0.1).half() if with_bias else None
    lay = SymmetricOTF2BitLinear(packed, scales, K, G, ovals, oidx, bias)
    d = dict(source="Symmetric2BitQuantizer.quantize_tensor + SymmetricOTF2BitLinear.forward (CPU LUT path)",
             act=act.numpy(), packed=packed.numpy(), scales=scales.numpy(),
             outliers=ovals.numpy(), outlier_idx=oidx.numpy(), mask=lay.outlier_mask_vector.numpy(),
             G=np.int64(G), ratio=np.float64(ratio))
    if N * K <= 65536:                                               # small cases keep W for quantizer checks
        d["W"] = W.numpy()
    if bias is not None:
        d["bias"] = bias.numpy()
    for M in Ms:
        x = torch.randn(M, K, generator=g).half()
        y = lay(x)                                                   # reference module forward
        d[f"x_m{M}"] = x.numpy()
        d[f"y_ref_m{M}"] = y.numpy()
        d[f"y_f64_m{M}"] = fp64_linear(x, packed, scales, G, lay.outlier_mask_vector, oidx, ovals, bias).numpy()
        yg = triton_symmetric_2bit_gemm(x, packed, scales, None, G, lay.outlier_mask_vector)
        d[f"y_gemm_m{M}"] = yg.numpy()                               # the gemm function alone
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **d)
    print(name, {k: v.shape for k, v in d.items() if hasattr(v, "shape")})


def asym_case(name, N, K, G, n_out, seed):
    g = torch.Generator().manual_seed(seed)
    packed = torch.randint(0, 256, (N, K // 4), generator=g, dtype=torch.int32).to(torch.uint8)
    scales = (torch.rand(N, K // G, generator=g) * 0.04 + 0.005).half()
    zeros = (torch.randn(N, K // G, generator=g) * 0.01).half()
    oidx = torch.randperm(K, generator=g)[:n_out]
    ovals = (torch.randn(N, n_out, generator=g) * 0.05).half()
    bias = (torch.randn(N, generator=g) * 0.1).half()
    qz = OTF2BitQuantizer(group_size=G)
    Wd = qz.unpack_2bit_uint8(packed, scales, zeros, K)            # reference dequant a7 (fp16)
    lay = OTF2BitLinear(packed, scales, zeros, K, G, ovals, oidx, bias)
    d = dict(source="OTF2BitQuantizer.unpack_2bit_uint8 (dequant incl. zeros); OTF2BitLinear.forward recorded "
                    "for reference (its kernel path drops zeros)",
             packed=packed.numpy(), scales=scales.numpy(), zeros=zeros.numpy(), outliers=ovals.numpy(),
             outlier_idx=oidx.numpy(), bias=bias.numpy(), mask=lay.outlier_mask_vector.numpy(),
             W_dequant=Wd.numpy(), G=np.int64(G))
    for M in (1, 3):
        x = torch.randn(M, K, generator=g).half()
        xm = x * lay.outlier_mask_vector
        y_a7 = xm.double() @ Wd.double().T + bias.double() + x.double()[:, oidx] @ ovals.double().T
        d[f"x_m{M}"] = x.numpy()
        d[f"y_a7_m{M}"] = y_a7.numpy()
        d[f"y_module_m{M}"] = lay(x).numpy()
        d[f"y_f64_m{M}"] = fp64_linear(x, packed, scales, G, lay.outlier_mask_vector, oidx, ovals, bias, zeros,
                                       cb16=False).numpy()
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **d)
    print(name, "ok")


def codes_case(name, N, K, seed):
    g = torch.Generator().manual_seed(seed)
    codes = torch.randint(0, 4, (N, K), generator=g, dtype=torch.int32).to(torch.uint8)
    packed = Symmetric2BitQuantizer().pack_2bit_uint8(codes)
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), source="Symmetric2BitQuantizer.pack_2bit_uint8",
                        codes=codes.numpy(), packed=packed.numpy())
    print(name, "ok")


def int8_case(name, V, D, seed):
    g = torch.Generator().manual_seed(seed)
    Wf = (torch.randn(V, D, generator=g) * 0.02).half()
    emb = QuantizedEmbedding(V, D)
    emb.quantize_from_fp16(Wf)
    head = QuantizedLinearHead(D, V)
    head.weight_int8 = emb.weight_int8                               # tied, as the runner does
    head.scales = emb.scales
    ids = torch.randint(0, V, (2, 7), generator=g)
    d = dict(source="QuantizedEmbedding.quantize_from_fp16/forward, QuantizedLinearHead.forward (tied)",
             W_fp16=Wf.numpy(), weight_int8=emb.weight_int8.numpy(), scales=emb.scales.numpy(), ids=ids.numpy(),
             emb_out=emb(ids).numpy())
    for M in (1, 5):
        x = torch.randn(M, D, generator=g).half()
        d[f"x_m{M}"] = x.numpy()
        d[f"logits_m{M}"] = head(x).numpy()
        d[f"logits_f64_m{M}"] = ((x.double() @ emb.weight_int8.double().T) * emb.scales.double().view(1, -1)).numpy()
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), **d)
    print(name, "ok")


def quant_case(name, N, K, G, ratio, seed):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(N, K, generator=g) * 0.02
    act = profile(K, g)
    packed, scales, ovals, oidx = Symmetric2BitQuantizer(G, ratio).quantize_tensor(W, activation_profile=act)
    np.savez_compressed(os.path.join(OUT, f"{name}.npz"), source="Symmetric2BitQuantizer.quantize_tensor",
                        W=W.numpy(), act=act.numpy(), packed=packed.numpy(), scales=scales.numpy(),
                        outliers=ovals.numpy(), outlier_idx=oidx.numpy(), G=np.int64(G), ratio=np.float64(ratio))
    print(name, "ok")


if __name__ == "__main__":
    sym_case("sym_g64_small", N=37, K=192, G=64, ratio=0.005, Ms=(1, 3), seed=1, with_bias=True)
    sym_case("sym_g64_k4096", N=256, K=4096, G=64, ratio=0.005, Ms=(1, 4), seed=2, with_bias=False)
    sym_case("sym_g32_legacy", N=64, K=512, G=32, ratio=0.035, Ms=(1, 2), seed=3, with_bias=True)
    sym_case("sym_g128", N=48, K=1024, G=128, ratio=0.01, Ms=(1,), seed=4, with_bias=False)
    asym_case("asym_g32", N=40, K=256, G=32, n_out=5, seed=5)
    codes_case("codes_pack", N=33, K=128, seed=6)
    int8_case("int8_v1000_d256", V=1000, D=256, seed=7)
    quant_case("quant_g64", N=64, K=256, G=64, ratio=0.02, seed=8)
