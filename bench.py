#!/usr/bin/env python
"""Benchmark: 2-bit GEMV HBM bandwidth on the Llama-2-7B decoder linear stack, batch 1.

One step = one decode token through all 32 layers x {q,k,v,o,gate,up,down} 2-bit
projections (G=64, 0.5% fp16 anchors) with fp16 RMSNorm, SiLU gate and residuals,
attention a single-position pass-through.  Weights are random-init W ~ N(0, 0.02^2)
per layer seed, quantised on the device with the layer's own quantizer.  The stack
holds 1.89 GB of weights, far larger than the 126 MB L2, so every step streams HBM.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]

N > 1 runs under torchrun: tensor parallel over N ranks (column shards of
q/k/v/gate/up, row shards of o/down, NCCL all-reduce after o and down); value is the
whole job's algorithmic bytes / max-over-ranks time.  --impl reference times the
reference's own CPU algorithm (the oracle's port of its LUT-dequant + matmul path)
on rank 0's host cores.  Prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "otf-llm-engine_b200")
for _p in (PKG, ROOT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "2-bit GEMV HBM GB/s (% of B200 peak); decode tok/s at 1/2/4/8 GPUs"
WORKLOAD = "Llama-2-7B 2-bit decoder linear stack, batch-1 decode step"


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def profile_traffic(name: str):
    """dram bytes per GEMV launch from a committed ncu summary, if it exists."""
    path = os.path.join(ROOT, "profiles", name)
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch="):
                return float(line.split("=", 1)[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="clk_", suffix=".csv")
            os.close(fd)
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.idx)], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.out.close()

    def summary(self):
        if self.proc is None or not self.path:
            return None
        sms, maxes, reasons = [], [], set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxes.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        os.unlink(self.path)
        if not sms:
            return None
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxes), "reasons": sorted(reasons),
                "samples": len(sms)}


_CPU_SAMPLE: dict = {}


def cpu_reference_sample(cfg, target_s: float, threads: int = 0):
    """Time the reference's CPU algorithm (oracle port) on whole layers of the stack.

    Inputs are synthetic codes/scales/anchors of the stack's shapes (the CPU cost does
    not depend on the values), built once per configuration and reused, so a call after the
    first times warm buffers.  Returns (GB/s, cores, sample description, seconds).
    """
    import numpy as np
    from oracle import oracle
    from otf_llm.decoder_stack import PROJECTIONS, linear_bytes

    if threads:
        oracle.set_num_threads(threads)
    cores = oracle.num_threads()
    shapes = cfg.shapes()
    key = (tuple(sorted(shapes.items())), cfg.group_size, cfg.outlier_ratio)
    if _CPU_SAMPLE.get("key") != key:     # one synthetic layer per configuration, reused by every call
        rng = np.random.default_rng(0)
        layer = []
        for name in PROJECTIONS:
            N, K = shapes[name]
            k = max(1, int(K * cfg.outlier_ratio))
            layer.append(dict(
                x=rng.standard_normal((1, K)).astype(np.float16),
                packed=rng.integers(0, 256, (N, K // 4), dtype=np.uint8),
                scales=(rng.random((N, K // cfg.group_size)) * 0.03 + 0.002).astype(np.float16),
                idx=rng.choice(K, k, replace=False).astype(np.int64),
                ov=(rng.standard_normal((N, k)) * 0.05).astype(np.float16),
                mask=np.ones(K, dtype=np.float16), N=N, K=K, k=k))
        for d in layer:
            d["mask"][d["idx"]] = 0
        _CPU_SAMPLE.update(key=key, layer=layer, wbuf=np.empty(max(d["N"] * d["K"] for d in layer), dtype=np.float16))
    layer, wbuf = _CPU_SAMPLE["layer"], _CPU_SAMPLE["wbuf"]
    nbytes, reps = 0, 0
    t0 = time.perf_counter()
    while True:
        for d in layer:
            oracle.lut_linear(d["x"], d["packed"], d["scales"], cfg.group_size, mask=d["mask"], outlier_idx=d["idx"],
                              outlier_vals=d["ov"], wbuf=wbuf)
            nbytes += linear_bytes(d["N"], d["K"], cfg.group_size, d["k"])
        reps += 1
        el = time.perf_counter() - t0
        if el >= target_s:
            break
    return nbytes / el / 1e9, cores, f"{reps} layer(s) x 7 projections of the stack, CPU LUT-dequant + matmul", el


def cpu_decode_sample(dec, layers, cfg, w8, sc, start: int, tokens, target_s: float):
    """Time the reference engine's decode step restated on the host cores (oracle.decode:
    LUT dequant + matmul per projection, fp32 attention, INT8 head) on the model the GPU just
    decoded.  The CPU continues from position ``start`` on a copy of the GPU run's KV cache of
    the prompt, fed the GPU's first generated token, and decodes greedily until ``target_s``
    has passed (at most 64 tokens).  Returns the cpu_baseline object."""
    import numpy as np
    from oracle import decode, oracle
    oracle.set_num_threads(os.cpu_count() or 1)
    cores = oracle.num_threads()
    ones = np.ones(cfg.hidden, np.float16)
    cl = [{n: decode.projection_of(m) for n, m in l.items()} for l in layers]
    w8h, sch = w8.cpu().numpy(), sc.cpu().numpy()
    cpu = decode.Decoder(cl, [(ones, ones)] * cfg.layers, ones, w8h, sch, w8h, sch, heads=cfg.heads,
                         kv_heads=cfg.kv_heads, head_dim=cfg.head_dim, rope_theta=cfg.rope_theta,
                         rms_eps=cfg.rms_eps, max_pos=start + 65)
    for li in range(cfg.layers):
        cpu.set_cache(li, dec.kc[li][:start].cpu().numpy(), dec.vc[li][:start].cpu().numpy())
    tok, picks = int(tokens[0]), []
    t0 = time.perf_counter()
    while True:
        tok = int(oracle.argmax_rows(cpu.step(tok, start + len(picks))[None])[0])
        picks.append(tok)
        el = time.perf_counter() - t0
        if el >= target_s or len(picks) >= 64:
            break
    same = sum(1 for i, t in enumerate(picks) if i + 1 < len(tokens) and int(tokens[i + 1]) == t)
    n = len(picks)
    return {"value": round(n / el, 3), "unit": "tokens/s", "cores": cores, "kind": "port",
            "sample": f"{n} greedy decode steps of the same model at positions {start}..{start + n - 1} on a copy of "
                      f"the GPU run's {start}-position KV cache, the reference engine's step restated on the host "
                      f"(LUT dequant + matmul per projection, fp32 attention, INT8 head); {el:.1f} s",
            "picks_equal_to_gpu": f"{same} of {n}"}


def run_reference(args, cfg):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from oracle import oracle
    # Every host core (torchrun sets OMP_NUM_THREADS=1 for its workers; rank 0 runs alone here).
    oracle.set_num_threads(os.cpu_count() or 1)
    cores = oracle.num_threads()
    vals = []
    for i in range(args.warmup + args.steps):
        gbs, cores, sample, _ = cpu_reference_sample(cfg, target_s=0.0)
        if i >= args.warmup:
            vals.append(gbs)
    v = statistics.median(vals)
    sample = "per step: 1 layer (7 projections) of the Llama-2-7B stack through the reference's CPU path"
    line = {"impl": "reference", "metric": METRIC, "value": round(v, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "fp16 activations x 2-bit codes, fp32 accumulate", "data": "synthetic",
            "config": {"workload": WORKLOAD, "layers": cfg.layers, "hidden": cfg.hidden,
                       "intermediate": cfg.intermediate, "group_size": cfg.group_size,
                       "outlier_ratio": cfg.outlier_ratio, "batch": 1},
            "cpu_baseline": {"value": round(v, 3), "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": round(v, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


class StepLaunches:
    """The decode step's own 2-bit GEMV launches (4 grouped launches per layer: RMSNorm +
    q/k/v, o + residual, RMSNorm + gate/up, SiLU + down + residual) captured as one CUDA graph
    without the step's output copy: the dominant kernel's per-launch duration is this
    graph's time divided by its launch count."""

    def __init__(self, stack):
        import torch
        dev = stack.norm_w.device
        self.x = torch.randn(1, stack.cfg.hidden, generator=torch.Generator(device=dev).manual_seed(17),
                             device=dev).half()
        s = torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(s):
            stack(self.x)
        torch.cuda.current_stream(dev).wait_stream(s)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            stack(self.x)
        torch.cuda.synchronize(dev)

    def replay(self) -> None:
        self.graph.replay()


def run_b200(args, cfg):
    import torch
    import torch.distributed as dist
    from otf_llm.decoder_stack import DecodeGraph, Llama2BitLinearStack

    world = args.gpus
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pg = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
        pg = dist.group.WORLD

    peer_ar = None
    if world > 1 and args.tp_exchange == "peer":
        from otf_llm.tp_allreduce import PeerAllReduce
        peer_ar = PeerAllReduce(cfg.hidden, group=pg, device=dev)
    stack = Llama2BitLinearStack(cfg, device=dev, seed=1, rank=rank, world=world, process_group=pg,
                                 peer_ar=peer_ar, persistent=args.decode == "persistent")
    graph = DecodeGraph(stack)
    # The dominant kernel timed on its own: the step's grouped GEMV launches, back to back in a
    # graph without the output copy (the roofline's per-launch duration).
    lin_graph = StepLaunches(stack) if stack.mk is None else None
    torch.cuda.synchronize()

    bytes_tok_rank = stack.bytes_per_token()
    lin_bytes = stack.linear_bytes_list()
    launches = stack.launches_per_token()

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    x0 = torch.randn(1, cfg.hidden, generator=torch.Generator().manual_seed(5)).half()
    graph.x.copy_(x0)
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()

    def timed(fn, steps):
        barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    with ClockSampler(local) as clk:
        ms = timed(graph.replay, args.steps)
    clocks = clk.summary()

    # The same token through the public API with host buffers: H2D input, replay, D2H output.
    xh = torch.empty(1, cfg.hidden, dtype=torch.float16).pin_memory()
    yh = torch.empty_like(xh).pin_memory()
    xh.copy_(x0)
    for _ in range(2):
        graph.step_host(xh, yh)
    ms_e2e = timed(lambda: graph.step_host(xh, yh), args.steps)

    # Dominant kernel: the step's grouped 2-bit GEMV launches on their own.
    roofline = None
    if lin_graph is not None:
        for _ in range(2):
            lin_graph.replay()
        ms_lin = timed(lin_graph.replay, args.steps)
        avg_s = ms_lin / 1e3 / (args.steps * launches)
        avg_bytes = bytes_tok_rank / launches
        peak, kind = measured_peak()
        achieved = avg_bytes / avg_s / 1e9
        tr = profile_traffic("gemv2b_group_7b_step_traffic.txt")
        roofline = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "traffic": tr, "peak_kind": kind,
                    "kernel": "k_gemv2b_group (grouped 2-bit GEMV: RMSNorm + q/k/v, o + residual, "
                              "RMSNorm + gate/up, SiLU + down + residual)",
                    "launches_per_step": launches, "avg_launch_us": round(avg_s * 1e6, 3),
                    "algorithmic_bytes_per_launch": round(avg_bytes)}

    total_bytes = bytes_tok_rank * world  # x/y of column shards counted per rank
    if world > 1:
        t = torch.tensor([float(bytes_tok_rank)], device=dev, dtype=torch.float64)
        dist.all_reduce(t)
        total_bytes = float(t.item())
    sec = ms / 1e3
    value = total_bytes * args.steps / sec / 1e9
    tok_s = args.steps / sec
    e2e = total_bytes * args.steps / (ms_e2e / 1e3) / 1e9

    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            gbs, cores, sample, el = cpu_reference_sample(cfg, target_s=args.cpu_seconds)
            cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                   "sample": f"{sample}; {el:.1f} s"}
        peak, kind = measured_peak()
        line = {"metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "fp16 activations x 2-bit codes (int MMA), "
                "fp32 accumulate", "data": "synthetic (random-init W ~ N(0,0.02^2), quantised on device)",
                "config": {"workload": WORKLOAD, "layers": cfg.layers, "hidden": cfg.hidden,
                           "intermediate": cfg.intermediate, "group_size": cfg.group_size,
                           "outlier_ratio": cfg.outlier_ratio, "batch": 1,
                           "parallelism": f"tp{world}" if world > 1 else "single",
                           "tp_exchange": (args.tp_exchange if world > 1 else None),
                           "decode": "persistent" if stack.mk is not None else "grouped launches",
                           "l2": "weights 1.89 GB >> 126 MB L2 (no flush needed)"},
                "tokens_per_s": round(tok_s, 1), "frac_of_peak": round(value / world / peak, 4),
                "peak_gbs": peak, "peak_kind": kind,
                "e2e": {"value": round(e2e, 1), "unit": "GB/s", "tokens_per_s": round(args.steps / (ms_e2e / 1e3), 1),
                        "h2d_bytes_per_step": xh.numel() * 2, "d2h_bytes_per_step": yh.numel() * 2},
                "gpu_launches": launches * args.steps, "roofline": roofline, "cpu_baseline": cpu, "clocks": clocks}
    del graph, lin_graph
    if world > 1:
        dist.barrier(device_ids=[local])
        if peer_ar is not None:
            torch.cuda.synchronize()
            peer_ar.close()
            dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if line is not None:
        print(json.dumps(line), flush=True)


def run_case(args):
    """Time (or let a profiler capture) one kernel on one shape: --case gemv:N:K or head:V:D."""
    import torch
    from otf_llm import _native
    from otf_llm.decoder_stack import StackConfig, linear_bytes, random_quantized_linear
    parts = args.case.split(":")
    kind, a, b = parts[0], int(parts[1]), int(parts[2])
    M = int(parts[3]) if len(parts) > 3 else 1
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    if kind in ("gemv", "gemm"):
        cfg = StackConfig()
        lay = random_quantized_linear(a, b, cfg, seed=3, device=dev)
        x = torch.randn(M, b, device=dev).half()
        y = torch.empty(M, a, dtype=torch.float16, device=dev)
        n_out = lay.outlier_indices.numel()
        fn = lambda: _native.linear_2bit(x, lay.packed_uint8, lay.scales, 64, lay.codebook,
                                         mask=lay.outlier_mask_vector, outlier_idx=lay.outlier_indices,
                                         outlier_vals=lay.outliers_fp16, out=y)
        nbytes = linear_bytes(a, b, 64, n_out, batch=M)
    else:
        w = torch.randint(-127, 128, (a, b), dtype=torch.int8, device=dev)
        s = (torch.rand(a, 1, device=dev) * 1e-3).half()
        x = torch.randn(1, b, device=dev).half()
        out = torch.empty(1, a, device=dev)
        fn = lambda: _native.i8_head(x, w, s, out)
        nbytes = a * b + a * 2 + b * 2 + a * 4
    for _ in range(args.warmup):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        fn()
    e1.record()
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    print(json.dumps({"case": args.case, "us_per_launch": round(us, 3), "bytes": nbytes,
                      "GBps_l2_warm": round(nbytes / us / 1e3, 1)}), flush=True)


def run_sweep(args):
    """Batch sweep of the skinny 2-bit GEMM at Llama-3-70B MLP shapes (K=8192 -> N=28672 and
    K=28672 -> N=8192, B in 1..64): one JSON line per (shape, B).  Codes/scales/anchors are
    uniform random (the kernels' time does not depend on the values); four weight copies
    rotate (235 MB > L2); CUDA graphs of the rotating launches, CUDA events."""
    import torch
    from otf_llm import _native
    from otf_llm.decoder_stack import linear_bytes
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(0)

    def layer(N, K, G=64):
        k = max(1, int(K * 0.005))
        packed = torch.randint(0, 256, (N, K // 4), dtype=torch.uint8, device=dev, generator=gen)
        scales = (torch.rand(N, K // G, device=dev, generator=gen) * 0.03 + 0.002).half()
        idx = torch.randperm(K, device=dev, generator=gen)[:k]
        ov = (torch.randn(N, k, device=dev, generator=gen) * 0.05).half()
        mask = torch.ones(K, dtype=torch.float16, device=dev)
        mask[idx] = 0
        return packed, scales, idx, ov, mask

    for (N, K) in [(28672, 8192), (8192, 28672)]:
        R = 4
        Ls = [layer(N, K) for _ in range(R)]
        for M in [1, 2, 4, 8, 9, 16, 32, 64, 128]:
            x = torch.randn(M, K, device=dev, generator=gen).half()
            y = torch.empty(M, N, dtype=torch.float16, device=dev)

            def run(i):
                p, sc, idx, ov, m = Ls[i % R]
                _native.linear_2bit(x, p, sc, 64, None, mask=m, outlier_idx=idx, outlier_vals=ov, out=y)

            for i in range(R):
                run(i)
            torch.cuda.synchronize()
            g = torch.cuda.CUDAGraph()
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(st):
                for i in range(R):
                    run(i)
            torch.cuda.current_stream().wait_stream(st)
            with torch.cuda.graph(g):
                for i in range(R):
                    run(i)
            for _ in range(max(3, args.warmup)):
                g.replay()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            reps = max(1, args.steps // R)
            e0.record()
            for _ in range(reps):
                g.replay()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / (reps * R)
            nb = linear_bytes(N, K, 64, max(1, int(K * 0.005)), batch=M)
            kernel = ("k_gemm2b_tmem (tcgen05, dequantised weights in tensor memory)" if M >= 9 else
                      "k_gemv2b" if M == 1 else "k_gemv2b_batch")
            print(json.dumps({"sweep": "70B MLP 2-bit GEMM", "N": N, "K": K, "B": M, "us": round(us, 2),
                              "GBps": round(nb / us / 1e3, 1), "TFLOPs": round(2 * M * N * K / us / 1e6, 1),
                              "kernel": kernel, "data": "synthetic codes/scales, 4 rotating copies",
                              "device_error": _native.device_error(True)}), flush=True)
            del g
        del Ls
        torch.cuda.empty_cache()


def run_e2e(args):
    """Greedy batch-1 decode of a random-init 2-bit model, every token step one CUDA graph of
    native kernels (otf_llm.decode_model): Llama-3.2-3B architecture (28 layers, hidden 3072,
    intermediate 8192, 24 q / 8 KV heads of 128) or Llama-3-70B (80 layers, hidden 8192,
    intermediate 28672, 64 q / 8 KV heads), RoPE theta 5e5, vocabulary 128256 with a tied INT8
    embedding / head.  P prompt tokens, then T generated tokens.  Under torchrun the model is
    tensor-parallel over the ranks (heads, MLP rows and vocabulary split; o/down exchanged by
    the fused peer stores or NCCL) and times are the max over ranks."""
    import torch
    import torch.distributed as dist
    from otf_llm import _native
    from otf_llm.decode_model import LLAMA3_70B, LLAMA32_3B, GreedyDecoder, ModelConfig, shard_layers
    from otf_llm.decoder_stack import StackConfig, random_quantized_linear, split_bounds
    from otf_llm.symmetric_2bit_engine import QuantizedEmbedding, QuantizedLinearHead
    P, T = args.e2e_prompt, args.e2e_tokens
    base = LLAMA3_70B if args.e2e_model == "llama3-70b" else LLAMA32_3B
    name = "Llama-3-70B" if base is LLAMA3_70B else "Llama-3.2-3B"
    cfg = ModelConfig(layers=args.e2e_layers or base.layers, hidden=base.hidden, intermediate=base.intermediate,
                      heads=base.heads, kv_heads=base.kv_heads, head_dim=base.head_dim, vocab=base.vocab,
                      rope_theta=base.rope_theta, max_pos=P + T + 8)
    world = args.gpus
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    pg = None
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
        pg = dist.group.WORLD
    peer_ar = None
    Bt = args.e2e_batch
    # the fused peer exchange lives in the batch-1 grouped launches; batched steps use NCCL
    exchange = (args.tp_exchange if Bt == 1 else "nccl") if world > 1 else None
    if exchange == "peer":
        from otf_llm.tp_allreduce import PeerAllReduce
        peer_ar = PeerAllReduce(cfg.hidden, group=pg, device=dev)
    std = 0.015 if base is LLAMA3_70B else 0.02
    qcfg = StackConfig(group_size=64, outlier_ratio=0.005, weight_std=std)
    shapes = {"q_proj": (cfg.heads * cfg.head_dim, cfg.hidden), "k_proj": (cfg.kv_heads * cfg.head_dim, cfg.hidden),
              "v_proj": (cfg.kv_heads * cfg.head_dim, cfg.hidden), "o_proj": (cfg.hidden, cfg.heads * cfg.head_dim),
              "gate_proj": (cfg.intermediate, cfg.hidden), "up_proj": (cfg.intermediate, cfg.hidden),
              "down_proj": (cfg.hidden, cfg.intermediate)}
    layers = []
    for li in range(cfg.layers):
        full = {n: random_quantized_linear(N, K, qcfg, 7000 + li * 7 + pi, dev)
                for pi, (n, (N, K)) in enumerate(shapes.items())}
        layers.append(shard_layers([full], cfg, rank, world)[0] if world > 1 else full)
        del full
    torch.cuda.synchronize()
    ones = torch.ones(cfg.hidden, dtype=torch.float16, device=dev)
    # tied INT8 embedding / head from W_emb ~ N(0, 0.02^2): row absmax / 127 on the device
    gen = torch.Generator(device=dev).manual_seed(11)
    w8 = torch.empty(cfg.vocab, cfg.hidden, dtype=torch.int8, device=dev)
    sc = torch.empty(cfg.vocab, 1, dtype=torch.float16, device=dev)
    for lo in range(0, cfg.vocab, 16384):
        hi = min(lo + 16384, cfg.vocab)
        w = (torch.randn(hi - lo, cfg.hidden, generator=gen, device=dev) * 0.02).half().float()
        step = w.abs().amax(dim=1, keepdim=True).div(127.0).clamp_min(1e-8)
        w8[lo:hi] = w.div(step).round().clamp(-127, 127).to(torch.int8)
        sc[lo:hi] = step.half()
    r0, r1 = split_bounds(cfg.vocab, rank, world) if world > 1 else (0, cfg.vocab)
    with torch.device("meta"):
        emb = QuantizedEmbedding(cfg.vocab, cfg.hidden)
        head = QuantizedLinearHead(cfg.hidden, r1 - r0)
    emb.weight_int8, emb.scales = w8, sc
    head.weight_int8, head.scales = w8[r0:r1], sc[r0:r1]
    if Bt > 1:
        from otf_llm.decode_model import BatchedGreedyDecoder
        dec = BatchedGreedyDecoder(cfg, layers, [(ones, ones)] * cfg.layers, emb, head, ones, dev, Bt, rank=rank,
                                   world=world, process_group=pg, head_row0=r0)
    else:
        dec = GreedyDecoder(cfg, layers, [(ones, ones)] * cfg.layers, emb, head, ones, dev, rank=rank, world=world,
                            process_group=pg, peer_ar=peer_ar, head_row0=r0)
    dec.capture()
    if world == 1 and Bt == 1:
        dec.capture_prefill(P)              # the timed prompt's prefill replays as one CUDA graph
    prompt = torch.randint(0, cfg.vocab, (Bt, P), generator=torch.Generator().manual_seed(5)).to(dev)
    for _ in range(max(1, args.warmup // 2)):
        dec.generate(prompt[:, :16] if Bt > 1 else prompt[0, :16], 8)
    torch.cuda.synchronize()
    dec.reset()
    if world > 1:
        dist.barrier(device_ids=[local])
    e0, e1, e2 = (torch.cuda.Event(enable_timing=True) for _ in range(3))
    with ClockSampler(local) as clk:
        e0.record()
        if world == 1:
            dec.prefill(prompt[0] if Bt == 1 else prompt)   # the prompt as one pass of Bt x P rows
        else:
            for i in range(P):
                dec.ids.copy_(prompt[:, i])
                dec.graph.replay()
        e1.record()
        out = torch.empty(T, Bt, dtype=torch.int64, device=dev)
        for i in range(T):
            out[i].copy_(dec.ids)
            dec.graph.replay()
        e2.record()
        torch.cuda.synchronize()
    t_pre = e0.elapsed_time(e1) / 1e3
    t_dec = e1.elapsed_time(e2) / 1e3
    lin_bytes = sum(m.packed_uint8.numel() + m.scales.shape[0] * m.scales.shape[1] * 2 +
                    (m.outliers_fp16.numel() * 2 + m.outlier_indices.numel() * 8 if m.has_outliers else 0)
                    for l in layers for m in l.values())
    head_bytes = (r1 - r0) * cfg.hidden + (r1 - r0) * 2
    if world > 1:
        t = torch.tensor([t_pre, t_dec], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        t_pre, t_dec = float(t[0]), float(t[1])
    peak, peak_kind = measured_peak()
    rank_gbs = (lin_bytes + head_bytes) * T / t_dec / 1e9
    line = {"metric": f"decode tokens/s, {name} architecture 2-bit (random init), batch {Bt}",
            "value": round(Bt * T / t_dec, 1), "unit": "tokens/s", "n_gpus": world, "higher_is_better": True,
            "batch": Bt, "prompt_tokens": P, "new_tokens": T, "ms_per_step": round(t_dec / T * 1e3, 4),
            "prefill_tokens_per_s": round(Bt * P / t_pre, 1),
            "prefill": ("one pass of batch x P rows (tensor-memory GEMM, causal prefill attention" +
                        ("; one CUDA graph)" if Bt == 1 else ")") if world == 1
                        else "token by token (graph replays)"),
            "hbm_gbs_per_gpu": round(rank_gbs, 1), "frac_of_peak_per_gpu": round(rank_gbs / peak, 4),
            "peak_gbs": peak, "peak_kind": peak_kind,
            "bytes_per_token_per_gpu": {"linears": lin_bytes, "int8_head": head_bytes,
                                        "kv_cache_at_end": Bt * 2 * cfg.layers * (P + T) * (cfg.kv_heads // world) *
                                        cfg.head_dim * 2},
            "data": "synthetic (random-init weights quantised on device; prompt = seeded uniform ids)",
            "config": {"workload": f"{name} 2-bit greedy decode", "layers": cfg.layers, "hidden": cfg.hidden,
                       "intermediate": cfg.intermediate, "heads": cfg.heads, "kv_heads": cfg.kv_heads,
                       "vocab": cfg.vocab, "rope": "default, theta 5e5", "group_size": 64, "outlier_ratio": 0.005,
                       "parallelism": f"tp{world}" if world > 1 else "single",
                       "tp_exchange": exchange},
            "gpu_launches_per_step": (11 * cfg.layers + 4) if Bt > 1 else (5 * cfg.layers + 5 + (1 if peer_ar is not None else 0)),
            "clocks": clk.summary(), "device_error": _native.device_error(),
            "first_tokens": [int(t) for t in out[:8, 0].cpu()]}
    if rank == 0 and world == 1 and Bt == 1 and base is LLAMA32_3B and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_sample(dec, layers, cfg, w8, sc, P, out[:, 0].cpu().tolist(),
                                                 args.cpu_seconds)
    dec.graph = None
    if world > 1:
        torch.cuda.synchronize()
        dist.barrier(device_ids=[local])
        if peer_ar is not None:
            peer_ar.close()
            dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps(line), flush=True)


def run_quantize(args):
    """GPU quantizer (otf2b_quantize: column impact, anchor ranking, anchor gather, five-round
    group fit) on one Llama-3-70B gate_proj: W 28672 x 8192 fp16 ~ N(0, 0.015^2), G = 64, 0.5%
    anchors, activation profile |N(0,1)|.  W (470 MB) exceeds L2, so each step reads HBM.  The
    CPU baseline is the oracle's restatement of the reference quantizer on a row sample."""
    import torch
    from otf_llm import _native
    N, K, G, ratio = 28672, 8192, 64, 0.005
    k = max(1, int(K * ratio))
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    gen = torch.Generator(device=dev).manual_seed(3)
    W = (torch.randn(N, K, generator=gen, device=dev) * 0.015).half()
    act = torch.randn(K, generator=gen, device=dev).abs()
    for _ in range(max(3, args.warmup)):
        _native.quantize_2b(W, G, k, act)
    torch.cuda.synchronize()
    steps = max(1, args.steps)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(0) as clk:
        e0.record()
        for _ in range(steps):
            _native.quantize_2b(W, G, k, act)
        e1.record()
        torch.cuda.synchronize()
    t = e0.elapsed_time(e1) / 1e3 / steps
    alg = N * K * 2 + N * K // 4 + N * (K // G) * 2 + N * k * 2
    peak, peak_kind = measured_peak()
    cpu = None
    if not args.no_cpu_baseline:
        from oracle import oracle
        rows = 4096
        Wc = W[:rows].float().cpu().numpy()
        ac = act.cpu().numpy()
        t0 = time.perf_counter()
        oracle.quantize_2b(Wc, G, ratio, ac)
        dt = time.perf_counter() - t0
        cpu = {"value": round(rows * K / dt / 1e9, 4), "unit": "Gweights/s", "cores": oracle.num_threads(),
               "kind": "port", "sample": f"{rows} rows x {K} of the same matrix (oracle quantize_2b, OpenMP)"}
    line = {"metric": "2-bit quantizer throughput (Llama-3-70B gate_proj)", "value": round(N * K / t / 1e9, 3),
            "unit": "Gweights/s", "n_gpus": 1, "steps": steps, "warmup": max(3, args.warmup),
            "ms_per_step": round(t * 1e3, 4), "higher_is_better": True, "dtype": "f32",
            "data": "synthetic (seeded N(0, 0.015^2) fp16 weights)",
            "config": {"workload": "quantize 28672 x 8192 fp16, G=64, 0.5% anchors", "l2": "inputs > L2"},
            "roofline": {"bound": "hbm", "achieved": round(alg / t / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(alg / t / 1e9 / peak, 4), "traffic": None, "peak_kind": peak_kind,
                         "note": "group fit bound by its IEEE fp32 divides (5 per weight), not by HBM"},
            "cpu_baseline": cpu, "clocks": clk.summary(), "device_error": _native.device_error()}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", default=None,
                    help="single-kernel timing/profiling case: gemv:N:K, gemm:N:K:M (batched) or head:V:D")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--cpu-seconds", type=float, default=12.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--decode", choices=("grouped", "persistent"), default="grouped",
                    help="decode step as 4 grouped launches per layer, or one persistent launch per token")
    ap.add_argument("--tp-exchange", choices=("peer", "nccl"), default="peer",
                    help="tensor-parallel exchange after o/down: fused NVLink peer stores, or NCCL all_reduce")
    ap.add_argument("--sweep", action="store_true", help="batch sweep at Llama-3-70B MLP shapes (JSON lines)")
    ap.add_argument("--e2e", action="store_true", help="greedy decode of a Llama-3.2-3B-architecture 2-bit model")
    ap.add_argument("--e2e-model", choices=("llama3.2-3b", "llama3-70b"), default="llama3.2-3b")
    ap.add_argument("--e2e-prompt", type=int, default=512)
    ap.add_argument("--e2e-batch", type=int, default=1, help="sequences decoded in lockstep (tensor-parallel batches exchange by NCCL)")
    ap.add_argument("--e2e-layers", type=int, default=0,
                    help="decoder layers of the e2e model (default: the architecture's; fewer for a profiling case)")
    ap.add_argument("--e2e-tokens", type=int, default=256)
    ap.add_argument("--quantize", action="store_true", help="GPU quantizer on a Llama-3-70B gate_proj matrix")
    args = ap.parse_args()
    from otf_llm.decoder_stack import StackConfig
    cfg = StackConfig(layers=args.layers)
    if args.case:
        run_case(args)
    elif args.sweep:
        run_sweep(args)
    elif args.e2e:
        run_e2e(args)
    elif args.quantize:
        run_quantize(args)
    elif args.impl == "reference":
        run_reference(args, cfg)
    else:
        run_b200(args, cfg)


if __name__ == "__main__":
    main()
