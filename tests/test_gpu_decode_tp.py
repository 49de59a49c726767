"""Tensor-parallel greedy decoding (GreedyDecoder with world > 1) on 2 GPUs (skipped with
fewer): each rank holds its heads' q/k/v, its K slice of o/down, its gate/up rows and its
vocabulary rows of the INT8 head.  Teacher-forced logits (gathered over ranks) against the
unsharded decoder on one GPU, with the exchange by NCCL all-reduce and fused into the GEMV
launches (peer stores), eagerly and as one CUDA graph per token; the greedy ids must be the
argmax of the gathered logits."""
import os
import socket

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _model(dev, seed=0):
    from otf_llm.decode_model import ModelConfig
    from otf_llm.decoder_stack import even_scale_rows
    from otf_llm.symmetric_2bit_engine import (QuantizedEmbedding, QuantizedLinearHead, Symmetric2BitQuantizer,
                                                SymmetricOTF2BitLinear)
    cfg = ModelConfig(layers=2, hidden=512, intermediate=1024, heads=8, kv_heads=4, head_dim=64, vocab=1000,
                      rope_theta=500000.0, max_pos=64)
    g = torch.Generator(device=dev).manual_seed(seed)
    shapes = {"q_proj": (512, 512), "k_proj": (256, 512), "v_proj": (256, 512), "o_proj": (512, 512),
              "gate_proj": (1024, 512), "up_proj": (1024, 512), "down_proj": (512, 1024)}
    qz = Symmetric2BitQuantizer(group_size=64, outlier_ratio=0.01)
    layers, norms = [], []
    for _ in range(cfg.layers):
        mods = {}
        for n, (o, i) in shapes.items():
            W = torch.randn(o, i, generator=g, device=dev) * 0.05
            act = torch.randn(i, generator=g, device=dev).abs()
            packed, scales, ov, oi = qz.quantize_tensor(W, act)
            mods[n] = even_scale_rows(SymmetricOTF2BitLinear(packed, scales, i, 64, ov, oi))
        layers.append(mods)
        norms.append(((1 + 0.1 * torch.randn(512, generator=g, device=dev)).half(),
                      (1 + 0.1 * torch.randn(512, generator=g, device=dev)).half()))
    E = (torch.randn(cfg.vocab, 512, generator=g, device=dev) * 0.5).half()
    emb = QuantizedEmbedding(cfg.vocab, 512)
    emb.quantize_from_fp16(E)
    emb.weight_int8, emb.scales = emb.weight_int8.to(dev), emb.scales.to(dev)
    fnorm = (1 + 0.1 * torch.randn(512, generator=g, device=dev)).half()
    return cfg, layers, norms, emb, fnorm


def _head_rows(emb, r0, r1):
    from otf_llm.symmetric_2bit_engine import QuantizedLinearHead
    with torch.device("meta"):
        h = QuantizedLinearHead(emb.embedding_dim, r1 - r0)
    h.weight_int8, h.scales = emb.weight_int8[r0:r1], emb.scales[r0:r1]
    return h


def _teacher_forced(dec, prompt):
    logits, ids = [], []
    dec.reset()
    for i in range(prompt.numel()):
        dec.ids.copy_(prompt[i:i + 1])
        dec.step()
        logits.append(dec.logits.clone())
        ids.append(dec.ids.clone())
    return torch.cat(logits), torch.cat(ids)


def _worker(rank, world, port, exchange, q):
    try:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        from otf_llm import _native
        from otf_llm.decode_model import GreedyDecoder, shard_layers
        from otf_llm.decoder_stack import split_bounds
        cfg, layers, norms, emb, fnorm = _model(dev)
        ar = None
        if exchange == "peer":
            from otf_llm.tp_allreduce import PeerAllReduce
            ar = PeerAllReduce(cfg.hidden, device=dev)
        r0, r1 = split_bounds(cfg.vocab, rank, world)
        dec = GreedyDecoder(cfg, shard_layers(layers, cfg, rank, world), norms, emb, _head_rows(emb, r0, r1), fnorm,
                            dev, rank=rank, world=world, process_group=dist.group.WORLD, peer_ar=ar, head_row0=r0)
        prompt = torch.from_numpy(np.random.default_rng(3).integers(0, cfg.vocab, 12)).to(dev)
        out = {}
        for mode in ("eager", "graph"):
            if mode == "graph":
                dec.capture()
            lg, ids = _teacher_forced(dec, prompt)
            parts = [torch.empty_like(lg) if r == rank else None for r in range(world)]
            sizes = [split_bounds(cfg.vocab, r, world)[1] - split_bounds(cfg.vocab, r, world)[0] for r in range(world)]
            parts = [torch.empty(lg.shape[0], n, dtype=lg.dtype, device=dev) for n in sizes]
            dist.all_gather(parts, lg.contiguous())
            out[mode] = (torch.cat(parts, dim=1).cpu().numpy(), ids.cpu().numpy())
        torch.cuda.synchronize()
        err = _native.device_error(clear=True)
        full = None
        if rank == 0:
            one = GreedyDecoder(cfg, layers, norms, emb, _head_rows(emb, 0, cfg.vocab), fnorm, dev)
            lg, ids = _teacher_forced(one, prompt)
            full = (lg.cpu().numpy(), ids.cpu().numpy())
        dec.graph = None
        dist.barrier()
        torch.cuda.synchronize()
        if ar is not None:
            ar.close()
        q.put((rank, out, full, err))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, e, None, -1))
        raise


@pytest.mark.parametrize("exchange", ["nccl", "peer"])
def test_tp2_decoder_matches_single_gpu(exchange):
    import torch.multiprocessing as mp
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, exchange, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    for r in res:
        assert not isinstance(r[1], Exception), r
    ref_logits, ref_ids = res[0][2]
    for rank, out, _, err in res:
        assert err == 0
        for mode, (lg, ids) in out.items():
            assert rel_err(lg, ref_logits) < 2e-2, (rank, mode)
            assert np.array_equal(ids, lg.argmax(axis=1)), (rank, mode)   # combined pick = argmax
        assert np.array_equal(out["graph"][0], out["eager"][0]), rank


def _teacher_forced_batch(dec, prompts):
    logits, ids = [], []
    dec.reset()
    for i in range(prompts.shape[1]):
        dec.ids.copy_(prompts[:, i])
        dec.step()
        logits.append(dec.logits.clone())
        ids.append(dec.ids.clone())
    return torch.stack(logits), torch.stack(ids)            # [T, B, V_rank], [T, B]


def _worker_batch(rank, world, port, q):
    try:
        import datetime

        import torch.distributed as dist
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=dev)
        from otf_llm import _native
        from otf_llm.decode_model import BatchedGreedyDecoder, shard_layers
        from otf_llm.decoder_stack import split_bounds
        cfg, layers, norms, emb, fnorm = _model(dev)
        B = 3
        r0, r1 = split_bounds(cfg.vocab, rank, world)
        dec = BatchedGreedyDecoder(cfg, shard_layers(layers, cfg, rank, world), norms, emb, _head_rows(emb, r0, r1),
                                   fnorm, dev, B, rank=rank, world=world, process_group=dist.group.WORLD, head_row0=r0)
        prompts = torch.from_numpy(np.random.default_rng(4).integers(0, cfg.vocab, (B, 10))).to(dev)
        sizes = [split_bounds(cfg.vocab, r, world)[1] - split_bounds(cfg.vocab, r, world)[0] for r in range(world)]
        out = {}
        for mode in ("eager", "graph"):
            if mode == "graph":
                dec.capture()
            lg, ids = _teacher_forced_batch(dec, prompts)
            parts = [torch.empty(lg.shape[0], B, n, dtype=lg.dtype, device=dev) for n in sizes]
            dist.all_gather(parts, lg.contiguous())
            out[mode] = (torch.cat(parts, dim=2).cpu().numpy(), ids.cpu().numpy())
        torch.cuda.synchronize()
        err = _native.device_error(clear=True)
        full = None
        if rank == 0:
            one = BatchedGreedyDecoder(cfg, layers, norms, emb, _head_rows(emb, 0, cfg.vocab), fnorm, dev, B)
            lg, ids = _teacher_forced_batch(one, prompts)
            full = (lg.cpu().numpy(), ids.cpu().numpy())
        dec.graph = None
        dist.barrier()
        torch.cuda.synchronize()
        q.put((rank, out, full, err))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, e, None, -1))
        raise


def test_tp2_batched_decoder_matches_single_gpu():
    """BatchedGreedyDecoder over 2 ranks (NCCL exchange, vocabulary-parallel head): every
    sequence's teacher-forced logits against the one-GPU batched decoder, the picks the argmax
    of the gathered logits, graph = eager bit for bit."""
    import torch.multiprocessing as mp
    world = 2
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker_batch, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted([q.get(timeout=300) for _ in range(world)], key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    for r in res:
        assert not isinstance(r[1], Exception), r
    ref_logits, ref_ids = res[0][2]
    for rank, out, _, err in res:
        assert err == 0
        for mode, (lg, ids) in out.items():
            assert lg.shape == ref_logits.shape
            assert rel_err(lg, ref_logits) < 2e-2, (rank, mode)
            assert np.array_equal(ids, lg.argmax(axis=2)), (rank, mode)
        assert np.array_equal(out["graph"][0], out["eager"][0]), rank
