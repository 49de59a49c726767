"""Tensor-parallel peer all-reduce (otf_ar_*) on the GPU.

* One GPU: a consumer whose producers never arrive gives up after its bounded wait and
  raises the device error flag (the GPU stays usable; nothing is faulted).
* Two and four GPUs (skipped with fewer): the standalone exchange is bit-exact against
  the fp32 rank-order sum, and a tensor-parallel decoder stack with the exchange fused
  into its launches matches the same stack with NCCL all-reduces and the unsharded stack,
  eagerly and as a CUDA graph (with ranks holding odd numbers of scale groups).
* One row-parallel layer (the o_proj / down_proj of Llama-2-7B, cut at group boundaries,
  anchors re-based per shard) with its fp32 partial rows exchanged by the fused producer
  and summed once: within 1e-3 of the fp32 oracle on the whole layer.
"""
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


def _init(rank, world, port, backend="nccl"):
    import datetime

    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    return dist


def test_wait_without_producer_times_out(cuda_dev):
    """A finish on a buffer nobody produced into: the wait runs out (~1 s), the kernel
    completes, otf_device_error reports it, and the next exchange works."""
    import torch.distributed as dist

    from otf_llm import _native
    from otf_llm.tp_allreduce import PeerAllReduce
    port = _free_port()
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        _native.device_error(clear=True)
        ar = PeerAllReduce(4096, device=cuda_dev)
        out = torch.empty(4096, dtype=torch.float16, device=cuda_dev)
        ar.finish(out, 0)
        torch.cuda.synchronize()
        assert _native.device_error(clear=True) == 1
        x = torch.randn(4096, device=cuda_dev).half()
        y = ar.all_reduce(x)
        torch.cuda.synchronize()
        assert torch.equal(y, x)                 # world 1: the sum is x itself
        assert _native.device_error(clear=True) == 0
        ar.close()
    finally:
        dist.destroy_process_group()


def _worker_exchange(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        from otf_llm import _native
        from otf_llm.tp_allreduce import PeerAllReduce
        dev = torch.device("cuda", rank)
        n = 11008
        ar = PeerAllReduce(n, device=dev)
        xs = [torch.randn(n, generator=torch.Generator().manual_seed(100 + r)).half() for r in range(world)]
        ref = torch.zeros(n, dtype=torch.float32)
        for r in range(world):
            ref += xs[r].float()
        ref = ref.clamp(-65504, 65504).half()
        x = xs[rank].to(dev)
        ok = True
        for _ in range(6):                        # alternating buffers, repeated use
            y = ar.all_reduce(x)
            ok = ok and torch.equal(y.cpu(), ref)
        torch.cuda.synchronize()
        err = _native.device_error(clear=True)
        dist.barrier()
        ar.close()
        q.put((rank, ok, err))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, e, -1))
        raise


def _worker_stack(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        from otf_llm import _native
        from otf_llm.decoder_stack import DecodeGraph, Llama2BitLinearStack, StackConfig
        from otf_llm.tp_allreduce import PeerAllReduce
        dev = torch.device("cuda", rank)
        # 5440 = 85 groups of 64: ranks hold odd group counts (padded scale rows)
        cfg = StackConfig(layers=3, hidden=2048, intermediate=5440, heads=16, kv_heads=16, head_dim=128)
        ar = PeerAllReduce(cfg.hidden, device=dev)
        pg = dist.group.WORLD
        peer = Llama2BitLinearStack(cfg, device=dev, seed=4, rank=rank, world=world, process_group=pg, peer_ar=ar)
        nccl = Llama2BitLinearStack(cfg, device=dev, seed=4, rank=rank, world=world, process_group=pg)
        h = torch.randn(1, cfg.hidden, generator=torch.Generator().manual_seed(9)).half().to(dev)
        y_peer = peer(h).clone()
        y_peer2 = peer(h).clone()                 # second step reuses both buffers
        y_nccl = nccl(h).clone()
        g = DecodeGraph(peer)
        g.x.copy_(h)
        g.replay()
        g.replay()
        y_graph = g.y.clone()
        torch.cuda.synchronize()
        err = _native.device_error(clear=True)
        full = None
        if rank == 0:
            one = Llama2BitLinearStack(cfg, device=dev, seed=4)
            full = one(h).float().cpu().numpy()
        res = (rank, y_peer.float().cpu().numpy(), y_peer2.float().cpu().numpy(), y_nccl.float().cpu().numpy(),
               y_graph.float().cpu().numpy(), full, err)
        del g
        dist.barrier()
        torch.cuda.synchronize()
        ar.close()
        q.put(res)
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, e))
        raise


def _worker_row_layer(rank, world, port, q):
    try:
        dist = _init(rank, world, port)
        from otf_llm import _native
        from otf_llm.decoder_stack import StackConfig, random_quantized_linear, shard_linear, split_bounds
        from otf_llm.tp_allreduce import PeerAllReduce
        dev = torch.device("cuda", rank)
        out = []
        ar = PeerAllReduce(4096, device=dev)
        for N, K in ((4096, 4096), (4096, 11008)):
            full = random_quantized_linear(N, K, StackConfig(), seed=N + K, device=dev)  # same weights on every rank
            shard = shard_linear(full, rank, world, "in")
            k0, k1 = split_bounds(K, rank, world, full.group_size)
            x = (torch.randn(1, K, generator=torch.Generator().manual_seed(K)) * 2).half().to(dev)
            xs = x[:, k0:k1].contiguous()
            buf = ar.next_buffer()
            unused = torch.empty(1, N, dtype=torch.float16, device=dev)
            _native.linear_group([_native.GroupItem(shard, xs, unused, ar=ar, ar_mode=_native.OTF_AR_PRODUCE,
                                                    ar_buf=buf)])
            y = torch.empty(N, dtype=torch.float16, device=dev)
            ar.finish(y, buf)
            torch.cuda.synchronize()
            ref = None
            if rank == 0:
                from oracle import oracle
                p = lambda t: t.cpu().numpy()
                ref = oracle.linear_f32(p(x), p(full.packed_uint8), p(full.scales), full.group_size,
                                        mask=p(full.outlier_mask_vector), outlier_idx=p(full.outlier_indices),
                                        outlier_vals=p(full.outliers_fp16))
            out.append((y.float().cpu().numpy(), ref))
        err = _native.device_error(clear=True)
        dist.barrier()
        ar.close()
        q.put((rank, out, err))
        dist.destroy_process_group()
    except Exception as e:
        q.put((rank, e, -1))
        raise


@pytest.mark.parametrize("world", [2, 4])
def test_row_parallel_layer_at_oracle_bar(world):
    res = _run(_worker_row_layer, world=world)
    for rank, out, err in res:
        assert err == 0
        for (y, _), (y0, ref) in zip(out, res[0][1]):
            assert np.array_equal(y, y0), "ranks disagree on the reduced rows"
    for y, ref in res[0][1]:
        assert rel_err(y, ref[0]) < 1e-3


def _run(target, world=2, timeout=300):
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=target, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=timeout) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
    for o in out:
        assert not any(isinstance(v, Exception) for v in o), o
    return sorted(out, key=lambda o: o[0])


def test_exchange_bit_exact_two_gpus():
    for rank, ok, err in _run(_worker_exchange):
        assert ok, f"rank {rank}: exchange differs from the rank-order fp32 sum"
        assert err == 0


@pytest.mark.parametrize("world", [2, 4])
def test_stack_with_fused_exchange(world):
    res = _run(_worker_stack, world=world)
    y0 = res[0][1]
    for rank, y_peer, y_peer2, y_nccl, y_graph, full, err in res:
        assert err == 0
        assert np.array_equal(y_peer, y0), "ranks disagree on the reduced hidden state"
        assert np.array_equal(y_peer2, y_peer)
        assert np.array_equal(y_graph, y_peer)
        assert rel_err(y_peer, y_nccl) < 3e-3
        assert y_peer.shape == (1, 2048)
    full = res[0][5]
    assert rel_err(y0, full) < 3e-3
