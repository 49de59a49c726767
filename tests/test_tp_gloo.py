"""Tensor-parallel sharding on CPU ranks (gloo, world size 2).

Each rank shards a quantized layer the way the decode stack does (column shards for
q/k/v/gate/up, row shards cut at group boundaries with anchors re-based for o/down),
evaluates its shard with the oracle, and the ranks all-reduce / all-gather.  The result
must equal the unsharded layer: the exchange step and the anchor re-basing are exact
up to fp32 summation order.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import load_golden, rel_err


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _oracle_layer(lay, x):
    from oracle import oracle
    p = lambda t: None if t is None else t.numpy()
    return oracle.linear_f32(x, p(lay.packed_uint8), p(lay.scales), lay.group_size,
                             mask=p(lay.outlier_mask_vector) if lay.has_outliers else None,
                             outlier_idx=p(lay.outlier_indices) if lay.has_outliers else None,
                             outlier_vals=p(lay.outliers_fp16) if lay.has_outliers else None)


def _worker(rank, world, port, name, q):
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from otf_llm.decoder_stack import shard_linear
        from otf_llm.symmetric_2bit_engine import SymmetricOTF2BitLinear
        gd = load_golden(name)
        K = gd["packed"].shape[1] * 4
        full = SymmetricOTF2BitLinear(torch.from_numpy(gd["packed"]), torch.from_numpy(gd["scales"]), K,
                                      int(gd["G"]), torch.from_numpy(gd["outliers"]),
                                      torch.from_numpy(gd["outlier_idx"]))
        x = gd["x_m1"]
        # row-parallel (o/down): shard K, all-reduce partial sums
        rs = shard_linear(full, rank, world, "in")
        k0 = rank * K // world
        part = torch.from_numpy(_oracle_layer(rs, x[:, k0:k0 + rs.d_in]).astype(np.float32))
        dist.all_reduce(part)
        # column-parallel (q/k/v/gate/up): shard N, all-gather
        cs = shard_linear(full, rank, world, "out")
        mine = torch.from_numpy(_oracle_layer(cs, x).astype(np.float32))
        gathered = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(gathered, mine)
        if rank == 0:
            q.put((part.numpy(), torch.cat(gathered, dim=1).numpy(), _oracle_layer(full, x)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # surface the failure to the parent
        q.put(e)
        raise


@pytest.mark.parametrize("name", ["sym_g64_k4096", "sym_g128"])
def test_tp_shards_reproduce_full_layer(name):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, name, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
    assert not isinstance(res, Exception), res
    row_par, col_par, full = res
    assert rel_err(row_par, full) < 1e-5
    assert rel_err(col_par, full) < 1e-6


def test_row_shard_rebases_anchors():
    from otf_llm.decoder_stack import shard_linear
    from otf_llm.symmetric_2bit_engine import SymmetricOTF2BitLinear
    gd = load_golden("sym_g64_k4096")
    full = SymmetricOTF2BitLinear(torch.from_numpy(gd["packed"]), torch.from_numpy(gd["scales"]), 4096, 64,
                                  torch.from_numpy(gd["outliers"]), torch.from_numpy(gd["outlier_idx"]))
    seen = []
    for r in range(4):
        s = shard_linear(full, r, 4, "in")
        if s.has_outliers:
            assert int(s.outlier_indices.min()) >= 0 and int(s.outlier_indices.max()) < 1024
            seen.extend((s.outlier_indices + r * 1024).tolist())
    assert sorted(seen) == sorted(gd["outlier_idx"].tolist())


def _ckpt_worker(rank, world, port, q):
    """Sharded checkpoint load + vocabulary-parallel greedy pick on gloo ranks."""
    try:
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from conftest import GOLDEN
        from otf_llm.checkpoint import load_checkpoint
        from otf_llm.vocab_parallel import combine_argmax
        d = os.path.join(GOLDEN, "ckpt_tied")
        ck = load_checkpoint(d, device="cpu", rank=rank, world=world)
        x = np.random.default_rng(5).standard_normal((3, 128)).astype(np.float16)
        # row-parallel down_proj: this rank's input slice, partial sums all-reduced
        m = ck.layers[1]["mlp.down_proj"]
        part = torch.from_numpy(_oracle_layer(m, x[:, rank * m.d_in:(rank + 1) * m.d_in]).astype(np.float32))
        dist.all_reduce(part)
        # greedy pick over vocabulary shards: equal maxima straddle the shard boundary
        V, M = 64, 6
        logits = torch.from_numpy(np.random.default_rng(9).standard_normal((M, V)).astype(np.float32))
        logits[1, 10] = logits[1, 40] = 9.0        # tie across ranks: the lower index wins
        logits[2, 33] = logits[2, 35] = 9.0        # tie inside rank 1
        logits[3, :] = -1.0                        # all equal: index 0
        logits[4, 63] = 50.0                       # maximum in the last row of the last shard
        logits[5, 31] = logits[5, 32] = 7.0        # tie on the shard boundary
        v0 = ck.head.row0
        loc = logits[:, v0:v0 + V // world]
        lm, li = loc.max(dim=1)
        ids = combine_argmax(lm, li, v0)
        if rank == 0:
            q.put((part.numpy(), ids.numpy(), torch.argmax(logits, dim=1).numpy()))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:
        q.put(e)
        raise


def test_sharded_checkpoint_and_vocab_argmax():
    from conftest import GOLDEN
    from otf_llm.checkpoint import load_checkpoint
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_ckpt_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=180)
    for p in procs:
        p.join(timeout=60)
    assert not isinstance(res, Exception), res
    part, ids, ref_ids = res
    full = load_checkpoint(os.path.join(GOLDEN, "ckpt_tied"), device="cpu").layers[1]["mlp.down_proj"]
    x = np.random.default_rng(5).standard_normal((3, 128)).astype(np.float16)
    assert rel_err(part, _oracle_layer(full, x)) < 1e-5
    assert np.array_equal(ids, ref_ids)


@pytest.mark.parametrize("world", [2, 4, 8])
def test_llama7b_shards_cover_every_group(world):
    """7B shapes at TP 2/4/8: the 172 groups of 64 of down_proj's input split into whole
    groups per rank (21 or 22 at TP 8), gate/up rows at the same points, q/k/v by heads."""
    from otf_llm.decoder_stack import LLAMA2_7B, split_bounds
    cfg = LLAMA2_7B
    inter = [split_bounds(cfg.intermediate, r, world, cfg.group_size) for r in range(world)]
    assert inter[0][0] == 0 and inter[-1][1] == cfg.intermediate
    assert all(a[1] == b[0] for a, b in zip(inter, inter[1:]))
    sizes = {hi - lo for lo, hi in inter}
    assert all(s % cfg.group_size == 0 for s in sizes) and max(sizes) - min(sizes) <= cfg.group_size
    heads = [split_bounds(cfg.heads * cfg.head_dim, r, world, cfg.head_dim) for r in range(world)]
    assert {hi - lo for lo, hi in heads} == {cfg.heads * cfg.head_dim // world}


@pytest.mark.parametrize("world", [2, 4, 8])
def test_decoder_shards_split_whole_heads(world):
    """shard_layers (tensor-parallel GreedyDecoder): q/k/v rows are whole heads, every rank
    gets heads/world query and kv_heads/world KV heads, gate/up rows line up with down_proj's
    K slice at group boundaries, and the shards put back together give the full layer."""
    from otf_llm.decode_model import ModelConfig, shard_layers
    from otf_llm.symmetric_2bit_engine import Symmetric2BitQuantizer, SymmetricOTF2BitLinear
    cfg = ModelConfig(layers=1, hidden=256, intermediate=1024, heads=8, kv_heads=8, head_dim=32, vocab=64)
    g = torch.Generator().manual_seed(0)
    qz = Symmetric2BitQuantizer(group_size=32, outlier_ratio=0.02)
    shapes = {"q_proj": (256, 256), "k_proj": (256, 256), "v_proj": (256, 256), "o_proj": (256, 256),
              "gate_proj": (1024, 256), "up_proj": (1024, 256), "down_proj": (256, 1024)}
    full = {}
    for n, (o, i) in shapes.items():
        p, s, ov, oi = qz.quantize_tensor(torch.randn(o, i, generator=g) * 0.02, torch.randn(i, generator=g).abs())
        full[n] = SymmetricOTF2BitLinear(p, s, i, 32, ov, oi)
    parts = [shard_layers([full], cfg, r, world)[0] for r in range(world)]
    for n in ("q_proj", "k_proj", "v_proj"):
        rows = [p[n].out_features for p in parts]
        assert all(r % cfg.head_dim == 0 for r in rows) and sum(rows) == 256
        assert torch.equal(torch.cat([p[n].packed_uint8 for p in parts]), full[n].packed_uint8)
    assert [p["q_proj"].out_features // 32 for p in parts] == [8 // world] * world
    for p in parts:
        assert p["gate_proj"].out_features == p["down_proj"].d_in == p["up_proj"].out_features
        assert p["o_proj"].d_in == p["q_proj"].out_features
    for n in ("o_proj", "down_proj"):
        assert torch.equal(torch.cat([p[n].packed_uint8 for p in parts], dim=1), full[n].packed_uint8)
        got = sorted(int(i) + sum(q[n].d_in for q in parts[:r]) for r, p in enumerate(parts) if p[n].has_outliers
                     for i in p[n].outlier_indices)
        assert got == sorted(full[n].outlier_indices.tolist())
    with pytest.raises(ValueError):
        shard_layers([full], ModelConfig(layers=1, hidden=256, intermediate=1024, heads=8, kv_heads=3,
                                         head_dim=32, vocab=64), 0, 2)
