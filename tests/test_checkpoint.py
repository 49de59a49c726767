"""Converted-checkpoint reader/writer against checkpoints the reference converter wrote
(tests/golden/ckpt_*/, made by tests/golden/make_checkpoints.py), on the CPU."""
import json
import os
import shutil

import pytest
import torch
from safetensors import safe_open
from safetensors.torch import load_file

from conftest import GOLDEN

FIXTURES = ("ckpt_tied", "ckpt_untied")


def _dir(name):
    return os.path.join(GOLDEN, name)


def _tensors(path):
    with safe_open(path, framework="pt", device="cpu") as f:
        return {k: f.get_tensor(k) for k in f.keys()}


@pytest.mark.parametrize("name", FIXTURES)
def test_loader_reads_reference_layout(name):
    from otf_llm.checkpoint import BASE_FILE, MODEL_FILE, load_checkpoint
    ck = load_checkpoint(_dir(name), device="cpu")
    meta = json.load(open(os.path.join(_dir(name), "source.json")))
    quant = _tensors(os.path.join(_dir(name), MODEL_FILE))
    base = _tensors(os.path.join(_dir(name), BASE_FILE))
    assert ck.num_layers == meta["layers"] and ck.group_size == meta["group_size"]
    for i, mods in enumerate(ck.layers):
        assert len(mods) == 7
        for proj, m in mods.items():
            pfx = f"model.layers.{i}.{proj}"
            assert torch.equal(m.packed_uint8, quant[f"{pfx}.packed_uint8"])
            assert torch.equal(m.scales, quant[f"{pfx}.scales"])
            assert m.d_in == quant[f"{pfx}.packed_uint8"].shape[1] * 4
            assert m.group_size == meta["group_size"]
            assert m.has_outliers
            assert torch.equal(m.outlier_indices, quant[f"{pfx}.outlier_indices"])
            assert torch.equal(m.outliers_fp16, quant[f"{pfx}.outlier_deltas"])
            mask = torch.ones(m.d_in, dtype=torch.float16)
            mask[quant[f"{pfx}.outlier_indices"]] = 0
            assert torch.equal(m.outlier_mask_vector, mask)
            if f"{pfx}.bias" in quant:
                assert m.has_bias and torch.equal(m.bias, quant[f"{pfx}.bias"])
            else:
                assert not m.has_bias
        for ln in ("input_layernorm", "post_attention_layernorm"):
            assert torch.equal(ck.layer_norms[i][ln], base[f"model.layers.{i}.{ln}.weight"])
    assert torch.equal(ck.final_norm, base["model.norm.weight"])
    assert torch.equal(ck.embed.weight_int8, base["model.embed_tokens.weight_int8"])
    assert torch.equal(ck.embed.scales, base["model.embed_tokens.scales"])
    if meta["tied"]:
        # the head reads the embedding's buffers in place (run_symmetric_2bit.py:132-135)
        assert ck.head_tied
        assert ck.head.weight_int8.data_ptr() == ck.embed.weight_int8.data_ptr()
        assert ck.head.scales.data_ptr() == ck.embed.scales.data_ptr()
    else:
        assert not ck.head_tied
        assert torch.equal(ck.head.weight_int8, base["lm_head.weight_int8"])
        assert torch.equal(ck.head.scales, base["lm_head.scales"])
    assert ck.head.out_features == meta["vocab"] and ck.head.in_features == meta["hidden"]


@pytest.mark.parametrize("name", FIXTURES)
def test_converter_matches_reference_converter(name, tmp_path):
    """The package's converter, on the same source weights and profile, writes the same tensors."""
    from otf_llm.checkpoint import BASE_FILE, CONFIG_FILE, MODEL_FILE, convert_symmetric_model
    src = tmp_path / "src"
    src.mkdir()
    shutil.copyfile(os.path.join(_dir(name), "source.safetensors"), src / "model.safetensors")
    prof = load_file(os.path.join(_dir(name), "profile.safetensors"))
    meta = json.load(open(os.path.join(_dir(name), "source.json")))
    out = tmp_path / "out"
    convert_symmetric_model(str(src), str(out), group_size=meta["group_size"], outlier_ratio=meta["outlier_ratio"],
                            act_profiles=prof, device="cpu")
    for fname in (MODEL_FILE, BASE_FILE):
        mine = _tensors(str(out / fname))
        ref = _tensors(os.path.join(_dir(name), fname))
        assert sorted(mine) == sorted(ref), fname
        for k in ref:
            assert mine[k].dtype == ref[k].dtype and mine[k].shape == ref[k].shape, k
            assert torch.equal(mine[k], ref[k]), k
    mine = json.load(open(out / CONFIG_FILE))
    ref = json.load(open(os.path.join(_dir(name), CONFIG_FILE)))
    for key in ("architecture", "group_size", "outlier_ratio", "num_layers", "projections"):
        assert mine[key] == ref[key], key


def test_config_defaults(tmp_path):
    """group_size 32 and the seven Llama projections when the config omits them (runner :75-77)."""
    from otf_llm.checkpoint import BASE_FILE, CONFIG_FILE, DEFAULT_PROJECTIONS, MODEL_FILE, load_checkpoint
    d = tmp_path / "ck"
    d.mkdir()
    for f in (MODEL_FILE, BASE_FILE):
        shutil.copyfile(os.path.join(_dir("ckpt_tied"), f), d / f)
    with open(d / CONFIG_FILE, "w") as fh:
        json.dump({"num_layers": 2}, fh)
    ck = load_checkpoint(str(d), device="cpu")
    assert ck.group_size == 32 and ck.projections == DEFAULT_PROJECTIONS
    # a projection list without the MLP loads only the attention projections
    with open(d / CONFIG_FILE, "w") as fh:
        json.dump({"num_layers": 1, "projections": DEFAULT_PROJECTIONS[:4]}, fh)
    ck = load_checkpoint(str(d), device="cpu")
    assert ck.num_layers == 1 and sorted(ck.layers[0]) == sorted(DEFAULT_PROJECTIONS[:4])


def test_group_size_mismatch_is_an_error(tmp_path):
    from otf_llm.checkpoint import BASE_FILE, CONFIG_FILE, MODEL_FILE, load_checkpoint
    d = tmp_path / "ck"
    d.mkdir()
    for f in (MODEL_FILE, BASE_FILE):
        shutil.copyfile(os.path.join(_dir("ckpt_tied"), f), d / f)
    with open(d / CONFIG_FILE, "w") as fh:
        json.dump({"num_layers": 2, "group_size": 64}, fh)     # scales were written for G=32
    with pytest.raises(ValueError, match="scales"):
        load_checkpoint(str(d), device="cpu")


@pytest.mark.parametrize("world", [2])
def test_tensor_parallel_shards_reassemble(world):
    """Column shards stack back by rows, row shards by columns with anchors re-based; the
    row-parallel bias stays on rank 0; head rows split by vocabulary (tied: views)."""
    from otf_llm.checkpoint import ROW_PARALLEL, load_checkpoint
    full = load_checkpoint(_dir("ckpt_tied"), device="cpu")
    shards = [load_checkpoint(_dir("ckpt_tied"), device="cpu", rank=r, world=world) for r in range(world)]
    for i, mods in enumerate(full.layers):
        for proj, m in mods.items():
            parts = [s.layers[i][proj] for s in shards]
            if proj in ROW_PARALLEL:
                assert torch.equal(torch.cat([p.packed_uint8 for p in parts], 1), m.packed_uint8)
                assert torch.equal(torch.cat([p.scales for p in parts], 1), m.scales)
                cols, vals = [], []
                for r, p in enumerate(parts):
                    assert p.d_in == m.d_in // world
                    if p.has_outliers:
                        assert int(p.outlier_indices.min()) >= 0 and int(p.outlier_indices.max()) < p.d_in
                        cols.append(p.outlier_indices + r * p.d_in)
                        vals.append(p.outliers_fp16)
                    assert p.has_bias == (m.has_bias and r == 0)
                order = torch.cat(cols).argsort()
                ref_order = m.outlier_indices.argsort()
                assert torch.equal(torch.cat(cols)[order], m.outlier_indices[ref_order])
                assert torch.equal(torch.cat(vals, 1)[:, order], m.outliers_fp16[:, ref_order])
            else:
                assert torch.equal(torch.cat([p.packed_uint8 for p in parts], 0), m.packed_uint8)
                assert torch.equal(torch.cat([p.scales for p in parts], 0), m.scales)
                assert torch.equal(torch.cat([p.outliers_fp16 for p in parts], 0), m.outliers_fp16)
                for p in parts:
                    assert torch.equal(p.outlier_indices, m.outlier_indices)
                if m.has_bias:
                    assert torch.equal(torch.cat([p.bias for p in parts]), m.bias)
    V = full.head.out_features
    for r, s in enumerate(shards):
        assert s.head.row0 == r * V // world and s.head.vocab_size == V
        w = s.head.shard.weight_int8
        assert torch.equal(w, full.head.weight_int8[r * V // world:(r + 1) * V // world])
        # a tied shard is a row view of this rank's replicated embedding
        assert w.data_ptr() == s.embed.weight_int8.data_ptr() + r * (V // world) * w.shape[1]


def test_uneven_group_count_splits_balanced():
    """down_proj has 3 groups of 64 per row: ranks take 1 and 2 groups, and gate/up rows are
    cut at the same points, so each rank's intermediate slice is its down_proj input."""
    from otf_llm.checkpoint import load_checkpoint
    full = load_checkpoint(_dir("ckpt_untied"), device="cpu")
    parts = [load_checkpoint(_dir("ckpt_untied"), device="cpu", rank=r, world=2) for r in range(2)]
    for r, p in enumerate(parts):
        down, gate, up = (p.layers[0][k] for k in ("mlp.down_proj", "mlp.gate_proj", "mlp.up_proj"))
        assert down.d_in == gate.out_features == up.out_features == 64 * (r + 1)
    for key in ("mlp.down_proj",):
        assert torch.equal(torch.cat([p.layers[0][key].packed_uint8 for p in parts], 1), full.layers[0][key].packed_uint8)
    for key in ("mlp.gate_proj", "mlp.up_proj"):
        assert torch.equal(torch.cat([p.layers[0][key].packed_uint8 for p in parts], 0), full.layers[0][key].packed_uint8)


def test_too_many_ranks_is_an_error():
    from otf_llm.checkpoint import load_checkpoint
    with pytest.raises(ValueError, match="split"):
        load_checkpoint(_dir("ckpt_tied"), device="cpu", rank=0, world=4)   # o_proj input: 2 groups of 32


def test_build_hf_model_injects_modules():
    """Meta skeleton -> checkpoint modules -> materialised norms and rotary tables (runner :81-187)."""
    transformers = pytest.importorskip("transformers")
    from otf_llm.checkpoint import build_hf_model
    from otf_llm.symmetric_2bit_engine import QuantizedEmbedding, QuantizedLinearHead, SymmetricOTF2BitLinear
    cfg = transformers.Qwen2Config(vocab_size=64, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=2, tie_word_embeddings=True,
                                   max_position_embeddings=64)
    model = build_hf_model(cfg, _dir("ckpt_tied"), device="cpu")
    base = _tensors(os.path.join(_dir("ckpt_tied"), "otf_2bit_base.safetensors"))
    assert isinstance(model.model.embed_tokens, QuantizedEmbedding)
    assert isinstance(model.lm_head, QuantizedLinearHead)
    assert model.lm_head.weight_int8.data_ptr() == model.model.embed_tokens.weight_int8.data_ptr()
    for i, layer in enumerate(model.model.layers):
        for proj in ("q_proj", "k_proj", "v_proj", "o_proj"):
            assert isinstance(getattr(layer.self_attn, proj), SymmetricOTF2BitLinear)
        for proj in ("gate_proj", "up_proj", "down_proj"):
            assert isinstance(getattr(layer.mlp, proj), SymmetricOTF2BitLinear)
        assert torch.equal(layer.input_layernorm.weight, base[f"model.layers.{i}.input_layernorm.weight"])
    assert torch.equal(model.model.norm.weight, base["model.norm.weight"])
    fresh = type(model.model.rotary_emb)(config=cfg, device="cpu")
    assert torch.equal(model.model.rotary_emb.inv_freq, fresh.inv_freq)


def test_stack_from_checkpoint_shapes():
    from otf_llm.checkpoint import load_checkpoint
    from otf_llm.decoder_stack import Llama2BitLinearStack
    ck = load_checkpoint(_dir("ckpt_tied"), device="cpu")
    st = Llama2BitLinearStack.from_checkpoint(ck, head_dim=16)
    assert (st.cfg.hidden, st.cfg.intermediate, st.cfg.heads, st.cfg.kv_heads) == (64, 128, 4, 2)
    assert st.fused and all(torch.equal(a, ck.layer_norms[i]["input_layernorm"]) for i, a in enumerate(st.in_norms))
    # three groups of 64 per down_proj row: the loader pads the scale rows to a 16-byte stride
    # (shape unchanged), which keeps the layer inside the tensor-pipe layout
    ck = load_checkpoint(_dir("ckpt_untied"), device="cpu")
    down = ck.layers[0]["mlp.down_proj"]
    assert down.scales.shape == (128, 3) and down.scales.stride(0) == 8
    assert torch.equal(down.scales, _tensors(os.path.join(_dir("ckpt_untied"), "otf_2bit_model.safetensors"))
                       ["model.layers.0.mlp.down_proj.scales"])
    st = Llama2BitLinearStack.from_checkpoint(ck, head_dim=32)
    assert st.fused
