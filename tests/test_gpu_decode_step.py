"""The persistent decode-step kernel (otf2b_decode_step): one launch per token for the whole
decoder linear stack, checked against the per-group launches and the CPU restatement."""
import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _pair(cfg, dev, seed):
    from otf_llm.decoder_stack import Llama2BitLinearStack
    mk = Llama2BitLinearStack(cfg, device=dev, seed=seed, persistent=True)
    ref = Llama2BitLinearStack(cfg, device=dev, seed=seed, persistent=False)
    assert mk.mk is not None and ref.mk is None
    return mk, ref


CONFIGS = {
    "mha_g64": dict(layers=2, hidden=1024, intermediate=2816, heads=8, kv_heads=8, head_dim=128),
    "gqa_g64": dict(layers=2, hidden=1024, intermediate=2816, heads=8, kv_heads=2, head_dim=128),
    "odd_groups": dict(layers=2, hidden=1024, intermediate=2880, heads=8, kv_heads=8, head_dim=128),  # 45 groups
    "g128": dict(layers=2, hidden=1024, intermediate=2816, heads=8, kv_heads=4, head_dim=128, group_size=128),
    "g32": dict(layers=1, hidden=512, intermediate=1536, heads=4, kv_heads=4, head_dim=128, group_size=32),
}


@pytest.mark.parametrize("name", list(CONFIGS))
def test_persistent_step_matches_group_launches(name, cuda_dev):
    from otf_llm import _native
    from otf_llm.decoder_stack import StackConfig
    cfg = StackConfig(**CONFIGS[name])
    mk, ref = _pair(cfg, cuda_dev, seed=2)
    h = torch.randn(1, cfg.hidden, generator=torch.Generator().manual_seed(3)).half().to(cuda_dev)
    y = mk(h).float().cpu().numpy()
    y_ref = ref(h).float().cpu().numpy()
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    assert rel_err(y, y_ref) < 3e-3
    # deterministic: a second step from the same input is bit-identical
    assert np.array_equal(mk(h).float().cpu().numpy(), y)


def test_persistent_step_in_cuda_graph(cuda_dev):
    from otf_llm import _native
    from otf_llm.decoder_stack import DecodeGraph, StackConfig
    cfg = StackConfig(**CONFIGS["gqa_g64"])
    mk, _ = _pair(cfg, cuda_dev, seed=5)
    h = torch.randn(1, cfg.hidden, generator=torch.Generator().manual_seed(6)).half().to(cuda_dev)
    eager = mk(h).clone()
    g = DecodeGraph(mk)
    g.x.copy_(h)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(g.y, eager)
    assert _native.device_error() == 0


def test_persistent_step_7b_layer_shapes(cuda_dev):
    """Two layers at the full Llama-2-7B shapes (the bench's per-layer work)."""
    from otf_llm import _native
    from otf_llm.decoder_stack import StackConfig
    cfg = StackConfig(layers=2)
    mk, ref = _pair(cfg, cuda_dev, seed=1)
    h = torch.randn(1, cfg.hidden, generator=torch.Generator().manual_seed(5)).half().to(cuda_dev)
    y = mk(h).float().cpu().numpy()
    y_ref = ref(h).float().cpu().numpy()
    torch.cuda.synchronize()
    assert _native.device_error() == 0
    assert rel_err(y, y_ref) < 3e-3
