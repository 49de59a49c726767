"""Batched greedy decoding (BatchedGreedyDecoder): B sequences in lockstep, each with its own
KV cache and position, the 2-bit projections at M = B rows (batched integer-MMA kernel for
B <= 8 and in 8-row slices to 16, the tcgen05 GEMM from 32).  Teacher-forced logits of every
sequence against the batch-1 decoder on the same prompt (tolerance 2e-2 of max|logit|, the
kernels accumulate in different orders), greedy ids = argmax of the logits, graph = eager."""
import numpy as np
import pytest
import torch

from conftest import rel_err
from test_gpu_decode_model import _tiny_model

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B", [3, 16, 32])
def test_batched_decoder_matches_batch1(B, cuda_dev):
    from otf_llm.decode_model import BatchedGreedyDecoder, GreedyDecoder
    cfg, layers, norms, emb, head, fnorm = _tiny_model(cuda_dev)
    T = 10
    prompts = torch.from_numpy(np.random.default_rng(B).integers(0, cfg.vocab, (B, T))).to(cuda_dev)
    bat = BatchedGreedyDecoder(cfg, layers, norms, emb, head, fnorm, cuda_dev, B)
    eager = []
    bat.generate(prompts, 1, logits_out=eager)
    bat.capture()
    graph = []
    bat.generate(prompts, 1, logits_out=graph)
    eager = torch.stack(eager, 1).float().cpu().numpy()               # [B, T, V]
    graph = torch.stack(graph, 1).float().cpu().numpy()
    assert np.array_equal(eager, graph)
    one = GreedyDecoder(cfg, layers, norms, emb, head, fnorm, cuda_dev)
    for s in (0, B // 2, B - 1):
        ref = []
        one.generate(prompts[s], 1, logits_out=ref)
        ref = torch.cat(ref).float().cpu().numpy()                    # [T, V]
        assert rel_err(eager[s], ref) < 2e-2, s
    # free-running: the ids each step feeds back are the argmax of that step's logits
    out = bat.generate(prompts[:, :4], 6)
    assert out.shape == (B, 6)
    assert int(bat.pos[0]) == 4 + 5
