"""GPU parity of the INT8 embedding (bit-exact) and LM head (max rel err 1e-3)."""
import numpy as np
import pytest
import torch

from conftest import load_golden, rel_err
from oracle import oracle

pytestmark = pytest.mark.gpu


def test_embedding_golden_bit_exact(cuda_dev):
    from otf_llm.symmetric_2bit_engine import QuantizedEmbedding
    gd = load_golden("int8_v1000_d256")
    emb = QuantizedEmbedding(*gd["weight_int8"].shape).to(cuda_dev)
    emb.weight_int8.copy_(torch.from_numpy(gd["weight_int8"]))
    emb.scales.copy_(torch.from_numpy(gd["scales"]))
    out = emb(torch.from_numpy(gd["ids"]).to(cuda_dev)).cpu().numpy()
    assert out.shape == gd["emb_out"].shape
    assert np.array_equal(out.view(np.uint16), gd["emb_out"].view(np.uint16))


def test_embedding_module_rejects_out_of_range_ids(cuda_dev):
    """QuantizedEmbedding.forward raises on ids outside [0, V), as the reference's
    F.embedding does (otf_llm/symmetric_2bit_engine.py:44)."""
    from otf_llm.symmetric_2bit_engine import QuantizedEmbedding
    emb = QuantizedEmbedding(100, 64).to(cuda_dev)
    emb(torch.tensor([[0, 99]], device=cuda_dev))
    for bad in ([[0, 100]], [[-1, 3]]):
        with pytest.raises(IndexError):
            emb(torch.tensor(bad, device=cuda_dev))


def test_embedding_large_vocab_bit_exact(cuda_dev):
    from otf_llm import _native
    V, D = 128256, 3072
    g = torch.Generator().manual_seed(11)
    w = torch.randint(-127, 128, (V, D), generator=g, dtype=torch.int32).to(torch.int8)
    s = (torch.rand(V, 1, generator=g) * 2e-4 + 1e-5).half()
    ids = torch.randint(0, V, (64,), generator=g)
    bad = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    out = _native.i8_embed(ids.to(cuda_dev), w.to(cuda_dev), s.to(cuda_dev), bad).cpu().numpy()
    ref = oracle.i8_embed(ids.numpy(), w.numpy(), s.numpy())
    assert np.array_equal(out.view(np.uint16), ref.view(np.uint16))
    assert int(bad.item()) == 0
    bad_ids = torch.tensor([0, V, -1], dtype=torch.int64, device=cuda_dev)
    out = _native.i8_embed(bad_ids, w.to(cuda_dev), s.to(cuda_dev), bad)
    assert int(bad.item()) == 1 and bool((out[1:] == 0).all())


@pytest.mark.parametrize("D", [100, 256, 8192, 16384, 16400])
def test_embedding_widths_bit_exact(D, cuda_dev):
    """Row widths on both sides of the 16-byte-piece gather (D a multiple of 16 up to 16384)
    and the strided form beyond it, bit for bit against the oracle."""
    from otf_llm import _native
    V = 300
    g = torch.Generator().manual_seed(D)
    w = torch.randint(-127, 128, (V, D), generator=g, dtype=torch.int32).to(torch.int8)
    s = (torch.rand(V, 1, generator=g) * 2e-3 + 1e-5).half()
    ids = torch.tensor([0, V - 1, 7, 7, 123], dtype=torch.int64)
    bad = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    out = _native.i8_embed(ids.to(cuda_dev), w.to(cuda_dev), s.to(cuda_dev), bad).cpu().numpy()
    ref = oracle.i8_embed(ids.numpy(), w.numpy(), s.numpy())
    assert np.array_equal(out.view(np.uint16), ref.view(np.uint16))
    assert int(bad.item()) == 0


def test_head_golden(cuda_dev):
    from otf_llm.symmetric_2bit_engine import QuantizedEmbedding, QuantizedLinearHead
    gd = load_golden("int8_v1000_d256")
    V, D = gd["weight_int8"].shape
    emb = QuantizedEmbedding(V, D).to(cuda_dev)
    emb.weight_int8.copy_(torch.from_numpy(gd["weight_int8"]))
    emb.scales.copy_(torch.from_numpy(gd["scales"]))
    head = QuantizedLinearHead(D, V).to(cuda_dev)
    head.weight_int8 = emb.weight_int8
    head.scales = emb.scales
    for M in (1, 5):
        lg = head(torch.from_numpy(gd[f"x_m{M}"]).to(cuda_dev).view(1, M, D)).view(M, V).cpu().numpy()
        assert lg.dtype == np.float32
        assert rel_err(lg, gd[f"logits_f64_m{M}"]) < 1e-3
        assert rel_err(lg, gd[f"logits_m{M}"]) < 1.5e-3


@pytest.mark.parametrize("V,D,M", [(128256, 3072, 1), (128256, 8192, 1), (1000, 200, 2), (4097, 64, 3),
                                   (17, 256, 1), (65, 128, 2), (1000, 4096, 1), (64000, 8192, 4), (300, 2064, 1)])
def test_head_shapes(V, D, M, cuda_dev):
    from otf_llm import _native
    g = torch.Generator().manual_seed(V + D)
    w = torch.randint(-127, 128, (V, D), generator=g, dtype=torch.int32).to(torch.int8)
    s = (torch.rand(V, 1, generator=g) * 2e-4 + 1e-5).half()
    x = torch.randn(M, D, generator=g).half()
    lg = _native.i8_head(x.to(cuda_dev), w.to(cuda_dev), s.to(cuda_dev)).cpu().numpy()
    ref = oracle.i8_head(x.numpy(), w.numpy(), s.numpy())
    assert rel_err(lg, ref) < 1e-3


@pytest.mark.parametrize("V,D,M", [(5000, 3072, 16), (3000, 8192, 16), (777, 272, 11), (4097, 64, 3)])
def test_head_rows_share_weight_boxes(V, D, M, cuda_dev):
    """Several activation rows per head launch (up to 8, as shared memory allows) read every
    weight box once for all of them; each row's logits and greedy pick are bit-identical to a
    launch of that row alone, with strided x and logits rows."""
    from otf_llm import _native
    g = torch.Generator().manual_seed(V * 7 + M)
    w = torch.randint(-127, 128, (V, D), generator=g, dtype=torch.int32).to(torch.int8).to(cuda_dev)
    s = (torch.rand(V, 1, generator=g) * 2e-3 + 1e-4).half().to(cuda_dev)
    xb = (torch.randn(M, D + 24, generator=g) * 2).half().to(cuda_dev)
    xb[M // 2, 7] = 900.0                            # a hot channel in one row only
    x = xb[:, :D]
    lb = torch.full((M, V + 5), -1.0, dtype=torch.float32, device=cuda_dev)
    logits = lb[:, :V]
    ids = _native.i8_head_argmax(x, w, s, logits)
    for m in range(M):
        one = torch.empty(1, V, dtype=torch.float32, device=cuda_dev)
        idm = _native.i8_head_argmax(x[m:m + 1].contiguous(), w, s, one)
        assert torch.equal(logits[m:m + 1], one), m
        assert int(ids[m]) == int(idm[0]), m
    assert bool((lb[:, V:] == -1.0).all())
    ref = oracle.i8_head(x.float().cpu().numpy().astype(np.float16), w.cpu().numpy(), s.cpu().numpy())
    assert rel_err(logits.cpu().numpy(), ref) < 1e-3
    assert _native.device_error() == 0


def test_head_graph_replay(cuda_dev):
    """The head's launch (its weight tensor map travels in the kernel parameters) replays
    from a CUDA graph exactly as it ran eagerly."""
    from otf_llm import _native
    g = torch.Generator().manual_seed(3)
    w = torch.randint(-127, 128, (20000, 3072), generator=g, dtype=torch.int32).to(torch.int8).to(cuda_dev)
    s = (torch.rand(20000, 1, generator=g) * 2e-4 + 1e-5).half().to(cuda_dev)
    x = torch.randn(1, 3072, generator=g).half().to(cuda_dev)
    out = torch.empty(1, 20000, dtype=torch.float32, device=cuda_dev)
    _native.i8_head(x, w, s, out)
    eager = out.clone()
    st = torch.cuda.Stream()
    st.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(st):
        _native.i8_head(x, w, s, out)
    torch.cuda.current_stream().wait_stream(st)
    gr = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gr):
        _native.i8_head(x, w, s, out)
    out.zero_()
    gr.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    assert _native.device_error() == 0


@pytest.mark.parametrize("V,D,M", [(128256, 3072, 1), (1000, 256, 3), (50000, 4096, 2), (777, 272, 2)])
def test_head_argmax(V, D, M, cuda_dev):
    """Fused greedy step: the index of the largest logit of each row (first maximum)."""
    from otf_llm import _native
    g = torch.Generator().manual_seed(V + D)
    w = torch.randint(-127, 128, (V, D), generator=g, dtype=torch.int32).to(torch.int8)
    s = (torch.rand(V, 1, generator=g) * 2e-3 + 1e-4).half()
    x = torch.randn(M, D, generator=g).half()
    wd, sd, xd = w.to(cuda_dev), s.to(cuda_dev), x.to(cuda_dev)
    logits = torch.empty(M, V, dtype=torch.float32, device=cuda_dev)
    ids = _native.i8_head_argmax(xd, wd, sd, logits)
    ref_logits = _native.i8_head(xd, wd, sd)
    assert torch.equal(logits, ref_logits)
    assert torch.equal(ids, torch.argmax(ref_logits, dim=1))
    ids2 = _native.i8_head_argmax(xd, wd, sd)          # logits not stored
    assert torch.equal(ids, ids2)
    # against the oracle: the chosen logit is the maximum up to the head's tolerance
    ref = oracle.i8_head(x.numpy(), w.numpy(), s.numpy())
    picked = ref[np.arange(M), ids.cpu().numpy()]
    assert np.all(picked >= ref.max(axis=1) - 1e-3 * np.abs(ref).max())
