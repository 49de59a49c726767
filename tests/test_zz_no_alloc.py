"""otf_attn_decode_noalloc: decode attention for callers that cannot allocate device memory
(a plugin host that hands over only the op's tensors, an allocator frozen after warm-up).
Its split-KV scratch is the library's own fixed device array; the result must match
otf_attn_decode with a caller-provided workspace, on consecutive calls that reuse that array.
This file is collected last on purpose."""
import math

import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu


def _call(N, fn, *args):
    st = fn(*args)
    assert st == 0, N.lib().otf_status_string(st)


@pytest.mark.parametrize("hd,heads,kv,max_pos,lengths", [
    (128, 24, 8, 1024, (700, 65)),
    (64, 8, 2, 1024, (700, 65)),
    # the largest cache the fixed array takes for 8 KV heads of 128: 63 splits, partials
    # ending 256 bytes before the end of the array
    (128, 64, 8, 4032, (4032, 4001)),
])
def test_noalloc_attention_matches_workspace_attention(hd, heads, kv, max_pos, lengths, cuda_dev):
    from otf_llm import _native as N
    L = N.lib()
    g = torch.Generator(device=cuda_dev).manual_seed(hd + heads)
    kc = torch.randn(max_pos, kv * hd, generator=g, device=cuda_dev).half()
    vc = torch.randn(max_pos, kv * hd, generator=g, device=cuda_dev).half()
    ws = torch.zeros(int(L.otf_attn_workspace_bytes(kv, hd, max_pos)), dtype=torch.uint8, device=cuda_dev)
    scale = 1.0 / math.sqrt(hd)
    st = N._stream(cuda_dev)
    # two calls in a row with different inputs and lengths: the second reuses the shared scratch
    for length in lengths:
        q = torch.randn(heads * hd, generator=g, device=cuda_dev).half()
        pos = torch.tensor([length - 1], dtype=torch.int32, device=cuda_dev)
        ref = torch.empty(heads * hd, dtype=torch.float16, device=cuda_dev)
        got = torch.empty_like(ref)
        _call(N, L.otf_attn_decode, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(), ref.data_ptr(),
              scale, heads, kv, hd, max_pos, ws.data_ptr(), ws.numel(), st)
        _call(N, L.otf_attn_decode_noalloc, q.data_ptr(), kc.data_ptr(), vc.data_ptr(), pos.data_ptr(),
              got.data_ptr(), scale, heads, kv, hd, max_pos, st)
        torch.cuda.synchronize()
        # the same kernel on the same inputs, only the scratch differs: identical bits
        assert torch.equal(got, ref), rel_err(got.float().cpu().numpy(), ref.float().cpu().numpy())


def test_noalloc_rejects_cache_beyond_scratch(cuda_dev):
    from otf_llm import _native as N
    L = N.lib()
    max_pos = 4033   # 8 KV heads of 128 need more than the fixed scratch beyond 4032 positions
    q = torch.zeros(24 * 128, dtype=torch.float16, device=cuda_dev)
    kc = torch.zeros(max_pos, 8 * 128, dtype=torch.float16, device=cuda_dev)
    out = torch.zeros_like(q)
    pos = torch.zeros(1, dtype=torch.int32, device=cuda_dev)
    st = L.otf_attn_decode_noalloc(q.data_ptr(), kc.data_ptr(), kc.data_ptr(), pos.data_ptr(), out.data_ptr(), 1.0,
                                   24, 8, 128, max_pos, N._stream(cuda_dev))
    assert st == 2   # OTF_ERR_UNSUPPORTED
