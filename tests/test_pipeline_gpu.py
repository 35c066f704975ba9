"""attn_forward_pinned: host-resident q/k/v through the pipelined copies,
against the device op on the same values (bitwise) and the oracle."""
import pytest
import torch

import oracle
from rocm_attn_b200.workloads import Shape, make_qkv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,dtype,causal,chunk", [
    (Shape(2, 8, 300, 300, 128), torch.float16, True, None),
    (Shape(1, 12, 512, 700, 64), torch.bfloat16, False, 5),
    (Shape(64, 8, 16, 16, 64), torch.float16, False, 100),   # short-sequence kernel
    (Shape(1, 3, 100, 100, 48), torch.float32, True, 1),     # general kernel
])
def test_pinned_matches_device_op(attn, shape, dtype, causal, chunk):
    q, k, v = (t.contiguous().pin_memory() for t in make_qkv(shape, dtype, seed=3))
    out = attn.attn_forward_pinned(q, k, v, causal=causal, chunk_slices=chunk)
    torch.cuda.synchronize()
    assert out.device.type == "cpu" and out.is_pinned() and out.shape == q.shape
    dev = attn.attn_forward(q.cuda(), k.cuda(), v.cuda(), causal=causal).cpu()
    assert torch.equal(out, dev)
    ok, err = oracle.check(out, oracle.sdpa_math_fp32(q, k, v, causal=causal), dtype)
    assert ok, err
    # a second call reuses the device buffers; new values must come through
    q2 = make_qkv(shape, dtype, seed=4)[0].contiguous().pin_memory()
    out2 = attn.attn_forward_pinned(q2, k, v, causal=causal, chunk_slices=chunk)
    torch.cuda.synchronize()
    assert torch.equal(out2, attn.attn_forward(q2.cuda(), k.cuda(), v.cuda(), causal=causal).cpu())


def test_pinned_buffer_cache_is_bounded(attn):
    from rocm_attn_b200 import pipeline
    shapes = [Shape(1, 2, 64 + 32 * i, 64 + 32 * i, 64) for i in range(pipeline.MAX_CACHED_SHAPES + 3)]
    for s in shapes:
        q, k, v = (t.contiguous().pin_memory() for t in make_qkv(s, torch.float16, seed=1))
        out = attn.attn_forward_pinned(q, k, v)
        torch.cuda.synchronize()
        assert torch.equal(out, attn.attn_forward(q.cuda(), k.cuda(), v.cuda()).cpu())
        assert len(pipeline._state) <= pipeline.MAX_CACHED_SHAPES
