"""CUDA-graph capture of the op (small-shape launch overhead): the launcher
allocates nothing and encodes its TMA descriptors on the host, so a captured
call replays with the descriptors baked into the graph.  The first call of
each kernel variant on a device must precede capture (it sets the kernel's
shared-memory attribute), which torch's own warm-up-then-capture pattern
already does."""
import pytest
import torch

import oracle
from rocm_attn_b200.workloads import Shape, make_qkv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape,dtype,causal", [
    (Shape(2, 16, 256, 256, 64), torch.float16, False),     # tensor-core kernel
    (Shape(16, 8, 128, 128, 128), torch.bfloat16, True),    # tensor-core kernel
    (Shape(16, 5, 40, 93, 16), torch.float16, False),       # general kernel (D=16)
    (Shape(2, 4, 100, 100, 64), torch.float32, True),       # general kernel (fp32)
], ids=["c5a", "c5d-causal", "d16-cross", "fp32"])
def test_capture_and_replay(attn, shape, dtype, causal):
    q, k, v = (t.cuda() for t in make_qkv(shape, dtype, seed=1))
    eager = attn.attn_forward(q, k, v, causal=causal)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = attn.attn_forward(q, k, v, causal=causal)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # new values in the captured input buffers are picked up by a replay
    q2, k2, v2 = make_qkv(shape, dtype, seed=2)
    q.copy_(q2)
    k.copy_(k2)
    v.copy_(v2)
    g.replay()
    torch.cuda.synchronize()
    ok, err = oracle.check(out.cpu(), oracle.sdpa_math_fp32(q2, k2, v2, causal=causal), dtype)
    assert ok, err
    assert attn.check_status(0) == 0
