"""The kernel watchdog, made to fire on purpose without faulting anything.

Every wait inside the tensor-core kernel's pipeline is bounded; when a wait
runs past its limit the kernel records ATTN_ERR_WATCHDOG in the device status
word, lets the copies and products it already issued land (under the default
2 s bound), frees its tensor memory and returns.  The limit is normally 2 s,
far above any legitimate wait (microseconds), so it never expires in use.
Here the test lowers it to 1 ns for one launch, so the first wait that is not
already satisfied expires; the test then checks that the launch returned,
that the status reports the watchdog, that reading the status cleared it, and
that a following launch under the default limit is correct and clean.
"""
import pytest
import torch

import oracle
from rocm_attn_b200.workloads import Shape, make_qkv

pytestmark = pytest.mark.gpu

ATTN_ERR_WATCHDOG = 7


@pytest.mark.parametrize("shape,dtype,causal", [
    (Shape(1, 4, 1024, 1024, 128), torch.float16, False),   # two-tile D=128 CTAs
    (Shape(2, 4, 1024, 1024, 64), torch.bfloat16, True),    # one-tile D=64 CTAs, 128-key blocks
    (Shape(8, 16, 256, 256, 64), torch.float16, False),     # one-tile D=64 CTAs, 64-key blocks
])
def test_watchdog_fires_and_recovers(attn, shape, dtype, causal):
    ext = attn.rocm_attn_ext
    q, k, v = (t.cuda() for t in make_qkv(shape, dtype, seed=5))
    assert attn.check_status(0) == 0
    prev = ext.set_wait_limit_ns(1)
    try:
        attn.attn_forward(q, k, v, causal=causal)
        torch.cuda.synchronize()
    finally:
        ext.set_wait_limit_ns(prev)
    assert attn.check_status(0) == ATTN_ERR_WATCHDOG
    assert attn.check_status(0) == 0  # reading the status cleared it
    out = attn.attn_forward(q, k, v, causal=causal)
    torch.cuda.synchronize()
    assert attn.check_status(0) == 0
    heads = [0, shape.bh - 1]
    qf, kf, vf, of = (t.reshape(-1, 1, *t.shape[2:]).cpu() for t in (q, k, v, out))
    ok, err = oracle.check(of[heads], oracle.sdpa_math_fp32(qf[heads], kf[heads], vf[heads], causal=causal), dtype)
    assert ok, f"after the watchdog: max abs err {err:.3e}"
