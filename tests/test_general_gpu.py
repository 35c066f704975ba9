"""The general kernel: fp32 inputs, head dims other than 64/128, and
fp16/bf16 buffers that are not 16-byte aligned, against the CPU oracle.

Includes the reference's own test cases run through this op: the ramp
known-answer test (src/tests/attn_test.cpp:51-98: B=1, H=1, S=2, D=4, fp32,
tolerance 1e-3) and the interface tests (python/test/test_torch_interface.py:
10-36: seed 0, fp32, D=16, self attention causal and not, cross attention
6x9, rtol = atol = 1e-3).
"""
import pytest
import torch

import oracle
from rocm_attn_b200.workloads import Shape, make_qkv

pytestmark = pytest.mark.gpu


def _check(attn, q, k, v, causal=False, scale=None, atol=None):
    out = attn.attn_forward(q.cuda(), k.cuda(), v.cuda(), causal=causal, scale=scale)
    torch.cuda.synchronize()
    assert out.shape == q.shape and out.dtype == q.dtype
    ref = oracle.sdpa_math_fp32(q, k, v, causal=causal, scale=scale)
    if atol is None:
        ok, err = oracle.check(out.cpu(), ref, q.dtype)
        assert ok, f"{tuple(q.shape)} x {tuple(k.shape)} {q.dtype} causal={causal}: max abs err {err:.3e}"
    else:
        err = (out.cpu().float() - ref).abs().max().item()
        assert err <= atol, err
    return out


def test_reference_ramp_known_answer(attn):
    # src/tests/attn_test.cpp:52-60: q = 0.01 (i+1), k = 0.02 (i+1), v = 0.03 (i+1)
    i = torch.arange(1, 9, dtype=torch.float32).view(1, 1, 2, 4)
    out = _check(attn, 0.01 * i, 0.02 * i, 0.03 * i, atol=1e-3)
    ref = oracle.c_oracle_forward(0.01 * i, 0.02 * i, 0.03 * i)
    assert (out.cpu() - ref).abs().max().item() <= 1e-3  # the test's own tolerance (attn_test.cpp:90)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
def test_reference_interface_cases(attn, dtype):
    # python/test/test_torch_interface.py:10-36 (seed 0, D=16), run in each dtype
    torch.manual_seed(0)
    q = torch.randn(1, 2, 8, 16).to(dtype)
    k = torch.randn(1, 2, 8, 16).to(dtype)
    v = torch.randn(1, 2, 8, 16).to(dtype)
    for causal in (False, True):
        _check(attn, q, k, v, causal=causal)
    qc = torch.randn(1, 2, 6, 16).to(dtype)
    kc = torch.randn(1, 2, 9, 16).to(dtype)
    vc = torch.randn(1, 2, 9, 16).to(dtype)
    _check(attn, qc, kc, vc)
    if dtype == torch.float32:
        # the reference's own tolerance for this test
        out = attn.attn_forward(q.cuda(), k.cuda(), v.cuda(), False).cpu()
        assert torch.allclose(out, oracle.sdpa_math_fp32(q, k, v), rtol=1e-3, atol=1e-3)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("D", [1, 4, 16, 24, 32, 48, 64, 80, 96, 128, 160, 200, 256])
def test_head_dims(attn, D, causal, dtype):
    s = Shape(2, 3, 77, 77, D)
    q, k, v = make_qkv(s, dtype, seed=D)
    _check(attn, q, k, v, causal=causal)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("shape", [Shape(1, 2, 6, 9, 16), Shape(2, 2, 300, 100, 32), Shape(1, 1, 100, 300, 96),
                                   Shape(16, 5, 40, 93, 16), Shape(1, 2, 1, 513, 200), Shape(1, 1, 700, 1, 48)],
                         ids=lambda s: f"{s.B}x{s.H}x{s.Lq}x{s.Lk}x{s.D}")
def test_cross_and_ragged(attn, shape, dtype):
    q, k, v = make_qkv(shape, dtype, seed=shape.Lq)
    for causal in (False, True):
        _check(attn, q, k, v, causal=causal)


@pytest.mark.parametrize("D", [64, 128])
def test_fp32_at_tensor_core_dims(attn, D):
    q, k, v = make_qkv(Shape(1, 4, 300, 300, D), torch.float32, seed=3)
    _check(attn, q, k, v, causal=True)
    _check(attn, q, k, v, causal=False, scale=0.3)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_unaligned_buffers_take_the_general_kernel(attn, dtype):
    # Views starting one element into their storage are not 16-byte aligned:
    # the tensor-core kernel cannot take them, the general kernel does.
    s = Shape(1, 2, 130, 130, 64)
    q, k, v = make_qkv(s, dtype, seed=9)
    n = q.numel()

    def offset_view(t):
        buf = torch.empty(n + 1, dtype=dtype, device="cuda")
        view = buf[1:].view(t.shape)
        view.copy_(t.cuda())
        return view

    qd, kd, vd = offset_view(q), offset_view(k), offset_view(v)
    assert qd.data_ptr() % 16 != 0
    out = attn.attn_forward(qd, kd, vd, causal=True)
    ok, err = oracle.check(out.cpu(), oracle.sdpa_math_fp32(q, k, v, causal=True), dtype)
    assert ok, err


def test_fp32_empty_keys_give_zeros(attn):
    q = torch.randn(1, 2, 7, 16, device="cuda")
    k = torch.randn(1, 2, 0, 16, device="cuda")
    out = attn.attn_forward(q, k, k)
    assert out.shape == q.shape and torch.count_nonzero(out) == 0
