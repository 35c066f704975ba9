"""Strided inputs read in place (no .contiguous() copies), against the CPU
oracle on contiguous copies of the same values.

The tensor-core kernel reads them through 4-D TMA maps when every stride is
a multiple of 16 bytes (e.g. the [B, L, H, D] layout viewed as [B, H, L, D],
benchmark/bench_attention.py:182-184 of the reference); other strides run the
general kernel.
"""
import ctypes

import pytest
import torch

import oracle
from rocm_attn_b200.workloads import Shape, make_qkv

pytestmark = pytest.mark.gpu


def _ref_check(attn, qd, kd, vd, causal):
    out = attn.attn_forward(qd, kd, vd, causal=causal)
    torch.cuda.synchronize()
    assert out.is_contiguous() and out.shape == qd.shape
    ref = oracle.sdpa_math_fp32(qd.cpu().contiguous(), kd.cpu().contiguous(), vd.cpu().contiguous(), causal=causal)
    ok, err = oracle.check(out.cpu(), ref, qd.dtype)
    assert ok, f"{tuple(qd.shape)} strides {qd.stride()} causal={causal}: max abs err {err:.3e}"


LAYOUTS = ["bshd", "hbld", "heads_sliced", "rows_sliced", "dim_sliced"]


def _make(layout, shape, dtype, seed):
    B, H, L, D = shape.B, shape.H, shape.Lq, shape.D
    q, k, v = (t.cuda() for t in make_qkv(shape, dtype, seed=seed))
    if layout == "bshd":           # [B, L, H, D] storage
        return tuple(t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
    if layout == "hbld":           # [H, B, L, D] storage
        return tuple(t.transpose(0, 1).contiguous().transpose(0, 1) for t in (q, k, v))
    if layout == "heads_sliced":   # every other head of a 2H tensor
        return tuple(torch.cat([t, t], dim=1)[:, ::2] for t in (q, k, v))
    if layout == "rows_sliced":    # rows 8.. of a longer sequence
        return tuple(torch.cat([torch.zeros_like(t[:, :, :8]), t], dim=2)[:, :, 8:] for t in (q, k, v))
    if layout == "dim_sliced":     # the first D columns of a 2D-wide tensor
        return tuple(torch.cat([t, t], dim=3)[..., :D] for t in (q, k, v))
    raise ValueError(layout)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("layout", LAYOUTS)
@pytest.mark.parametrize("L", [300, 200])  # tcgen05 kernel, 64-row warp-level kernel
def test_tensor_core_strided(attn, layout, D, dtype, L):
    qd, kd, vd = _make(layout, Shape(2, 3, L, L, D), dtype, seed=D)
    assert not qd.is_contiguous()
    for causal in (False, True):
        _ref_check(attn, qd, kd, vd, causal)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
@pytest.mark.parametrize("layout", ["bshd", "heads_sliced", "dim_sliced"])
def test_general_strided(attn, layout, dtype):
    qd, kd, vd = _make(layout, Shape(2, 3, 100, 100, 48), dtype, seed=5)
    for causal in (False, True):
        _ref_check(attn, qd, kd, vd, causal)


def test_broadcast_kv_heads(attn):
    # K/V shared by all heads (stride 0 over heads, as an expand() gives)
    s = Shape(2, 4, 200, 200, 64)
    q, k, v = (t.cuda() for t in make_qkv(s, torch.float16, seed=8))
    kd, vd = k[:, :1].expand(-1, 4, -1, -1), v[:, :1].expand(-1, 4, -1, -1)
    assert kd.stride(1) == 0
    _ref_check(attn, q, kd, vd, causal=True)


def test_bshd_matches_contiguous_bitwise(attn):
    s = Shape(1, 8, 1000, 1000, 128)
    q, k, v = (t.cuda() for t in make_qkv(s, torch.float16, seed=2))
    a = attn.attn_forward(q, k, v, causal=True)
    qb, kb, vb = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
    b = attn.attn_forward(qb, kb, vb, causal=True)
    assert torch.equal(a, b)  # same kernel, same tiles: only the addressing differs


def test_c_abi_strided_entry_point(attn):
    lib = ctypes.CDLL(attn.KERNEL_LIB_PATH)
    LL3 = ctypes.c_longlong * 3
    lib.launch_attn_forward_strided.argtypes = ([ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 +
                                                [ctypes.c_bool, ctypes.c_float, ctypes.c_int] +
                                                [ctypes.POINTER(ctypes.c_longlong)] * 3 + [ctypes.c_void_p])
    B, H, L, D = 2, 4, 256, 128
    s = Shape(B, H, L, L, D)
    q, k, v = make_qkv(s, torch.float16, seed=4)
    # [B, L, H, D] storage
    qb, kb, vb = (t.transpose(1, 2).contiguous().cuda() for t in (q, k, v))
    st = LL3(L * H * D, D, H * D)
    out = torch.empty(B, H, L, D, dtype=torch.float16, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    rc = lib.launch_attn_forward_strided(qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), out.data_ptr(), B, H, L, L, D,
                                         False, -1.0, 0, st, st, st, stream)
    assert rc == 0
    torch.cuda.synchronize()
    ok, err = oracle.check(out.cpu(), oracle.sdpa_math_fp32(q, k, v), torch.float16)
    assert ok, err
    # negative strides are refused before any launch
    bad = LL3(-1, D, H * D)
    assert lib.launch_attn_forward_strided(qb.data_ptr(), kb.data_ptr(), vb.data_ptr(), out.data_ptr(), B, H, L, L,
                                           D, False, -1.0, 0, bad, st, st, stream) == 1
