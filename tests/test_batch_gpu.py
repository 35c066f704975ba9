"""Several problems in one call: ``attn_forward_batch`` / the C entry point
``launch_attn_forward_batch``.

The reference's benchmark runs its shape lists one launch per shape
(benchmark/bench_attention.py:81-100,171-175): the C5 sweep of five shapes and
the UnifoLM preset list (benchmark/attn_shapes_unifolm_infer.txt:1-17).  The
batch entry point runs such a list with the tensor-core problems of one
instantiation in one grid.  Every problem's output must be bit for bit the
output of its own ``attn_forward`` call, and within the path's tolerance of
the CPU oracle (torch SDPA math, fp32).
"""
import ctypes

import pytest
import torch

import oracle
from rocm_attn_b200.workloads import WORKLOADS, Shape, make_qkv

pytestmark = pytest.mark.gpu


def _inputs(shapes, dtype, seed=0):
    return [tuple(t.cuda() for t in make_qkv(s, dtype, seed=seed + i)) for i, s in enumerate(shapes)]


def _check_oracle(shape, q, k, v, out, dtype, causal, heads=2):
    qf, kf, vf, of = (t.reshape(-1, 1, *t.shape[2:]) for t in (q, k, v, out))
    idx = sorted({0, shape.bh - 1})[:heads]
    rows = list(range(shape.Lq)) if shape.Lq <= 256 else list(range(128)) + list(range(shape.Lq - 128, shape.Lq))
    ref = oracle.sdpa_rows_fp32(qf[idx].cpu(), kf[idx].cpu(), vf[idx].cpu(), rows, causal=causal)
    ok, err = oracle.check(of[idx][:, :, rows].cpu(), ref, dtype)
    assert ok, f"{shape} causal={causal}: max abs err {err:.3e}"


def _batch_equals_single(attn, shapes, dtype, causal, seed=0, oracle_check=True):
    ins = _inputs(shapes, dtype, seed)
    outs = attn.attn_forward_batch([t[0] for t in ins], [t[1] for t in ins], [t[2] for t in ins], causal=causal)
    singles = [attn.attn_forward(*t, causal=causal) for t in ins]
    torch.cuda.synchronize()
    assert len(outs) == len(shapes)
    for s, o, r in zip(shapes, outs, singles):
        assert o.shape == r.shape and o.dtype == r.dtype
        assert torch.equal(o, r), f"{s}: batched output differs from the single call"
    if oracle_check:
        for s, t, o in zip(shapes, ins, outs):
            _check_oracle(s, *t, o, dtype, causal)
    assert attn.check_status(0) == 0


def test_c5_sweep_batched(attn):
    _batch_equals_single(attn, list(WORKLOADS["c5"].shapes), torch.float16, False)


def test_unifolm_preset_batched(attn):
    _batch_equals_single(attn, list(WORKLOADS["unifolm"].shapes), torch.float16, False)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("causal", [False, True])
def test_mixed_routes_batched(attn, dtype, causal):
    # tensor-core D=128 and D=64 (both key-block sizes), the short, mid-length
    # and general kernels, cross attention and ragged tails in one call
    shapes = [Shape(1, 4, 1024, 1024, 128), Shape(2, 3, 300, 200, 128), Shape(1, 2, 130, 700, 64),
              Shape(64, 8, 256, 256, 64), Shape(8, 4, 16, 16, 64), Shape(2, 4, 40, 93, 64),
              Shape(1, 2, 100, 100, 48), Shape(1, 2, 2048, 2048, 128), Shape(3, 2, 77, 77, 64)]
    _batch_equals_single(attn, shapes, dtype, causal, seed=7)


def test_more_problems_than_one_grid_holds(attn):
    # 20 problems of one instantiation: two grids (16 + 4)
    shapes = [Shape(1, 2, 128 + 64 * i, 128 + 96 * i, 128) for i in range(20)]
    _batch_equals_single(attn, shapes, torch.bfloat16, True, seed=3, oracle_check=False)
    ins = _inputs(shapes[-3:], torch.bfloat16, 3 + 17)
    outs = attn.attn_forward_batch([t[0] for t in ins], [t[1] for t in ins], [t[2] for t in ins], causal=True)
    for s, t, o in zip(shapes[-3:], ins, outs):
        _check_oracle(s, *t, o, torch.bfloat16, True)


def test_strided_problems_batched(attn):
    # the flash-style [B, L, H, D] storage viewed as [B, H, L, D], and a
    # stride-0 (broadcast) K/V that TMA cannot describe (general kernel)
    s1, s2 = Shape(2, 4, 512, 512, 128), Shape(2, 4, 300, 300, 64)
    q1, k1, v1 = (t.cuda().transpose(1, 2).contiguous().transpose(1, 2) for t in make_qkv(s1, torch.float16, 1))
    q2, k2, v2 = (t.cuda() for t in make_qkv(s2, torch.float16, 2))
    k2b, v2b = k2[:, :1].expand(-1, 4, -1, -1), v2[:, :1].expand(-1, 4, -1, -1)
    outs = attn.attn_forward_batch([q1, q2], [k1, k2b], [v1, v2b])
    assert torch.equal(outs[0], attn.attn_forward(q1, k1, v1))
    assert torch.equal(outs[1], attn.attn_forward(q2, k2b, v2b))
    _check_oracle(s1, q1, k1, v1, outs[0], torch.float16, False)
    _check_oracle(s2, q2, k2b.contiguous(), v2b.contiguous(), outs[1], torch.float16, False)


def test_batch_argument_errors(attn):
    x = torch.zeros(1, 1, 8, 64, device="cuda", dtype=torch.float16)
    y = torch.zeros(1, 1, 8, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="same dtype"):
        attn.attn_forward_batch([x, y], [x, y], [x, y])
    with pytest.raises(RuntimeError, match="same length"):
        attn.attn_forward_batch([x], [x, x], [x])
    assert attn.attn_forward_batch([], [], []) == []


class AttnProblem(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("B", ctypes.c_int), ("H", ctypes.c_int), ("Sq", ctypes.c_int), ("Skv", ctypes.c_int),
                ("D", ctypes.c_int), ("causal", ctypes.c_bool), ("softmax_scale", ctypes.c_float),
                ("q_strides", ctypes.c_void_p), ("k_strides", ctypes.c_void_p), ("v_strides", ctypes.c_void_p)]


def test_batch_through_the_c_abi(attn):
    lib = ctypes.CDLL(attn.KERNEL_LIB_PATH)
    lib.launch_attn_forward_batch.argtypes = [ctypes.POINTER(AttnProblem), ctypes.c_int, ctypes.c_int,
                                              ctypes.c_void_p]
    lib.launch_attn_forward_batch.restype = ctypes.c_int
    shapes = [Shape(2, 4, 700, 700, 128), Shape(1, 8, 256, 900, 128), Shape(4, 4, 16, 16, 64)]
    ins = _inputs(shapes, torch.float16, 11)
    outs = [torch.empty_like(t[0]) for t in ins]
    arr = (AttnProblem * len(shapes))()
    for i, (s, (q, k, v), o) in enumerate(zip(shapes, ins, outs)):
        arr[i] = AttnProblem(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), s.B, s.H, s.Lq, s.Lk, s.D,
                             True, -1.0, None, None, None)
    st = lib.launch_attn_forward_batch(arr, len(shapes), 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert st == 0
    torch.cuda.synchronize()
    for s, t, o in zip(shapes, ins, outs):
        assert torch.equal(o, attn.attn_forward(*t, causal=True))
        _check_oracle(s, *t, o, torch.float16, True)
    # an unsupported problem anywhere in the list: nothing is launched
    bad = (AttnProblem * 2)()
    bad[0] = arr[0]
    bad[1] = AttnProblem(ins[1][0].data_ptr(), ins[1][1].data_ptr(), ins[1][2].data_ptr(), outs[1].data_ptr(),
                         1, 8, 256, 900, 1000, False, -1.0, None, None, None)
    assert lib.launch_attn_forward_batch(bad, 2, 0, None) == 2  # ATTN_ERR_UNSUPPORTED


def test_short_problems_grouped_through_the_c_abi(attn):
    # 21 short problems (<= 16 queries) for the warp-level tensor-core kernel,
    # each with its own causal flag: 17 of one head dim and key-group count
    # (two grids, 16 + 1), three with 17-32 keys (another group), and one
    # whose K rows are 136 bytes apart, which the grouped kernel cannot stage
    # with 16-byte copies: it runs alone (general kernel).  Every output must
    # equal its own strided single call bit for bit, and meet the oracle.
    lib = ctypes.CDLL(attn.KERNEL_LIB_PATH)
    lib.launch_attn_forward_batch.argtypes = [ctypes.POINTER(AttnProblem), ctypes.c_int, ctypes.c_int,
                                              ctypes.c_void_p]
    lib.launch_attn_forward_batch.restype = ctypes.c_int
    lib.launch_attn_forward_strided.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [
        ctypes.c_bool, ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
        ctypes.c_void_p]
    lib.launch_attn_forward_strided.restype = ctypes.c_int
    shapes = [Shape(1 + i % 5, 1 + i % 3, 1 + i % 16, 1 + (5 * i) % 16, 64) for i in range(17)]
    shapes += [Shape(3, 2, 16, 17 + 5 * i, 64) for i in range(3)]
    shapes += [Shape(2, 3, 12, 16, 64)]
    causal = [i % 2 == 1 for i in range(len(shapes))]
    ins = _inputs(shapes, torch.float16, 21)
    # the last problem's K: rows of 68 elements in storage, 64 used
    s = shapes[-1]
    kpad = torch.zeros(s.B, s.H, s.Lk, 68, device="cuda", dtype=torch.float16)
    kpad[..., :64] = ins[-1][1]
    ins[-1] = (ins[-1][0], kpad[..., :64], ins[-1][2])
    strides = []
    for q, k, v in ins:
        strides.append(tuple((ctypes.c_longlong * 3)(*t.stride()[:3]) for t in (q, k, v)))
    outs = [torch.empty_like(t[0]) for t in ins]
    arr = (AttnProblem * len(shapes))()
    for i, (sh, (q, k, v), o, st) in enumerate(zip(shapes, ins, outs, strides)):
        arr[i] = AttnProblem(q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr(), sh.B, sh.H, sh.Lq, sh.Lk, sh.D,
                             causal[i], -1.0, ctypes.addressof(st[0]), ctypes.addressof(st[1]),
                             ctypes.addressof(st[2]))
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.launch_attn_forward_batch(arr, len(shapes), 0, stream) == 0
    singles = [torch.empty_like(t[0]) for t in ins]
    for i, (sh, (q, k, v), r, st) in enumerate(zip(shapes, ins, singles, strides)):
        assert lib.launch_attn_forward_strided(q.data_ptr(), k.data_ptr(), v.data_ptr(), r.data_ptr(), sh.B, sh.H,
                                               sh.Lq, sh.Lk, sh.D, causal[i], -1.0, 0, ctypes.addressof(st[0]),
                                               ctypes.addressof(st[1]), ctypes.addressof(st[2]), stream) == 0
    torch.cuda.synchronize()
    for i, (sh, o, r) in enumerate(zip(shapes, outs, singles)):
        assert torch.equal(o, r), f"problem {i} {sh} causal={causal[i]}: batched output differs from the single call"
    for i, (sh, (q, k, v), o) in enumerate(zip(shapes, ins, outs)):
        _check_oracle(sh, q, k.contiguous(), v, o, torch.float16, causal[i])
    assert attn.check_status(0) == 0
