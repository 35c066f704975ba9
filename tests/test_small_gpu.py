"""The short-sequence kernel (Sq <= 32, Skv <= 64: one warp per (batch, head)
slice), against the CPU oracle, including the reference's UnifoLM inference
shapes with 16-row sequences (benchmark/attn_shapes_unifolm_infer.txt:1-9)."""
import pytest
import torch

import oracle
from rocm_attn_b200.workloads import Shape, WORKLOADS, make_qkv

pytestmark = pytest.mark.gpu


def _check(attn, shape, dtype, causal, seed=0, heads=None):
    q, k, v = make_qkv(shape, dtype, seed=seed)
    out = attn.attn_forward(q.cuda(), k.cuda(), v.cuda(), causal=causal).cpu()
    assert out.shape == q.shape and torch.isfinite(out.float()).all()
    if heads is None:
        ref = oracle.sdpa_math_fp32(q, k, v, causal=causal)
        ok, err = oracle.check(out, ref, dtype)
    else:
        qf, kf, vf, of = (t.reshape(-1, 1, *t.shape[2:]) for t in (q, k, v, out))
        ref = oracle.sdpa_math_fp32(qf[heads], kf[heads], vf[heads], causal=causal)
        ok, err = oracle.check(of[heads], ref, dtype)
    assert ok, f"{shape} {dtype} causal={causal}: max abs err {err:.3e}"


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("sq,skv,d", [(1, 1, 64), (5, 7, 16), (16, 16, 64), (16, 16, 128), (16, 64, 128),
                                      (17, 3, 64), (32, 32, 32), (32, 64, 64), (8, 40, 96), (24, 9, 48)])
def test_small_shapes(attn, sq, skv, d, causal, dtype):
    _check(attn, Shape(3, 5, sq, skv, d), dtype, causal, seed=sq * 100 + skv)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("sq,skv", [(1, 64), (8, 40), (8, 17), (8, 16), (3, 64)])
def test_fp32_d128_decode_shapes(attn, sq, skv, causal):
    # fp32 at D = 128 with 17-64 keys: the SIMT short kernel's fp32 K and V would
    # need 256 KiB of shared memory, so the dispatcher sends these to the
    # general kernel; with up to 16 keys the SIMT kernel takes them.
    _check(attn, Shape(2, 3, sq, skv, 128), torch.float32, causal, seed=sq * 1000 + skv)


@pytest.mark.parametrize("idx", [0, 2, 4, 6, 8])
def test_unifolm_short_shapes(attn, idx):
    s = WORKLOADS["unifolm"].shapes[idx]
    assert s.Lq == 16 and s.Lk == 16
    _check(attn, s, torch.float16, False, seed=idx, heads=[0, 1, s.bh // 2, s.bh - 1])


def test_small_strided_and_broadcast(attn):
    s = Shape(64, 8, 16, 16, 64)
    q, k, v = (t.cuda() for t in make_qkv(s, torch.float16, seed=3))
    qb, kb, vb = (t.transpose(1, 2).contiguous().transpose(1, 2) for t in (q, k, v))
    a = attn.attn_forward(q, k, v)
    b = attn.attn_forward(qb, kb, vb)
    assert torch.equal(a, b)
    kx, vx = k[:, :1].expand(-1, 8, -1, -1), v[:, :1].expand(-1, 8, -1, -1)
    out = attn.attn_forward(q, kx, vx, causal=True).cpu()
    ref = oracle.sdpa_math_fp32(q.cpu(), kx.cpu().contiguous(), vx.cpu().contiguous(), causal=True)
    ok, err = oracle.check(out, ref, torch.float16)
    assert ok, err
