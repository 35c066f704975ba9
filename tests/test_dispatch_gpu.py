"""Seeded random shapes around the dispatcher's boundaries, against the oracle.

The dispatcher picks a kernel from (dtype, D, Sq, Skv, causal, grid size):
the short-sequence kernels (Sq <= 16 / 32, Skv <= 64), the mid-length
warp-level kernel (D = 16 / 32, or D = 64 with Sq <= 64 and Skv <= 256), the
tcgen05 kernel (D = 64 with 64- or 128-key blocks, D = 128) and the general
kernel (fp32, other head dims).  These cases draw sizes on both sides of
every limit so that each route and its tails are exercised.
"""
import random

import pytest
import torch

import oracle
from rocm_attn_b200.workloads import Shape, make_qkv

pytestmark = pytest.mark.gpu

_EDGES_Q = [1, 15, 16, 17, 31, 33, 63, 64, 65, 127, 128, 129, 200, 255, 257, 383]
_EDGES_K = [1, 15, 16, 63, 64, 65, 93, 128, 255, 256, 257, 351, 384, 385, 700]
DT = {"fp16": torch.float16, "bf16": torch.bfloat16, "fp32": torch.float32}


def _cases(n=48, seed=20251202):
    rng = random.Random(seed)
    out = []
    for _ in range(n):
        D = rng.choice([16, 32, 48, 64, 64, 64, 128, 128])
        dtype = rng.choice(["fp16", "bf16", "fp16", "bf16", "fp32"])
        Lq, Lk = rng.choice(_EDGES_Q), rng.choice(_EDGES_K)
        causal = rng.random() < 0.5
        # enough (batch, head) slices for some cases to pass the grid-size
        # limit of the 64-key blocks (two CTAs per SM), few for others
        BH = rng.choice([1, 3, 8, 40, 320])
        B = rng.choice([b for b in (1, 2, 4, 8) if BH % b == 0])
        out.append(pytest.param(Shape(B, BH // B, Lq, Lk, D), dtype, causal,
                                id=f"{B}x{BH // B}x{Lq}x{Lk}x{D}-{dtype}-{'c' if causal else 'n'}"))
    return out


@pytest.mark.parametrize("shape,dtype,causal", _cases())
def test_random_dispatch_boundaries(attn, shape, dtype, causal):
    q, k, v = make_qkv(shape, DT[dtype], seed=shape.Lq * 7 + shape.Lk)
    out = attn.attn_forward(q.cuda(), k.cuda(), v.cuda(), causal=causal)
    torch.cuda.synchronize()
    assert out.shape == q.shape and out.dtype == q.dtype
    ref = oracle.sdpa_math_fp32(q, k, v, causal=causal)
    ok, err = oracle.check(out, ref, DT[dtype])
    assert ok, f"{shape} {dtype} causal={causal}: max abs err {err:.3e}"
