"""The oracle, pinned against the reference (CPU only).

* the reference's own known-answer test (src/tests/attn_test.cpp:51-98),
  compiled from its sources against the C oracle, passes;
* both oracles reproduce the golden vectors that the reference's own
  ``_sdpa_fallback`` produced (tests/golden/make_golden.py);
* the C oracle and torch SDPA math agree on random shapes, causal and cross;
* the checker rejects planted mistakes.
"""
import math
import os

import numpy as np
import pytest
import torch

import oracle
from golden_util import cases, load

def test_reference_known_answer_test():
    if not os.path.exists(oracle.REF_KAT_BIN):
        if not oracle.reference_dir():
            pytest.skip("reference sources absent and the known-answer binary was not built")
        oracle.build()
    ok, out = oracle.run_reference_kat()
    assert ok, out


def test_ramp_known_answer_values():
    # src/tests/attn_test.cpp:52-60: q=0.01(i+1), k=0.02(i+1), v=0.03(i+1)
    i = torch.arange(1, 9, dtype=torch.float32).view(1, 1, 2, 4)
    q, k, v = 0.01 * i, 0.02 * i, 0.03 * i
    out = oracle.c_oracle_forward(q, k, v)
    qd, kd, vd = (t.double().view(2, 4).numpy() for t in (q, k, v))
    s = qd @ kd.T / 2.0
    p = np.exp(s - s.max(1, keepdims=True))
    exp = (p / p.sum(1, keepdims=True)) @ vd
    assert np.abs(out.view(2, 4).numpy() - exp).max() < 1e-6


@pytest.mark.parametrize("name", cases())
def test_oracles_reproduce_reference_golden(name):
    g = load(name)
    for fn in (oracle.sdpa_math_fp32, oracle.c_oracle_forward):
        out = fn(g["q"], g["k"], g["v"], causal=g["causal"])
        # fp32 reference path on the same upcast inputs: agreement to fp32 noise
        assert oracle.max_abs_err(out, g["out_ref_fp32"]) < 2e-5, fn.__name__
        # reference output in the input dtype: within the path's tolerance
        ok, err = oracle.check(g["out_ref"], out, g["dtype"])
        assert ok, f"{fn.__name__}: {err}"


@pytest.mark.parametrize("D", [4, 16, 64, 128])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("lq,lk", [(1, 1), (7, 7), (33, 50), (50, 33), (129, 129)])
def test_c_oracle_matches_sdpa_math(D, causal, lq, lk):
    g = torch.Generator().manual_seed(D * 1000 + lq * 10 + lk)
    q = torch.randn(2, 3, lq, D, generator=g)
    k = torch.randn(2, 3, lk, D, generator=g)
    v = torch.randn(2, 3, lk, D, generator=g)
    a = oracle.c_oracle_forward(q, k, v, causal=causal)
    b = oracle.sdpa_math_fp32(q, k, v, causal=causal)
    assert oracle.max_abs_err(a, b) < 2e-5


def test_explicit_scale_and_empty_keys():
    g = torch.Generator().manual_seed(5)
    q = torch.randn(1, 2, 9, 64, generator=g)
    k = torch.randn(1, 2, 11, 64, generator=g)
    v = torch.randn(1, 2, 11, 64, generator=g)
    for sc in (0.1, 0.5, 1.0 / math.sqrt(64)):
        assert oracle.max_abs_err(oracle.c_oracle_forward(q, k, v, scale=sc),
                                  oracle.sdpa_math_fp32(q, k, v, scale=sc)) < 2e-5
    empty = torch.zeros(1, 2, 0, 64)
    # reference rule: an empty denominator gives 0 (src/attn_kernel_torch.cu:335-336)
    assert torch.count_nonzero(oracle.c_oracle_forward(q, empty, empty)) == 0
    assert torch.count_nonzero(oracle.sdpa_math_fp32(q, empty, empty)) == 0


def test_checker_rejects_planted_mistakes():
    g = torch.Generator().manual_seed(9)
    q, k, v = (torch.randn(1, 2, 40, 64, generator=g).half() for _ in range(3))
    ref = oracle.sdpa_math_fp32(q, k, v)
    good = ref.half()
    assert oracle.check(good, ref, torch.float16)[0]
    bad = good.clone()
    bad[0, 1, 17, 5] += 0.01          # one wrong element
    assert not oracle.check(bad, ref, torch.float16)[0]
    nan = good.clone()
    nan[0, 0, 0, 0] = float("nan")    # a non-finite value
    assert not oracle.check(nan, ref, torch.float16)[0]
    # a wrong mask (causal result checked against the non-causal oracle)
    wrong_mask = oracle.sdpa_math_fp32(q, k, v, causal=True).half()
    assert not oracle.check(wrong_mask, ref, torch.float16)[0]


def test_reference_sdpa_path_matches_oracle():
    g = torch.Generator().manual_seed(3)
    q, k, v = (torch.randn(1, 2, 100, 128, generator=g) for _ in range(3))
    for causal in (False, True):
        assert oracle.max_abs_err(oracle.reference_sdpa_path(q, k, v, causal),
                                  oracle.sdpa_math_fp32(q, k, v, causal)) < 2e-5
