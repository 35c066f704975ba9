"""The golden vectors of tests/golden through the CUDA path.

Each case holds inputs and the output of the reference's own code: its
``_sdpa_fallback`` (python/rocm_attn_op/__init__.py:7-26) on the fp32 upcast
of the inputs, written by tests/golden/make_golden.py.  The cases are seven
hot-path shapes (fp16/bf16, D = 64/128, self and cross attention, causal and
not, ragged tails), the seeded cases of the reference's Python test
(python/test/test_torch_interface.py:10-36, fp32, D = 16) and the ramp
known-answer case of its native test (src/tests/attn_test.cpp:52-60, fp32,
D = 4).  Each goes through ``rocm_attn_op.attn_forward`` on the GPU and is
compared with the reference output at the path's tolerances: max abs error
<= 2e-3 (fp16), 1e-2 (bf16), 1e-3 (fp32, the reference tests' own rtol=atol).
"""
import pytest
import torch

import oracle
from golden_util import cases, load

pytestmark = pytest.mark.gpu


def test_every_golden_case_is_listed():
    assert len(cases()) == 11, cases()


@pytest.mark.parametrize("name", cases())
def test_golden_case_through_cuda_path(attn, name):
    import rocm_attn_op

    g = load(name)
    q, k, v = (g[x].cuda() for x in ("q", "k", "v"))
    out = rocm_attn_op.attn_forward(q, k, v, causal=g["causal"])
    torch.cuda.synchronize()
    assert out.dtype == g["dtype"] and out.shape == q.shape
    ok, err = oracle.check(out, g["out_ref_fp32"], g["dtype"])
    assert ok, f"{name}: max abs err {err:.3e} against the reference output (tolerance {oracle.ATOL[g['dtype']]})"
    assert attn.check_status(0) == 0
