"""Generates the golden vectors in this folder from the reference itself.

Imports JoursBleu/rocm_attn's own Python package (python/rocm_attn_op) from
a checkout of the reference, with its compiled HIP extension replaced by an
empty stub module (the package only needs it for non-SDPA calls), and calls
the reference's ``_sdpa_fallback`` (python/rocm_attn_op/__init__.py:7-26) --
the code every fp16/bf16, D >= 64 call of the reference runs -- on CPU
tensors.  Each case stores the inputs (16-bit values as raw bits), the
reference output in the input dtype and the reference output on the fp32
upcast of the same inputs.

Also stores the reference's own test inputs: the seeded cases of
python/test/test_torch_interface.py:10-36 and the ramp known-answer case of
src/tests/attn_test.cpp:52-60.

    python tests/golden/make_golden.py [/path/to/reference]   (default: $ROCM_ATTN_REF)

Run once where the reference checkout exists; the .npz files are committed.
"""
import importlib
import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(ref_dir):
    stub = types.ModuleType("rocm_attn_op.rocm_attn_ext")
    sys.modules["rocm_attn_op.rocm_attn_ext"] = stub
    sys.path.insert(0, os.path.join(ref_dir, "python"))
    for name in [m for m in sys.modules if m == "rocm_attn_op"]:
        del sys.modules[name]
    mod = importlib.import_module("rocm_attn_op")
    assert os.path.abspath(mod.__file__).startswith(os.path.abspath(ref_dir)), mod.__file__
    return mod


def bits(t):
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.contiguous().view(torch.int16).numpy().view(np.uint16)
    return t.contiguous().numpy()


def main():
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
    import oracle
    ref_dir = sys.argv[1] if len(sys.argv) > 1 else oracle.reference_dir()
    if not ref_dir:
        raise SystemExit("usage: make_golden.py /path/to/reference (or set ROCM_ATTN_REF)")
    ref = load_reference(ref_dir)
    cases = []
    # hot-path cases: fp16/bf16, D in {64, 128}, self and cross, causal and not
    g = torch.Generator().manual_seed(20240601)
    hot = [("f16_d64_self", torch.float16, (1, 2, 64, 64, 64), False),
           ("f16_d64_self_causal", torch.float16, (1, 2, 64, 64, 64), True),
           ("f16_d128_tail_causal", torch.float16, (1, 2, 130, 130, 128), True),
           ("f16_d128_cross", torch.float16, (1, 1, 70, 200, 128), False),
           ("bf16_d64_cross", torch.bfloat16, (2, 1, 96, 160, 64), False),
           ("bf16_d128_self_causal", torch.bfloat16, (1, 1, 257, 257, 128), True),
           ("bf16_d64_tail", torch.bfloat16, (1, 3, 33, 33, 64), False)]
    for name, dt, (B, H, Lq, Lk, D), causal in hot:
        q = torch.randn(B, H, Lq, D, generator=g).to(dt)
        k = torch.randn(B, H, Lk, D, generator=g).to(dt)
        v = torch.randn(B, H, Lk, D, generator=g).to(dt)
        cases.append((name, q, k, v, causal))
    # the reference's own Python test inputs (fp32, D=16)
    torch.manual_seed(0)
    q = torch.randn(1, 2, 8, 16, dtype=torch.float32)
    k = torch.randn_like(q)
    v = torch.randn_like(q)
    cases.append(("reftest_self", q, k, v, False))
    cases.append(("reftest_self_causal", q, k, v, True))
    qx = torch.randn(1, 2, 6, 16, dtype=torch.float32)
    kx = torch.randn(1, 2, 9, 16, dtype=torch.float32)
    vx = torch.randn_like(kx)
    cases.append(("reftest_cross", qx, kx, vx, False))
    # the reference's native known-answer ramp (B=1,H=1,S=2,D=4)
    n = 8
    ramp = torch.arange(1, n + 1, dtype=torch.float32).view(1, 1, 2, 4)
    cases.append(("refkat_ramp", ramp * 0.01, ramp * 0.02, ramp * 0.03, False))

    for name, q, k, v, causal in cases:
        out_dt = ref._sdpa_fallback(q, k, v, causal)
        out_32 = ref._sdpa_fallback(q.float(), k.float(), v.float(), causal)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), q=bits(q), k=bits(k), v=bits(v),
                            dtype=str(q.dtype).replace("torch.", ""), causal=np.array(causal),
                            out_ref=bits(out_dt), out_ref_fp32=out_32.numpy())
        print("wrote", name, tuple(q.shape), tuple(k.shape), q.dtype, "causal" if causal else "")


if __name__ == "__main__":
    main()
