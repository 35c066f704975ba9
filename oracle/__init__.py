"""TEST INFRASTRUCTURE -- CPU oracles for the attention forward path.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs
(``cpu_baseline`` and ``--impl reference``) use this package, and only as the
checker or the timed CPU reference; the product path never imports it.

Three oracles, each citing what it restates from JoursBleu/rocm_attn:

* :func:`sdpa_math_fp32` -- torch ``scaled_dot_product_attention`` on the
  MATH backend, fp32, on the CPU.  This is the correctness oracle of the
  path: at every fp16/bf16, D >= 64 call the reference runs torch SDPA
  (python/rocm_attn_op/__init__.py:30-31 -> :7-26), and its Python test
  compares against SDPA (python/test/test_torch_interface.py:17-18,24,34).
* :func:`reference_sdpa_path` -- the reference's ``_sdpa_fallback``
  (python/rocm_attn_op/__init__.py:7-26) run on CPU tensors: FLASH backend
  first, then EFFICIENT, then default.  Timed as the CPU baseline.
* :func:`c_oracle_forward` -- ``attn_oracle.c``, a restatement of the
  reference's native CPU attention (src/tests/attn_test.cpp:10-49) extended
  with causal masking, Skv != Sq and an explicit scale, accumulated in double.

Parity is pinned by (a) the reference's own known-answer test
(src/tests/attn_test.cpp:51-98) compiled from its sources against the C
oracle (``_ref/attn_test_kat``, see Makefile), and (b) golden vectors that
``tests/golden/make_golden.py`` produced by importing the reference's own
``rocm_attn_op`` package and calling its ``_sdpa_fallback``.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))
C_ORACLE_LIB = os.path.join(HERE, "libattn_oracle.so")
REF_KAT_BIN = os.path.join(HERE, "_ref", "attn_test_kat")

# Pass criteria of the path: max |O - O_ref| (north_star tolerances).
ATOL = {torch.float16: 2e-3, torch.bfloat16: 1e-2, torch.float32: 1e-3}


def reference_dir() -> Optional[str]:
    """Checkout of the reference's sources, if one is present: the directory
    named by the ROCM_ATTN_REF environment variable, else a ``reference``
    directory beside this repository.  None when neither exists."""
    cand = os.environ.get("ROCM_ATTN_REF") or os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference")
    return cand if os.path.isfile(os.path.join(cand, "src", "tests", "attn_test.cpp")) else None


def build(ref_dir: Optional[str] = None) -> None:
    """Compile the C oracle and, when the reference sources are present
    (``ref_dir``, else :func:`reference_dir`), the reference's known-answer
    test against it (outputs stay in oracle/)."""
    ref = ref_dir or reference_dir() or ""
    subprocess.run(["make", "-s", "-C", HERE, f"REF={ref}"], check=True)


_lib = None


def _c_lib():
    global _lib
    if _lib is None:
        if not os.path.exists(C_ORACLE_LIB):
            build()
        lib = ctypes.CDLL(C_ORACLE_LIB)
        fp = ctypes.POINTER(ctypes.c_float)
        lib.attn_oracle_rows.argtypes = [fp, fp, fp, fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                         ctypes.c_int, ctypes.c_int, ctypes.c_float, ctypes.c_longlong,
                                         ctypes.c_longlong]
        lib.attn_oracle_rows.restype = None
        _lib = lib
    return _lib


def c_oracle_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                     scale: Optional[float] = None, threads: Optional[int] = None) -> torch.Tensor:
    """Naive three-pass attention in double precision (attn_oracle.c).
    Inputs are upcast to fp32 on the CPU; returns an fp32 CPU tensor."""
    lib = _c_lib()
    qf = q.detach().to("cpu", torch.float32).contiguous()
    kf = k.detach().to("cpu", torch.float32).contiguous()
    vf = v.detach().to("cpu", torch.float32).contiguous()
    B, H, Sq, D = qf.shape
    Skv = kf.shape[2]
    out = torch.empty_like(qf)
    fp = ctypes.POINTER(ctypes.c_float)
    args = [ctypes.cast(t.data_ptr(), fp) for t in (qf, kf, vf, out)]
    total = B * H * Sq
    n = max(1, min(threads or os.cpu_count() or 1, total))
    bounds = [total * i // n for i in range(n + 1)]
    sc = 0.0 if scale is None else float(scale)

    def run(i):
        lib.attn_oracle_rows(*args, B, H, Sq, Skv, D, int(bool(causal)), sc, bounds[i], bounds[i + 1])

    if n == 1:
        run(0)
    else:  # ctypes releases the GIL for the duration of each call
        with ThreadPoolExecutor(n) as ex:
            list(ex.map(run, range(n)))
    return out


def sdpa_math_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                   scale: Optional[float] = None) -> torch.Tensor:
    """torch SDPA, MATH backend, fp32, CPU.  Inputs are the dtype-rounded
    values the GPU sees, upcast to fp32.  Returns an fp32 CPU tensor."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    qf = q.detach().to("cpu", torch.float32)
    kf = k.detach().to("cpu", torch.float32)
    vf = v.detach().to("cpu", torch.float32)
    if kf.shape[2] == 0:
        return torch.zeros_like(qf)
    with sdpa_kernel(SDPBackend.MATH):
        return F.scaled_dot_product_attention(qf, kf, vf, attn_mask=None, dropout_p=0.0, is_causal=bool(causal),
                                              scale=scale)


def sdpa_rows_fp32(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, rows, causal: bool = False,
                   scale: Optional[float] = None) -> torch.Tensor:
    """:func:`sdpa_math_fp32` for the query rows ``rows`` (absolute row
    indices, the same for every (b, h)) only: the causal rule keeps key j for
    query row i when j <= i, as for the full problem.  Returns an fp32 CPU
    tensor [B, H, len(rows), D]."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    idx = torch.as_tensor(list(rows), dtype=torch.long)
    qf = q.detach().to("cpu", torch.float32)[:, :, idx]
    kf = k.detach().to("cpu", torch.float32)
    vf = v.detach().to("cpu", torch.float32)
    if kf.shape[2] == 0:
        return torch.zeros_like(qf)
    mask = None
    if causal:
        mask = torch.arange(kf.shape[2])[None, :] <= idx[:, None]
    with sdpa_kernel(SDPBackend.MATH):
        return F.scaled_dot_product_attention(qf, kf, vf, attn_mask=mask, dropout_p=0.0, scale=scale)


def reference_sdpa_path(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False) -> torch.Tensor:
    """The reference's ``_sdpa_fallback`` (python/rocm_attn_op/__init__.py:7-26)
    restated for CPU tensors: FLASH backend, else EFFICIENT, else default."""
    from torch.nn.attention import SDPBackend, sdpa_kernel

    def call():
        return F.scaled_dot_product_attention(q, k, v, attn_mask=None, dropout_p=0.0, is_causal=bool(causal))

    try:
        with sdpa_kernel(SDPBackend.FLASH_ATTENTION):
            return call()
    except Exception:
        try:
            with sdpa_kernel(SDPBackend.EFFICIENT_ATTENTION):
                return call()
        except Exception:
            return call()


def max_abs_err(out: torch.Tensor, ref: torch.Tensor) -> float:
    d = (out.detach().to("cpu", torch.float32) - ref.detach().to("cpu", torch.float32)).abs()
    return float(d.max()) if d.numel() else 0.0


# Half-ulp relative rounding error of the 16-bit types (11 and 8 significant bits).
HALF_ULP = {torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8, torch.float32: 2.0 ** -24}


def check(out: torch.Tensor, ref: torch.Tensor, dtype: torch.dtype, output_rounding_slack: bool = False,
          v_absmax: Optional[float] = None) -> tuple[bool, float]:
    """North-star pass criterion: finite output and max abs error <= ATOL[dtype].

    Stress inputs (a nearly one-hot softmax, |O| of a few units) get two
    further terms, both rounding errors any 16-bit flash-attention kernel has:
    ``output_rounding_slack`` adds the error of rounding the exact result
    itself to ``dtype``; ``v_absmax`` adds the effect of holding the
    probabilities P in ``dtype`` for the P*V product, at most
    half-ulp(dtype) * max|V| (sum_j |P~_j - p_j| |v_j| / sum_j p_j)."""
    o = out.detach().to("cpu", torch.float32)
    r = ref.detach().to("cpu", torch.float32)
    finite = bool(torch.isfinite(o).all())
    err = max_abs_err(o, r)
    bound = ATOL[dtype]
    if output_rounding_slack and r.numel():
        bound += float((r.to(dtype).float() - r).abs().max())
    if v_absmax is not None:
        bound += HALF_ULP[dtype] * float(v_absmax)
    return finite and err <= bound, err


def run_reference_kat() -> tuple[bool, str]:
    """Run the reference's known-answer test linked against the C oracle."""
    if not os.path.exists(REF_KAT_BIN):
        return False, "not built"
    r = subprocess.run([REF_KAT_BIN], capture_output=True, text=True)
    return r.returncode == 0 and "PASSED" in r.stdout, r.stdout.strip()


__all__ = ["ATOL", "HALF_ULP", "build", "reference_dir", "c_oracle_forward", "sdpa_math_fp32", "sdpa_rows_fp32", "reference_sdpa_path", "max_abs_err", "check",
           "run_reference_kat"]
