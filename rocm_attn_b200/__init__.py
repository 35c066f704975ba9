"""B200-native fused attention forward.

Python surface of the operator, mirroring ``rocm_attn_op.attn_forward`` of
JoursBleu/rocm_attn (python/rocm_attn_op/__init__.py:29-32).  The reference
sends fp16/bf16 CUDA calls with D >= 64 to torch SDPA
(python/rocm_attn_op/__init__.py:7-26,30-31); here every call goes to the
hand-written sm_100a kernel in ``librocm_attn.so`` through the PyTorch binding
``rocm_attn_ext``.  There is no fallback: when the native extension is absent
the import fails loudly.
"""
from __future__ import annotations

import importlib.util
import os
import sysconfig
from typing import Optional, Sequence

import torch

_PKG_DIR = os.path.dirname(os.path.abspath(__file__))
KERNEL_LIB_PATH = os.path.join(_PKG_DIR, "librocm_attn.so")


def _load_ext():
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    path = os.path.join(_PKG_DIR, "rocm_attn_ext" + suffix)
    if not os.path.exists(path) or not os.path.exists(KERNEL_LIB_PATH):
        raise ImportError(
            "rocm_attn_b200: native extension not built (expected %s and %s); "
            "run `python rocm_attn_b200/build.py`" % (path, KERNEL_LIB_PATH))
    spec = importlib.util.spec_from_file_location(__name__ + ".rocm_attn_ext", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


rocm_attn_ext = _load_ext()

# Head dims and dtypes of the tcgen05 tensor-core kernel; every other call
# with 1 <= D <= MAX_HEAD_DIM (and fp32 at any such D) runs the general
# fp32-arithmetic kernel.
SUPPORTED_HEAD_DIMS = (64, 128)
SUPPORTED_DTYPES = (torch.float16, torch.bfloat16)
MAX_HEAD_DIM = 256


def attn_forward(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, causal: bool = False,
                 scale: Optional[float] = None) -> torch.Tensor:
    """Scaled dot-product attention forward.

    q: [B, H, Lq, D], k/v: [B, H, Lk, D], fp16, bf16 or fp32 CUDA tensors,
    1 <= D <= 256.  fp16/bf16 with D in {64, 128} run the tcgen05
    tensor-core kernel; other calls run the general kernel (fp32 math).
    ``causal`` masks key j for query i when j > i (top-left aligned, as torch
    SDPA ``is_causal=True``).  ``scale`` defaults to 1/sqrt(D).  Returns O
    [B, H, Lq, D] in q's dtype.
    """
    return rocm_attn_ext.attn_forward(q, k, v, bool(causal), -1.0 if scale is None else float(scale))


def attn_forward_batch(qs: Sequence[torch.Tensor], ks: Sequence[torch.Tensor], vs: Sequence[torch.Tensor],
                       causal: bool = False, scale: Optional[float] = None) -> list:
    """Several independent attention problems (e.g. a sequence of shapes) in
    one call: returns ``[attn_forward(q, k, v, causal, scale) for ...]``, the
    same values bit for bit, with the problems that run the tcgen05 kernel at
    the same head dim and tile shape sharing one grid (longest units first),
    so they pay one launch and one partial last wave instead of one each.
    All problems share dtype, device, ``causal`` and ``scale``."""
    return list(rocm_attn_ext.attn_forward_batch(list(qs), list(ks), list(vs), bool(causal),
                                                 -1.0 if scale is None else float(scale)))


def check_status(device: int = 0) -> int:
    """Synchronise ``device`` and return (and clear) the kernel watchdog
    status: 0 when every earlier launch completed, non-zero when a kernel gave
    up on a wait (its output is then invalid)."""
    return int(rocm_attn_ext.check_status(int(device)))


from .pipeline import attn_forward_pinned  # noqa: E402  (host-resident inputs, transfers overlapped)

__all__ = ["attn_forward", "attn_forward_batch", "attn_forward_pinned", "check_status", "rocm_attn_ext", "KERNEL_LIB_PATH",
           "SUPPORTED_HEAD_DIMS", "SUPPORTED_DTYPES", "MAX_HEAD_DIM"]
