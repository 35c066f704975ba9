"""Drop-in package name of JoursBleu/rocm_attn's operator.

``from rocm_attn_op import attn_forward`` and
``from rocm_attn_op import rocm_attn_ext`` keep working for callers of the
reference (python/rocm_attn_op/__init__.py:29, setup.py:62,68); both resolve
to the sm_100a implementation in ``rocm_attn_b200``.
"""
import sys as _sys

from rocm_attn_b200 import attn_forward, attn_forward_batch, check_status, rocm_attn_ext

_sys.modules[__name__ + ".rocm_attn_ext"] = rocm_attn_ext

__all__ = ["attn_forward", "attn_forward_batch", "check_status", "rocm_attn_ext"]
