"""The C-ABI library and the bindings, without a GPU.

Loads librocm_attn.so, checks that it exports every entry point
include/attn_kernel.h declares, and exercises the argument checks that run
before any CUDA call (so nothing here launches or allocates on a device).
"""
import ctypes
import os
import re

import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(REPO, "include", "attn_kernel.h")
LIB = os.path.join(REPO, "rocm_attn_b200", "librocm_attn.so")

ATTN_OK, ATTN_ERR_INVALID_ARGUMENT, ATTN_ERR_UNSUPPORTED, ATTN_ERR_MISALIGNED = 0, 1, 2, 3


def declared_symbols():
    text = open(HEADER).read()
    # return types may be several words ("unsigned long long")
    return re.findall(r"ATTN_API\s+(?:\w+\s+)+?\**(\w+)\s*\(", text)


@pytest.fixture(scope="module")
def lib():
    assert os.path.exists(LIB), "librocm_attn.so not built (run __graft_entry__.build())"
    lib = ctypes.CDLL(LIB)
    lib.launch_attn_forward.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [
        ctypes.c_bool, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    lib.launch_attn_forward.restype = ctypes.c_int
    lib.attn_get_status.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    lib.attn_get_status.restype = ctypes.c_int
    return lib


def test_header_declares_entry_points():
    syms = declared_symbols()
    assert "launch_attn_forward" in syms and "attn_get_status" in syms and "attn_library_version" in syms


def test_library_exports_every_declared_symbol(lib):
    for name in declared_symbols():
        assert hasattr(lib, name), f"{name} declared in attn_kernel.h but not exported"


def test_dtype_enum_matches_reference_values():
    # reference src/attn_kernel.h:12-16: ATTN_F16=0, ATTN_BF16=1, ATTN_F32=2
    text = open(HEADER).read()
    assert re.search(r"ATTN_F16\s*=\s*0", text) and re.search(r"ATTN_BF16\s*=\s*1", text)
    assert re.search(r"ATTN_F32\s*=\s*2", text)


def test_version(lib):
    assert lib.attn_library_version() == 200


def test_wait_limit_setter_round_trips(lib):
    # a host-side setting only: no CUDA call, nothing launched
    lib.attn_set_wait_limit_ns.argtypes = [ctypes.c_ulonglong]
    lib.attn_set_wait_limit_ns.restype = ctypes.c_ulonglong
    assert lib.attn_set_wait_limit_ns(12345) == 0
    assert lib.attn_set_wait_limit_ns(0) == 12345
    assert lib.attn_set_wait_limit_ns(0) == 0


def _call(lib, q=0x1000, k=0x1000, v=0x1000, o=0x1000, B=1, H=1, Sq=8, Skv=8, D=64, causal=False, scale=-1.0,
          dtype=0):
    return lib.launch_attn_forward(q, k, v, o, B, H, Sq, Skv, D, causal, scale, dtype, None)


def test_argument_checks_before_any_cuda_call(lib):
    # Every call here fails (or finishes) before the device is touched; the
    # pointers are fake.
    assert _call(lib, D=257) == ATTN_ERR_UNSUPPORTED            # general kernel takes D <= 256
    assert _call(lib, D=1000) == ATTN_ERR_UNSUPPORTED
    assert _call(lib, dtype=7) == ATTN_ERR_UNSUPPORTED
    assert _call(lib, D=0) == ATTN_ERR_INVALID_ARGUMENT
    assert _call(lib, B=-1) == ATTN_ERR_INVALID_ARGUMENT
    assert _call(lib, Sq=-3) == ATTN_ERR_INVALID_ARGUMENT
    assert _call(lib, q=None) == ATTN_ERR_INVALID_ARGUMENT
    assert _call(lib, o=None) == ATTN_ERR_INVALID_ARGUMENT
    assert _call(lib, q=0x1001) == ATTN_ERR_MISALIGNED          # not aligned to the 2-byte element
    assert _call(lib, v=0x1003, dtype=1) == ATTN_ERR_MISALIGNED
    assert _call(lib, k=0x1002, dtype=2) == ATTN_ERR_MISALIGNED  # fp32 needs 4-byte alignment
    # empty problems are a successful no-op
    assert _call(lib, B=0) == ATTN_OK
    assert _call(lib, Sq=0) == ATTN_OK


class _AttnProblem(ctypes.Structure):
    _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("B", ctypes.c_int), ("H", ctypes.c_int), ("Sq", ctypes.c_int), ("Skv", ctypes.c_int),
                ("D", ctypes.c_int), ("causal", ctypes.c_bool), ("softmax_scale", ctypes.c_float),
                ("q_strides", ctypes.c_void_p), ("k_strides", ctypes.c_void_p), ("v_strides", ctypes.c_void_p)]


def test_batch_argument_checks_before_any_cuda_call(lib):
    # The batch entry checks every problem before launching any; these fail
    # (or finish) before the device is touched.  The pointers are fake.
    lib.launch_attn_forward_batch.argtypes = [ctypes.POINTER(_AttnProblem), ctypes.c_int, ctypes.c_int,
                                              ctypes.c_void_p]
    lib.launch_attn_forward_batch.restype = ctypes.c_int
    good = _AttnProblem(0x1000, 0x1000, 0x1000, 0x1000, 0, 1, 8, 8, 64, False, -1.0, None, None, None)  # empty
    bad_d = _AttnProblem(0x1000, 0x1000, 0x1000, 0x1000, 1, 1, 8, 8, 1000, False, -1.0, None, None, None)
    bad_ptr = _AttnProblem(None, 0x1000, 0x1000, 0x1000, 1, 1, 8, 8, 64, False, -1.0, None, None, None)
    arr = (_AttnProblem * 3)(good, bad_d, good)
    assert lib.launch_attn_forward_batch(arr, 3, 0, None) == ATTN_ERR_UNSUPPORTED
    arr = (_AttnProblem * 2)(good, bad_ptr)
    assert lib.launch_attn_forward_batch(arr, 2, 0, None) == ATTN_ERR_INVALID_ARGUMENT
    assert lib.launch_attn_forward_batch(None, 1, 0, None) == ATTN_ERR_INVALID_ARGUMENT
    assert lib.launch_attn_forward_batch(None, -1, 0, None) == ATTN_ERR_INVALID_ARGUMENT
    assert lib.launch_attn_forward_batch(None, 0, 0, None) == ATTN_OK
    arr = (_AttnProblem * 2)(good, good)
    assert lib.launch_attn_forward_batch(arr, 2, 0, None) == ATTN_OK  # only empty problems
    assert lib.launch_attn_forward_batch(arr, 2, 9, None) == ATTN_ERR_UNSUPPORTED  # unknown dtype


def test_status_requires_output_pointer(lib):
    assert lib.attn_get_status(None, None) == ATTN_ERR_INVALID_ARGUMENT


def test_bindings_load_and_check_devices():
    import rocm_attn_op
    import rocm_attn_b200

    assert rocm_attn_op.attn_forward is rocm_attn_b200.attn_forward
    import rocm_attn_op.rocm_attn_ext as ext  # the reference's module path keeps working
    assert ext.library_version() == 200
    x = torch.zeros(1, 1, 8, 64, dtype=torch.float16)
    with pytest.raises(RuntimeError, match="CUDA"):
        rocm_attn_op.attn_forward(x, x, x)
    with pytest.raises(RuntimeError, match="CUDA"):
        rocm_attn_op.rocm_attn_ext.attn_forward(x, x, x, False)


def test_product_path_does_not_import_oracle():
    for root, _, files in os.walk(os.path.join(REPO, "rocm_attn_b200")):
        for f in files:
            if f.endswith((".py", ".cpp", ".cu", ".cuh", ".h")):
                text = open(os.path.join(root, f)).read()
                assert "import oracle" not in text and "from oracle" not in text, f
