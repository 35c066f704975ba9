"""The kernel watchdog, made to fire on purpose without faulting anything.

Every wait inside the tensor-core kernel's pipeline is bounded: when a wait
runs past its limit the kernel records ATTN_ERR_WATCHDOG in the device status
word, lets the copies and products it already issued land (under the default
2 s bound), frees its tensor memory and returns.  A legitimate wait ends
inside the hardware's own suspension of ``mbarrier.try_wait``, so the limit
only ever expires when an arrival is lost.

This test loses one on purpose.  ``librocm_attn_wdtest.so`` is the library
built from the same sources with RA_WATCHDOG_TEST (rocm_attn_b200/build.py);
after ``attn_test_drop_arrival(1)`` its launches skip one P-ready arrival in
CTA 0 (a flag nothing else sets), so the MMA warp's wait for it can only end by
the watchdog.  The limit is lowered to 1 ms for that launch.  The test then
checks, through the C ABI: the launch returned and the stream synchronises,
the status reports the watchdog, reading the status cleared it, and a
following launch with nothing dropped is correct and clean.  The product
library is not the one loaded here; it has no way to drop an arrival.
"""
import ctypes
import os

import pytest
import torch

import oracle
from rocm_attn_b200.workloads import Shape, make_qkv

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
WDTEST_LIB = os.path.join(REPO, "rocm_attn_b200", "librocm_attn_wdtest.so")
ATTN_OK, ATTN_ERR_WATCHDOG = 0, 7
DTYPE_CODE = {torch.float16: 0, torch.bfloat16: 1}


@pytest.fixture(scope="module")
def wdlib():
    assert os.path.exists(WDTEST_LIB), "librocm_attn_wdtest.so not built (run __graft_entry__.build())"
    lib = ctypes.CDLL(WDTEST_LIB)
    lib.launch_attn_forward.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [
        ctypes.c_bool, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    lib.launch_attn_forward.restype = ctypes.c_int
    lib.attn_get_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    lib.attn_get_status.restype = ctypes.c_int
    lib.attn_set_wait_limit_ns.argtypes = [ctypes.c_ulonglong]
    lib.attn_set_wait_limit_ns.restype = ctypes.c_ulonglong
    lib.attn_test_drop_arrival.argtypes = [ctypes.c_int]
    lib.attn_test_drop_arrival.restype = None
    yield lib
    lib.attn_test_drop_arrival(0)
    lib.attn_set_wait_limit_ns(0)


def _stream():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def _launch(lib, q, k, v, out, causal):
    B, H, Sq, D = q.shape
    st = lib.launch_attn_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), B, H, Sq, k.shape[2], D,
                                 causal, -1.0, DTYPE_CODE[q.dtype], _stream())
    assert st == ATTN_OK, f"launch status {st}"


def _status(lib):
    s = ctypes.c_int(-1)
    assert lib.attn_get_status(_stream(), ctypes.byref(s)) == ATTN_OK
    return s.value


@pytest.mark.parametrize("shape,dtype,causal", [
    (Shape(1, 4, 1024, 1024, 128), torch.float16, False),   # two-tile D=128 CTAs
    (Shape(1, 2, 200, 100, 128), torch.bfloat16, True),     # one key block per CTA
    (Shape(2, 4, 1024, 1024, 64), torch.bfloat16, True),    # one-tile D=64 CTAs, 128-key blocks
    (Shape(64, 8, 256, 256, 64), torch.float16, False),     # one-tile D=64 CTAs, 64-key blocks
])
def test_watchdog_fires_and_recovers(wdlib, shape, dtype, causal):
    q, k, v = (t.cuda() for t in make_qkv(shape, dtype, seed=5))
    out = torch.empty_like(q)
    assert _status(wdlib) == ATTN_OK
    wdlib.attn_set_wait_limit_ns(1_000_000)
    wdlib.attn_test_drop_arrival(1)
    try:
        _launch(wdlib, q, k, v, out, causal)
        torch.cuda.synchronize()
    finally:
        wdlib.attn_test_drop_arrival(0)
        wdlib.attn_set_wait_limit_ns(0)
    assert _status(wdlib) == ATTN_ERR_WATCHDOG
    assert _status(wdlib) == ATTN_OK  # reading the status cleared it
    _launch(wdlib, q, k, v, out, causal)
    torch.cuda.synchronize()
    assert _status(wdlib) == ATTN_OK
    heads = [0, shape.bh - 1]
    qf, kf, vf, of = (t.reshape(-1, 1, *t.shape[2:]).cpu() for t in (q, k, v, out))
    ok, err = oracle.check(of[heads], oracle.sdpa_math_fp32(qf[heads], kf[heads], vf[heads], causal=causal), dtype)
    assert ok, f"after the watchdog: max abs err {err:.3e}"


def test_product_library_cannot_drop_arrivals():
    import rocm_attn_b200
    lib = ctypes.CDLL(rocm_attn_b200.KERNEL_LIB_PATH)
    assert not hasattr(lib, "attn_test_drop_arrival")
