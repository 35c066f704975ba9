"""Several host threads calling the C ABI at once, each on its own stream.

The launcher keeps per-device state that is set up on first use (shared-memory
opt-ins, attribute and tensor-map entry-point lookups), and the boundary
promises that it is safe to call from several host threads.  The check runs in
a fresh interpreter, so those first uses really race: eight threads start
together (a barrier) and call ``launch_attn_forward`` / the batch entry point
through ctypes, which releases the GIL for the call, on problems that take
every kernel family.  Each thread's outputs must equal, bit for bit, those of
the same calls made one at a time afterwards.
"""
import os
import subprocess
import sys
import textwrap

import pytest

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CHILD = textwrap.dedent(r"""
    import ctypes, os, sys, threading
    import torch
    sys.path.insert(0, sys.argv[1])
    from rocm_attn_b200.workloads import Shape, make_qkv
    lib = ctypes.CDLL(os.path.join(sys.argv[1], "rocm_attn_b200", "librocm_attn.so"))
    lib.launch_attn_forward.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int] * 5 + [
        ctypes.c_bool, ctypes.c_float, ctypes.c_int, ctypes.c_void_p]
    lib.launch_attn_forward.restype = ctypes.c_int

    class AttnProblem(ctypes.Structure):
        _fields_ = [("q", ctypes.c_void_p), ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
                    ("out", ctypes.c_void_p), ("B", ctypes.c_int), ("H", ctypes.c_int), ("Sq", ctypes.c_int),
                    ("Skv", ctypes.c_int), ("D", ctypes.c_int), ("causal", ctypes.c_bool),
                    ("softmax_scale", ctypes.c_float), ("q_strides", ctypes.c_void_p),
                    ("k_strides", ctypes.c_void_p), ("v_strides", ctypes.c_void_p)]
    lib.launch_attn_forward_batch.argtypes = [ctypes.POINTER(AttnProblem), ctypes.c_int, ctypes.c_int,
                                              ctypes.c_void_p]
    lib.launch_attn_forward_batch.restype = ctypes.c_int

    # (shape, dtype, causal): tcgen05 D=128 and D=64 (both key-block sizes),
    # short-sequence, mid-length and general kernels
    cases = [(Shape(1, 4, 640, 640, 128), torch.float16, False), (Shape(2, 2, 300, 300, 128), torch.bfloat16, True),
             (Shape(1, 4, 512, 512, 64), torch.bfloat16, False), (Shape(64, 8, 256, 256, 64), torch.float16, False),
             (Shape(64, 4, 16, 16, 64), torch.float16, False), (Shape(4, 4, 40, 93, 64), torch.bfloat16, True),
             (Shape(2, 2, 100, 100, 48), torch.float32, True), (Shape(2, 4, 200, 200, 32), torch.float16, False)]
    code = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
    inputs = [tuple(t.cuda() for t in make_qkv(s, dt, seed=i)) for i, (s, dt, _) in enumerate(cases)]
    streams = [torch.cuda.Stream() for _ in cases]
    outs = [torch.empty_like(t[0]) for t in inputs]
    batch_outs = [torch.empty_like(inputs[i][0]) for i in (0, 3, 4)]
    torch.cuda.synchronize()
    start = threading.Barrier(len(cases))
    status = [None] * len(cases)

    def call(i, out, stream):
        (s, dt, causal), (q, k, v) = cases[i], inputs[i]
        return lib.launch_attn_forward(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), s.B, s.H, s.Lq,
                                       s.Lk, s.D, causal, -1.0, code[dt], ctypes.c_void_p(stream.cuda_stream))

    def batch(stream):
        idx = (0, 3, 4)  # fp16 problems: tcgen05 D=128, tcgen05 D=64 with 64-key blocks, short kernel
        arr = (AttnProblem * 3)(*[AttnProblem(inputs[i][0].data_ptr(), inputs[i][1].data_ptr(),
                                              inputs[i][2].data_ptr(), o.data_ptr(), cases[i][0].B, cases[i][0].H,
                                              cases[i][0].Lq, cases[i][0].Lk, cases[i][0].D, cases[i][2], -1.0,
                                              None, None, None) for i, o in zip(idx, batch_outs)])
        return lib.launch_attn_forward_batch(arr, 3, 0, ctypes.c_void_p(stream.cuda_stream))

    def worker(i):
        start.wait()
        st = [call(i, outs[i], streams[i]) for _ in range(3)]
        if i == 0:  # one thread also runs a fp16 batch of three problems
            st.append(batch(streams[i]))
        status[i] = st

    threads = [threading.Thread(target=worker, args=(i,)) for i in range(len(cases))]
    for t in threads: t.start()
    for t in threads: t.join()
    torch.cuda.synchronize()
    assert all(s is not None and all(x == 0 for x in s) for s in status), status
    for i in range(len(cases)):  # the same calls, one at a time
        ref = torch.empty_like(outs[i])
        assert call(i, ref, torch.cuda.current_stream()) == 0
        torch.cuda.synchronize()
        assert torch.equal(outs[i], ref), f"case {i} differs from its single-threaded call"
    for o, i in zip(batch_outs, (0, 3, 4)):
        assert torch.equal(o, outs[i]), f"batched case {i} differs"
    s = ctypes.c_int(-1)
    lib.attn_get_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int)]
    assert lib.attn_get_status(None, ctypes.byref(s)) == 0 and s.value == 0
    print("threads ok")
""")


def test_concurrent_host_threads_fresh_process():
    r = subprocess.run([sys.executable, "-c", CHILD, REPO], capture_output=True, text=True, timeout=600)
    assert r.returncode == 0 and "threads ok" in r.stdout, r.stdout[-2000:] + r.stderr[-4000:]
