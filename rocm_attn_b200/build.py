"""In-tree build of the native parts.

* ``librocm_attn.so``  -- the sm_100a kernels and the C-ABI launcher
  (``csrc/attn_kernel.cu``: tensor-core kernel and dispatch;
  ``csrc/attn_group.cu``: grouped launches of several problems;
  ``csrc/attn_general.cu``: fp32 / other head dims), compiled by nvcc for
  ``sm_100a`` only, with the
  CUDA runtime linked statically so the library loads without torch.
* ``librocm_attn_wdtest.so`` -- the same kernels built with
  RA_WATCHDOG_TEST for the watchdog's GPU test (see WATCHDOG_TEST_LIB).
* ``rocm_attn_ext*.so`` -- the PyTorch binding (``csrc/attn_torch.cpp``),
  linked against ``librocm_attn.so`` through an ``$ORIGIN`` rpath.

Both land next to this file so they travel with the source tree.  Run as
``python rocm_attn_b200/build.py`` (or through ``__graft_entry__.build()``).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
KERNEL_LIB = os.path.join(PKG_DIR, "librocm_attn.so")

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-cudart", "static",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the sm_100a kernels need the CUDA toolkit to build")


def _newer(target: str, sources: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _kernel_sources() -> list[str]:
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC))
            if f.endswith((".cu", ".cuh", ".h"))] + [os.path.join(INCLUDE, "attn_kernel.h")]


# The watchdog test build: the same sources with RA_WATCHDOG_TEST, which can
# lose one pipeline arrival on request so that a GPU test can make a wait run
# out (tests/test_watchdog_gpu.py).  Never loaded by the package.
WATCHDOG_TEST_LIB = os.path.join(PKG_DIR, "librocm_attn_wdtest.so")
OBJ_DIR = os.path.join(PKG_DIR, "_build", "kernels")


def _deps(src: str) -> list[str]:
    """The source and the local headers it includes, transitively."""
    seen, todo = [], [src]
    while todo:
        f = todo.pop()
        if f in seen or not os.path.exists(f):
            continue
        seen.append(f)
        for line in open(f):
            line = line.strip()
            if line.startswith('#include "'):
                name = line.split('"')[1]
                todo += [os.path.join(CSRC, name), os.path.join(INCLUDE, name)]
    return seen


def _compile(src: str, obj: str, defines=(), verbose: bool = False) -> str:
    if _newer(obj, _deps(src)):
        os.makedirs(os.path.dirname(obj), exist_ok=True)
        cmd = [_nvcc(), *NVCC_FLAGS, *(f"-D{d}" for d in defines), "-I", INCLUDE, "-c", src, "-o", obj + ".tmp"]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
        os.replace(obj + ".tmp", obj)
    return obj


def _link(objs: list[str], lib: str) -> None:
    subprocess.run([_nvcc(), *NVCC_FLAGS, "-shared", *objs, "-o", lib + ".tmp"], check=True)
    os.replace(lib + ".tmp", lib)


def build_kernel_lib(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/*.cu into librocm_attn.so (sm_100a), and the watchdog
    test build of the same sources into librocm_attn_wdtest.so."""
    if force or _newer(KERNEL_LIB, _kernel_sources()) or _newer(WATCHDOG_TEST_LIB, _kernel_sources()):
        if force and os.path.isdir(OBJ_DIR):
            shutil.rmtree(OBJ_DIR)
        # The translation units compile in parallel (each takes about a minute).
        jobs = [("attn_general.cu", "attn_general.o", ()), ("attn_kernel.cu", "attn_kernel.o", ()),
                ("attn_group.cu", "attn_group.o", ()),
                ("attn_kernel.cu", "attn_kernel_wdtest.o", ("RA_WATCHDOG_TEST",))]
        with ThreadPoolExecutor(len(jobs)) as ex:
            general, kernel, group, wd = ex.map(
                lambda j: _compile(os.path.join(CSRC, j[0]), os.path.join(OBJ_DIR, j[1]), defines=j[2],
                                   verbose=verbose), jobs)
        _link([kernel, group, general], KERNEL_LIB)
        _link([wd, group, general], WATCHDOG_TEST_LIB)
    return KERNEL_LIB


def ext_path() -> str | None:
    suffix = sysconfig.get_config_var("EXT_SUFFIX") or ".so"
    p = os.path.join(PKG_DIR, "rocm_attn_ext" + suffix)
    return p if os.path.exists(p) else None


def build_torch_ext(force: bool = False) -> str:
    """Build the PyTorch binding in place (rocm_attn_b200/rocm_attn_ext*.so)."""
    src = os.path.join(CSRC, "attn_torch.cpp")
    existing = ext_path()
    if not force and existing and not _newer(existing, [src, KERNEL_LIB, os.path.join(INCLUDE, "attn_kernel.h")]):
        return existing
    from setuptools import setup
    from torch.utils.cpp_extension import BuildExtension, CUDAExtension

    build_temp = os.path.join(PKG_DIR, "_build")
    ext = CUDAExtension(
        name="rocm_attn_b200.rocm_attn_ext",
        sources=[os.path.relpath(src, REPO_DIR)],
        include_dirs=[INCLUDE],
        library_dirs=[PKG_DIR],
        libraries=["rocm_attn"],
        extra_compile_args={"cxx": ["-O3"]},
        extra_link_args=["-Wl,-rpath,$ORIGIN"],
    )
    # Link against the system libstdc++ the rest of the process (torch) uses.
    # A toolchain wrapper that resolves -lstdc++ to a partial static copy puts
    # a second set of iostream/locale internals into the module, and the first
    # `ostream << int` on an error path then crashes in a mismatched facet.
    env_save = {k: os.environ.get(k) for k in ("CXX", "CC")}
    for var, exe in (("CXX", "/usr/bin/g++"), ("CC", "/usr/bin/gcc")):
        if os.path.exists(exe):
            os.environ[var] = exe
    cwd = os.getcwd()
    os.chdir(REPO_DIR)
    try:
        setup(
            name="rocm_attn_b200_ext",
            ext_modules=[ext],
            cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
            script_args=["-q", "build_ext", "--inplace", "--build-temp", build_temp],
        )
    finally:
        os.chdir(cwd)
        for k, v in env_save.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v
    p = ext_path()
    if p is None:
        raise RuntimeError("PyTorch extension build produced no module")
    return p


def build_all(force: bool = False, verbose: bool = False) -> None:
    build_kernel_lib(force=force, verbose=verbose)
    build_torch_ext(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print("built", KERNEL_LIB, ext_path())
