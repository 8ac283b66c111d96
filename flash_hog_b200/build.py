"""Build the in-tree CUDA library for sm_100a with nvcc.

``libflashhog_b200.so`` -- the attention kernels and the C ABI declared in
``include/flash_hog_b200.h`` -- is written next to this file so it travels with
the source tree. Object files are cached under ``_build/`` keyed by source and
header modification times, so an unchanged tree rebuilds in well under a second.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(PKG, "csrc")
ROOT = os.path.dirname(PKG)
BUILD_DIR = os.path.join(ROOT, "_build")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O2", "--expt-relaxed-constexpr",
              "-I" + os.path.join(ROOT, "include"), "-I" + CSRC]

MAIN_SOURCES = ["capi.cu", "fwd.cu", "bwd.cu", "bwdbwd.cu", "rowdot.cu", "f32.cu", "ln_gelu.cu", "xent.cu"]

MAIN_LIB = os.path.join(PKG, "libflashhog_b200.so")


def nvcc() -> str:
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build flash_hog_b200")


def _headers_mtime() -> float:
    paths = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    inc = os.path.join(ROOT, "include")
    paths += [os.path.join(inc, f) for f in os.listdir(inc) if f.endswith(".h")]
    return max(os.path.getmtime(p) for p in paths)


def _compile(src: str, verbose: bool) -> str:
    os.makedirs(BUILD_DIR, exist_ok=True)
    path = os.path.join(CSRC, src)
    obj = os.path.join(BUILD_DIR, src.replace(".cu", ".o"))
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(path), _headers_mtime()):
        return obj
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", path, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{res.stdout}\n{res.stderr}")
    if verbose and res.stderr:
        print(res.stderr, file=sys.stderr)
    return obj


def _link(objs, out):
    cmd = [nvcc(), *ARCH, "-shared", "-o", out, *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link of {os.path.basename(out)} failed:\n{res.stdout}\n{res.stderr}")


def build(verbose: bool = False) -> None:
    """Compile every CUDA source of the library for sm_100a and link it."""
    srcs = MAIN_SOURCES
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = dict(zip(srcs, ex.map(lambda s: _compile(s, verbose), srcs)))
    _link([objs[s] for s in MAIN_SOURCES], MAIN_LIB)


XLA_FFI_SOURCE = os.path.join(CSRC, "xla_ffi.cc")
XLA_FFI_LIB = os.path.join(PKG, "libfh_xla_ffi.so")


def xla_ffi_include_dir():
    """jaxlib's FFI header directory, or None where JAX is not installed (this image)."""
    try:
        import jax.ffi

        return jax.ffi.include_dir()
    except Exception:  # noqa: BLE001 - any failure means the headers are not available
        return None


def build_xla_ffi():
    """Compiles ``csrc/xla_ffi.cc`` (the XLA FFI handlers FhAttnFwd, FhAttnBwd, FhBwdBwd,
    FhBwdBwdO) into ``libfh_xla_ffi.so``, linked against ``libflashhog_b200.so``.
    Returns the library path, or None without building where jaxlib's FFI headers are
    absent -- as on this image, where the handlers are therefore not built."""
    inc = xla_ffi_include_dir()
    if inc is None:
        return None
    build()
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-x", "cu", "-shared", "-I" + inc, XLA_FFI_SOURCE, "-o", XLA_FFI_LIB,
           "-L" + PKG, "-lflashhog_b200", "-Xlinker", "-rpath,$ORIGIN"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on xla_ffi.cc:\n{res.stdout}\n{res.stderr}")
    return XLA_FFI_LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv)
    print("built", MAIN_LIB)
    ffi_lib = build_xla_ffi()
    print("built", ffi_lib) if ffi_lib else print("XLA FFI handlers not built: jaxlib's FFI headers are absent")
