"""Build step of the GPU unit test of the tcgen05 building blocks.

Compiles ``tests/csrc/selftest.cu`` (against the library's ``tc05.cuh``,
``tmap.h`` and ``attn_common.cuh``) for sm_100a into ``tests/csrc/libfh_selftest.so``, the library
``tests/test_gpu_primitives.py`` loads. Test infrastructure: the product
library does not contain this kernel.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
SRC = os.path.join(HERE, "selftest.cu")
LIB = os.path.join(HERE, "libfh_selftest.so")


def build() -> str:
    sys.path.insert(0, ROOT)
    from flash_hog_b200.build import ARCH, CSRC, NVCC_FLAGS, nvcc

    deps = [SRC] + [os.path.join(CSRC, f) for f in ("tc05.cuh", "tmap.h", "attn_common.cuh")]
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(p) for p in deps):
        return LIB
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-shared", SRC, "-o", LIB]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on selftest.cu:\n{res.stdout}\n{res.stderr}")
    return LIB


if __name__ == "__main__":
    print("built", build())
