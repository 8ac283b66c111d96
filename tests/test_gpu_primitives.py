"""GPU unit test of the tcgen05 / TMA / TMEM conventions (tests/csrc/selftest.cu,
built by tests/csrc/build_selftest.py into tests/csrc/libfh_selftest.so).

Every attention kernel builds its operands from the same panels and
descriptors; this test isolates them on a single 128 x N x K GEMM against a
plain fp32 torch matmul of the same bf16 inputs.
"""

import ctypes
import os

import pytest
import torch

LIB = os.path.join(os.path.dirname(os.path.abspath(__file__)), "csrc", "libfh_selftest.so")


@pytest.mark.gpu
@pytest.mark.parametrize("a_threads", [0, 1])
@pytest.mark.parametrize("b_mn", [0, 1])
@pytest.mark.parametrize("n,k", [(64, 64), (128, 64), (64, 128), (256, 128)])
def test_umma_tile(n, k, b_mn, a_threads):
    lib = ctypes.CDLL(LIB)
    g = torch.Generator().manual_seed(n * 1000 + k + 10 * b_mn + a_threads)
    a = torch.randn(128, k, generator=g).to(torch.bfloat16).cuda()
    if b_mn:
        b = torch.randn(k, n, generator=g).to(torch.bfloat16).cuda()
        ref = a.float() @ b.float()
    else:
        b = torch.randn(n, k, generator=g).to(torch.bfloat16).cuda()
        ref = a.float() @ b.float().T
    c = torch.full((128, n), float("nan"), device="cuda")
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.fh_selftest_umma(
        ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()), ctypes.c_void_p(c.data_ptr()),
        n, k, b_mn, a_threads, ctypes.c_void_p(status.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert rc == 0
    assert int(status.item()) == 0
    err = (c - ref).abs().max().item()
    assert err <= 1e-3 * max(1.0, ref.abs().max().item()), f"max abs err {err}"
