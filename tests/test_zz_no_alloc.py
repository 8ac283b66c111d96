"""fh_attn_bwdbwd_noalloc: the double backward for callers that cannot allocate.

Callers such as an XLA FFI handler (which only receives the buffers XLA
assigned up front, on a GPU mostly reserved by JAX's own pool) or a server that
reserved its whole memory budget at start-up cannot allocate the per-query
scratch (D, dD, B) the standard entry point takes. This entry point keeps that
scratch in a static device array inside the library. Here it is called through
the C ABI, twice in a row on different problems, and compared with the standard
entry point (fh_attn_rowdot + fh_attn_bwdbwd with caller scratch) at the parity
tolerance the other GPU tests use. The file name makes pytest collect it last.
"""

import ctypes

import pytest
import torch

from parity_util import BF16_REL_TOL, case_inputs, np64

from oracle import attention_oracle as ora


def _call_noalloc(x, outs, causal, status):
    from flash_hog_b200 import _capi

    dims = _capi.make_dims(x["q"], x["k"])
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    return _capi.lib().fh_attn_bwdbwd_noalloc(
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(dims),
        p(x["q"]), p(x["k"]), p(x["v"]), p(x["o"]), p(x["do"]), p(x["ddq"]), p(x["ddk"]), p(x["ddv"]),
        p(x["lse"]), p(outs[0]), p(outs[1]), p(outs[2]), p(outs[3]), ctypes.c_float(64 ** -0.5), int(causal),
        p(status))


def _standard(x, causal):
    from flash_hog_b200 import _capi

    b, t, h, _ = x["q"].shape
    delta, dd, bv = (torch.empty((b, h, t), dtype=torch.float32, device="cuda") for _ in range(3))
    outs = [torch.empty_like(x["q"]), torch.empty_like(x["q"]), torch.empty_like(x["k"]), torch.empty_like(x["k"])]
    _capi.attn_rowdot(x["o"], x["do"], delta)
    _capi.attn_bwdbwd(x["q"], x["k"], x["v"], x["do"], x["ddq"], x["ddk"], x["ddv"], x["lse"], delta,
                      outs[0], outs[1], outs[2], outs[3], dd, bv, 64 ** -0.5, causal)
    return outs


@pytest.mark.gpu
def test_noalloc_matches_standard_entry_on_two_calls_in_a_row():
    from flash_hog_b200 import _capi

    cases = [((1, 2, 256, 256), True, 21), ((2, 3, 384, 256), False, 22)]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for (b, h, tq, tk), causal, seed in cases:
        x = {k: v.cuda() for k, v in case_inputs(b, h, tq, tk, seed=seed, causal=causal).items()}
        ref = _standard(x, causal)
        got = [torch.full_like(r, float("nan")) for r in ref]
        rc = _call_noalloc(x, got, causal, status)
        assert rc == 0, _capi.lib().fh_last_error().decode()
        torch.cuda.synchronize()
        assert int(status.item()) == 0
        for name, g, r in zip(("dQ2", "ddO", "dK2", "dV2"), got, ref):
            err = ora.rel_err(np64(g), np64(r))
            assert err <= BF16_REL_TOL, f"{name}: rel err {err:.3e}"


def test_noalloc_rejects_problems_beyond_its_static_scratch():
    """Validation happens before any CUDA call, so this runs without a GPU."""
    from flash_hog_b200 import _capi

    s = _capi.FhStrides(2 * 8192 * 64, 64 * 64, 64)
    dims = _capi.FhAttnDims(2, 64, 8192, 8192, 64, s, s)  # 2 * 64 * 8192 = 1,048,576 rows > 524,288
    p = ctypes.c_void_p(256)
    rc = _capi.lib().fh_attn_bwdbwd_noalloc(None, ctypes.byref(dims), *([p] * 13), ctypes.c_float(0.125), 1, None)
    assert rc == 1
    assert b"static" in _capi.lib().fh_last_error() and b"524288" in _capi.lib().fh_last_error()
