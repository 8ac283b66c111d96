"""fh_attn_bwdbwd_noalloc: the double backward for callers that cannot allocate.

Some callers cannot allocate device memory while they run: an XLA FFI handler
only receives the buffers XLA assigned up front, on a GPU whose memory JAX's
own pool has mostly reserved, and a server that reserved its whole memory
budget at start-up never allocates per request. Neither has anywhere to put the
per-query scratch (D, dD, B) that the standard entry point takes, so this entry
point keeps that scratch in a static device array inside the library.

Here it is called through the C ABI on a sequence of problems, largest first
(exactly the array's 524,288-row capacity), so that every later call runs on
the leftovers of a larger one; each problem is called twice in a row. Each call
must equal the standard entry point (fh_attn_bwdbwd_o with caller scratch, the
same two kernels) bit for bit, and the smaller problems are also checked
against the CPU oracle at the bf16 parity bar. The file name makes pytest
collect it last.
"""

import ctypes

import numpy as np
import pytest
import torch

from parity_util import BF16_REL_TOL, np64

from oracle import attention_oracle as ora

CAP_ROWS = 1 << 19  # batch * heads * seq_q the static scratch holds


def _inputs(b, h, tq, tk, d, seed, causal, kv_heads=None, window=0):
    """Seeded bf16 inputs on the GPU with the forward's O and L: the oracle's for the
    small problems, the library's forward kernel for the capacity-sized one (whose
    float64 forward on the host would take gigabytes)."""
    x = ora.make_inputs(b, h, tq, tk, d, seed=seed, kv_heads=kv_heads)
    if b * h * tq * tk <= 1 << 24:
        o, lse = ora.attention_fwd(np64(x["q"]), np64(x["k"]), np64(x["v"]), causal=causal, window=window)
        x["o"] = torch.from_numpy(o).to(torch.bfloat16)
        x["lse"] = torch.from_numpy(lse).float()
        return {k: v.cuda() for k, v in x.items()}
    from flash_hog_b200 import _capi

    x = {k: v.cuda() for k, v in x.items()}
    x["o"] = torch.empty_like(x["q"])
    x["lse"] = torch.empty((b, h, tq), dtype=torch.float32, device="cuda")
    _capi.attn_fwd(x["q"], x["k"], x["v"], x["o"], x["lse"], d ** -0.5, causal, window)
    return x


def _call_noalloc(x, outs, causal, window, status):
    from flash_hog_b200 import _capi

    dims = _capi.make_dims(x["q"], x["k"], window)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    return _capi.lib().fh_attn_bwdbwd_noalloc(
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream), ctypes.byref(dims),
        p(x["q"]), p(x["k"]), p(x["v"]), p(x["o"]), p(x["do"]), p(x["ddq"]), p(x["ddk"]), p(x["ddv"]),
        p(x["lse"]), p(outs[0]), p(outs[1]), p(outs[2]), p(outs[3]), ctypes.c_float(x["q"].shape[-1] ** -0.5),
        int(causal), p(status))


def _standard(x, causal, window):
    from flash_hog_b200 import _capi

    b, t, h, d = x["q"].shape
    delta, dd, bv = (torch.empty((b, h, t), dtype=torch.float32, device="cuda") for _ in range(3))
    outs = [torch.empty_like(x["q"]), torch.empty_like(x["q"]), torch.empty_like(x["k"]), torch.empty_like(x["k"])]
    _capi.attn_bwdbwd_o(x["q"], x["k"], x["v"], x["o"], x["do"], x["ddq"], x["ddk"], x["ddv"], x["lse"],
                        outs[0], outs[1], outs[2], outs[3], delta, dd, bv, d ** -0.5, causal, window=window)
    return outs


# (b, h, kv_heads, tq, tk, d, causal, window, check against the oracle), largest first
CASES = [
    (1, 1, None, CAP_ROWS, 128, 64, 0, 0, False),  # exactly the static capacity
    (2, 4, 2, 384, 320, 128, 1, 96, True),         # head_dim 128, GQA, sliding window
    (1, 2, None, 256, 256, 64, 1, 0, True),
    (2, 3, None, 200, 136, 64, 0, 0, True),        # ragged, non-causal
]


@pytest.mark.gpu
def test_noalloc_matches_standard_entry_on_calls_in_a_row():
    from flash_hog_b200 import _capi

    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    for i, (b, h, hk, tq, tk, d, causal, window, oracle) in enumerate(CASES):
        assert b * h * tq <= CAP_ROWS
        x = _inputs(b, h, tq, tk, d, seed=31 + i, causal=causal, kv_heads=hk, window=window)
        ref = _standard(x, causal, window)
        for call in range(2):
            got = [torch.full_like(r, float("nan")) for r in ref]
            rc = _call_noalloc(x, got, causal, window, status)
            assert rc == 0, _capi.lib().fh_last_error().decode()
            torch.cuda.synchronize()
            assert int(status.item()) == 0, f"case {i} call {call}: device status {int(status.item())}"
            for name, g, r in zip(("dQ2", "ddO", "dK2", "dV2"), got, ref):
                assert torch.equal(g, r), f"case {i} call {call}: {name} differs from fh_attn_bwdbwd_o"
        if oracle:
            arrs = {n: np64(x[n]) for n in ("q", "k", "v", "o", "lse", "do", "ddq", "ddk", "ddv")}
            want = ora.bwdbwd_stats(arrs["q"], arrs["k"], arrs["v"], arrs["o"], arrs["lse"], arrs["do"],
                                    arrs["ddq"], arrs["ddk"], arrs["ddv"], causal=causal, window=window)
            for name, g, w in zip(("dQ2", "dK2", "dV2", "ddO"), (got[0], got[2], got[3], got[1]), want):
                err = ora.rel_err(np64(g), w)
                assert err <= BF16_REL_TOL, f"case {i}: {name} rel err {err:.3e} against the oracle"
        else:
            # Query-side outputs of sampled query rows depend only on those rows.
            rows = torch.tensor([0, 1, 4095, 131071, CAP_ROWS - 1], device="cuda")
            arrs = {n: np64(x[n].index_select(1, rows)) if n in ("q", "o", "do", "ddq")
                    else np64(x[n]) for n in ("q", "k", "v", "o", "do", "ddq", "ddk", "ddv")}
            lse = np64(x["lse"].index_select(2, rows))
            wq2, _, _, wdo = ora.bwdbwd_stats(arrs["q"], arrs["k"], arrs["v"], arrs["o"], lse, arrs["do"],
                                              arrs["ddq"], arrs["ddk"], arrs["ddv"], causal=causal)
            for name, g, w in (("dQ2", got[0], wq2), ("ddO", got[1], wdo)):
                err = ora.rel_err(np64(g.index_select(1, rows)), w)
                assert err <= BF16_REL_TOL, f"cap case: {name} rel err {err:.3e} on sampled rows"
            assert np.isfinite(np64(got[2])).all() and np.isfinite(np64(got[3])).all()
        del x, ref, got
        torch.cuda.empty_cache()


def test_noalloc_rejects_problems_beyond_its_static_scratch():
    """Validation happens before any CUDA call, so this runs without a GPU."""
    from flash_hog_b200 import _capi

    s = _capi.FhStrides(2 * 8192 * 64, 64 * 64, 64)
    dims = _capi.FhAttnDims(2, 64, 8192, 8192, 64, s, s)  # 2 * 64 * 8192 = 1,048,576 rows > 524,288
    p = ctypes.c_void_p(256)
    rc = _capi.lib().fh_attn_bwdbwd_noalloc(None, ctypes.byref(dims), *([p] * 13), ctypes.c_float(0.125), 1, None)
    assert rc == 1
    assert b"static" in _capi.lib().fh_last_error() and b"524288" in _capi.lib().fh_last_error()
    # One row past the capacity is rejected too.
    dims = _capi.FhAttnDims(1, 1, CAP_ROWS + 1, 128, 64, _capi.FhStrides(0, 64, 0), _capi.FhStrides(0, 64, 0))
    rc = _capi.lib().fh_attn_bwdbwd_noalloc(None, ctypes.byref(dims), *([p] * 13), ctypes.c_float(0.125), 0, None)
    assert rc == 1
