"""The oracle, pinned to the reference's own known-answer vectors (CPU only).

``tests/golden/kat_bwdbwd.npz`` holds the reference's ``test_data.zip``
(inputs and double-backward outputs written by
``flash_hog/_jax_refs/jax_impl.py:404-477``; regenerate with
``tests/golden/make_golden.py``). The explicit-formula oracle reproduces it to
~1e-4 when the reference's bf16 dtype flow is emulated, and to the bf16-grade
~5e-3 when evaluated in float64. The other oracle statements (tiled 4-pass
schedule, torch double autograd of naive attention, forward / first-order
backward) are then checked against each other in float64.
"""

import os

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "kat_bwdbwd.npz")
NAMES = ("dq2", "dk2", "dv2", "ddo")


def _golden():
    d = np.load(GOLDEN)
    bf = lambda n: torch.from_numpy(d[n + "_bf16"].view(np.int16)).view(torch.bfloat16).float()
    inp = {n: bf(n) for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")}
    inp["o"] = torch.from_numpy(d["o"])
    inp["L"] = torch.from_numpy(d["L"])
    out = {n: d[n].astype(np.float64) for n in NAMES}
    return inp, out, float(d["scale"]), bool(d["causal"])


def test_golden_file_shape_and_quirk():
    inp, out, scale, causal = _golden()
    assert inp["q"].shape == (128, 64) and inp["k"].shape == (256, 64)
    assert scale == 0.125 and not causal
    # dO was drawn from the same key as Q in the generator (jax_impl.py:608,611).
    assert torch.equal(inp["do"], inp["q"])


def test_kat_dtype_flow_emulation_is_tight():
    inp, out, scale, _ = _golden()
    got = ora.bwdbwd_stats_jax_dtype_flow(inp["q"], inp["k"], inp["v"], inp["o"], inp["L"], inp["do"], inp["ddq"],
                                          inp["ddk"], inp["ddv"], scale)
    tol = dict(dq2=1e-4, dk2=1e-4, dv2=1e-4, ddo=5e-4)
    for n, g in zip(NAMES, got):
        assert ora.max_abs(g.numpy(), out[n]) <= tol[n], n


def test_kat_float64_formulas():
    inp, out, scale, _ = _golden()
    a = {n: inp[n].double().numpy()[None, :, None, :] for n in ("q", "k", "v", "o", "do", "ddq", "ddk", "ddv")}
    lse = inp["L"].double().numpy()[None, None, :]
    got = ora.bwdbwd_stats(a["q"], a["k"], a["v"], a["o"], lse, a["do"], a["ddq"], a["ddk"], a["ddv"], scale=scale)
    for n, g in zip(NAMES, got):
        assert ora.max_abs(g[0, :, 0], out[n]) <= 1e-2, n
        assert ora.rel_err(g[0, :, 0], out[n]) <= 1e-2, n


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("tq,tk", [(96, 160), (160, 96), (64, 64)])
def test_oracle_statements_agree(causal, tq, tk):
    x = ora.make_inputs(2, 2, tq, tk, 64, seed=tq + tk, dtype=torch.float64)
    q, k, v, do, ddq, ddk, ddv = (x[n].numpy() for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv"))
    o, lse = ora.attention_fwd(q, k, v, causal=causal)
    stats, (d, dd, bb) = ora.bwdbwd_stats(q, k, v, o, lse, do, ddq, ddk, ddv, causal=causal, return_stats=True)
    tiled, (d4, dd4, bb4) = ora.bwdbwd_4pass(q, k, v, o, lse, do, ddq, ddk, ddv, causal=causal)
    auto = ora.autograd_all(*(x[n] for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")), causal=causal)
    for a, b_, n in zip(stats, tiled, NAMES):
        assert ora.max_abs(a, b_) < 1e-10, n
        assert ora.max_abs(a, auto[n].numpy()) < 1e-10, n
    for a, b_ in ((d, d4), (dd, dd4), (bb, bb4)):
        assert ora.max_abs(a, b_) < 1e-10
    assert ora.max_abs(o, auto["o"].numpy()) < 1e-12
    g1 = ora.attention_bwd(q, k, v, o, lse, do, causal=causal)
    for a, n in zip(g1, ("dq", "dk", "dv")):
        assert ora.max_abs(a, auto[n].numpy()) < 1e-10, n


def test_credited_flops_headline():
    # B4 H16 S2048 D64 causal: 22 GEMM-equivalents x 2 x D per kept pair.
    assert ora.causal_pairs(4, 16, 2048, 2048, True) == 134_283_264
    assert abs(ora.bwdbwd_flops(4, 16, 2048, 2048, 64, True) / 1e9 - 378.1) < 0.1


@pytest.mark.parametrize("causal", [False, True])
def test_oracle_grouped_query_heads(causal):
    """Grouped-query attention (4 query heads on 2 key heads): the explicit
    formulas, with key head n // group for query head n and key-side gradients
    summed over each group, agree with torch double autograd of naive attention
    whose key/value heads are repeated the same way."""
    x = ora.make_inputs(2, 4, 48, 48 if causal else 64, 16, seed=3, dtype=torch.float64, kv_heads=2)
    a = ora.autograd_all(*(x[n] for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")), causal=causal)
    q, k, v, do, ddq, ddk, ddv = (x[n].numpy() for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv"))
    o, lse = ora.attention_fwd(q, k, v, causal=causal)
    assert np.abs(o - a["o"].numpy()).max() < 1e-12
    for got, name in zip(ora.attention_bwd(q, k, v, o, lse, do, causal=causal), ("dq", "dk", "dv")):
        assert np.abs(got - a[name].numpy()).max() < 1e-12, name
    for got, name in zip(ora.bwdbwd_stats(q, k, v, o, lse, do, ddq, ddk, ddv, causal=causal),
                         ("dq2", "dk2", "dv2", "ddo")):
        assert got.shape == a[name].shape
        assert np.abs(got - a[name].numpy()).max() < 1e-12, name


@pytest.mark.parametrize("causal,window,kv_heads,tq,tk", [(0, 0, None, 200, 136), (1, 0, 2, 160, 160),
                                                          (2, 48, None, 96, 200), (1, 0, None, 300, 100)])
def test_chunked_statement_matches_explicit_formulas(causal, window, kv_heads, tq, tk):
    """The chunked matmul statement used by the full-size GPU checks equals the explicit
    formulas, including masks that cut across chunk edges and grouped-query heads."""
    x = ora.make_inputs(2, 4, tq, tk, 32, seed=tq * tk, dtype=torch.float64, kv_heads=kv_heads)
    q, k, v, do, ddq, ddk, ddv = (x[n].numpy() for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv"))
    o, lse = ora.attention_fwd(q, k, v, causal=causal, window=window)
    want, wstats = ora.bwdbwd_stats(q, k, v, o, lse, do, ddq, ddk, ddv, causal=causal, window=window,
                                    return_stats=True)
    got, gstats = ora.bwdbwd_stats_rows(q, k, v, o, lse, do, ddq, ddk, ddv, causal=causal, window=window, chunk=48)
    for a, b_, n in zip(got, want, NAMES):
        assert a.shape == b_.shape and ora.max_abs(a, b_) < 1e-11, n
    for a, b_ in zip(gstats, wstats):
        assert ora.max_abs(a, b_) < 1e-11
