"""Bottom-right causal alignment and sliding windows.

The reference's public path masks top-left only; its JAX statements use a
bottom-right causal mask with a sliding window (``get_mask_bottom_right``,
``flash_hog/_jax_refs/jax_impl.py:104-109``: ``qi = qi + ks - qs``,
``(qi >= kj) & (qi - kj < sliding_window_length)``). Every kernel takes that band.
A query that sees no key (bottom-right with seq_q > seq_k) gets O = 0, L = -inf
and zero gradients.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from tests.parity_util import assert_close, np64


def _mask_loop(nq, nk, causal, window):
    keep = np.zeros((nq, nk), dtype=bool)
    for i in range(nq):
        qi = i + (nk - nq if causal == 2 else 0)
        for j in range(nk):
            keep[i, j] = qi >= j and (window == 0 or qi - j < window)
    return keep


@pytest.mark.parametrize("nq,nk,causal,window", [(10, 20, 2, 5), (20, 10, 2, 0), (16, 16, 1, 4), (7, 13, 1, 0),
                                                 (13, 7, 2, 3)])
def test_band_mask_matches_the_reference_formula(nq, nk, causal, window):
    assert np.array_equal(ora.causal_mask(nq, nk, causal, window), _mask_loop(nq, nk, causal, window))


def test_oracle_statements_agree_on_band_masks():
    """Explicit formulas (numpy) against double autograd of naive attention (torch)."""
    for causal, window, tq, tk in ((2, 0, 24, 40), (1, 7, 32, 32), (2, 9, 30, 44)):
        x = ora.make_inputs(1, 2, tq, tk, 16, seed=2, dtype=torch.float64)
        a = {n: t.numpy() for n, t in x.items()}
        ref = ora.autograd_all(*(x[n] for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")), causal=causal,
                               window=window)
        o, lse = ora.attention_fwd(a["q"], a["k"], a["v"], causal=causal, window=window)
        assert ora.rel_err(o, ref["o"].numpy()) < 1e-12
        got = ora.bwdbwd_stats(a["q"], a["k"], a["v"], o, lse, a["do"], a["ddq"], a["ddk"], a["ddv"], causal=causal,
                               window=window)
        for name, g in zip(("dq2", "dk2", "dv2", "ddo"), got):
            assert ora.rel_err(g, ref[name].numpy()) < 1e-10, name


def test_keyless_queries_are_zero_in_the_oracle():
    x = ora.make_inputs(1, 1, 12, 8, 16, seed=4, dtype=torch.float64)
    a = {n: t.numpy() for n, t in x.items()}
    o, lse = ora.attention_fwd(a["q"], a["k"], a["v"], causal=2)
    assert np.all(o[:, :4] == 0) and np.all(np.isneginf(lse[..., :4])) and np.isfinite(lse[..., 4:]).all()
    dq, dk, dv = ora.attention_bwd(a["q"], a["k"], a["v"], o, lse, a["do"], causal=2)
    assert np.all(dq[:, :4] == 0) and np.isfinite(dk).all() and np.isfinite(dv).all()


# ----------------------------------------------------------------------------------------
# GPU: every kernel against the oracle
# ----------------------------------------------------------------------------------------

MASK_CASES = [  # b, h, hk, tq, tk, causal, window, d
    (1, 2, 2, 200, 328, 2, 0, 64),     # bottom-right, seq_q < seq_k
    (1, 2, 2, 328, 200, 2, 0, 64),     # bottom-right, 128 queries see no key
    (2, 2, 2, 256, 256, 1, 96, 64),    # top-left sliding window
    (1, 2, 2, 300, 260, 2, 70, 64),    # bottom-right window, keyless queries, ragged tiles
    (1, 4, 2, 256, 384, 2, 128, 64),   # grouped-query attention
    (1, 2, 2, 256, 320, 2, 100, 128),  # head_dim 128
    (1, 2, 1, 520, 520, 1, 200, 128),  # long window, several key tiles per row
]


def _inputs(b, h, hk, tq, tk, d, seed=3):
    x = ora.make_inputs(b, h, tq, tk, d, seed=seed, kv_heads=hk)
    x["tdo"] = torch.randn(x["do"].shape, generator=torch.Generator().manual_seed(seed + 1)).to(torch.bfloat16)
    return x


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,hk,tq,tk,causal,window,d", MASK_CASES)
def test_band_masks_match_oracle(b, h, hk, tq, tk, causal, window, d):
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200._attention_impl import MaskType, SlidingWindow
    from flash_hog_b200.bwdbwd import flash_bwdbwd

    x = _inputs(b, h, hk, tq, tk, d)
    c = {n: t.cuda() for n, t in x.items()}
    mt = MaskType(causal)
    mask = SlidingWindow(mt, window) if window else mt
    sc = d ** -0.5
    a = {n: np64(t) for n, t in x.items()}
    kw = dict(scale=sc, causal=causal, window=window)

    # forward: O and L, including the queries that see no key
    o, lse = impl.cuda_dot_product_attention(c["q"], c["k"], c["v"], mask, sc, return_residual=True)
    o_r, lse_r = ora.attention_fwd(a["q"], a["k"], a["v"], **kw)
    assert_close("O", np64(o), o_r)
    lse_np = lse.cpu().numpy()
    assert np.array_equal(np.isneginf(lse_np), np.isneginf(lse_r))
    fin = np.isfinite(lse_r)
    assert np.abs(lse_np[fin] - lse_r[fin]).max() < 2e-2

    # the rest runs from the kernels' own (O, L), as the autograd rules do
    a["o"], a["lse"] = np64(o), lse.double().cpu().numpy()
    res = (c["q"], c["k"], c["v"], lse, o)
    dq, dk, dv = impl.dot_product_attention_bwd_rule(mask, sc, res, c["do"])
    for name, got, want in zip(("dQ", "dK", "dV"), (dq, dk, dv),
                               ora.attention_bwd(a["q"], a["k"], a["v"], a["o"], a["lse"], a["do"], **kw)):
        assert_close(name, np64(got), want)

    outs = flash_bwdbwd(c["q"], c["k"], c["v"], o, c["do"], c["ddq"], c["ddk"], c["ddv"], lse, mask_type=mask, scale=sc)
    ref = ora.bwdbwd_stats(a["q"], a["k"], a["v"], a["o"], a["lse"], a["do"], a["ddq"], a["ddk"], a["ddv"], **kw)
    for name, got, want in zip(("dQ'", "dK'", "dV'", "ddO"), outs, ref):
        assert_close(name, np64(got), want)

    tdq, tdk, tdv = impl.dot_product_attention_bwd_jvp(mask, sc, res, c["do"], (c["ddq"], c["ddk"], c["ddv"], c["tdo"]))
    ref = ora.jvp_bwd(a["q"], a["k"], a["v"], a["o"], a["lse"], a["do"], a["ddq"], a["ddk"], a["ddv"], a["tdo"], **kw)
    for name, got, want in zip(("tdQ", "tdK", "tdV"), (tdq, tdk, tdv), ref):
        assert_close(name, np64(got), want)
    from flash_hog_b200 import _capi

    assert _capi.device_status() == 0  # no bounded wait expired, no spurious error code


@pytest.mark.gpu
def test_public_op_bottom_right_window_double_backward():
    """dot_product_attention(..., causal_alignment="bottom_right", sliding_window_length=W)
    differentiated twice by torch autograd, against double autograd of naive attention."""
    from flash_hog_b200.attention import dot_product_attention

    x = ora.make_inputs(1, 2, 192, 256, 64, seed=6)
    ref = ora.autograd_all(*(x[n].double() for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")), causal=2, window=80)
    c = {n: t.cuda() for n, t in x.items()}
    q, k, v, do = (c[n].clone().requires_grad_(True) for n in ("q", "k", "v", "do"))
    o = dot_product_attention(q, k, v, is_causal=True, causal_alignment="bottom_right", sliding_window_length=80)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), do, create_graph=True)
    dq2, dk2, dv2, ddo = torch.autograd.grad((dq, dk, dv), (q, k, v, do), (c["ddq"], c["ddk"], c["ddv"]))
    assert_close("O", np64(o), ref["o"].numpy())
    for name, got in (("dq", dq), ("dk", dk), ("dv", dv), ("dq2", dq2), ("dk2", dk2), ("dv2", dv2), ("ddo", ddo)):
        assert_close(name, np64(got), ref[name].numpy())


def test_public_op_rejects_bad_mask_arguments():
    from flash_hog_b200.attention import dot_product_attention

    q = torch.zeros(1, 4, 1, 64)
    with pytest.raises(ValueError):
        dot_product_attention(q, q, q, is_causal=False, sliding_window_length=8)
    with pytest.raises(ValueError):
        dot_product_attention(q, q, q, is_causal=True, causal_alignment="middle")


EDGE_CASES = [  # b, h, hk, tq, tk, causal, window, d
    (1, 2, 2, 64, 64, 1, 1, 64),       # window 1: each query sees only its diagonal key
    (1, 2, 2, 1, 1, 1, 0, 64),         # one query, one key
    (1, 2, 1, 1, 300, 2, 0, 64),       # one query sees every key (bottom-right), GQA
    (1, 2, 2, 300, 1, 2, 0, 64),       # one key; only the last query sees it
    (1, 2, 2, 200, 100, 1, 0, 64),     # top-left with seq_q > seq_k: late rows see all keys
    (1, 2, 2, 333, 129, 2, 17, 128),   # bottom-right window, ragged, most rows keyless
    (2, 4, 1, 130, 390, 2, 65, 64),    # GQA group of 4 with a window crossing tile edges
]


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,hk,tq,tk,causal,window,d", EDGE_CASES)
def test_band_mask_edge_cases(b, h, hk, tq, tk, causal, window, d):
    """Forward, backward and double backward on the band's edge cases, against the oracle."""
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200 import _capi
    from flash_hog_b200._attention_impl import MaskType, SlidingWindow
    from flash_hog_b200.bwdbwd import flash_bwdbwd

    x = _inputs(b, h, hk, tq, tk, d, seed=11)
    c = {n: t.cuda() for n, t in x.items()}
    mt = MaskType(causal)
    mask = SlidingWindow(mt, window) if window else mt
    sc = d ** -0.5
    a = {n: np64(t) for n, t in x.items()}
    kw = dict(scale=sc, causal=causal, window=window)
    o, lse = impl.cuda_dot_product_attention(c["q"], c["k"], c["v"], mask, sc, return_residual=True)
    o_r, lse_r = ora.attention_fwd(a["q"], a["k"], a["v"], **kw)
    if np.abs(o_r).max() > 0:
        assert_close("O", np64(o), o_r)
    assert np.array_equal(np.isneginf(lse.cpu().numpy()), np.isneginf(lse_r))
    a["o"], a["lse"] = np64(o), lse.double().cpu().numpy()
    res = (c["q"], c["k"], c["v"], lse, o)
    grads = impl.dot_product_attention_bwd_rule(mask, sc, res, c["do"])
    outs = flash_bwdbwd(c["q"], c["k"], c["v"], o, c["do"], c["ddq"], c["ddk"], c["ddv"], lse, mask_type=mask, scale=sc)
    refs = ora.attention_bwd(a["q"], a["k"], a["v"], a["o"], a["lse"], a["do"], **kw) + ora.bwdbwd_stats(
        a["q"], a["k"], a["v"], a["o"], a["lse"], a["do"], a["ddq"], a["ddk"], a["ddv"], **kw)
    for name, got, want in zip(("dQ", "dK", "dV", "dQ'", "dK'", "dV'", "ddO"), list(grads) + list(outs), refs):
        g = np64(got)
        assert np.isfinite(g).all(), name
        if np.abs(want).max() < 1e-3:
            # (Near-)exact cancellation (one visible key: P = 1, O = V): the kernels
            # round O to bf16 before D = rowsum(dO o O), so ~1e-6 remains where the
            # float64 oracle gives ~0; a relative bar is meaningless there.
            assert np.abs(g).max() < 1e-3, name
        else:
            assert_close(name, g, want)
    assert _capi.device_status() == 0
