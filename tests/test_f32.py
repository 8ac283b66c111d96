"""fp32 inputs: the fp32 kernels (``fh_attn_*_f32``) against the float64 oracle at 1e-3.

The reference keeps fp32 inputs in fp32 (its Pallas double backward casts each
score-like operand to the dtype of the tensor it multiplies,
``flash_hog/jax/_pallas_gpu_kernel.py:251-256``) and its XLA reference is fp32
attention differentiated twice (``flash_hog/_jax_refs/jax_impl.py:194-247``); the
bar for fp32 inputs is max|gpu - oracle| / max|oracle| <= 1e-3. Configuration 1 of
the benchmark table (B1 H2 S256 D64 fp32, causal and not) is the first case.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from tests.parity_util import assert_close, np64

F32_REL_TOL = 1e-3

F32_CASES = [  # b, h, hk, tq, tk, causal, window, d
    (1, 2, 2, 256, 256, 0, 0, 64),     # configuration 1, no mask
    (1, 2, 2, 256, 256, 1, 0, 64),     # configuration 1, causal
    (1, 2, 2, 200, 328, 2, 0, 64),     # bottom-right, seq_q < seq_k, ragged tiles
    (1, 2, 2, 328, 200, 2, 0, 64),     # bottom-right, 128 queries see no key
    (2, 2, 2, 256, 256, 1, 96, 64),    # top-left sliding window
    (1, 4, 2, 256, 384, 2, 128, 64),   # grouped-query attention
    (1, 2, 2, 256, 320, 2, 100, 128),  # head_dim 128
    (1, 4, 1, 300, 300, 0, 0, 128),    # head_dim 128, GQA group of 4, ragged, no mask
]


def _inputs(b, h, hk, tq, tk, d, seed=21):
    x = ora.make_inputs(b, h, tq, tk, d, seed=seed, dtype=torch.float32, kv_heads=hk)
    x["tdo"] = torch.randn(x["do"].shape, generator=torch.Generator().manual_seed(seed + 1))
    return x


def test_f32_entry_points_are_bound():
    """The binding routes fp32 inputs to the fp32 entry points (no GPU needed)."""
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200 import _capi

    for name in ("fh_attn_fwd_f32", "fh_attn_bwd_f32", "fh_attn_bwdbwd_f32", "fh_attn_jvp_bwd_f32"):
        assert name in _capi.EXPORTED_SYMBOLS
    assert impl._is_f32(torch.zeros(1, dtype=torch.float32))
    assert not impl._is_f32(torch.zeros(1, dtype=torch.bfloat16))
    assert not impl._is_f32(torch.zeros(1, dtype=torch.float16))


def test_fp32_policy_switch(monkeypatch):
    """FLASH_HOG_B200_FP32=bf16 sends fp32 inputs to the bf16 kernels (the reference's
    native-plugin behaviour); anything but fp32/bf16 is refused."""
    from flash_hog_b200 import _attention_impl as impl

    x = torch.zeros(1, dtype=torch.float32)
    monkeypatch.setenv(impl.FP32_POLICY_ENV, "bf16")
    assert impl.fp32_policy() == "bf16" and not impl._is_f32(x)
    monkeypatch.setenv(impl.FP32_POLICY_ENV, "fp32")
    assert impl._is_f32(x)
    monkeypatch.setenv(impl.FP32_POLICY_ENV, "tf32")
    with pytest.raises(ValueError):
        impl.fp32_policy()


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,hk,tq,tk,causal,window,d", F32_CASES)
def test_f32_kernels_match_oracle(b, h, hk, tq, tk, causal, window, d):
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200 import _capi
    from flash_hog_b200._attention_impl import MaskType, SlidingWindow
    from flash_hog_b200.bwdbwd import flash_bwdbwd

    x = _inputs(b, h, hk, tq, tk, d)
    c = {n: t.cuda() for n, t in x.items()}
    mt = MaskType(causal)
    mask = SlidingWindow(mt, window) if window else mt
    sc = d ** -0.5
    a = {n: np64(t) for n, t in x.items()}
    kw = dict(scale=sc, causal=causal, window=window)
    n0 = _capi.launch_count()

    o, lse = impl.cuda_dot_product_attention(c["q"], c["k"], c["v"], mask, sc, return_residual=True)
    assert o.dtype == torch.float32
    o_r, lse_r = ora.attention_fwd(a["q"], a["k"], a["v"], **kw)
    assert_close("O", np64(o), o_r, F32_REL_TOL)
    lse_np = lse.double().cpu().numpy()
    assert np.array_equal(np.isneginf(lse_np), np.isneginf(lse_r))
    fin = np.isfinite(lse_r)
    assert np.abs(lse_np[fin] - lse_r[fin]).max() < 1e-4

    a["o"], a["lse"] = np64(o), lse_np
    res = (c["q"], c["k"], c["v"], lse, o)
    grads = impl.dot_product_attention_bwd_rule(mask, sc, res, c["do"])
    for name, got, want in zip(("dQ", "dK", "dV"), grads,
                               ora.attention_bwd(a["q"], a["k"], a["v"], a["o"], a["lse"], a["do"], **kw)):
        assert got.dtype == torch.float32
        assert_close(name, np64(got), want, F32_REL_TOL)

    outs, stats = flash_bwdbwd(c["q"], c["k"], c["v"], o, c["do"], c["ddq"], c["ddk"], c["ddv"], lse, mask_type=mask,
                               scale=sc, return_stats=True)
    ref, ref_stats = ora.bwdbwd_stats(a["q"], a["k"], a["v"], a["o"], a["lse"], a["do"], a["ddq"], a["ddk"],
                                      a["ddv"], return_stats=True, **kw)
    for name, got, want in zip(("dQ'", "dK'", "dV'", "ddO"), outs, ref):
        assert got.dtype == torch.float32
        assert_close(name, np64(got), want, F32_REL_TOL)
    for name, got, want in zip(("D", "dD", "B"), stats, ref_stats):
        assert_close(name, np64(got), want, F32_REL_TOL)

    tdq, tdk, tdv = impl.dot_product_attention_bwd_jvp(mask, sc, res, c["do"], (c["ddq"], c["ddk"], c["ddv"], c["tdo"]))
    ref = ora.jvp_bwd(a["q"], a["k"], a["v"], a["o"], a["lse"], a["do"], a["ddq"], a["ddk"], a["ddv"], a["tdo"], **kw)
    for name, got, want in zip(("tdQ", "tdK", "tdV"), (tdq, tdk, tdv), ref):
        assert_close(name, np64(got), want, F32_REL_TOL)

    to, tlse = impl.dot_product_attention_fwd_jvp(mask, sc, res, (c["ddq"], c["ddk"], c["ddv"]))
    to_r, tlse_r = ora.jvp_fwd(a["q"], a["k"], a["v"], a["o"], a["lse"], a["ddq"], a["ddk"], a["ddv"], **kw)
    assert_close("tO", np64(to), to_r, F32_REL_TOL)
    fin = np.isfinite(tlse_r)
    assert_close("tL", np64(tlse)[fin], tlse_r[fin], F32_REL_TOL)

    # fwd 1, bwd 3, bwdbwd 3, jvp_bwd 6, fwd jvp 2 kernels: all from this library.
    assert _capi.launch_count() - n0 == 15


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [False, True])
def test_f32_public_op_double_backward_config1(causal):
    """Configuration 1 through the public op: dot_product_attention on fp32 inputs,
    differentiated twice by torch autograd, against double autograd of naive
    attention in float64 (the statement of the reference's XLA reference)."""
    from flash_hog_b200.attention import dot_product_attention

    x = ora.make_inputs(1, 2, 256, 256, 64, seed=5, dtype=torch.float32)
    ref = ora.autograd_all(*(x[n].double() for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")), causal=causal)
    c = {n: t.cuda() for n, t in x.items()}
    q, k, v, do = (c[n].clone().requires_grad_(True) for n in ("q", "k", "v", "do"))
    o = dot_product_attention(q, k, v, is_causal=causal)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), do, create_graph=True)
    dq2, dk2, dv2, ddo = torch.autograd.grad((dq, dk, dv), (q, k, v, do), (c["ddq"], c["ddk"], c["ddv"]))
    for name, got in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv), ("dq2", dq2), ("dk2", dk2), ("dv2", dv2),
                      ("ddo", ddo)):
        assert got.dtype == torch.float32, name
        assert_close(name, np64(got), ref[name].numpy(), F32_REL_TOL)


@pytest.mark.gpu
def test_f32_strided_bhtd_views():
    """The C ABI reads the (batch, head, seq) strides: a BHTD tensor viewed as BTNH
    gives the same results as its contiguous copy, bit for bit."""
    from flash_hog_b200 import _capi

    g = torch.Generator().manual_seed(9)
    b, h, t, d = 2, 3, 200, 64
    q, k, v, do, ddq, ddk, ddv = (torch.randn(b, h, t, d, generator=g).cuda().transpose(1, 2) for _ in range(7))
    assert not q.is_contiguous()

    def run(q, k, v, do, ddq, ddk, ddv):
        o = torch.empty_like(q)
        lse = torch.empty(b, h, t, device="cuda")
        _capi.attn_fwd_f32(q, k, v, o, lse, d ** -0.5, 1)
        outs = [torch.empty_like(q), torch.empty_like(q), torch.empty_like(k), torch.empty_like(k)]
        st = torch.empty(3, b, h, t, device="cuda")
        _capi.attn_bwdbwd_f32(q, k, v, o, do, ddq, ddk, ddv, lse, *outs, st[0], st[1], st[2], d ** -0.5, 1)
        return [o, lse] + outs

    strided = run(q, k, v, do, ddq, ddk, ddv)
    dense = run(*(x.contiguous() for x in (q, k, v, do, ddq, ddk, ddv)))
    for s_, d_ in zip(strided, dense):
        assert torch.equal(s_, d_)


@pytest.mark.gpu
def test_f32_kernels_on_the_golden_inputs():
    """The reference's known-answer inputs (non-causal, Nq 128, Nk 256, D 64, scale 1/8)
    through the fp32 double backward: within 1e-3 of the float64 oracle on the same
    inputs, and within the golden file's own bf16-grade 1e-2 of its outputs."""
    from flash_hog_b200.bwdbwd import flash_bwdbwd

    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "kat_bwdbwd.npz"))
    bf = lambda n: torch.from_numpy(d[n + "_bf16"].view(np.int16)).view(torch.bfloat16).float()
    inp = {n: bf(n)[None, :, None, :] for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")}
    inp["o"] = torch.from_numpy(d["o"]).float()[None, :, None, :]
    inp["L"] = torch.from_numpy(d["L"]).float()[None, None, :]
    scale = float(d["scale"])
    c = {n: t.cuda() for n, t in inp.items()}
    got = flash_bwdbwd(c["q"], c["k"], c["v"], c["o"], c["do"], c["ddq"], c["ddk"], c["ddv"], c["L"], scale=scale)
    a = {n: t.double().numpy() for n, t in inp.items()}
    ref = ora.bwdbwd_stats(a["q"], a["k"], a["v"], a["o"], a["L"], a["do"], a["ddq"], a["ddk"], a["ddv"], scale=scale)
    for name, g, r in zip(("dq2", "dk2", "dv2", "ddo"), got, ref):
        assert_close(name, np64(g), r, F32_REL_TOL)
        assert ora.rel_err(np64(g)[0, :, 0], d[name].astype(np.float64)) <= 1e-2, name


@pytest.mark.gpu
def test_fp16_inputs_run_the_bf16_kernels():
    """fp16 inputs are cast to bf16, as the reference's native plugin casts every dtype
    (``flash_hog/jax/_tk_gpu.py:90-92``); results come back in fp16 within the bf16 bar."""
    from flash_hog_b200.attention import dot_product_attention

    x = ora.make_inputs(1, 2, 192, 192, 64, seed=8, dtype=torch.float16)
    ref = ora.autograd_all(*(x[n].double() for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")), causal=True)
    c = {n: t.cuda() for n, t in x.items()}
    q, k, v, do = (c[n].clone().requires_grad_(True) for n in ("q", "k", "v", "do"))
    o = dot_product_attention(q, k, v, is_causal=True)
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), do, create_graph=True)
    dq2, dk2, dv2, ddo = torch.autograd.grad((dq, dk, dv), (q, k, v, do), (c["ddq"], c["ddk"], c["ddv"]))
    for name, got in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv), ("dq2", dq2), ("dk2", dk2), ("dv2", dv2),
                      ("ddo", ddo)):
        assert got.dtype == torch.float16, name
        assert_close(name, np64(got), ref[name].numpy())


F32_EDGE_CASES = [  # b, h, hk, tq, tk, causal, window, d
    (1, 2, 2, 64, 64, 1, 1, 64),       # window 1: each query sees only its diagonal key
    (1, 2, 2, 1, 1, 1, 0, 64),         # one query, one key
    (1, 2, 1, 1, 300, 2, 0, 64),       # one query sees every key (bottom-right), GQA
    (1, 2, 2, 300, 1, 2, 0, 64),       # one key; only the last query sees it
    (1, 2, 2, 333, 129, 2, 17, 128),   # bottom-right window, ragged, most rows keyless
    (2, 4, 1, 130, 390, 2, 65, 64),    # GQA group of 4 with a window crossing tile edges
]


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,hk,tq,tk,causal,window,d", F32_EDGE_CASES)
def test_f32_band_mask_edge_cases(b, h, hk, tq, tk, causal, window, d):
    """The fp32 kernels (including their prefetching loops: one streamed tile, one item,
    several query heads per key head) on the band's edge cases, at the 1e-3 bar."""
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200._attention_impl import MaskType, SlidingWindow
    from flash_hog_b200.bwdbwd import flash_bwdbwd

    x = _inputs(b, h, hk, tq, tk, d, seed=31)
    c = {n: t.cuda() for n, t in x.items()}
    mt = MaskType(causal)
    mask = SlidingWindow(mt, window) if window else mt
    sc = d ** -0.5
    a = {n: np64(t) for n, t in x.items()}
    kw = dict(scale=sc, causal=causal, window=window)
    o, lse = impl.cuda_dot_product_attention(c["q"], c["k"], c["v"], mask, sc, return_residual=True)
    o_r, lse_r = ora.attention_fwd(a["q"], a["k"], a["v"], **kw)
    assert np.array_equal(np.isneginf(lse.cpu().numpy()), np.isneginf(lse_r))
    a["o"], a["lse"] = np64(o), lse.double().cpu().numpy()
    res = (c["q"], c["k"], c["v"], lse, o)
    grads = impl.dot_product_attention_bwd_rule(mask, sc, res, c["do"])
    outs = flash_bwdbwd(c["q"], c["k"], c["v"], o, c["do"], c["ddq"], c["ddk"], c["ddv"], lse, mask_type=mask, scale=sc)
    refs = [o_r] + list(ora.attention_bwd(a["q"], a["k"], a["v"], a["o"], a["lse"], a["do"], **kw)) + list(
        ora.bwdbwd_stats(a["q"], a["k"], a["v"], a["o"], a["lse"], a["do"], a["ddq"], a["ddk"], a["ddv"], **kw))
    for name, got, want in zip(("O", "dQ", "dK", "dV", "dQ'", "dK'", "dV'", "ddO"), [o] + list(grads) + list(outs),
                               refs):
        g = np64(got)
        assert np.isfinite(g).all(), name
        if np.abs(want).max() < 1e-4:
            # (Near-)exact cancellation (one visible key: P = 1, O = V) leaves fp32
            # rounding where the float64 oracle gives ~0; a relative bar is meaningless.
            assert np.abs(g).max() < 1e-4, name
        else:
            assert_close(name, g, want, F32_REL_TOL)


@pytest.mark.gpu
def test_fp32_inputs_under_the_bf16_policy(monkeypatch):
    """Under FLASH_HOG_B200_FP32=bf16 fp32 inputs run the bf16 kernels: fp32 outputs,
    within the bf16 bar, and visibly less exact than the default fp32 policy."""
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200.attention import dot_product_attention

    x = ora.make_inputs(1, 2, 256, 256, 64, seed=12, dtype=torch.float32)
    ref = ora.autograd_all(*(x[n].double() for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")), causal=True)
    c = {n: t.cuda() for n, t in x.items()}
    errs = {}
    for policy in ("bf16", "fp32"):
        monkeypatch.setenv(impl.FP32_POLICY_ENV, policy)
        q, k, v, do = (c[n].clone().requires_grad_(True) for n in ("q", "k", "v", "do"))
        o = dot_product_attention(q, k, v, is_causal=True)
        dq, dk, dv = torch.autograd.grad(o, (q, k, v), do, create_graph=True)
        dq2, dk2, dv2, ddo = torch.autograd.grad((dq, dk, dv), (q, k, v, do), (c["ddq"], c["ddk"], c["ddv"]))
        assert all(t.dtype == torch.float32 for t in (o, dq, dq2, ddo))
        errs[policy] = max(assert_close(n, np64(t), ref[n].numpy()) for n, t in
                           (("o", o), ("dq", dq), ("dk", dk), ("dv", dv), ("dq2", dq2), ("dk2", dk2), ("dv2", dv2),
                            ("ddo", ddo)))
    assert errs["fp32"] <= F32_REL_TOL < errs["bf16"]


@pytest.mark.gpu
def test_fp32_policy_is_kept_from_the_forward(monkeypatch):
    """The policy the forward decided holds for the whole graph: switching the variable
    between the forward and the backward changes nothing (no mix of fp32-kernel and
    bf16-kernel results in one graph)."""
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200.attention import dot_product_attention

    x = ora.make_inputs(1, 2, 256, 256, 64, seed=13, dtype=torch.float32)
    ref = ora.autograd_all(*(x[n].double() for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")), causal=True)
    c = {n: t.cuda() for n, t in x.items()}
    monkeypatch.setenv(impl.FP32_POLICY_ENV, "fp32")
    q, k, v, do = (c[n].clone().requires_grad_(True) for n in ("q", "k", "v", "do"))
    o = dot_product_attention(q, k, v, is_causal=True)
    monkeypatch.setenv(impl.FP32_POLICY_ENV, "bf16")  # too late: the forward decided fp32
    dq, dk, dv = torch.autograd.grad(o, (q, k, v), do, create_graph=True)
    dq2, dk2, dv2, ddo = torch.autograd.grad((dq, dk, dv), (q, k, v, do), (c["ddq"], c["ddk"], c["ddv"]))
    for n, t in (("o", o), ("dq", dq), ("dk", dk), ("dv", dv), ("dq2", dq2), ("dk2", dk2), ("dv2", dv2),
                 ("ddo", ddo)):
        assert_close(n, np64(t), ref[n].numpy(), tol=F32_REL_TOL)
