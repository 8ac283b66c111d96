"""Forward mode: jvp of the forward and of the first-order backward.

The reference differentiates attention in reverse mode only (nested custom_vjp,
``flash_hog/jax/attention.py:100-130``); forward-over-reverse Hessian-vector
products are the first extension its hot path is ranked for. The kernels compute
them from the identity jvp(bwd)(tQ, tK, tV, tdO) = bwdbwd(ddQ=tQ, ddK=tK, ddV=tV)
+ bwd(dO=tdO) (the backward is the gradient of <O, dO>, whose Hessian is
symmetric); the forward tangent is the double backward's ddO at dO = 0.

CPU tests: the identity in float64 against torch.func (an independent statement),
and the autograd plumbing (setup_context, jvp rules, dual tensors, torch.func
reverse transforms) with the kernel calls replaced by the oracle. GPU tests: the
kernels against the oracle at the bf16 bar, and a forward-over-reverse HVP through
the public op.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch
import torch.autograd.forward_ad as fwAD
import torch.func as tf

from oracle import attention_oracle as ora
from tests.parity_util import assert_close, case_inputs, np64


def _np(t):
    return t.detach().cpu().numpy()


@pytest.mark.parametrize("causal,kv_heads,tq,tk", [(False, None, 24, 20), (True, None, 24, 24), (True, 1, 24, 24),
                                                   (False, 1, 17, 33)])
def test_identity_matches_torch_func(causal, kv_heads, tq, tk):
    x = ora.make_inputs(1, 2, tq, tk, 16, seed=3, dtype=torch.float64, kv_heads=kv_heads)
    tdo = torch.randn(x["do"].shape, generator=torch.Generator().manual_seed(9), dtype=torch.float64)
    sc = 0.3
    ref = ora.autograd_jvp(x["q"], x["k"], x["v"], x["do"], x["ddq"], x["ddk"], x["ddv"], tdo, scale=sc,
                           causal=causal)
    q, k, v, do = (_np(x[n]) for n in ("q", "k", "v", "do"))
    t = [_np(x[n]) for n in ("ddq", "ddk", "ddv")]
    o, lse = ora.attention_fwd(q, k, v, scale=sc, causal=causal)
    to, tl = ora.jvp_fwd(q, k, v, o, lse, *t, scale=sc, causal=causal)
    tdq, tdk, tdv = ora.jvp_bwd(q, k, v, o, lse, do, *t, _np(tdo), scale=sc, causal=causal)
    for name, got, want in (("tO", to, ref["to"]), ("tL", tl, ref["tlse"]), ("tdQ", tdq, ref["tdq"]),
                            ("tdK", tdk, ref["tdk"]), ("tdV", tdv, ref["tdv"])):
        assert ora.rel_err(got, _np(want)) < 1e-12, name


def _oracle_impl(monkeypatch):
    """Replaces the kernel calls of the implementation layer by float64 oracle calls."""
    from flash_hog_b200 import _attention_impl as impl

    T = lambda a: torch.from_numpy(np.ascontiguousarray(a))
    causal = impl._is_causal

    def fwd(query, key, value, mask_type, scale, return_residual=False, policy=None):
        o, l = ora.attention_fwd(_np(query), _np(key), _np(value), scale=scale, causal=causal(mask_type))
        return (T(o), T(l)) if return_residual else T(o)

    def bwd_fwd(mask_type, scale, res, g, policy=None):
        q, k, v, l, o = res
        d = ora.attention_bwd(*map(_np, (q, k, v, o, l, g)), scale=scale, causal=causal(mask_type))
        return tuple(map(T, d)), (q, k, v, o, l, g)

    def bwd_bwd(mask_type, scale, res, g, policy=None):
        r = ora.bwdbwd_stats(*map(_np, res), *map(_np, g), scale=scale, causal=causal(mask_type))
        return (T(r[0]), T(r[1]), T(r[2]), None, None), T(r[3])

    def fwd_jvp(mask_type, scale, res, tangents, policy=None):
        q, k, v, l, o = res
        impl._require_plain(*res, *tangents)
        t = impl._zeros_if_none(tangents, (q, k, v))
        to, tl = ora.jvp_fwd(*map(_np, (q, k, v, o, l)), *map(_np, t), scale=scale, causal=causal(mask_type))
        return T(to), T(tl)

    def bwd_jvp(mask_type, scale, res, g, tangents, policy=None):
        q, k, v, l, o = res
        impl._require_plain(*res, g, *tangents)
        t = impl._zeros_if_none(tangents[:3], (q, k, v))
        tdo = None if tangents[3] is None else _np(tangents[3])
        return tuple(map(T, ora.jvp_bwd(*map(_np, (q, k, v, o, l, g)), *map(_np, t), tdo, scale=scale,
                                        causal=causal(mask_type))))

    for name, fn in (("cuda_dot_product_attention", fwd), ("dot_product_attention_bwd_rule_fwd_rule", bwd_fwd),
                     ("dot_product_attention_bwd_rule_bwd_rule", bwd_bwd),
                     ("dot_product_attention_fwd_jvp", fwd_jvp), ("dot_product_attention_bwd_jvp", bwd_jvp)):
        monkeypatch.setattr(impl, name, fn)


def _problem(device="cpu", dtype=torch.float64, causal=True, d=8, seed=1):
    x = ora.make_inputs(1, 2, 16, 16, d, seed=seed, dtype=torch.float32)
    x = {n: t.to(device=device, dtype=dtype) for n, t in x.items()}
    x["w"] = torch.randn(x["q"].shape, generator=torch.Generator().manual_seed(4)).to(device=device, dtype=dtype)
    return x


def _loss(attn, w):  # non-linear in O, so the cotangent of O has a tangent too
    return lambda q, k, v: ((attn(q, k, v).double() * w.double()).sum()) ** 2


def _ref(scale, causal):
    return lambda q, k, v: ora._torch_attention(q, k, v, scale, causal)


def _fwd_over_rev_hvp(f, prim, tan):
    """Forward-over-reverse HVP with dual tensors and torch.autograd.grad."""
    with fwAD.dual_level():
        duals = [fwAD.make_dual(p.detach().clone().requires_grad_(True), t) for p, t in zip(prim, tan)]
        g = torch.autograd.grad(f(*duals), duals)
        return [fwAD.unpack_dual(x).tangent for x in g]


def test_plumbing_forward_mode(monkeypatch):
    from flash_hog_b200.attention import dot_product_attention

    _oracle_impl(monkeypatch)
    x = _problem()
    loss = lambda attn: _loss(attn, x["w"])
    ref = _ref(8 ** -0.5, True)
    ours = lambda q, k, v: dot_product_attention(q, k, v, is_causal=True)
    prim, tan = (x["q"], x["k"], x["v"]), (x["ddq"], x["ddk"], x["ddv"])
    _, to_ref = tf.jvp(ref, prim, tan)
    with fwAD.dual_level():
        od = ours(*(fwAD.make_dual(p, t) for p, t in zip(prim, tan)))
        assert ora.rel_err(_np(fwAD.unpack_dual(od).tangent), _np(to_ref)) < 1e-12
    _, h_ref = tf.jvp(tf.grad(loss(ref), argnums=(0, 1, 2)), prim, tan)
    for got, want in zip(_fwd_over_rev_hvp(loss(ours), prim, tan), h_ref):
        assert ora.rel_err(_np(got), _np(want)) < 1e-12
    # Reverse-over-reverse through torch.func (setup_context form) and classic autograd agree.
    hv_func = tf.vjp(tf.grad(loss(ours), argnums=(0, 1, 2)), *prim)[1](tan)
    for got, want in zip(hv_func, h_ref):  # symmetric Hessian: the vjp equals the jvp
        assert ora.rel_err(_np(got), _np(want)) < 1e-12
    # The torch.func.jvp transform is refused with a clear error (no silent wrong path).
    with pytest.raises(NotImplementedError, match="forward_ad"):
        tf.jvp(ours, prim, tan)


# ----------------------------------------------------------------------------------------
# GPU: kernels against the oracle
# ----------------------------------------------------------------------------------------

JVP_CASES = [  # b, h, hk, tq, tk, causal, d
    (2, 4, 4, 256, 256, True, 64),
    (1, 4, 4, 200, 328, False, 64),
    (1, 4, 2, 192, 192, True, 64),
    (1, 2, 2, 256, 256, True, 128),
    (1, 2, 1, 130, 130, False, 128),
]


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,hk,tq,tk,causal,d", JVP_CASES)
def test_jvp_kernels_match_oracle(b, h, hk, tq, tk, causal, d):
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200._attention_impl import MaskType

    x = case_inputs(b, h, tq, tk, d=d, seed=7, causal=causal, kv_heads=hk)
    g = torch.Generator().manual_seed(11)
    x["tdo"] = torch.randn(x["do"].shape, generator=g).to(torch.bfloat16)
    c = {n: t.cuda() for n, t in x.items()}
    mask = MaskType.CAUSAL if causal else MaskType.NO_MASK
    sc = d ** -0.5
    res = (c["q"], c["k"], c["v"], c["lse"], c["o"])
    to, tl = impl.dot_product_attention_fwd_jvp(mask, sc, res, (c["ddq"], c["ddk"], c["ddv"]))
    tdq, tdk, tdv = impl.dot_product_attention_bwd_jvp(mask, sc, res, c["do"], (c["ddq"], c["ddk"], c["ddv"], c["tdo"]))
    a = {n: np64(x[n]) for n in ("q", "k", "v", "o", "do", "ddq", "ddk", "ddv", "tdo")}
    lse = x["lse"].double().numpy()
    to_r, tl_r = ora.jvp_fwd(a["q"], a["k"], a["v"], a["o"], lse, a["ddq"], a["ddk"], a["ddv"], scale=sc, causal=causal)
    ref = ora.jvp_bwd(a["q"], a["k"], a["v"], a["o"], lse, a["do"], a["ddq"], a["ddk"], a["ddv"], a["tdo"], scale=sc,
                      causal=causal)
    assert_close("tO", np64(to), to_r)
    assert_close("tL", np64(tl), tl_r)
    for name, got, want in zip(("tdQ", "tdK", "tdV"), (tdq, tdk, tdv), ref):
        assert_close(name, np64(got), want)


@pytest.mark.gpu
def test_jvp_without_tdo_is_the_double_backward():
    """tdO = None: the jvp of the backward is the double backward's (dQ', dK', dV')."""
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200._attention_impl import MaskType
    from flash_hog_b200.bwdbwd import flash_bwdbwd

    x = {n: t.cuda() for n, t in case_inputs(1, 4, 256, 256, seed=5, causal=True).items()}
    res = (x["q"], x["k"], x["v"], x["lse"], x["o"])
    got = impl.dot_product_attention_bwd_jvp(MaskType.CAUSAL, 0.125, res, x["do"], (x["ddq"], x["ddk"], x["ddv"], None))
    want = flash_bwdbwd(x["q"], x["k"], x["v"], x["o"], x["do"], x["ddq"], x["ddk"], x["ddv"], x["lse"],
                        mask_type=MaskType.CAUSAL, scale=0.125)[:3]
    for a, b in zip(got, want):
        assert torch.equal(a, b)


@pytest.mark.gpu
@pytest.mark.parametrize("causal", [True, False])
def test_forward_over_reverse_hvp_on_gpu(causal):
    """HVP through the public op with dual tensors: the forward jvp, the backward and
    its jvp (double backward + backward) all on the kernels, against torch.func on
    float64 math attention."""
    from flash_hog_b200.attention import dot_product_attention

    x = _problem(device="cuda", dtype=torch.bfloat16, causal=causal, d=64, seed=2)
    ours = lambda q, k, v: dot_product_attention(q, k, v, is_causal=causal)
    prim, tan = (x["q"], x["k"], x["v"]), (x["ddq"], x["ddk"], x["ddv"])
    hv = _fwd_over_rev_hvp(_loss(ours, x["w"]), prim, tan)
    x64 = {n: t.double().cpu() for n, t in x.items()}  # the same bf16 values, in float64
    _, h_ref = tf.jvp(tf.grad(_loss(_ref(64 ** -0.5, causal), x64["w"]), argnums=(0, 1, 2)),
                      (x64["q"], x64["k"], x64["v"]), (x64["ddq"], x64["ddk"], x64["ddv"]))
    for name, got, want in zip(("q", "k", "v"), hv, h_ref):
        assert_close(f"hvp_{name}", np64(got), _np(want), tol=3e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("b,h,hk,tq,tk,causal,d,window", [(1, 4, 2, 256, 384, 0, 64, 0), (2, 2, 2, 200, 200, 1, 128, 0),
                                                          (1, 2, 1, 320, 256, 2, 64, 96)])
def test_forward_tangent_pass_equals_the_query_pass_at_zero_do(b, h, hk, tq, tk, causal, d, window):
    """FH_PASS_FWD_TANGENT (the query pass without the products that vanish at dO = 0)
    writes the tO and tL of FH_PASS_QUERY with a zero-filled dO, to within rounding (its
    statistics sum may fuse a multiply into an add that the full pass keeps apart); both
    match the oracle's jvp of the forward."""
    from flash_hog_b200 import _capi

    x = {n: t.cuda() for n, t in ora.make_inputs(b, h, tq, tk, d, seed=tq + d, kv_heads=hk).items()}
    o, lse = torch.empty_like(x["q"]), torch.empty((b, h, tq), dtype=torch.float32, device="cuda")
    _capi.attn_fwd(x["q"], x["k"], x["v"], o, lse, d ** -0.5, causal, window)
    st = torch.empty((3, b, h, tq), dtype=torch.float32, device="cuda")
    to_ref, dq2 = torch.empty_like(o), torch.empty_like(o)
    _capi.attn_bwdbwd_o(x["q"], x["k"], x["v"], o, torch.zeros_like(o), x["ddq"], x["ddk"], x["ddv"], lse, dq2, to_ref,
                        None, None, st[0], st[1], st[2], d ** -0.5, causal, which=_capi.PASS_QUERY, window=window)
    to, tl = torch.empty_like(o), torch.empty((b, h, tq), dtype=torch.float32, device="cuda")
    _capi.attn_bwdbwd_o(x["q"], x["k"], x["v"], None, None, x["ddq"], x["ddk"], x["ddv"], lse, None, to, None, None,
                        None, tl, None, d ** -0.5, causal, which=_capi.PASS_FWD_TANGENT, window=window)
    torch.cuda.synchronize()
    assert _capi.device_status() == 0
    assert torch.allclose(tl, st[1], rtol=1e-5, atol=1e-6)
    assert (to.float() - to_ref.float()).abs().max().item() <= 2 ** -7 * to_ref.float().abs().max().item()
    n = lambda t: t.detach().double().cpu().numpy()
    want_o, want_l = ora.jvp_fwd(n(x["q"]), n(x["k"]), n(x["v"]), n(o), n(lse), n(x["ddq"]), n(x["ddk"]), n(x["ddv"]),
                                 causal=causal, window=window)
    assert ora.rel_err(n(to), want_o) <= 2e-2
    finite = np.isfinite(want_l)
    assert ora.rel_err(n(tl)[finite], want_l[finite]) <= 2e-2
