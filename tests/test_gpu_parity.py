"""GPU parity of the sm_100a kernels against the CPU oracle (through the C ABI).

Edge cases follow what the reference exercises or documents: causal and
non-causal, Nq != Nk cross attention (the golden file's 128 x 256 shape),
BTNH and BHTD layouts, ragged lengths that are not tile multiples, and the
headline configuration at full size checked on sampled heads.
"""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from parity_util import assert_close, assert_elementwise, case_inputs, np64, oracle_bwdbwd, select_heads

pytestmark = pytest.mark.gpu

CASES = [
    # b, h, tq, tk, causal
    (1, 2, 128, 128, True),
    (1, 2, 128, 128, False),
    (1, 1, 128, 256, False),   # golden-file shape: Nq=128, Nk=256
    (2, 2, 256, 256, True),
    (1, 2, 256, 384, False),
    (1, 2, 384, 256, True),
    (1, 1, 200, 200, True),    # ragged: not a multiple of any tile
    (1, 2, 72, 136, False),    # ragged cross attention
    (2, 3, 512, 512, True),
]


def _cuda(x):
    return {k: v.cuda() for k, v in x.items()}


@pytest.mark.parametrize("b,h,tq,tk,causal", CASES)
def test_bwdbwd_matches_oracle(b, h, tq, tk, causal):
    from flash_hog_b200 import MaskType, flash_bwdbwd
    from flash_hog_b200._capi import device_status

    x = case_inputs(b, h, tq, tk, seed=11 * tq + tk, causal=causal)
    (rq2, rk2, rv2, rdo), (rd, rdd, rb) = oracle_bwdbwd(x, causal)
    g = _cuda(x)
    mask = MaskType.CAUSAL if causal else MaskType.NO_MASK
    (dq2, dk2, dv2, ddo), (d, dd, bv) = flash_bwdbwd(g["q"], g["k"], g["v"], g["o"], g["do"], g["ddq"], g["ddk"],
                                                     g["ddv"], g["lse"], mask_type=mask, return_stats=True)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert_close("D", np64(d), rd)
    assert_close("dD", np64(dd), rdd)
    assert_close("B", np64(bv), rb)
    assert_close("dQ2", np64(dq2), rq2)
    assert_close("dK2", np64(dk2), rk2)
    assert_close("dV2", np64(dv2), rv2)
    assert_close("ddO", np64(ddo), rdo)


@pytest.mark.parametrize("b,h,tq,tk,causal", CASES)
def test_fwd_bwd_match_oracle(b, h, tq, tk, causal):
    from flash_hog_b200 import MaskType
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200._capi import device_status

    x = case_inputs(b, h, tq, tk, seed=7 * tq + tk, causal=causal)
    g = _cuda(x)
    mask = MaskType.CAUSAL if causal else MaskType.NO_MASK
    scale = 64 ** -0.5
    out, lse = impl.cuda_dot_product_attention(g["q"], g["k"], g["v"], mask, scale, return_residual=True)
    torch.cuda.synchronize()
    assert device_status() == 0
    ro, rl = ora.attention_fwd(np64(x["q"]), np64(x["k"]), np64(x["v"]), causal=causal)
    assert_close("O", np64(out), ro)
    assert ora.max_abs(np64(lse), rl) <= 2e-3
    # first-order backward from the oracle's residuals
    dq, dk, dv = impl.dot_product_attention_bwd_rule(mask, scale, (g["q"], g["k"], g["v"], g["lse"], g["o"]),
                                                     g["do"])
    torch.cuda.synchronize()
    assert device_status() == 0
    rq, rk, rv = ora.attention_bwd(np64(x["q"]), np64(x["k"]), np64(x["v"]), np64(x["o"]), np64(x["lse"]),
                                   np64(x["do"]), causal=causal)
    assert_close("dQ", np64(dq), rq)
    assert_close("dK", np64(dk), rk)
    assert_close("dV", np64(dv), rv)


GQA_CASES = [
    # b, q_heads, kv_heads, tq, tk, causal, head_dim -- grouped-query attention
    (1, 4, 2, 128, 128, True, 64),
    (2, 4, 1, 256, 384, False, 64),
    (1, 8, 2, 200, 200, True, 64),
    (1, 4, 2, 256, 256, True, 128),
    (1, 6, 3, 72, 136, False, 128),
]


@pytest.mark.parametrize("b,h,hk,tq,tk,causal,d", GQA_CASES)
def test_gqa_matches_oracle(b, h, hk, tq, tk, causal, d):
    """q_heads a multiple of kv_heads: forward, backward and double backward."""
    from flash_hog_b200 import MaskType, flash_bwdbwd
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200._capi import device_status

    x = case_inputs(b, h, tq, tk, d=d, seed=17 * tq + tk + h, causal=causal, kv_heads=hk)
    g = _cuda(x)
    mask = MaskType.CAUSAL if causal else MaskType.NO_MASK
    scale = d ** -0.5
    out, lse = impl.cuda_dot_product_attention(g["q"], g["k"], g["v"], mask, scale, return_residual=True)
    dq, dk, dv = impl.dot_product_attention_bwd_rule(mask, scale, (g["q"], g["k"], g["v"], g["lse"], g["o"]),
                                                     g["do"])
    (dq2, dk2, dv2, ddo), (dd_, dd, bv) = flash_bwdbwd(g["q"], g["k"], g["v"], g["o"], g["do"], g["ddq"],
                                                       g["ddk"], g["ddv"], g["lse"], mask_type=mask,
                                                       return_stats=True)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert dk.shape == x["k"].shape and dk2.shape == x["k"].shape and dv2.shape == x["v"].shape
    ro, rl = ora.attention_fwd(np64(x["q"]), np64(x["k"]), np64(x["v"]), causal=causal)
    assert_close("O", np64(out), ro)
    assert ora.max_abs(np64(lse), rl) <= 2e-3
    rq, rk, rv = ora.attention_bwd(np64(x["q"]), np64(x["k"]), np64(x["v"]), np64(x["o"]), np64(x["lse"]),
                                   np64(x["do"]), causal=causal)
    assert_close("dQ", np64(dq), rq)
    assert_close("dK", np64(dk), rk)
    assert_close("dV", np64(dv), rv)
    (rq2, rk2, rv2, rdo), (rd, rdd, rb) = oracle_bwdbwd(x, causal)
    assert_close("dD", np64(dd), rdd)
    assert_close("B", np64(bv), rb)
    assert_close("dQ2", np64(dq2), rq2)
    assert_close("dK2", np64(dk2), rk2)
    assert_close("dV2", np64(dv2), rv2)
    assert_close("ddO", np64(ddo), rdo)


HD128_CASES = [
    # b, h, tq, tk, causal -- head_dim 128 (the long-sequence and cross-attention configs)
    (1, 2, 128, 128, True),
    (1, 2, 256, 384, False),
    (1, 1, 200, 200, True),
    (1, 2, 72, 136, False),
    (2, 2, 512, 512, True),
    (2, 2, 512, 256, False),   # non-causal cross attention with more queries than keys (configuration 4's form)
]


@pytest.mark.parametrize("b,h,tq,tk,causal", HD128_CASES)
def test_bwdbwd_matches_oracle_hd128(b, h, tq, tk, causal):
    from flash_hog_b200 import MaskType, flash_bwdbwd
    from flash_hog_b200._capi import device_status

    x = case_inputs(b, h, tq, tk, d=128, seed=13 * tq + tk, causal=causal)
    (rq2, rk2, rv2, rdo), (rd, rdd, rb) = oracle_bwdbwd(x, causal)
    g = _cuda(x)
    mask = MaskType.CAUSAL if causal else MaskType.NO_MASK
    (dq2, dk2, dv2, ddo), (d, dd, bv) = flash_bwdbwd(g["q"], g["k"], g["v"], g["o"], g["do"], g["ddq"], g["ddk"],
                                                     g["ddv"], g["lse"], mask_type=mask, return_stats=True)
    torch.cuda.synchronize()
    assert device_status() == 0
    assert_close("D", np64(d), rd)
    assert_close("dD", np64(dd), rdd)
    assert_close("B", np64(bv), rb)
    assert_close("dQ2", np64(dq2), rq2)
    assert_close("dK2", np64(dk2), rk2)
    assert_close("dV2", np64(dv2), rv2)
    assert_close("ddO", np64(ddo), rdo)


@pytest.mark.parametrize("b,h,tq,tk,causal", HD128_CASES)
def test_fwd_bwd_match_oracle_hd128(b, h, tq, tk, causal):
    from flash_hog_b200 import MaskType
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200._capi import device_status

    x = case_inputs(b, h, tq, tk, d=128, seed=5 * tq + tk, causal=causal)
    g = _cuda(x)
    mask = MaskType.CAUSAL if causal else MaskType.NO_MASK
    scale = 128 ** -0.5
    out, lse = impl.cuda_dot_product_attention(g["q"], g["k"], g["v"], mask, scale, return_residual=True)
    torch.cuda.synchronize()
    assert device_status() == 0
    ro, rl = ora.attention_fwd(np64(x["q"]), np64(x["k"]), np64(x["v"]), causal=causal)
    assert_close("O", np64(out), ro)
    assert ora.max_abs(np64(lse), rl) <= 2e-3
    dq, dk, dv = impl.dot_product_attention_bwd_rule(mask, scale, (g["q"], g["k"], g["v"], g["lse"], g["o"]),
                                                     g["do"])
    torch.cuda.synchronize()
    assert device_status() == 0
    rq, rk, rv = ora.attention_bwd(np64(x["q"]), np64(x["k"]), np64(x["v"]), np64(x["o"]), np64(x["lse"]),
                                   np64(x["do"]), causal=causal)
    assert_close("dQ", np64(dq), rq)
    assert_close("dK", np64(dk), rk)
    assert_close("dV", np64(dv), rv)


@pytest.mark.parametrize("causal,kv_heads,d", [(True, 2, 64), (False, 2, 64), (True, 1, 64), (True, 2, 128)])
def test_nested_autograd_matches_double_autograd(causal, kv_heads, d):
    """grad-of-grad through the public API vs torch double autograd of naive
    attention (kv_heads < 2: grouped-query attention)."""
    import flash_hog_b200 as fhb

    x = ora.make_inputs(2, 2, 256, 256, d, seed=5, kv_heads=kv_heads)
    ref = ora.autograd_all(*(x[n].double() for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")), causal=causal)
    q, k, v, do = (x[n].cuda().requires_grad_(True) for n in ("q", "k", "v", "do"))
    out = fhb.dot_product_attention(q, k, v, is_causal=causal)
    dq, dk, dv = torch.autograd.grad(out, (q, k, v), do, create_graph=True)
    dq2, dk2, dv2, ddo = torch.autograd.grad((dq, dk, dv), (q, k, v, do),
                                             (x["ddq"].cuda(), x["ddk"].cuda(), x["ddv"].cuda()))
    torch.cuda.synchronize()
    for name, got in dict(o=out, dq=dq, dk=dk, dv=dv, dq2=dq2, dk2=dk2, dv2=dv2, ddo=ddo).items():
        assert_close(name, np64(got), ref[name].numpy())


def test_unbatched_and_bhtd_layouts():
    """TNH inputs (reference's unbatched form) and BHTD-strided views give the BTNH results."""
    from flash_hog_b200 import MaskType, flash_bwdbwd

    x = _cuda(case_inputs(1, 2, 256, 256, seed=3, causal=True))
    args = [x[n] for n in ("q", "k", "v", "o", "do", "ddq", "ddk", "ddv")]
    full = flash_bwdbwd(*args, x["lse"], mask_type=MaskType.CAUSAL)
    unb = flash_bwdbwd(*(a[0] for a in args), x["lse"][0], mask_type=MaskType.CAUSAL)
    # BHTD storage, presented to the kernels as a strided BTNH view
    bhtd = [a.transpose(1, 2).contiguous().transpose(1, 2) for a in args]
    from flash_hog_b200 import _capi
    q, k, v, o, do, ddq, ddk, ddv = bhtd
    delta = torch.empty_like(x["lse"])
    dd, bv = torch.empty_like(delta), torch.empty_like(delta)
    dq2, ddo = torch.empty_like(q), torch.empty_like(q)
    dk2, dv2 = torch.empty_like(k), torch.empty_like(k)
    _capi.attn_bwdbwd_o(q, k, v, o, do, ddq, ddk, ddv, x["lse"], dq2, ddo, dk2, dv2, delta, dd, bv, 0.125, True)
    # The delta-input entry (D from fh_attn_rowdot) sums D in another order: equal
    # up to bf16 rounding of the outputs.
    delta_r, dd_r, bv_r = (torch.empty_like(delta) for _ in range(3))
    r2 = [torch.empty_like(t) for t in (dq2, ddo, dk2, dv2)]
    _capi.attn_rowdot(o, do, delta_r)
    _capi.attn_bwdbwd(q, k, v, do, ddq, ddk, ddv, x["lse"], delta_r, r2[0], r2[1], r2[2], r2[3], dd_r, bv_r,
                      0.125, True)
    torch.cuda.synchronize()
    for a, u, s in zip(full, unb, (dq2, dk2, dv2, ddo)):
        assert torch.equal(a[0], u)
        assert torch.equal(a, s)
    assert torch.allclose(delta_r, delta, rtol=1e-5, atol=1e-5)
    for got, ref in zip(r2, (dq2, ddo, dk2, dv2)):
        err = (got.float() - ref.float()).abs().max().item() / ref.float().abs().max().item()
        assert err < 1e-2, err


def test_headline_config_full_size_sampled_heads():
    """B4 H16 S2048 D64 causal at full size; oracle on sampled (batch, head) pairs;
    determinism (bitwise) and batch x heads sharding (a shard's result equals the
    matching slice of the full run, bit for bit)."""
    from flash_hog_b200 import MaskType, flash_bwdbwd

    b, h, s = 4, 16, 2048
    x = ora.make_inputs(b, h, s, s, 64, seed=0)
    g = _cuda(x)
    from flash_hog_b200 import _attention_impl as impl
    o, lse = impl.cuda_dot_product_attention(g["q"], g["k"], g["v"], MaskType.CAUSAL, 0.125, return_residual=True)
    args = [g[n] for n in ("q", "k", "v")] + [o] + [g[n] for n in ("do", "ddq", "ddk", "ddv")] + [lse]
    out1 = flash_bwdbwd(*args, mask_type=MaskType.CAUSAL)
    out2 = flash_bwdbwd(*args, mask_type=MaskType.CAUSAL)
    torch.cuda.synchronize()
    for a1, a2 in zip(out1, out2):
        assert torch.equal(a1, a2), "double backward is not deterministic"
    # sharding: batch 1..2 and heads 4..11 as an independent call
    sl = [a[1:3, :, 4:12].contiguous() for a in args[:-1]] + [lse[1:3, 4:12].contiguous()]
    shard = flash_bwdbwd(*sl, mask_type=MaskType.CAUSAL)
    torch.cuda.synchronize()
    for full, part in zip(out1, shard):
        assert torch.equal(full[1:3, :, 4:12], part)
    heads = [(0, 0), (3, 15), (2, 7), (1, 3), (0, 11), (3, 0), (2, 14), (1, 8)]
    arrs = {n: select_heads(x[n], heads) for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")}
    want, _ = ora.bwdbwd_stats_rows(arrs["q"], arrs["k"], arrs["v"], select_heads(o, heads),
                                    select_heads(lse, heads, stat=True), arrs["do"], arrs["ddq"], arrs["ddk"],
                                    arrs["ddv"], causal=True)
    for name, got, ref in zip(("dQ2", "dK2", "dV2", "ddO"), out1, want):
        assert_close(name, select_heads(got, heads), ref)
        assert_elementwise(name, select_heads(got, heads), ref)


def test_golden_inputs_through_the_bf16_kernels():
    """The reference's own known-answer vectors (``test_data.zip``, written by
    ``flash_hog/_jax_refs/jax_impl.py:404-477``: bf16 Q, K, V, dO, ddQ, ddK, ddV with
    fp32 O and L, non-causal, Nq 128, Nk 256, scale 1/8) through the bf16 tensor-core
    double backward: with D = rowsum(dO o O) from the stored fp32 O (the reference
    computes D in fp32 too) via ``fh_attn_bwdbwd``, and with O rounded to bf16 via the
    fused ``fh_attn_bwdbwd_o``. Both match the stored outputs to 1e-2 max-abs."""
    import os

    from flash_hog_b200 import _capi

    d = np.load(os.path.join(os.path.dirname(__file__), "golden", "kat_bwdbwd.npz"))
    bf = lambda n: torch.from_numpy(d[n + "_bf16"].view(np.int16)).view(torch.bfloat16)[None, :, None].cuda()
    q, k, v, do, ddq, ddk, ddv = (bf(n) for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv"))
    o32 = torch.from_numpy(d["o"])[None, :, None].cuda()
    lse = torch.from_numpy(d["L"])[None, None].cuda().contiguous()
    scale = float(d["scale"])
    assert not bool(d["causal"])
    delta = (do.float() * o32).sum(-1).permute(0, 2, 1).contiguous()
    outs = [torch.empty_like(q), torch.empty_like(q), torch.empty_like(k), torch.empty_like(k)]
    dd, bv = torch.empty_like(delta), torch.empty_like(delta)
    _capi.attn_bwdbwd(q, k, v, do, ddq, ddk, ddv, lse, delta, outs[0], outs[1], outs[2], outs[3], dd, bv, scale, 0)
    fused = [torch.empty_like(t) for t in outs]
    delta2, dd2, bv2 = (torch.empty_like(delta) for _ in range(3))
    _capi.attn_bwdbwd_o(q, k, v, o32.to(torch.bfloat16), do, ddq, ddk, ddv, lse, fused[0], fused[1], fused[2],
                        fused[3], delta2, dd2, bv2, scale, 0)
    torch.cuda.synchronize()
    assert _capi.device_status() == 0
    for variant in (outs, fused):
        for name, got in zip(("dq2", "ddo", "dk2", "dv2"), variant):
            got = np64(got)[0, :, 0]
            ref = d[name].astype(np.float64)
            assert ora.max_abs(got, ref) <= 1e-2, f"{name}: max abs {ora.max_abs(got, ref):.3e}"
            assert ora.rel_err(got, ref) <= 2e-2, f"{name}: rel err {ora.rel_err(got, ref):.3e}"


def test_device_status_clean_and_fp32_inputs():
    """fp32 inputs run the fp32-product kernels and the result returns in fp32 (held
    here to the bf16 bar; ``tests/test_f32.py`` holds them to 1e-3); no device error
    is recorded."""
    import flash_hog_b200 as fhb
    from flash_hog_b200._capi import device_status

    x = ora.make_inputs(1, 2, 256, 256, 64, seed=9, dtype=torch.float32)
    q, k, v = (x[n].cuda() for n in ("q", "k", "v"))
    out = fhb.dot_product_attention(q, k, v, is_causal=True)
    assert out.dtype == torch.float32
    ro, _ = ora.attention_fwd(np64(x["q"]), np64(x["k"]), np64(x["v"]), causal=True)
    assert_close("O fp32-in", np64(out), ro)
    assert device_status() == 0


def test_sharded_entry_slices_equal_the_full_run():
    """sharded_flash_bwdbwd for each rank of a 4-way split (emulated one rank after the
    other on this GPU; grouped-query heads, so key heads split with their groups): every
    rank's result is the matching slice of the unsharded call, bit for bit."""
    from flash_hog_b200 import MaskType, flash_bwdbwd
    from flash_hog_b200.sharding import sharded_flash_bwdbwd

    x = _cuda(case_inputs(2, 8, 256, 384, d=128, seed=8, causal=False, kv_heads=4))
    args = [x[n] for n in ("q", "k", "v", "o", "do", "ddq", "ddk", "ddv", "lse")]
    full = flash_bwdbwd(*args, mask_type=MaskType.NO_MASK)
    host = [a.cpu() for a in args]  # the global batch as a caller would hold it
    for rank in range(4):
        part, sh = sharded_flash_bwdbwd(*host, mask_type=MaskType.NO_MASK, rank=rank, world=4)
        sb, hs = sh.slices(rank)
        ks = sh.kv_slice(rank)
        for i, (f, p) in enumerate(zip(full, part)):
            assert torch.equal(f[sb, :, ks if i in (1, 2) else hs], p), (rank, i)
