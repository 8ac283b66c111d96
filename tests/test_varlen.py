"""Packed variable-length batches (cu_seqlens) through the C ABI and the public API.

The reference's JAX statements give every (qs, ks) pair its own bottom-right
mask and sliding window (``flash_hog/_jax_refs/jax_impl.py:104-130``). Here such
pairs are packed into one call: sequence b is query rows [cu_q[b], cu_q[b+1])
against key rows [cu_k[b], cu_k[b+1]). Each sequence's results must equal, bit
for bit, the dense call on that sequence alone (the kernels tile every sequence
from its own first row), and the CPU oracle evaluated per sequence within the
bf16 bar. Edge cases: ragged lengths, a sequence with no queries, one with no
keys (its queries get O = 0, L = -inf and zero gradients), grouped-query heads,
head_dim 128, a sliding window, and all three masks.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from parity_util import assert_close, np64

# (query lengths, key lengths, causal code, window, heads, kv heads, head_dim)
CASES = [
    ([200, 64, 333], [150, 300, 333], 2, 0, 2, 2, 64),
    ([128, 0, 77, 256], [128, 40, 0, 300], 1, 48, 4, 2, 128),
    ([96, 300], [500, 64], 0, 0, 2, 1, 64),
]


def _packed_inputs(lq, lk, h, hk, d, seed):
    g = torch.Generator().manual_seed(seed)
    tq, tk = sum(lq), sum(lk)
    mk = lambda t, n: torch.randn((1, t, n, d), generator=g).to(torch.bfloat16)
    x = dict(q=mk(tq, h), k=mk(tk, hk), v=mk(tk, hk), do=mk(tq, h), ddq=mk(tq, h), ddk=mk(tk, hk), ddv=mk(tk, hk))
    cq = torch.tensor(np.concatenate([[0], np.cumsum(lq)]), dtype=torch.int32)
    ck = torch.tensor(np.concatenate([[0], np.cumsum(lk)]), dtype=torch.int32)
    return x, cq, ck


def _seq(t, c, b):
    """Rows of sequence b of a packed (1, total, ...) tensor."""
    return t[:, int(c[b]):int(c[b + 1])]


@pytest.mark.gpu
@pytest.mark.parametrize("lq,lk,causal,window,h,hk,d", CASES)
def test_packed_batch_equals_per_sequence_calls(lq, lk, causal, window, h, hk, d):
    from flash_hog_b200 import _capi

    x, cq, ck = _packed_inputs(lq, lk, h, hk, d, seed=sum(lq) + d)
    g = {n: t.cuda() for n, t in x.items()}
    vl = _capi.Varlen(cq.cuda(), ck.cuda(), max(lq), max(lk))
    scale = d ** -0.5
    tq = sum(lq)
    o, lse = torch.empty_like(g["q"]), torch.empty((1, h, tq), dtype=torch.float32, device="cuda")
    _capi.attn_fwd(g["q"], g["k"], g["v"], o, lse, scale, causal, window, varlen=vl)
    dq, dk, dv = torch.empty_like(g["q"]), torch.empty_like(g["k"]), torch.empty_like(g["v"])
    delta = torch.empty_like(lse)
    _capi.attn_bwd(g["q"], g["k"], g["v"], o, g["do"], lse, dq, dk, dv, delta, scale, causal, window, varlen=vl)
    outs = [torch.empty_like(g["q"]), torch.empty_like(g["q"]), torch.empty_like(g["k"]), torch.empty_like(g["k"])]
    st = [torch.empty_like(lse) for _ in range(3)]
    _capi.attn_bwdbwd_o(g["q"], g["k"], g["v"], o, g["do"], g["ddq"], g["ddk"], g["ddv"], lse, *outs, *st, scale,
                        causal, window=window, varlen=vl)
    torch.cuda.synchronize()
    assert _capi.device_status() == 0
    dq2, ddo, dk2, dv2 = outs
    for b in range(len(lq)):
        qs = lambda t: _seq(t, cq, b)
        ks = lambda t: _seq(t, ck, b)
        ls = lse[:, :, int(cq[b]):int(cq[b + 1])]
        if lq[b] == 0:
            if lk[b]:  # keys no query sees: zero gradients
                for t in (dk, dv, dk2, dv2):
                    assert not ks(t).float().abs().max().item()
            continue
        if lk[b] == 0:  # queries that see no key
            assert torch.isinf(ls).all() and (ls < 0).all()
            for t in (o, dq, dq2, ddo):
                assert not qs(t).float().abs().max().item()
            continue
        # The dense call on this sequence alone.
        s = {n: (qs if n in ("q", "do", "ddq") else ks)(g[n]).contiguous() for n in g}
        o1, l1 = torch.empty_like(s["q"]), torch.empty((1, h, lq[b]), dtype=torch.float32, device="cuda")
        _capi.attn_fwd(s["q"], s["k"], s["v"], o1, l1, scale, causal, window)
        d1 = [torch.empty_like(s["q"]), torch.empty_like(s["k"]), torch.empty_like(s["v"])]
        _capi.attn_bwd(s["q"], s["k"], s["v"], o1, s["do"], l1, *d1, torch.empty_like(l1), scale, causal, window)
        r1 = [torch.empty_like(s["q"]), torch.empty_like(s["q"]), torch.empty_like(s["k"]), torch.empty_like(s["k"])]
        _capi.attn_bwdbwd_o(s["q"], s["k"], s["v"], o1, s["do"], s["ddq"], s["ddk"], s["ddv"], l1, *r1,
                            *[torch.empty_like(l1) for _ in range(3)], scale, causal, window=window)
        torch.cuda.synchronize()
        assert torch.equal(qs(o), o1) and torch.equal(ls, l1), f"sequence {b}: forward"
        for name, got, want in (("dQ", qs(dq), d1[0]), ("dK", ks(dk), d1[1]), ("dV", ks(dv), d1[2]),
                                ("dQ2", qs(dq2), r1[0]), ("ddO", qs(ddo), r1[1]), ("dK2", ks(dk2), r1[2]),
                                ("dV2", ks(dv2), r1[3])):
            assert torch.equal(got, want), f"sequence {b}: {name} differs from the dense call"
        # The oracle on this sequence, with its own mask.
        a = {n: np64(s[n].cpu()) for n in s}
        want = ora.bwdbwd_stats(a["q"], a["k"], a["v"], np64(o1.cpu()), np64(l1.cpu()), a["do"], a["ddq"], a["ddk"],
                                a["ddv"], causal=causal, window=window)
        for name, got, w in zip(("dQ2", "dK2", "dV2", "ddO"), (qs(dq2), ks(dk2), ks(dv2), qs(ddo)), want):
            assert_close(f"sequence {b} {name}", np64(got.cpu()), w)
        ro, rl = ora.attention_fwd(a["q"], a["k"], a["v"], causal=causal, window=window)
        assert_close(f"sequence {b} O", np64(o1.cpu()), ro)


@pytest.mark.gpu
def test_public_varlen_op_twice_differentiable():
    """``dot_product_attention_varlen`` differentiated twice equals the dense public op
    on each sequence, bit for bit (bottom-right mask per sequence)."""
    import flash_hog_b200 as fhb

    lq, lk = [150, 256, 40], [200, 256, 90]
    x, cq, ck = _packed_inputs(lq, lk, 2, 2, 64, seed=5)
    g = {n: t.cuda()[0] for n, t in x.items()}  # (total, heads, head_dim)
    q, k, v, do = (g[n].clone().requires_grad_(True) for n in ("q", "k", "v", "do"))
    out = fhb.dot_product_attention_varlen(q, k, v, cq.cuda(), ck.cuda(), max(lq), max(lk), is_causal=True,
                                           causal_alignment="bottom_right")
    grads = torch.autograd.grad(out, (q, k, v), do, create_graph=True)
    second = torch.autograd.grad(grads, (q, k, v, do), (g["ddq"], g["ddk"], g["ddv"]))
    for b in range(len(lq)):
        sq, sk = slice(int(cq[b]), int(cq[b + 1])), slice(int(ck[b]), int(ck[b + 1]))
        qb, kb, vb, dob = (t[sl].detach().clone().unsqueeze(0).requires_grad_(True)
                           for t, sl in ((q, sq), (k, sk), (v, sk), (do, sq)))
        ob = fhb.dot_product_attention(qb, kb, vb, is_causal=True, causal_alignment="bottom_right")
        gb = torch.autograd.grad(ob, (qb, kb, vb), dob, create_graph=True)
        sb = torch.autograd.grad(gb, (qb, kb, vb, dob), (g["ddq"][sq][None], g["ddk"][sk][None], g["ddv"][sk][None]))
        assert torch.equal(out[sq], ob[0])
        for got, want, sl in zip(grads, gb, (sq, sk, sk)):
            assert torch.equal(got[sl], want[0])
        for got, want, sl in zip(second, sb, (sq, sk, sk, sq)):
            assert torch.equal(got[sl], want[0])


def test_varlen_validation_without_a_gpu():
    """Argument checks that run before any CUDA call."""
    from flash_hog_b200 import _capi

    lib = _capi.lib()
    s = _capi.FhStrides(0, 64, 64)
    cu = (ctypes.c_int32 * 3)(0, 100, 200)
    p = ctypes.c_void_p(256)
    dims = _capi.FhAttnDims(2, 1, 200, 200, 64, s, s, 1, 0, ctypes.cast(cu, ctypes.c_void_p), None, 100, 100)
    assert lib.fh_attn_fwd(None, ctypes.byref(dims), p, p, p, p, p, ctypes.c_float(0.125), 1) == 1  # one cu missing
    assert b"cu_seqlens_q and cu_seqlens_k" in lib.fh_last_error()
    dims.cu_seqlens_k = ctypes.cast(cu, ctypes.c_void_p)
    dims.max_seqlen_q = 300  # longer than the packed rows
    assert lib.fh_attn_fwd(None, ctypes.byref(dims), p, p, p, p, p, ctypes.c_float(0.125), 1) == 1
    dims.max_seqlen_q = 100
    assert lib.fh_attn_fwd_f32(None, ctypes.byref(dims), p, p, p, p, p, ctypes.c_float(0.125), 1) == 2
    assert b"bf16" in lib.fh_last_error()
    with pytest.raises(ValueError):
        _capi.Varlen(torch.zeros(3, dtype=torch.int64), torch.zeros(3, dtype=torch.int32), 1, 1)
    with pytest.raises(ValueError):
        _capi.Varlen(torch.zeros(3, dtype=torch.int32), torch.zeros(4, dtype=torch.int32), 1, 1)
