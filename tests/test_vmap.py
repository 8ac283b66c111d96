"""Batching rules: ``torch.func.vmap`` over ``flash_bwdbwd`` and the public op.

The reference gives its double backward a ``custom_vmap`` rule that folds the vmapped
axis into the batch axis (``flash_hog/jax/_pallas_gpu.py:85-102``). Here
``flash_bwdbwd`` is a torch operator with that rule, and the two autograd Functions
of ``dot_product_attention`` have ``vmap`` staticmethods doing the same.

CPU tests replace the device calls with the float64 oracle (the host logic of the
rules -- moving, folding, broadcasting and unfolding axes -- is what they check); GPU
tests check the kernels under vmap against per-slice calls, bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora


def _np(x):
    return x.detach().double().numpy()


def _oracle_bwdbwd_device(Q, K, V, O, dO, ddQ, ddK, ddV, L, causal, window, scale, policy=None, packed=None):
    b, t, n, _ = Q.shape
    outs, stats = ora.bwdbwd_stats(*(_np(x) for x in (Q, K, V, O)), L.reshape(b, n, t).double().numpy(),
                                   *(_np(x) for x in (dO, ddQ, ddK, ddV)), scale=scale, causal=causal, window=window,
                                   return_stats=True)
    return tuple(torch.from_numpy(x).to(Q.dtype) for x in outs) + (torch.from_numpy(np.stack(stats)).float(),)


def _oracle_fwd(query, key, value, mask_type, scale, return_residual=False, policy=None):
    from flash_hog_b200._attention_impl import _mask_args

    causal, window = _mask_args(mask_type)
    o, lse = ora.attention_fwd(_np(query), _np(key), _np(value), scale=scale, causal=causal, window=window)
    out = torch.from_numpy(o).to(query.dtype)
    return (out, torch.from_numpy(lse).float()) if return_residual else out


def _oracle_bwd(mask_type, scale, res, g, policy=None):
    from flash_hog_b200._attention_impl import _mask_args

    query, key, value, activation, out = res
    causal, window = _mask_args(mask_type)
    grads = ora.attention_bwd(*(_np(x) for x in (query, key, value, out)), _np(activation), _np(g), scale=scale,
                              causal=causal, window=window)
    return tuple(torch.from_numpy(x).to(query.dtype) for x in grads)


@pytest.fixture
def oracle_device(monkeypatch):
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200 import bwdbwd as bb

    monkeypatch.setattr(bb, "_bwdbwd_device", _oracle_bwdbwd_device)
    monkeypatch.setattr(impl, "cuda_dot_product_attention", _oracle_fwd)
    monkeypatch.setattr(impl, "dot_product_attention_bwd_rule", _oracle_bwd)


def _stacked_inputs(nv, b, h, t, s, d, dtype=torch.float64, seed=0):
    """Seven stacked input sets (a leading vmapped axis of size nv) plus O and L."""
    xs = [ora.make_inputs(b, h, t, s, d, seed=seed + i, dtype=dtype) for i in range(nv)]
    st = {n: torch.stack([x[n] for x in xs]) for n in xs[0]}
    o, lse = zip(*(ora.attention_fwd(*(_np(x[n]) for n in ("q", "k", "v")), causal=1) for x in xs))
    st["o"] = torch.from_numpy(np.stack(o)).to(dtype)
    st["lse"] = torch.from_numpy(np.stack(lse)).float()
    return st


NAMES = ("q", "k", "v", "o", "do", "ddq", "ddk", "ddv", "lse")


def test_fold_and_unfold_axes():
    from flash_hog_b200._attention_impl import _fold, _unfold

    x = torch.arange(2 * 3 * 5 * 4).reshape(3, 2, 5, 4)  # vmapped axis 1 (size 2), batch 3
    f = _fold(x, 1, 2)
    assert f.shape == (6, 5, 4)
    assert torch.equal(f[3:], x[:, 1])
    assert torch.equal(_unfold(f, 2), x.movedim(1, 0))
    b = _fold(torch.ones(3, 5), None, 4)  # not vmapped: broadcast
    assert b.shape == (12, 5)


def test_vmap_rule_of_flash_bwdbwd_folds_into_batch(oracle_device):
    from flash_hog_b200.bwdbwd import flash_bwdbwd

    st = _stacked_inputs(3, 2, 2, 24, 40, 16)
    fn = lambda *a: flash_bwdbwd(*a, mask_type=__import__("flash_hog_b200").MaskType.CAUSAL, scale=0.25)
    got = torch.func.vmap(fn)(*(st[n] for n in NAMES))
    for i in range(3):
        want = fn(*(st[n][i] for n in NAMES))
        for g, w in zip(got, want):
            assert torch.equal(g[i], w)
    # vmapped axis not first, and one input not vmapped (broadcast)
    moved = [st[n].movedim(0, 1) for n in NAMES]
    in_dims = (1,) * 8 + (None,)
    moved[8] = st["lse"][0]
    got = torch.func.vmap(fn, in_dims=in_dims)(*moved)
    for i in range(3):
        want = fn(*(st[n][i] for n in NAMES[:8]), st["lse"][0])
        for g, w in zip(got, want):
            assert torch.equal(g[i], w)


def test_nested_vmap_of_flash_bwdbwd(oracle_device):
    from flash_hog_b200 import MaskType
    from flash_hog_b200.bwdbwd import flash_bwdbwd

    st = _stacked_inputs(4, 1, 2, 16, 16, 16)
    grid = {n: st[n].reshape(2, 2, *st[n].shape[1:]) for n in NAMES}
    fn = lambda *a: flash_bwdbwd(*a, mask_type=MaskType.CAUSAL, scale=0.25)
    got = torch.func.vmap(torch.func.vmap(fn))(*(grid[n] for n in NAMES))
    want = fn(*(st[n][3] for n in NAMES))
    for g, w in zip(got, want):
        assert torch.equal(g[1, 1], w)


def test_vmap_of_public_op_and_its_gradients(oracle_device):
    from flash_hog_b200.attention import dot_product_attention

    st = _stacked_inputs(3, 1, 2, 20, 20, 16)
    q, k, v, do = (st[n] for n in ("q", "k", "v", "do"))
    attn = lambda q_, k_, v_: dot_product_attention(q_, k_, v_, is_causal=True)
    out = torch.func.vmap(attn)(q, k, v)
    for i in range(3):
        assert torch.equal(out[i], attn(q[i], k[i], v[i]))

    # reverse mode under vmap: the backward Function's batching rule
    phi = lambda q_, k_, v_, do_: (attn(q_, k_, v_) * do_).sum()
    grads = torch.func.vmap(torch.func.grad(phi, argnums=(0, 1, 2)))(q, k, v, do)
    for i in range(3):
        ref = ora.attention_bwd(*(_np(x[i]) for x in (q, k, v, st["o"])), _np(st["lse"][i]), _np(do[i]), causal=1)
        for g, r in zip(grads, ref):
            assert ora.max_abs(_np(g[i]), r) < 1e-10

    # second order under vmap: the gradient of <dQ, ddQ> reaches flash_bwdbwd's rule
    ddq = st["ddq"]

    def dq_dot(q_, k_, v_, do_, ddq_):
        dq = torch.func.grad(phi, argnums=0)(q_, k_, v_, do_)
        return (dq * ddq_).sum()

    g2 = torch.func.vmap(torch.func.grad(dq_dot, argnums=(0, 1, 2, 3)))(q, k, v, do, ddq)
    for i in range(3):
        z = torch.zeros_like(st["ddk"][i])
        ref = ora.bwdbwd_stats(*(_np(x[i]) for x in (q, k, v, st["o"])), _np(st["lse"][i]), _np(do[i]), _np(ddq[i]),
                               _np(z), _np(z), causal=1)
        for g, r in zip(g2, ref):  # (dQ2, dK2, dV2, ddO)
            assert ora.max_abs(_np(g[i]), r) < 1e-10


@pytest.mark.gpu
def test_vmap_of_flash_bwdbwd_on_the_kernels_is_bitwise_per_slice():
    from flash_hog_b200 import MaskType
    from flash_hog_b200.bwdbwd import flash_bwdbwd
    from flash_hog_b200 import _attention_impl as impl

    st = _stacked_inputs(3, 2, 4, 256, 256, 64, dtype=torch.bfloat16, seed=7)
    c = {n: st[n].cuda() for n in NAMES}
    o, lse = impl.cuda_dot_product_attention(*(c[n].flatten(0, 1) for n in ("q", "k", "v")), MaskType.CAUSAL, 0.125,
                                             return_residual=True)
    c["o"], c["lse"] = o.unflatten(0, (3, 2)), lse.unflatten(0, (3, 2))
    fn = lambda *a: flash_bwdbwd(*a, mask_type=MaskType.CAUSAL, scale=0.125)
    got = torch.func.vmap(fn)(*(c[n] for n in NAMES))
    for i in range(3):
        want = fn(*(c[n][i] for n in NAMES))
        for g, w in zip(got, want):
            assert torch.equal(g[i], w)


@pytest.mark.gpu
def test_vmap_of_hessian_vector_products_on_the_kernels():
    """vmap over a grad-of-grad of the public op (fp32 inputs, so the result can be held
    to 1e-3 of the float64 oracle per slice)."""
    from flash_hog_b200.attention import dot_product_attention

    st = _stacked_inputs(2, 1, 2, 128, 192, 64, dtype=torch.float32, seed=3)
    c = {n: st[n].cuda() for n in ("q", "k", "v", "do", "ddq")}
    phi = lambda q_, k_, v_, do_: (dot_product_attention(q_, k_, v_) * do_).sum()

    def dq_dot(q_, k_, v_, do_, ddq_):
        return (torch.func.grad(phi, argnums=0)(q_, k_, v_, do_) * ddq_).sum()

    g2 = torch.func.vmap(torch.func.grad(dq_dot, argnums=(0, 1, 2, 3)))(c["q"], c["k"], c["v"], c["do"], c["ddq"])
    for i in range(2):
        a = {n: _np(st[n][i]) for n in ("q", "k", "v", "do", "ddq")}
        o, lse = ora.attention_fwd(a["q"], a["k"], a["v"])
        z = np.zeros_like(a["k"])
        ref = ora.bwdbwd_stats(a["q"], a["k"], a["v"], o, lse, a["do"], a["ddq"], z, z)
        for g, r in zip(g2, ref):
            assert ora.rel_err(_np(g[i].cpu()), r) <= 1e-3
