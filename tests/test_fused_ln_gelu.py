"""Fused LayerNorm and GELU (forward, backward, double backward) of the GPT step.

CPU: the closed forms of ``oracle/ln_gelu_oracle.py`` (what the kernels evaluate)
against torch's double autograd of ``layer_norm`` / ``gelu`` in float64.
GPU: the kernels through the C ABI and the autograd Functions of
``flash_hog_b200.fused`` against the same torch double autograd.
"""

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import ln_gelu_oracle as lno

# rows, cols: a multiple of 128, one that is not, and the GPT width
SHAPES = [(64, 128), (37, 200), (300, 768)]


def _ln_case(rows, cols, seed, dtype=torch.float64):
    g = torch.Generator().manual_seed(seed)
    r = lambda *s: torch.randn(*s, generator=g, dtype=dtype)
    return dict(x=r(rows, cols) * 2 + 0.5, w=r(cols), b=r(cols), dy=r(rows, cols), u=r(rows, cols), vb=r(cols),
                cb=r(cols))


def _torch_ln_second_order(c, eps=1e-5):
    x, w, b, dy = (c[n].clone().requires_grad_(True) for n in ("x", "w", "b", "dy"))
    y = F.layer_norm(x, (x.shape[-1],), w, b, eps)
    dx, dw, db = torch.autograd.grad(y, (x, w, b), dy, create_graph=True)
    gx, gw, gdy = torch.autograd.grad((dx, dw, db), (x, w, dy), (c["u"], c["vb"], c["cb"]))
    return y.detach(), (dx.detach(), dw.detach(), db.detach()), (gx, gw, gdy)


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


@pytest.mark.parametrize("rows,cols", SHAPES)
def test_layernorm_closed_forms_match_torch_double_autograd(rows, cols):
    c = _ln_case(rows, cols, seed=rows + cols)
    y, first, second = _torch_ln_second_order(c)
    n = {k: v.numpy() for k, v in c.items()}
    assert _rel(lno.layernorm_fwd(n["x"], n["w"], n["b"])[0], y) < 1e-12
    for got, want in zip(lno.layernorm_bwd(n["x"], n["w"], n["dy"]), first):
        assert _rel(got, want) < 1e-12
    for got, want in zip(lno.layernorm_bwd_bwd(n["x"], n["w"], n["dy"], n["u"], n["vb"], n["cb"]), second):
        assert _rel(got, want) < 1e-10


def test_gelu_closed_forms_match_torch_double_autograd():
    g = torch.Generator().manual_seed(3)
    a = (torch.randn(4000, generator=g, dtype=torch.float64) * 3).requires_grad_(True)
    dh = torch.randn(4000, generator=g, dtype=torch.float64).requires_grad_(True)
    c = torch.randn(4000, generator=g, dtype=torch.float64)
    h = F.gelu(a)
    (da,) = torch.autograd.grad(h, a, dh, create_graph=True)
    ga, gdh = torch.autograd.grad(da, (a, dh), c)
    v, d1, d2 = lno.gelu_terms(a.detach().numpy())
    assert _rel(v, h.detach()) < 1e-12
    assert _rel(dh.detach().numpy() * d1, da.detach()) < 1e-12
    assert _rel(c.numpy() * d1, gdh) < 1e-12
    assert _rel(c.numpy() * dh.detach().numpy() * d2, ga) < 1e-10


@pytest.mark.gpu
@pytest.mark.parametrize("rows,cols", SHAPES)
def test_layernorm_kernels(rows, cols):
    """fp32 kernels against float64 torch: forward, backward, double backward (also
    with absent cotangents), through the public autograd Functions."""
    from flash_hog_b200 import fused

    c = _ln_case(rows, cols, seed=7 * rows + cols)
    y64, first64, second64 = _torch_ln_second_order(c)
    g = {k: v.float().cuda() for k, v in c.items()}
    x, w, b, dy = (g[n].clone().requires_grad_(True) for n in ("x", "w", "b", "dy"))
    y = fused.layer_norm(x, w, b)
    dx, dw, db = torch.autograd.grad(y, (x, w, b), dy, create_graph=True)
    gx, gw, gdy = torch.autograd.grad((dx, dw, db), (x, w, dy), (g["u"], g["vb"], g["cb"]))
    torch.cuda.synchronize()
    assert _rel(y.detach().cpu(), y64) < 2e-6
    for got, want in zip((dx, dw, db), first64):
        assert _rel(got.detach().cpu(), want) < 2e-5
    for name, got, want in zip(("gx", "gw", "gdy"), (gx, gw, gdy), second64):
        assert _rel(got.cpu(), want) < 1e-4, name
    # Only dx receives a cotangent (dw, db unused): the closed form with vb = cb = 0.
    x2, w2, b2, dy2 = (g[n].clone().requires_grad_(True) for n in ("x", "w", "b", "dy"))
    dx2, _, _ = torch.autograd.grad(fused.layer_norm(x2, w2, b2), (x2, w2, b2), dy2, create_graph=True)
    gx2, gw2, gdy2 = torch.autograd.grad(dx2, (x2, w2, dy2), g["u"])
    n = {k: v.numpy() for k, v in c.items()}
    want = lno.layernorm_bwd_bwd(n["x"], n["w"], n["dy"], n["u"])
    for got, w_ in zip((gx2, gw2, gdy2), want):
        assert _rel(got.cpu(), w_) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 1e-2)])
def test_gelu_kernels(dtype, tol):
    from flash_hog_b200 import fused

    gen = torch.Generator().manual_seed(11)
    a64 = torch.randn(3, 1000, generator=gen, dtype=torch.float64) * 3
    dh64 = torch.randn(3, 1000, generator=gen, dtype=torch.float64)
    c64 = torch.randn(3, 1000, generator=gen, dtype=torch.float64)
    # torch reference on the values the kernels see (inputs rounded to the dtype)
    a_r, dh_r, c_r = (t.to(dtype).double() for t in (a64, dh64, c64))
    v, d1, d2 = (torch.from_numpy(t) for t in lno.gelu_terms(a_r.numpy()))
    a = a_r.to(dtype).cuda().requires_grad_(True)
    dh = dh_r.to(dtype).cuda().requires_grad_(True)
    h = fused.gelu(a)
    (da,) = torch.autograd.grad(h, a, dh, create_graph=True)
    ga, gdh = torch.autograd.grad(da, (a, dh), c_r.to(dtype).cuda())
    assert h.dtype == dtype and da.dtype == dtype and ga.dtype == dtype
    assert _rel(h.detach().double().cpu(), v) < tol
    assert _rel(da.detach().double().cpu(), dh_r * d1) < tol
    assert _rel(gdh.double().cpu(), c_r * d1) < tol
    assert _rel(ga.double().cpu(), c_r * dh_r * d2) < tol


def _torch_xent_second_order(z, t, u):
    """torch float64: loss, dz (= d loss / dz) and the cotangents of z and of the upstream
    scalar g for the cotangent u of dz."""
    z = z.clone().requires_grad_(True)
    g = torch.ones((), dtype=z.dtype, requires_grad=True)
    loss = F.cross_entropy(z, t)
    (dz,) = torch.autograd.grad(loss, z, g, create_graph=True)
    gz, gg = torch.autograd.grad(dz, (z, g), u)
    return loss.detach(), dz.detach(), gz, gg


@pytest.mark.parametrize("rows,vocab", [(5, 37), (16, 512)])
def test_xent_closed_forms_match_torch_double_autograd(rows, vocab):
    gen = torch.Generator().manual_seed(rows + vocab)
    z = torch.randn(rows, vocab, generator=gen, dtype=torch.float64) * 3
    t = torch.randint(0, vocab, (rows,), generator=gen)
    u = torch.randn(rows, vocab, generator=gen, dtype=torch.float64)
    loss, dz, gz, gg = _torch_xent_second_order(z, t, u)
    lse, loss_r = lno.xent_fwd(z.numpy(), t.numpy())
    assert abs(loss_r.mean() - float(loss)) < 1e-12
    assert _rel(lno.xent_bwd(z.numpy(), t.numpy(), 1.0, 1.0 / rows), dz) < 1e-12
    gz_o, gg_o = lno.xent_bwd_bwd(z.numpy(), t.numpy(), 1.0, 1.0 / rows, u.numpy())
    assert _rel(gz_o, gz) < 1e-10
    assert abs(gg_o - float(gg)) < 1e-10 * max(1.0, abs(float(gg)))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,tol", [(torch.float32, 2e-5), (torch.bfloat16, 1e-2)])
@pytest.mark.parametrize("rows,vocab,pad", [(64, 1000, 0), (33, 517, 0), (48, 768, 24)])
def test_xent_kernels(dtype, tol, rows, vocab, pad):
    """Forward, backward and backward's backward through the autograd Functions against
    torch float64 on the values the kernels see; vocab not a multiple of 8 (scalar tail)
    and a row stride above vocab (pad) included."""
    from flash_hog_b200 import fused

    gen = torch.Generator().manual_seed(rows * vocab + pad)
    zfull = (torch.randn(rows, vocab + pad, generator=gen) * 3).to(dtype)
    t = torch.randint(0, vocab, (rows,), generator=gen)
    u = torch.randn(rows, vocab, generator=gen).to(dtype)
    z64 = zfull[:, :vocab].double()
    loss64, dz64, gz64, gg64 = _torch_xent_second_order(z64, t, u.double())
    zg = zfull.cuda()[:, :vocab].requires_grad_(True)
    assert zg.stride(0) == vocab + pad
    g = torch.ones((), device="cuda", requires_grad=True)
    loss = fused.cross_entropy(zg, t.cuda())
    (dz,) = torch.autograd.grad(loss, zg, g, create_graph=True)
    gz, gg = torch.autograd.grad(dz, (zg, g), u.cuda())
    torch.cuda.synchronize()
    assert dz.dtype == dtype and gz.dtype == dtype
    assert abs(float(loss) - float(loss64)) < 1e-5 * max(1.0, abs(float(loss64)))
    assert _rel(dz.detach().double().cpu(), dz64) < tol
    assert _rel(gz.double().cpu(), gz64) < tol
    assert abs(float(gg) - float(gg64)) < 1e-4 * max(1.0, abs(float(gg64)))


@pytest.mark.gpu
def test_xent_targets_outside_the_vocabulary():
    """A target outside [0, vocab) is caught by the kernels' own bounds check: its row's
    loss is NaN and its gradient has no one-hot term (softmax / rows); other rows are
    unaffected."""
    from flash_hog_b200 import _capi

    rows, vocab = 4, 40
    z = torch.randn(rows, vocab, generator=torch.Generator().manual_seed(3)).cuda()
    t = torch.tensor([3, -1, vocab, 7], dtype=torch.int64, device="cuda")
    lse = torch.empty(rows, device="cuda")
    loss = torch.empty(rows, device="cuda")
    _capi.xent_fwd(z, t, lse, loss)
    g = torch.ones(1, device="cuda")
    dz = torch.empty_like(z)
    _capi.xent_bwd(z, t, lse, g, 1.0 / rows, dz)
    torch.cuda.synchronize()
    assert torch.isnan(loss[1]) and torch.isnan(loss[2])
    ref = torch.nn.functional.cross_entropy(z[[0, 3]].double().cpu(), t[[0, 3]].cpu(), reduction="none")
    assert torch.allclose(loss[[0, 3]].double().cpu(), ref, rtol=1e-5, atol=1e-5)
    p = torch.softmax(z.double(), -1).cpu() / rows
    assert torch.allclose(dz[1:3].double().cpu(), p[1:3], rtol=1e-4, atol=1e-7)
