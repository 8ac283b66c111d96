"""CPU statements of the LayerNorm, GELU and cross-entropy double backward -- TEST INFRASTRUCTURE ONLY.

Nothing in the product package imports this module; ``tests/`` use it as the
checker of ``flash_hog_b200/csrc/ln_gelu.cu`` and ``csrc/xent.cu``. The formulas are the closed forms
the kernels evaluate, restated in float64 numpy; ``tests/test_fused_ln_gelu.py``
checks them against torch's double autograd of ``layer_norm`` and ``gelu`` on the
CPU, and the kernels against torch on the GPU. (The reference has no model code:
these ops belong to the grad-norm-penalty model step, configuration 5.)
"""

from __future__ import annotations

import math

import numpy as np


def layernorm_fwd(x, w, b, eps=1e-5):
    """y = (x - mean) rstd w + b over the last dimension; returns (y, mean, rstd)."""
    x = np.asarray(x, np.float64)
    mu = x.mean(-1, keepdims=True)
    r = 1.0 / np.sqrt(((x - mu) ** 2).mean(-1, keepdims=True) + eps)
    return (x - mu) * r * w + b, mu[..., 0], r[..., 0]


def layernorm_bwd(x, w, dy, eps=1e-5):
    """(dx, dw, db): dx = r (g - mean(g) - xh mean(g xh)), g = dy w."""
    _, mu, r = layernorm_fwd(x, w, np.zeros_like(w), eps)
    mu, r = mu[..., None], r[..., None]
    xh = (x - mu) * r
    g = dy * w
    dx = r * (g - g.mean(-1, keepdims=True) - xh * (g * xh).mean(-1, keepdims=True))
    red = tuple(range(x.ndim - 1))
    return dx, (dy * xh).sum(red), dy.sum(red)


def layernorm_bwd_bwd(x, w, dy, u=None, vb=None, cb=None, eps=1e-5):
    """Gradient of <u, dx> + <vb, dw> + <cb, db> w.r.t. (x, w, dy), the closed form of
    ``ln_gelu.cu`` (with t = r (u - mean(u) - xh mean(u xh)) and G the partial in xh)."""
    x = np.asarray(x, np.float64)
    n = x.shape[-1]
    u = np.zeros_like(x) if u is None else u
    vb = np.zeros_like(w) if vb is None else vb
    cb = np.zeros_like(w) if cb is None else cb
    _, mu, r = layernorm_fwd(x, w, np.zeros_like(w), eps)
    mu, r = mu[..., None], r[..., None]
    xh = (x - mu) * r
    g = dy * w
    s = lambda a: a.sum(-1, keepdims=True)
    su, sux, sg, sgx, sug = s(u), s(u * xh), s(g), s(g * xh), s(u * g)
    t = r * (u - su / n - xh * sux / n)
    gdy = w * t + vb * xh + cb
    red = tuple(range(x.ndim - 1))
    gw = (dy * t).sum(red)
    G = -(r / n) * (sux * g + sgx * u) + vb * dy
    phi_r = sug - sg * su / n - sgx * sux / n
    gx = r * (G - G.mean(-1, keepdims=True) - xh * (G * xh).mean(-1, keepdims=True)) - (r * r / n) * xh * phi_r
    return gx, gw, gdy


_ERF = np.vectorize(math.erf)


def gelu_terms(a):
    """(gelu(a), gelu'(a), gelu''(a)) of the exact GELU a Phi(a)."""
    a = np.asarray(a, np.float64)
    cdf = 0.5 * (1.0 + _ERF(a / math.sqrt(2.0)))
    pdf = np.exp(-0.5 * a * a) / math.sqrt(2.0 * math.pi)
    return a * cdf, cdf + a * pdf, pdf * (2.0 - a * a)


def xent_fwd(z, t):
    """Per-row (lse, loss) of logits z (rows, vocab) against integer targets t."""
    z = np.asarray(z, np.float64)
    m = z.max(-1, keepdims=True)
    lse = (m + np.log(np.exp(z - m).sum(-1, keepdims=True)))[:, 0]
    return lse, lse - z[np.arange(z.shape[0]), t]


def xent_bwd(z, t, g, s):
    """dz = g s (softmax(z) - onehot(t))."""
    z = np.asarray(z, np.float64)
    lse, _ = xent_fwd(z, t)
    p = np.exp(z - lse[:, None])
    p[np.arange(z.shape[0]), t] -= 1.0
    return g * s * p


def xent_bwd_bwd(z, t, g, s, u):
    """Cotangents of (z, g) for the cotangent u of dz: (g s p (u - <p, u>), sum_r s (<p_r, u_r> - u_r,t_r))."""
    z, u = np.asarray(z, np.float64), np.asarray(u, np.float64)
    lse, _ = xent_fwd(z, t)
    p = np.exp(z - lse[:, None])
    dot = (p * u).sum(-1, keepdims=True)
    gz = g * s * p * (u - dot)
    gg = (s * (dot[:, 0] - u[np.arange(z.shape[0]), t])).sum()
    return gz, gg
