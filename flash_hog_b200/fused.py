"""LayerNorm, GELU and cross entropy with fused first- and second-order backward kernels.

The grad-norm-penalty step (L + lam ||dL/dtheta||^2, configuration 5) differentiates
every layer's backward once more. In torch autograd the double backward of
LayerNorm and of GELU is a composite of many elementwise and reduction kernels;
here each pass is one kernel of ``csrc/ln_gelu.cu`` through the C ABI
(``fh_layernorm_*``, ``fh_gelu``), with two nested autograd Functions per op in the
same pattern as the attention op (``flash_hog/jax/attention.py:52-60, 100-130``):
the outer Function's backward is the inner Function, whose backward is the
double backward. Third-order derivatives raise.

* ``LayerNorm`` (module) / ``layer_norm(x, w, b, eps)``: fp32 arithmetic; under
  autocast the inputs are cast to fp32, as autocast does for torch's layer_norm.
* ``gelu(x)``: exact GELU (x Phi(x)) in the input dtype (fp32 or bf16; fp32
  arithmetic), as ``torch.nn.functional.gelu`` under autocast.
* ``cross_entropy(logits, targets)``: the mean cross entropy of (rows, vocab) logits
  (fp32 or bf16, fp32 arithmetic) as ``torch.nn.functional.cross_entropy`` on the
  logits cast to fp32; its gradient comes back in the logits' dtype, as autocast
  would cast it for the head's matmul (``csrc/xent.cu``, ``fh_xent_*``).
* ``sum_of_squares(tensors)``: the penalty sum_i ||t_i||^2 with torch's multi-tensor
  kernels (one norm pass forward, one scaled copy backward), differentiable once.
"""

from __future__ import annotations

import torch
import torch.nn as nn

from flash_hog_b200 import _capi


def _contig(t):
    return t if t.is_contiguous() else t.contiguous()


class _LayerNormBwd(torch.autograd.Function):
    """(dx, dw, db) of LayerNorm from (x, w, mean, rstd, dy); its backward is the double backward."""

    @staticmethod
    def forward(ctx, x, w, mean, rstd, dy):
        dy = _contig(dy.float())
        dx, dw, db = torch.empty_like(x), torch.empty_like(w), torch.empty_like(w)
        _capi.layernorm_bwd(x, w, mean, rstd, dy, dx, dw, db)
        ctx.save_for_backward(x, w, mean, rstd, dy)
        return dx, dw, db

    @staticmethod
    def backward(ctx, gdx, gdw, gdb):
        x, w, mean, rstd, dy = ctx.saved_tensors
        if any(ctx.needs_input_grad) and torch.is_grad_enabled():
            raise NotImplementedError("third-order derivatives of the fused LayerNorm are not supported")
        gx, gw, gdy = torch.empty_like(x), torch.empty_like(w), torch.empty_like(dy)
        _capi.layernorm_bwd_bwd(x, w, mean, rstd, dy, None if gdx is None else _contig(gdx.float()),
                                None if gdw is None else _contig(gdw.float()),
                                None if gdb is None else _contig(gdb.float()), gx, gw, gdy)
        return gx, gw, None, None, gdy


class _LayerNorm(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w, b, eps):
        y, mean, rstd = torch.empty_like(x), x.new_empty(x.shape[:-1]), x.new_empty(x.shape[:-1])
        _capi.layernorm_fwd(x, w, b, eps, y, mean, rstd)
        ctx.save_for_backward(x, w, mean, rstd)
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w, mean, rstd = ctx.saved_tensors
        dx, dw, db = _LayerNormBwd.apply(x, w, mean, rstd, dy)
        return dx, dw, db, None


def layer_norm(x, weight, bias, eps: float = 1e-5):
    """LayerNorm over the last dimension in fp32 (fused kernels, differentiable twice)."""
    cast = lambda t: _contig(t.float())
    with torch.autocast(device_type="cuda", enabled=False):
        return _LayerNorm.apply(cast(x), cast(weight), cast(bias), float(eps))


class LayerNorm(nn.LayerNorm):
    """``nn.LayerNorm`` (same parameters and state dict) on the fused kernels."""

    def forward(self, x):
        return layer_norm(x, self.weight, self.bias, self.eps)


class _GeluBwd(torch.autograd.Function):
    """dh gelu'(a); its backward is the double backward (one kernel for both cotangents)."""

    @staticmethod
    def forward(ctx, a, dh):
        ctx.dh_dtype = dh.dtype
        dh = _contig(dh.to(a.dtype))
        da = torch.empty_like(a)
        _capi.gelu(1, a, dh, None, da, None)
        ctx.save_for_backward(a, dh)
        return da

    @staticmethod
    def backward(ctx, c):
        a, dh = ctx.saved_tensors
        if any(ctx.needs_input_grad) and torch.is_grad_enabled():
            raise NotImplementedError("third-order derivatives of the fused GELU are not supported")
        c = _contig(c.to(a.dtype))
        gdh, ga = torch.empty_like(a), torch.empty_like(a)
        _capi.gelu(2, a, dh, c, gdh, ga)
        return ga, gdh.to(ctx.dh_dtype)


class _Gelu(torch.autograd.Function):
    @staticmethod
    def forward(ctx, a):
        h = torch.empty_like(a)
        _capi.gelu(0, a, None, None, h, None)
        ctx.save_for_backward(a)
        return h

    @staticmethod
    def backward(ctx, dh):
        (a,) = ctx.saved_tensors
        return _GeluBwd.apply(a, dh)


def gelu(x):
    """Exact GELU in the input dtype (fp32 or bf16), differentiable twice on the fused kernels."""
    return _Gelu.apply(_contig(x))


class _CrossEntropyBwd(torch.autograd.Function):
    """dz = g (softmax(z) - onehot(t)) / rows; its backward is the double backward."""

    @staticmethod
    def forward(ctx, z, t, lse, g):
        g32 = _contig(g.detach().float().reshape(1))
        dz = torch.empty(z.shape, dtype=z.dtype, device=z.device)
        _capi.xent_bwd(z, t, lse, g32, 1.0 / z.shape[0], dz)
        ctx.save_for_backward(z, t, lse, g32)
        ctx.g_shape, ctx.g_dtype = g.shape, g.dtype
        return dz

    @staticmethod
    def backward(ctx, u):
        z, t, lse, g32 = ctx.saved_tensors
        if any(ctx.needs_input_grad) and torch.is_grad_enabled():
            raise NotImplementedError("third-order derivatives of the fused cross entropy are not supported")
        u = _contig(u.to(z.dtype))
        gz = torch.empty(z.shape, dtype=z.dtype, device=z.device)
        gg = torch.empty(z.shape[0], dtype=torch.float32, device=z.device)
        _capi.xent_bwd_bwd(z, t, lse, g32, 1.0 / z.shape[0], u, gz, gg)
        return gz, None, None, gg.sum().to(ctx.g_dtype).reshape(ctx.g_shape)


class _CrossEntropy(torch.autograd.Function):
    @staticmethod
    def forward(ctx, z, t):
        lse = torch.empty(z.shape[0], dtype=torch.float32, device=z.device)
        loss = torch.empty_like(lse)
        _capi.xent_fwd(z, t, lse, loss)
        ctx.save_for_backward(z, t, lse)
        return loss.mean()

    @staticmethod
    def backward(ctx, g):
        z, t, lse = ctx.saved_tensors
        return _CrossEntropyBwd.apply(z, t, lse, g), None


def cross_entropy(logits, targets):
    """Mean cross entropy of (rows, vocab) logits against int64 targets, differentiable
    twice on the fused kernels (fp32 result; the logits' gradient in their dtype)."""
    if logits.stride(-1) != 1:
        logits = logits.contiguous()
    return _CrossEntropy.apply(logits, _contig(targets.long()))


class _SumOfSquares(torch.autograd.Function):
    """sum_i ||t_i||^2 over a list of tensors with multi-tensor kernels: one pass for the
    norms forward, one scaled copy of every tensor backward (instead of a square, a
    reduction and their gradients per tensor)."""

    @staticmethod
    def forward(ctx, *ts):
        ctx.save_for_backward(*ts)
        return torch.stack(torch._foreach_norm(list(ts), 2)).float().square().sum()

    @staticmethod
    def backward(ctx, g):
        ts = ctx.saved_tensors
        return tuple(torch._foreach_mul(list(ts), 2.0 * g))


def sum_of_squares(tensors):
    """sum_i ||t_i||^2 (fp32), differentiable once (the penalty term of the step)."""
    return _SumOfSquares.apply(*tensors)
