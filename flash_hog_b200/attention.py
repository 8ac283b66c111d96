"""Public attention API with higher-order gradients on B200.

Mirrors ``flash_hog/jax/attention.py``: ``dot_product_attention(query, key,
value, is_causal=False, scale=None)`` on BTNH (or unbatched TNH) tensors. The
reference nests two ``jax.custom_vjp``s so that differentiating the backward
reaches a dedicated double-backward rule (``attention.py:52-60, 100-130``);
here the same nesting is two ``torch.autograd.Function``s:

* ``_DotProductAttention`` -- forward saves ``(q, k, v, L, O)``; its backward
  calls ``_DotProductAttentionBwd`` (``attention.py:64-72``);
* ``_DotProductAttentionBwd`` -- forward is the first-order backward and saves
  ``(q, k, v, O, L, dO)`` (``attention.py:110-116``); its backward is the
  double backward (``attention.py:119-125``).

So ``torch.autograd.grad(..., create_graph=True)`` followed by a second
``grad`` (grad-of-grad, Hessian-vector products) runs fwd -> bwd -> bwdbwd on
the sm_100a kernels, as nested ``jax.grad`` does in the reference.

Beyond the reference, both Functions also have forward-mode (``jvp``) rules
and the ``setup_context`` form, so ``torch.func`` transforms compose over them:
``torch.func.jvp(torch.func.grad(f), primals, tangents)`` -- forward-over-reverse
Hessian-vector products -- runs fwd, bwd, the forward jvp (the double
backward's query pass at dO = 0) and the backward's jvp (double backward plus
first-order backward, ``fh_attn_jvp_bwd``) on the kernels.

Both Functions, and ``flash_bwdbwd``, also have batching rules for
``torch.func.vmap``: the vmapped axis is folded into the batch axis and the
kernels run once, the rule the reference gives its double backward
(``flash_hog/jax/_pallas_gpu.py:85-102``).
"""

from __future__ import annotations

import torch

from flash_hog_b200 import _attention_impl as attn_impl
from flash_hog_b200._attention_impl import MaskType, PackedSequences, SlidingWindow


def dot_product_attention(query, key, value, is_causal: bool = False, scale: float | None = None, *,
                          causal_alignment: str = "top_left", sliding_window_length: int | None = None):
    """softmax(scale * query key^T [+ causal mask]) value.

    Dimensions: T query length, S key/value length, N heads, H head dim.
    query (B, T, N, H) or (T, N H); key, value (B, S, N, H) or (S, N, H).

    Keyword-only extensions of the reference signature, with ``is_causal``:
    ``causal_alignment`` "top_left" (query i sees keys j <= i, the reference API's
    mask) or "bottom_right" (j <= i + S - T, the alignment of the reference's JAX
    statements, ``flash_hog/_jax_refs/jax_impl.py:104-109``), and
    ``sliding_window_length`` W (each query sees the W keys ending at its diagonal).
    A query that sees no key gets a zero output.
    """
    if scale is None:
        scale = query.shape[-1] ** -0.5
    if not (query.dtype == key.dtype == value.dtype):
        raise TypeError("query, key and value must share a dtype")
    if causal_alignment not in ("top_left", "bottom_right"):
        raise ValueError(f"causal_alignment must be 'top_left' or 'bottom_right', got {causal_alignment!r}")
    if not is_causal and (sliding_window_length is not None or causal_alignment != "top_left"):
        raise ValueError("causal_alignment and sliding_window_length apply to causal attention only")
    mask_type = MaskType.NO_MASK
    if is_causal:
        mask_type = MaskType.CAUSAL if causal_alignment == "top_left" else MaskType.CAUSAL_BOTTOM_RIGHT
        if sliding_window_length is not None:
            mask_type = SlidingWindow(mask_type, int(sliding_window_length))
    unbatched = query.ndim == 3
    if unbatched:
        query, key, value = query.unsqueeze(0), key.unsqueeze(0), value.unsqueeze(0)
    # The fp32 policy is decided once here and kept with the residuals: the backward,
    # double backward and forward-mode rules of this graph all follow it.
    result, _ = _DotProductAttention.apply(query, key, value, mask_type, float(scale), attn_impl.fp32_policy())
    if unbatched:
        result = result.squeeze(0)
    return result


def dot_product_attention_varlen(query, key, value, cu_seqlens_q, cu_seqlens_k, max_seqlen_q: int,
                                 max_seqlen_k: int, is_causal: bool = False, scale: float | None = None, *,
                                 causal_alignment: str = "top_left", sliding_window_length: int | None = None):
    """``dot_product_attention`` over a packed batch of variable-length sequences,
    differentiable twice like it (fwd -> bwd -> bwdbwd on the kernels).

    query (total_q, N, H); key, value (total_k, Nkv, H); sequence b is query rows
    [cu_seqlens_q[b], cu_seqlens_q[b+1]) against key rows [cu_seqlens_k[b],
    cu_seqlens_k[b+1]) (int32 tensors on the tensors' device, sequences + 1 entries,
    non-decreasing from 0); ``max_seqlen_q``/``max_seqlen_k`` bound the lengths. Masks
    apply per sequence: "bottom_right" aligns each sequence's own diagonal, the mask of
    the reference's JAX statements for a (qs, ks) pair
    (``flash_hog/_jax_refs/jax_impl.py:104-130``). Each sequence's result equals the
    dense call on that sequence alone. Computes with bf16 operands (any input dtype;
    results in the input dtype).
    """
    if query.ndim != 3 or key.ndim != 3 or value.ndim != 3:
        raise ValueError("packed tensors are (total, heads, head_dim)")
    if scale is None:
        scale = query.shape[-1] ** -0.5
    if causal_alignment not in ("top_left", "bottom_right"):
        raise ValueError(f"causal_alignment must be 'top_left' or 'bottom_right', got {causal_alignment!r}")
    if not is_causal and (sliding_window_length is not None or causal_alignment != "top_left"):
        raise ValueError("causal_alignment and sliding_window_length apply to causal attention only")
    mask = MaskType.NO_MASK
    if is_causal:
        mask = MaskType.CAUSAL if causal_alignment == "top_left" else MaskType.CAUSAL_BOTTOM_RIGHT
        if sliding_window_length is not None:
            mask = SlidingWindow(mask, int(sliding_window_length))
    packed = PackedSequences(mask, cu_seqlens_q, cu_seqlens_k, int(max_seqlen_q), int(max_seqlen_k))
    result, _ = _DotProductAttention.apply(query.unsqueeze(0), key.unsqueeze(0), value.unsqueeze(0), packed,
                                           float(scale), "bf16")
    return result.squeeze(0)


def _no_packed_vmap(mask_type):
    if isinstance(mask_type, PackedSequences):
        raise NotImplementedError("packed variable-length batches are not vmapped: pack the sequences instead")


class _DotProductAttention(torch.autograd.Function):
    """Forward (outputs O and the log-sum-exp L, the latter non-differentiable)."""

    @staticmethod
    def forward(query, key, value, mask_type, scale, policy):
        return attn_impl.cuda_dot_product_attention(query, key, value, mask_type=mask_type, scale=scale,
                                                    return_residual=True, policy=policy)

    @staticmethod
    def setup_context(ctx, inputs, output):
        query, key, value, mask_type, scale, policy = inputs
        out, activation = output
        ctx.mark_non_differentiable(activation)
        ctx.save_for_backward(query, key, value, activation, out)
        ctx.save_for_forward(query, key, value, activation, out)
        ctx.mask_type, ctx.scale, ctx.policy = mask_type, scale, policy

    @staticmethod
    def backward(ctx, g, _g_activation):
        query, key, value, activation, out = ctx.saved_tensors
        dq, dk, dv = _DotProductAttentionBwd.apply(query, key, value, activation, out, g, ctx.mask_type, ctx.scale,
                                                   ctx.policy)
        return dq, dk, dv, None, None, None

    @staticmethod
    def jvp(ctx, tq, tk, tv, _t_mask, _t_scale, _t_policy):
        res = ctx.saved_tensors
        t_out, _ = attn_impl.dot_product_attention_fwd_jvp(ctx.mask_type, ctx.scale, res, (tq, tk, tv),
                                                           policy=ctx.policy)
        return t_out, None

    @staticmethod
    def vmap(info, in_dims, query, key, value, mask_type, scale, policy):
        # Fold the vmapped axis into batch (the rule of flash_hog/jax/_pallas_gpu.py:85-102).
        _no_packed_vmap(mask_type)
        size = info.batch_size
        q, k, v = (attn_impl._fold(x, d, size) for x, d in zip((query, key, value), in_dims[:3]))
        out, activation = _DotProductAttention.apply(q, k, v, mask_type, scale, policy)
        return (attn_impl._unfold(out, size), attn_impl._unfold(activation, size)), (0, 0)


class _DotProductAttentionBwd(torch.autograd.Function):
    """First-order backward (dQ, dK, dV); reverse mode gives the double backward,
    forward mode its jvp."""

    @staticmethod
    def forward(query, key, value, activation, out, g, mask_type, scale, policy):
        (dq, dk, dv), _ = attn_impl.dot_product_attention_bwd_rule_fwd_rule(
            mask_type=mask_type, scale=scale, res=(query, key, value, activation, out), g=g, policy=policy)
        return dq, dk, dv

    @staticmethod
    def setup_context(ctx, inputs, output):
        query, key, value, activation, out, g, mask_type, scale, policy = inputs
        # The residual order of the reference's bwd-of-bwd rule (_attention_impl.py:264-275).
        ctx.save_for_backward(query, key, value, out, activation, g)
        ctx.save_for_forward(query, key, value, activation, out, g)
        ctx.mask_type, ctx.scale, ctx.policy = mask_type, scale, policy

    @staticmethod
    def backward(ctx, ddq, ddk, ddv):
        res = ctx.saved_tensors
        zeros = [torch.zeros_like(t) if c is None else c for c, t in zip((ddq, ddk, ddv), res[:3])]
        (dq2, dk2, dv2, _, _), ddo = attn_impl.dot_product_attention_bwd_rule_bwd_rule(
            mask_type=ctx.mask_type, scale=ctx.scale, res=res, g=tuple(zeros), policy=ctx.policy)
        return dq2, dk2, dv2, None, None, ddo, None, None, None

    @staticmethod
    def jvp(ctx, tq, tk, tv, _t_activation, _t_out, tg, _t_mask, _t_scale, _t_policy):
        query, key, value, activation, out, g = ctx.saved_tensors
        return attn_impl.dot_product_attention_bwd_jvp(ctx.mask_type, ctx.scale, (query, key, value, activation, out),
                                                      g, (tq, tk, tv, tg), policy=ctx.policy)

    @staticmethod
    def vmap(info, in_dims, query, key, value, activation, out, g, mask_type, scale, policy):
        _no_packed_vmap(mask_type)
        size = info.batch_size
        args = [attn_impl._fold(x, d, size) for x, d in zip((query, key, value, activation, out, g), in_dims[:6])]
        dq, dk, dv = _DotProductAttentionBwd.apply(*args, mask_type, scale, policy)
        return tuple(attn_impl._unfold(x, size) for x in (dq, dk, dv)), (0, 0, 0)
