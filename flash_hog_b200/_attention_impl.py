"""Forward, backward and double-backward rules of the attention op.

Mirrors ``flash_hog/jax/_attention_impl.py:224-303`` function by function,
with the cuDNN custom calls and the Pallas/ThunderKittens double backward
replaced by this package's sm_100a kernels (``_capi``). Tensors are BTNH torch
CUDA tensors; the log-sum-exp ``activation`` is (B, N, T) fp32.

Residual tuples keep the reference's order:
  * forward residual ``(query, key, value, activation, out)``
    (``_attention_impl.py:246``);
  * backward residual ``(query, key, value, out, activation, dO)``
    (``_attention_impl.py:274``).
"""

from __future__ import annotations

import enum

import torch

from flash_hog_b200 import _capi


class MaskType(enum.Enum):
    """The two masks of the reference path (``_pallas_gpu_kernel.py:100``)."""

    NO_MASK = 0
    CAUSAL = 1


def _is_causal(mask_type: MaskType) -> bool:
    if mask_type not in (MaskType.NO_MASK, MaskType.CAUSAL):
        raise ValueError(f"unsupported mask type {mask_type}")
    return mask_type is MaskType.CAUSAL


def _bf16(x: torch.Tensor) -> torch.Tensor:
    """bf16 BTNH with a contiguous head_dim (the kernels' operand type).

    fp32 inputs are cast like the reference's native plugin does
    (``flash_hog/jax/_tk_gpu.py:90-92``)."""
    x = x.to(torch.bfloat16)
    return x if x.is_contiguous() else x.contiguous()


def _check_inputs(query, key, value):
    if query.ndim != 4 or key.ndim != 4 or value.ndim != 4:
        raise ValueError("expected BTNH tensors")
    if not (query.is_cuda and key.is_cuda and value.is_cuda):
        raise ValueError("flash_hog_b200 runs on CUDA tensors only")
    if key.shape != value.shape or query.shape[0] != key.shape[0] or query.shape[3] != key.shape[3]:
        raise ValueError(f"incompatible shapes q{tuple(query.shape)} k{tuple(key.shape)} v{tuple(value.shape)}")
    if query.shape[2] % key.shape[2] != 0:
        raise ValueError(f"q_heads ({query.shape[2]}) must be a multiple of kv_heads ({key.shape[2]})")


def cuda_dot_product_attention(query, key, value, mask_type: MaskType, scale: float, return_residual=False):
    """Forward. Returns ``out`` or ``(out, activation)`` (activation = L, (B, N, T) fp32)."""
    _check_inputs(query, key, value)
    q, k, v = _bf16(query), _bf16(key), _bf16(value)
    b, t, n, _ = q.shape
    out = torch.empty_like(q)
    lse = torch.empty((b, n, t), dtype=torch.float32, device=q.device)
    _capi.attn_fwd(q, k, v, out, lse, scale, _is_causal(mask_type))
    out = out.to(query.dtype)
    return (out, lse) if return_residual else out


def dot_product_attention_fwd(query, key, value, mask_type: MaskType, scale: float):
    """Forward pass, no saving (``_attention_impl.py:224-229``)."""
    return cuda_dot_product_attention(query, key, value, mask_type=mask_type, scale=scale)


def dot_product_attention_fwd_rule(query, key, value, mask_type: MaskType, scale: float):
    """Forward saving ``(query, key, value, activation, out)`` (``_attention_impl.py:232-239``)."""
    out, activation = cuda_dot_product_attention(query, key, value, mask_type=mask_type, scale=scale,
                                                 return_residual=True)
    return out, (query, key, value, activation, out)


def dot_product_attention_bwd_rule(mask_type: MaskType, scale: float, res, g):
    """First-order backward: (dQ, dK, dV) (``_attention_impl.py:242-261``)."""
    query, key, value, activation, out = res
    q, k, v, o, do = _bf16(query), _bf16(key), _bf16(value), _bf16(out), _bf16(g)
    b, t, n, _ = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty((b, n, t), dtype=torch.float32, device=q.device)
    _capi.attn_bwd(q, k, v, o, do, activation.float().contiguous(), dq, dk, dv, delta, scale,
                   _is_causal(mask_type))
    return dq.to(query.dtype), dk.to(key.dtype), dv.to(value.dtype)


def dot_product_attention_bwd_rule_fwd_rule(mask_type: MaskType, scale: float, res, g):
    """Backward saving ``(query, key, value, out, activation, dO)`` (``_attention_impl.py:264-275``)."""
    query, key, value, activation, out = res
    grads = dot_product_attention_bwd_rule(mask_type=mask_type, scale=scale, res=res, g=g)
    return grads, (query, key, value, out, activation, g)


def dot_product_attention_bwd_rule_bwd_rule(mask_type: MaskType, scale: float, res, g):
    """Backward through the backward (``_attention_impl.py:278-303``).

    Returns ``((dQ2, dK2, dV2, None, None), ddO)``: cotangents of the forward
    residual ``(query, key, value, activation, out)`` and of ``dO``. The None
    entries match the reference: the double-backward formulas already carry the
    dependence of L and O on (Q, K, V).
    """
    from flash_hog_b200.bwdbwd import flash_bwdbwd

    query, key, value, out, activation, dO = res
    ddQ, ddK, ddV = g
    dQ2, dK2, dV2, ddO = flash_bwdbwd(Q=query, K=key, V=value, O=out, dO=dO, ddQ=ddQ, ddK=ddK, ddV=ddV,
                                      L=activation, mask_type=mask_type, scale=scale)
    return (dQ2, dK2, dV2, None, None), ddO
