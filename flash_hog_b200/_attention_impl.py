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

import dataclasses
import enum
import os

import torch

from flash_hog_b200 import _capi


class MaskType(enum.Enum):
    """Masks: the two of the reference path (``_pallas_gpu_kernel.py:100``) and the
    bottom-right alignment of the reference's JAX statements for seq_q != seq_k
    (``flash_hog/_jax_refs/jax_impl.py:104-109``: query i sees keys j <= i + Tk - Tq).
    The values are the C ABI's ``causal`` codes."""

    NO_MASK = 0
    CAUSAL = 1
    CAUSAL_BOTTOM_RIGHT = 2


@dataclasses.dataclass(frozen=True)
class SlidingWindow:
    """A causal mask (``mask_type`` CAUSAL or CAUSAL_BOTTOM_RIGHT) limited to the
    ``length`` keys ending at each query's diagonal -- ``get_mask_bottom_right``'s
    ``qi - kj < sliding_window_length`` (``flash_hog/_jax_refs/jax_impl.py:104-109``).
    Accepted wherever a ``MaskType`` is."""

    mask_type: MaskType
    length: int


@dataclasses.dataclass(frozen=True, eq=False)
class PackedSequences:
    """A packed variable-length batch: ``mask`` (a MaskType or SlidingWindow) applied
    to each sequence on its own. Tensors are (1, total rows, heads, head_dim) (or
    (total, heads, head_dim)); sequence b is query rows [cu_seqlens_q[b],
    cu_seqlens_q[b+1]) and key rows [cu_seqlens_k[b], cu_seqlens_k[b+1]) (int32
    device tensors); ``max_seqlen_q``/``max_seqlen_k`` bound the sequence lengths.
    CAUSAL_BOTTOM_RIGHT aligns each sequence's own diagonal, as the reference's JAX
    statements do for every (qs, ks) pair (``flash_hog/_jax_refs/jax_impl.py:104-130``).
    Accepted wherever a MaskType is; packed batches run the bf16 kernels."""

    mask: object
    cu_seqlens_q: torch.Tensor
    cu_seqlens_k: torch.Tensor
    max_seqlen_q: int
    max_seqlen_k: int

    def capi(self) -> "_capi.Varlen":
        return _capi.Varlen(self.cu_seqlens_q, self.cu_seqlens_k, self.max_seqlen_q, self.max_seqlen_k)


def _varlen_kw(mask) -> dict:
    """``{"varlen": ...}`` for the bf16 C ABI wrappers when ``mask`` packs sequences."""
    return {"varlen": mask.capi()} if isinstance(mask, PackedSequences) else {}


def _mask_args(mask) -> tuple[int, int]:
    """(causal code, window length) of a MaskType or SlidingWindow, for the C ABI."""
    if isinstance(mask, PackedSequences):
        return _mask_args(mask.mask)
    if isinstance(mask, SlidingWindow):
        if mask.mask_type not in (MaskType.CAUSAL, MaskType.CAUSAL_BOTTOM_RIGHT) or mask.length < 1:
            raise ValueError(f"a sliding window needs a causal mask type and a length >= 1, got {mask}")
        return mask.mask_type.value, int(mask.length)
    if not isinstance(mask, MaskType):
        raise ValueError(f"unsupported mask type {mask}")
    return mask.value, 0


def _is_causal(mask) -> bool:
    return _mask_args(mask)[0] != 0


FP32_POLICY_ENV = "FLASH_HOG_B200_FP32"


def fp32_policy() -> str:
    """How fp32 inputs are computed: "fp32" (default) -- the fp32-product kernels, as
    the reference's Pallas rule keeps fp32 operands in fp32
    (``flash_hog/jax/_pallas_gpu_kernel.py:251-256``); or "bf16" -- cast to bf16 for the
    tensor-core kernels, as the reference's native plugin does
    (``flash_hog/jax/_tk_gpu.py:90-92``), with results returned in fp32. Set by the
    ``FLASH_HOG_B200_FP32`` environment variable, read at each call."""
    policy = os.environ.get(FP32_POLICY_ENV, "fp32").strip().lower() or "fp32"
    if policy not in ("fp32", "bf16"):
        raise ValueError(f"{FP32_POLICY_ENV} must be 'fp32' or 'bf16', got {policy!r}")
    return policy


def _is_f32(x: torch.Tensor, policy: str | None = None, mask=None) -> bool:
    """Whether ``x``'s call runs the fp32 kernels (``fh_attn_*_f32``): fp32 inputs under
    the "fp32" policy. Every other case runs the bf16 tensor-core kernels. ``policy``
    is the one the forward decided (kept with its residuals so that the backward,
    the double backward and the forward-mode rules of one graph all follow it);
    None reads ``fp32_policy()`` now. Packed variable-length batches (``mask`` a
    PackedSequences) always run the bf16 kernels."""
    if isinstance(mask, PackedSequences):
        return False
    return x.dtype == torch.float32 and (fp32_policy() if policy is None else policy) == "fp32"


def _operand(x: torch.Tensor, f32: bool) -> torch.Tensor:
    """BTNH with a contiguous layout in the kernels' operand type (fp32 or bf16)."""
    x = x.to(torch.float32 if f32 else torch.bfloat16)
    return x if x.is_contiguous() else x.contiguous()


def _bf16(x: torch.Tensor) -> torch.Tensor:
    """bf16 BTNH with a contiguous layout (the tensor-core kernels' operand type);
    a cast like the one of the reference's native plugin (``flash_hog/jax/_tk_gpu.py:90-92``)."""
    return _operand(x, False)


def _fold(x: torch.Tensor, dim, size: int) -> torch.Tensor:
    """For a batching (vmap) rule: moves the vmapped dimension ``dim`` (None: not
    vmapped, broadcast) to the front and merges it with the batch dimension,
    (size, B, ...) -> (size * B, ...), as ``flash_hog/jax/_pallas_gpu.py:92-93`` does."""
    x = x.movedim(dim, 0) if dim is not None else x.unsqueeze(0).expand(size, *x.shape)
    return x.reshape(size * x.shape[1], *x.shape[2:])


def _unfold(x: torch.Tensor, size: int) -> torch.Tensor:
    """Inverse of ``_fold`` on a result: (size * B, ...) -> (size, B, ...)."""
    return x.reshape(size, x.shape[0] // size, *x.shape[1:])


def _check_inputs(query, key, value):
    if query.ndim != 4 or key.ndim != 4 or value.ndim != 4:
        raise ValueError("expected BTNH tensors")
    if not (query.is_cuda and key.is_cuda and value.is_cuda):
        raise ValueError("flash_hog_b200 runs on CUDA tensors only")
    if key.shape != value.shape or query.shape[0] != key.shape[0] or query.shape[3] != key.shape[3]:
        raise ValueError(f"incompatible shapes q{tuple(query.shape)} k{tuple(key.shape)} v{tuple(value.shape)}")
    if query.shape[2] % key.shape[2] != 0:
        raise ValueError(f"q_heads ({query.shape[2]}) must be a multiple of kv_heads ({key.shape[2]})")


def cuda_dot_product_attention(query, key, value, mask_type: MaskType, scale: float, return_residual=False,
                               policy: str | None = None):
    """Forward. Returns ``out`` or ``(out, activation)`` (activation = L, (B, N, T) fp32)."""
    _check_inputs(query, key, value)
    f32 = _is_f32(query, policy, mask_type)
    q, k, v = (_operand(x, f32) for x in (query, key, value))
    b, t, n, _ = q.shape
    out = torch.empty_like(q)
    lse = torch.empty((b, n, t), dtype=torch.float32, device=q.device)
    if f32:
        _capi.attn_fwd_f32(q, k, v, out, lse, scale, *_mask_args(mask_type))
    else:
        _capi.attn_fwd(q, k, v, out, lse, scale, *_mask_args(mask_type), **_varlen_kw(mask_type))
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


def dot_product_attention_bwd_rule(mask_type: MaskType, scale: float, res, g, policy: str | None = None):
    """First-order backward: (dQ, dK, dV) (``_attention_impl.py:242-261``)."""
    query, key, value, activation, out = res
    f32 = _is_f32(query, policy, mask_type)
    q, k, v, o, do = (_operand(x, f32) for x in (query, key, value, out, g))
    b, t, n, _ = q.shape
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    delta = torch.empty((b, n, t), dtype=torch.float32, device=q.device)
    if f32:
        _capi.attn_bwd_f32(q, k, v, o, do, activation.float().contiguous(), dq, dk, dv, delta, scale,
                           *_mask_args(mask_type))
    else:
        _capi.attn_bwd(q, k, v, o, do, activation.float().contiguous(), dq, dk, dv, delta, scale,
                       *_mask_args(mask_type), **_varlen_kw(mask_type))
    return dq.to(query.dtype), dk.to(key.dtype), dv.to(value.dtype)


def dot_product_attention_bwd_rule_fwd_rule(mask_type: MaskType, scale: float, res, g, policy: str | None = None):
    """Backward saving ``(query, key, value, out, activation, dO)`` (``_attention_impl.py:264-275``)."""
    query, key, value, activation, out = res
    grads = dot_product_attention_bwd_rule(mask_type=mask_type, scale=scale, res=res, g=g, policy=policy)
    return grads, (query, key, value, out, activation, g)


def _zeros_if_none(ts, like):
    return tuple(torch.zeros_like(x) if t is None else t for t, x in zip(ts, like))


def _require_plain(*ts) -> None:
    """The forward-mode rules hand tensors to the C ABI by address. Under the
    ``torch.func.jvp`` transform their saved tensors are functorch wrappers with
    no storage, so that transform is refused with a clear message; forward mode
    through ``torch.autograd.forward_ad`` (dual tensors) passes plain tensors."""
    if any(t is not None and torch._C._functorch.is_functorch_wrapped_tensor(t) for t in ts):
        raise NotImplementedError(
            "flash_hog_b200 forward-mode rules run under torch.autograd.forward_ad (dual tensors), not under "
            "the torch.func.jvp transform; torch.func.grad / vjp are supported")


def dot_product_attention_fwd_jvp(mask_type: MaskType, scale: float, res, tangents, policy: str | None = None):
    """Forward-mode derivative of the forward: ``(t_out, t_activation)``.

    No counterpart in the reference, which has reverse-mode rules only
    (``flash_hog/jax/attention.py:52-60``). The tangents are the double
    backward's query-pass outputs for dO = 0 and (ddQ, ddK, ddV) = (tQ, tK, tV):
    with tS = scale (tQ K^T + Q tK^T) and tP = P o (tS - rowsum(P o tS)),
    ddO = tP V + P tV = t_out and dD = rowsum(P o tS) = t_lse (the double
    backward's formulas, ``flash_hog/_jax_refs/jax_impl.py:273-336``, at dO = 0).
    """
    query, key, value, activation, out = res
    _require_plain(query, key, value, activation, out, *tangents)
    tq, tk, tv = _zeros_if_none(tangents, (query, key, value))
    f32 = _is_f32(query, policy, mask_type)
    q, k, v, o, tq, tk, tv = (_operand(x, f32) for x in (query, key, value, out, tq, tk, tv))
    b, t, n, _ = q.shape
    t_lse = torch.empty((b, n, t), dtype=torch.float32, device=q.device)
    t_out = torch.empty_like(q)
    causal, window = _mask_args(mask_type)
    lse = activation.float().contiguous()
    if f32:
        stats = torch.empty((2, b, n, t), dtype=torch.float32, device=q.device)
        _capi.attn_bwdbwd_f32(q, k, v, o, torch.zeros_like(q), tq, tk, tv, lse, None, t_out, None, None, stats[0],
                              t_lse, stats[1], scale, causal, which=_capi.PASS_QUERY, window=window)
    else:
        # The forward-tangent pass: the query pass at dO = 0, without the products that vanish there.
        _capi.attn_bwdbwd_o(q, k, v, None, None, tq, tk, tv, lse, None, t_out, None, None, None, t_lse, None, scale,
                            causal, which=_capi.PASS_FWD_TANGENT, window=window, **_varlen_kw(mask_type))
    return t_out.to(out.dtype), t_lse


def dot_product_attention_bwd_jvp(mask_type: MaskType, scale: float, res, g, tangents, policy: str | None = None):
    """Forward-mode derivative of the first-order backward: ``(tdQ, tdK, tdV)``.

    ``res`` = (query, key, value, activation, out), ``g`` = dO, ``tangents`` =
    (tQ, tK, tV, tdO) (None = zero). The backward is the gradient of
    phi = <O, dO>, so its jvp is Hess(phi) (tQ, tK, tV) -- the double backward
    with (ddQ, ddK, ddV) = (tQ, tK, tV), the Hessian being symmetric -- plus the
    first-order backward of tdO (``fh_attn_jvp_bwd``). The tangents of the
    residuals L and O are not used: they are functions of (Q, K, V), whose
    tangents already carry them (the reference's bwd-of-bwd rule returns None
    for them likewise, ``flash_hog/jax/_attention_impl.py:302-303``).
    """
    query, key, value, activation, out = res
    _require_plain(query, key, value, activation, out, g, *tangents)
    tq, tk, tv = _zeros_if_none(tangents[:3], (query, key, value))
    tdo = tangents[3]
    f32 = _is_f32(query, policy, mask_type)
    q, k, v, o, do, tq, tk, tv = (_operand(x, f32) for x in (query, key, value, out, g, tq, tk, tv))
    tdo = None if tdo is None else _operand(tdo, f32)
    b, t, n, _ = q.shape
    stats = torch.empty((3, b, n, t), dtype=torch.float32, device=q.device)
    tdq, t_out = torch.empty_like(q), torch.empty_like(q)
    tdk, tdv = torch.empty_like(k), torch.empty_like(v)
    (_capi.attn_jvp_bwd_f32 if f32 else _capi.attn_jvp_bwd)(
        q, k, v, o, do, activation.float().contiguous(), tq, tk, tv, tdo, tdq, tdk, tdv, t_out,
        stats[0], stats[1], stats[2], scale, *_mask_args(mask_type), **({} if f32 else _varlen_kw(mask_type)))
    return tdq.to(query.dtype), tdk.to(key.dtype), tdv.to(value.dtype)


def dot_product_attention_bwd_rule_bwd_rule(mask_type: MaskType, scale: float, res, g, policy: str | None = None):
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
                                      L=activation, mask_type=mask_type, scale=scale, _policy=policy)
    return (dQ2, dK2, dV2, None, None), ddO
