"""``flash_bwdbwd``: the attention double backward on the GPU.

Mirrors the reference's double-backward entry points
``flash_hog/jax/_pallas_gpu.py:51-114`` (``flash_bwdbwd``) and
``flash_hog/jax/_tk_gpu.py:83-103`` (the native-plugin variant): same
arguments, same return order ``(dQ2, dK2, dV2, ddO)``, unbatched (T, N, H)
inputs accepted by adding a batch dimension (``_pallas_gpu.py:65-68``), and
D = rowsum(dO o O) computed on the device before the kernels (``_tk_gpu.py:93``).

Under ``torch.func.vmap`` the vmapped axis is folded into the batch axis and
the kernels run once, the reference's batching rule (``_pallas_gpu.py:85-102``).

Unlike the reference's TK path there is no per-call fallback and no gate on
GPU generation: every call runs the sm_100a kernels or raises.
"""

from __future__ import annotations

import dataclasses

import torch

from flash_hog_b200 import _capi
from flash_hog_b200._attention_impl import (MaskType, PackedSequences, _fold, _is_f32, _mask_args, _operand, _unfold,
                                            _varlen_kw, fp32_policy)


@dataclasses.dataclass(frozen=True)
class TuningConfig:
    """Accepted for signature compatibility with ``_pallas_gpu_kernel.py:22-29``.

    Tile shapes are fixed by the sm_100a kernels (128 resident rows x 64
    streamed rows); the fields are ignored.
    """

    tile_q: int = 128
    tile_k: int = 64
    max_concurrent_steps: int = 3
    epilogue_tile_n: int = 64
    grid_minor_dim: int = 0
    grid_tile_width: int = 1


def flash_bwdbwd(Q, K, V, O, dO, ddQ, ddK, ddV, L, mask_type: MaskType = MaskType.NO_MASK, scale=None,
                 config: TuningConfig | None = None, return_stats: bool = False, _policy: str | None = None):
    """Double backward of attention; BTNH in, ``(dQ2, dK2, dV2, ddO)`` out.

    ``L`` is the forward log-sum-exp, (B, N, T) fp32 (natural log). Outputs
    have the input dtype. With ``return_stats`` also returns the fp32 row
    statistics ``(D, dD, B)``, each (B, N, T). ``_policy`` (internal): the fp32
    policy the forward of the same graph decided; None reads it now.
    """
    if Q.ndim == 3:
        batched = [x.unsqueeze(0) for x in (Q, K, V, O, dO, ddQ, ddK, ddV, L)]
        res = flash_bwdbwd(*batched, mask_type=mask_type, scale=scale, config=config, return_stats=return_stats,
                           _policy=_policy)
        outs = tuple(x.squeeze(0) for x in res[0]) if return_stats else tuple(x.squeeze(0) for x in res)
        if return_stats:
            return outs, tuple(x.squeeze(0) for x in res[1])
        return outs
    if scale is None:
        scale = Q.shape[-1] ** -0.5
    if Q.shape[2] % K.shape[2] != 0:
        raise ValueError(f"q_heads ({Q.shape[2]}) must be a multiple of kv_heads ({K.shape[2]})")
    causal, window = _mask_args(mask_type)
    policy = fp32_policy() if _policy is None else _policy
    packed = mask_type if isinstance(mask_type, PackedSequences) else None
    dq2, dk2, dv2, ddo, stats = _FlashBwdBwd.apply(Q, K, V, O, dO, ddQ, ddK, ddV, L, causal, window, float(scale),
                                                   policy, packed)
    outs = (dq2, dk2, dv2, ddo)
    if return_stats:
        return outs, (stats[0], stats[1], stats[2])
    return outs


def _bwdbwd_device(Q, K, V, O, dO, ddQ, ddK, ddV, L, causal: int, window: int, scale: float, policy: str,
                   packed: PackedSequences | None = None):
    """The kernels on 4-D BTNH tensors: ``(dQ2, dK2, dV2, ddO, stats)``, stats = (D, dD, B) stacked.
    ``packed``: the tensors are (1, total, heads, head_dim) packed sequences."""
    f32 = _is_f32(Q, policy, packed)
    q, k, v, o, do, ddq, ddk, ddv = (_operand(x, f32) for x in (Q, K, V, O, dO, ddQ, ddK, ddV))
    b, t, n, _ = q.shape
    lse = L.reshape(b, n, t).float().contiguous()
    stats = torch.empty((3, b, n, t), dtype=torch.float32, device=q.device)
    delta, dd, bvec = stats[0], stats[1], stats[2]
    dq2, ddo = torch.empty_like(q), torch.empty_like(q)
    dk2, dv2 = torch.empty_like(k), torch.empty_like(k)
    # D = rowsum(dO * O) is computed on the device as part of the call.
    entry = _capi.attn_bwdbwd_f32 if f32 else _capi.attn_bwdbwd_o
    entry(q, k, v, o, do, ddq, ddk, ddv, lse, dq2, ddo, dk2, dv2, delta, dd, bvec, scale, causal, window=window,
          **({} if f32 else _varlen_kw(packed)))
    return dq2.to(Q.dtype), dk2.to(K.dtype), dv2.to(V.dtype), ddo.to(dO.dtype), stats


class _FlashBwdBwd(torch.autograd.Function):
    """The double backward as an autograd Function, so that ``torch.func`` transforms
    reach its batching rule instead of handing batched wrappers to the C ABI.
    Returns ``(dQ2, dK2, dV2, ddO, stats)``."""

    @staticmethod
    def forward(Q, K, V, O, dO, ddQ, ddK, ddV, L, causal, window, scale, policy, packed):
        return _bwdbwd_device(Q, K, V, O, dO, ddQ, ddK, ddV, L, causal, window, scale, policy, packed)

    @staticmethod
    def setup_context(ctx, inputs, output):
        ctx.mark_non_differentiable(output[4])

    @staticmethod
    def backward(ctx, *grads):
        raise NotImplementedError(
            "flash_bwdbwd has no derivative: third-order derivatives of attention are not supported (the "
            "reference's double-backward rule is the last one it defines, flash_hog/jax/attention.py:100-130)")

    @staticmethod
    def vmap(info, in_dims, Q, K, V, O, dO, ddQ, ddK, ddV, L, causal, window, scale, policy, packed):
        """Batching rule of ``flash_hog/jax/_pallas_gpu.py:85-102``: the vmapped axis is
        folded into the batch axis, the kernels run once, and the results are unfolded.
        The reference requires every input to be vmapped; here an input that is not is
        broadcast along the vmapped axis first."""
        if packed is not None:
            raise NotImplementedError("packed variable-length batches are not vmapped: pack the sequences instead")
        size = info.batch_size
        args = [_fold(x, d, size) for x, d in zip((Q, K, V, O, dO, ddQ, ddK, ddV, L), in_dims[:9])]
        dq2, dk2, dv2, ddo, stats = _FlashBwdBwd.apply(*args, causal, window, scale, policy, None)
        stats = stats.reshape(3, size, stats.shape[1] // size, *stats.shape[2:])
        return (_unfold(dq2, size), _unfold(dk2, size), _unfold(dv2, size), _unfold(ddo, size), stats), (0, 0, 0, 0, 1)

