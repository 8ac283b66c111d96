"""CPU oracle for Flash Hog's attention hot path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product package imports this module. Only ``tests/``,
``__graft_entry__.smoke()`` and ``bench.py`` (its ``cpu_baseline`` leg and the
``--impl reference`` arm) call it, and only as the checker / the timed CPU
baseline, never as the thing measured or shipped.

Parity is pinned: ``tests/test_oracle_kat.py`` checks ``bwdbwd_stats`` against
the reference's own known-answer vectors (``tests/golden/kat_bwdbwd.npz``,
extracted from the reference's ``test_data.zip``), and checks that the three
independent statements below (explicit formulas, the tiled 4-pass schedule,
and double autograd of naive attention) agree with each other.

Conventions (all functions):

* tensors are BTNH -- (batch, seq, heads, head_dim) -- like the reference API
  ``flash_hog/jax/attention.py:19-49``;
* the log-sum-exp ``L`` is (batch, heads, seq_q), natural log, the layout the
  cuDNN forward returns (``flash_hog/jax/_attention_impl.py:114-139``);
* the causal mask is top-left (query i sees keys j <= i), the mask of
  ``flash_hog/jax/_pallas_gpu_kernel.py:37-41`` and of
  ``jax.nn.dot_product_attention(is_causal=True)`` that the reference tests
  compare against (``tests/test_jax_fhog.py:14-15``);
* masked scores are -inf, so masked probabilities are exactly 0
  (``_pallas_gpu_kernel.py:34``).

The numpy statements compute in float64; ``autograd_*`` run torch autograd in
the dtype of their inputs (float64 for truth, float32 for the timed baseline).
"""

from __future__ import annotations

import math

import numpy as np

try:  # torch is only needed by the autograd statement and the bf16 helpers
    import torch
except ImportError:  # pragma: no cover
    torch = None


# --------------------------------------------------------------------------------------
# helpers
# --------------------------------------------------------------------------------------

def default_scale(head_dim: int) -> float:
    """``scale = head_dim ** -0.5`` (``flash_hog/jax/attention.py:34-35``)."""
    return head_dim ** -0.5


def causal_mask(nq: int, nk: int, causal=1, window: int = 0) -> np.ndarray:
    """Causal band mask, True where the score is kept: query i sees key j iff
    j <= i + diag and (window == 0 or i + diag - j < window), with diag = 0 for
    ``causal`` 1 / True (top-left, ``_pallas_gpu_kernel.py:37-41``) and nk - nq for
    ``causal`` 2 (bottom-right: ``get_mask_bottom_right``'s ``qi = qi + ks - qs``,
    ``(qi >= kj) & (qi - kj < sliding_window_length)``,
    ``flash_hog/_jax_refs/jax_impl.py:104-109``)."""
    qi = np.arange(nq)[:, None] + (nk - nq if int(causal) == 2 else 0)
    kj = np.arange(nk)[None, :]
    keep = qi >= kj
    if window:
        keep &= (qi - kj) < window
    return keep


def _heads(x: np.ndarray) -> np.ndarray:
    """BTNH -> (B, N, T, H) float64 view for per-head matmuls."""
    return np.ascontiguousarray(np.transpose(np.asarray(x, dtype=np.float64), (0, 2, 1, 3)))


def _btnh(x: np.ndarray) -> np.ndarray:
    return np.ascontiguousarray(np.transpose(x, (0, 2, 1, 3)))


def _expand(xh: np.ndarray, group: int) -> np.ndarray:
    """Key-side heads (B, Hkv, T, D) repeated for grouped-query attention: query
    head n uses key head n // group, the reference's "(kv_heads group)" split
    (``flash_hog/jax/_pallas_gpu_kernel.py:106-107``)."""
    return xh if group == 1 else np.repeat(xh, group, axis=1)


def _group_sum(xh: np.ndarray, group: int) -> np.ndarray:
    """Sums a key-side gradient computed per query head back onto its key head."""
    if group == 1:
        return xh
    b, h, t, d = xh.shape
    return xh.reshape(b, h // group, group, t, d).sum(axis=2)


def _group(q, k) -> int:
    if q.shape[2] % k.shape[2]:
        raise ValueError("q_heads must be a multiple of kv_heads")
    return q.shape[2] // k.shape[2]


def _scores(q, k, scale, causal, window=0):
    s = np.einsum("bhqd,bhkd->bhqk", q, k) * scale
    if causal:
        s = np.where(causal_mask(q.shape[2], k.shape[2], causal, window), s, -np.inf)
    return s


def _probs(s, lse):
    """P = exp(S - L); a query that sees no key (L = -inf) has P = 0."""
    lse = np.asarray(lse, np.float64)[..., None]
    p = np.exp(s - np.where(np.isfinite(lse), lse, 0.0))
    return np.where(np.isfinite(s), p, 0.0)


# --------------------------------------------------------------------------------------
# forward and first-order backward
# --------------------------------------------------------------------------------------

def attention_fwd(q, k, v, scale=None, causal=False, window=0):
    """O = softmax(scale*Q K^T + mask) V and L = logsumexp(scale*Q K^T + mask).

    Restates the forward the reference delegates to cuDNN
    (``flash_hog/jax/_attention_impl.py:224-239``; semantics of
    ``jax.nn.dot_product_attention``, ``tests/test_jax_fhog.py:14-15``).
    Returns (O BTNH, L (B,N,T)). ``causal`` 1 (or True) masks top-left, 2 bottom-right;
    ``window`` > 0 is a sliding window (``causal_mask``). A query that sees no key
    gets O = 0 and L = -inf (the kernels' convention; softmax over an empty set is
    undefined, and the reference's XLA statement gives NaN there).
    """
    scale = default_scale(q.shape[-1]) if scale is None else scale
    g = _group(q, k)
    qh, kh, vh = _heads(q), _expand(_heads(k), g), _expand(_heads(v), g)
    s = _scores(qh, kh, scale, causal, window)
    m = s.max(axis=-1, keepdims=True)
    m = np.where(np.isfinite(m), m, 0.0)
    e = np.exp(s - m)
    den = e.sum(axis=-1, keepdims=True)
    p = e / np.where(den > 0, den, 1.0)
    o = np.einsum("bhqk,bhkd->bhqd", p, vh)
    with np.errstate(divide="ignore"):
        lse = np.where(den > 0, m + np.log(den), -np.inf)[..., 0]
    return _btnh(o), lse


def attention_bwd(q, k, v, o, lse, do, scale=None, causal=False, window=0):
    """First-order backward (dQ, dK, dV) from the saved (O, L).

    Restates ``flash_hog/_jax_refs/jax_impl.py:142-191`` (``attn_bwd``) with
    P recomputed as exp(S - L) and D = rowsum(dO * O), the residual form the
    cuDNN backward uses (``flash_hog/jax/_attention_impl.py:242-261``).
    """
    scale = default_scale(q.shape[-1]) if scale is None else scale
    g = _group(q, k)
    qh, oh, doh = map(_heads, (q, o, do))
    kh, vh = (_expand(_heads(x), g) for x in (k, v))
    s = _scores(qh, kh, scale, causal, window)
    p = _probs(s, lse)
    dp = np.einsum("bhqd,bhkd->bhqk", doh, vh)
    d = np.einsum("bhqd,bhqd->bhq", doh, oh)[..., None]
    ds = scale * p * (dp - d)
    dq = np.einsum("bhqk,bhkd->bhqd", ds, kh)
    dk = _group_sum(np.einsum("bhqk,bhqd->bhkd", ds, qh), g)
    dv = _group_sum(np.einsum("bhqk,bhqd->bhkd", p, doh), g)
    return _btnh(dq), _btnh(dk), _btnh(dv)


# --------------------------------------------------------------------------------------
# double backward: the reference's dtype flow (pins the formulas to the golden file)
# --------------------------------------------------------------------------------------

def bwdbwd_stats_jax_dtype_flow(q, k, v, o, lse, do, ddq, ddk, ddv, scale):
    """``attn_bwd_bwd_stats`` on one head, rounding where the reference's JAX run rounds.

    The golden file was written by ``flash_hog/_jax_refs/jax_impl.py:404-477``
    calling ``attn_bwd_bwd_stats`` (``jax_impl.py:273-336``) on bf16 q, k, v,
    do, ddq, ddk, ddv with fp32 o and L, under
    ``jax_default_matmul_precision = BF16_BF16_F32`` (``jax_impl.py:33``). So:

    * a bf16 @ bf16 product (dO V^T, ddQ K^T, Q ddK^T, dO ddV^T) is rounded to bf16;
    * bf16 op bf16 elementwise results (the ddS sum and scale, dP * ddS) are bf16;
    * an fp32 @ bf16 product rounds its fp32 operand to bf16 and accumulates in fp32;
    * everything else is fp32.

    Inputs are unbatched (T, D) torch tensors holding the stored values.
    Returns (dq2, dk2, dv2, ddo) as float64 torch tensors. With this rounding
    the restatement reproduces the stored outputs to ~1e-4 (max-abs), which pins
    the formulas far below the ~5e-3 bf16-grade gap of a pure float64 evaluation.
    """
    r = lambda x: x.to(torch.bfloat16).double()
    f = lambda x: x.float().double()
    q, k, v, o, do, ddq, ddk, ddv = (t.double() for t in (q, k, v, o, do, ddq, ddk, ddv))
    lse = lse.double()
    mmb = lambda a, b: r(r(a) @ r(b))
    mmf = lambda a, b: f(r(a) @ r(b))
    s = f(q @ k.T) * scale                      # precision=F32_F32_F32 (jax_impl.py:301)
    p = f(torch.exp(s - lse[:, None]))
    dp = mmb(do, v.T)
    dds = r(r(mmb(ddq, k.T) + mmb(q, ddk.T)) * scale)
    d = f((o * do).sum(-1, keepdim=True))
    dd = f((dds * p).sum(-1, keepdim=True))
    dp2 = f(f(f(mmb(do, ddv.T) - f(dp * dd)) - f(dds * d)) + r(dp * dds))
    bb = f((dp2 * p).sum(-1, keepdim=True))
    ddp = f(p * f(dds - dd))
    ds2 = f(f(scale * p) * f(dp2 - bb))
    ds = f(f(scale * p) * f(dp - d))
    dq2 = mmf(ds, ddk) + mmf(ds2, k)
    dk2 = mmf(ds.T, ddq) + mmf(ds2.T, q)
    dv2 = mmf(ddp.T, do)
    ddo = mmf(p, ddv) + mmf(ddp, v)
    return dq2, dk2, dv2, ddo


# --------------------------------------------------------------------------------------
# double backward: explicit formulas
# --------------------------------------------------------------------------------------

def bwdbwd_stats(q, k, v, o, lse, do, ddq, ddk, ddv, scale=None, causal=False, return_stats=False, window=0):
    """Double backward (dQ', dK', dV', ddO) from the saved (O, L).

    Restates ``flash_hog/_jax_refs/jax_impl.py:273-336`` (``attn_bwd_bwd_stats``),
    the function that wrote the reference's known-answer vectors::

        P   = exp(S - L)                 dP  = dO V^T
        ddS = scale (ddQ K^T + Q ddK^T)  D   = rowsum(dO o O)
        dD  = rowsum(ddS o P)
        dP2 = dO ddV^T - dP dD - ddS D + dP o ddS
        B   = rowsum(dP2 o P)
        dS  = scale P o (dP - D)         dS2 = scale P o (dP2 - B)
        ddP = P o (ddS - dD)
        dQ' = dS ddK + dS2 K             dK' = dS^T ddQ + dS2^T Q
        dV' = ddP^T dO                   ddO = P ddV + ddP V

    With ``return_stats`` also returns (D, dD, B), each (B, N, T). Grouped-query
    inputs (fewer key heads) use key head n // group for query head n, and
    dK', dV' are summed over each group.
    """
    scale = default_scale(q.shape[-1]) if scale is None else scale
    g = _group(q, k)
    qh, oh, doh, ddqh = map(_heads, (q, o, do, ddq))
    kh, vh, ddkh, ddvh = (_expand(_heads(x), g) for x in (k, v, ddk, ddv))
    s = _scores(qh, kh, scale, causal, window)
    p = _probs(s, lse)
    dp = np.einsum("bhqd,bhkd->bhqk", doh, vh)
    dds = scale * (np.einsum("bhqd,bhkd->bhqk", ddqh, kh) + np.einsum("bhqd,bhkd->bhqk", qh, ddkh))
    d = np.einsum("bhqd,bhqd->bhq", oh, doh)[..., None]
    dd = (dds * p).sum(-1, keepdims=True)
    dp2 = np.einsum("bhqd,bhkd->bhqk", doh, ddvh) - dp * dd - dds * d + dp * dds
    bb = (dp2 * p).sum(-1, keepdims=True)
    ddp = p * (dds - dd)
    ds2 = scale * p * (dp2 - bb)
    ds = scale * p * (dp - d)
    dq2 = np.einsum("bhqk,bhkd->bhqd", ds, ddkh) + np.einsum("bhqk,bhkd->bhqd", ds2, kh)
    dk2 = _group_sum(np.einsum("bhqk,bhqd->bhkd", ds, ddqh) + np.einsum("bhqk,bhqd->bhkd", ds2, qh), g)
    dv2 = _group_sum(np.einsum("bhqk,bhqd->bhkd", ddp, doh), g)
    ddo = np.einsum("bhqk,bhkd->bhqd", p, ddvh) + np.einsum("bhqk,bhkd->bhqd", ddp, vh)
    out = (_btnh(dq2), _btnh(dk2), _btnh(dv2), _btnh(ddo))
    if return_stats:
        return out, (d[..., 0], dd[..., 0], bb[..., 0])
    return out


def bwdbwd_stats_rows(q, k, v, o, lse, do, ddq, ddk, ddv, scale=None, causal=False, window=0, chunk=1024):
    """``bwdbwd_stats`` evaluated over chunks of ``chunk`` query rows, in float64 with
    BLAS matmuls -- for the long sequences of the full-size checks (S = 8192), where
    one (Nq, Nk) float64 array per product would take gigabytes per head.

    Same formulas (``flash_hog/_jax_refs/jax_impl.py:273-336``). The split is exact:
    a query row's statistics D, dD and B need only that row's scores over all keys,
    so each chunk yields its dQ' and ddO rows and adds its share to dK' and dV'.
    Returns (dq2, dk2, dv2, ddo), BTNH, plus (D, dD, B) each (B, N, Tq).
    """
    scale = default_scale(q.shape[-1]) if scale is None else scale
    g = _group(q, k)
    qh, oh, doh, ddqh = map(_heads, (q, o, do, ddq))
    kh, vh, ddkh, ddvh = (_expand(_heads(x), g) for x in (k, v, ddk, ddv))
    lse = np.asarray(lse, np.float64)
    nq, nk = qh.shape[2], kh.shape[2]
    dq2, ddo = np.zeros_like(qh), np.zeros_like(qh)
    dk2, dv2 = np.zeros_like(kh), np.zeros_like(kh)
    stats = np.zeros((3,) + qh.shape[:3])
    kt, vt, ddkt, ddvt = (np.swapaxes(x, -1, -2) for x in (kh, vh, ddkh, ddvh))
    keep_all = causal_mask(nq, nk, causal, window) if causal else None
    for r0 in range(0, nq, chunk):
        rs = slice(r0, min(r0 + chunk, nq))
        qc, oc, doc, ddqc = qh[:, :, rs], oh[:, :, rs], doh[:, :, rs], ddqh[:, :, rs]
        s = np.matmul(qc, kt) * scale
        if causal:
            s = np.where(keep_all[rs], s, -np.inf)
        p = _probs(s, lse[:, :, rs])
        dp = np.matmul(doc, vt)
        dds = scale * (np.matmul(ddqc, kt) + np.matmul(qc, ddkt))
        d = (oc * doc).sum(-1, keepdims=True)
        dd = (dds * p).sum(-1, keepdims=True)
        dp2 = np.matmul(doc, ddvt) - dp * dd - dds * d + dp * dds
        bb = (dp2 * p).sum(-1, keepdims=True)
        ddp = p * (dds - dd)
        ds2 = scale * p * (dp2 - bb)
        ds = scale * p * (dp - d)
        dq2[:, :, rs] = np.matmul(ds, ddkh) + np.matmul(ds2, kh)
        ddo[:, :, rs] = np.matmul(p, ddvh) + np.matmul(ddp, vh)
        dk2 += np.matmul(np.swapaxes(ds, -1, -2), ddqc) + np.matmul(np.swapaxes(ds2, -1, -2), qc)
        dv2 += np.matmul(np.swapaxes(ddp, -1, -2), doc)
        stats[0][:, :, rs], stats[1][:, :, rs], stats[2][:, :, rs] = d[..., 0], dd[..., 0], bb[..., 0]
    out = (_btnh(dq2), _btnh(_group_sum(dk2, g)), _btnh(_group_sum(dv2, g)), _btnh(ddo))
    return out, (stats[0], stats[1], stats[2])


def bwdbwd_4pass(q, k, v, o, lse, do, ddq, ddk, ddv, scale=None, causal=False,
                 tile_q=32, tile_k=32):
    """Tiled 4-pass schedule of the reference's Pallas kernels, in float64.

    Follows ``flash_hog/jax/_pallas_gpu_kernel.py``: D precomputed by einsum
    (line 110); stage 1 over query tiles (126-305) with a dD sweep (149-186), a
    B sweep (191-225) and a dQ'/ddO sweep (227-278), each skipping key tiles
    that the causal mask removes entirely (172-183, 215-222, 259-270); stage 2
    over key tiles (309-416) with the dK'/dV' sweep (333-370, 372-382). No
    (Nq, Nk) array larger than one tile pair is formed. Returns the four
    outputs plus (D, dD, B) -- the stage-1 -> stage-2 scratch vectors.
    """
    scale = default_scale(q.shape[-1]) if scale is None else scale
    qh, kh, vh, oh, doh, ddqh, ddkh, ddvh = map(_heads, (q, k, v, o, do, ddq, ddk, ddv))
    lse = np.asarray(lse, np.float64)
    nb, nh, nq, hd = qh.shape
    nk = kh.shape[2]
    dq2 = np.zeros_like(qh)
    ddo = np.zeros_like(qh)
    dk2 = np.zeros_like(kh)
    dv2 = np.zeros_like(kh)
    dvec = np.einsum("bhqd,bhqd->bhq", doh, oh)
    ddvec = np.zeros((nb, nh, nq))
    bvec = np.zeros((nb, nh, nq))

    def tile_terms(b, h, qs, ks, d_i, dd_i):
        q_i, do_i, ddq_i = qh[b, h, qs], doh[b, h, qs], ddqh[b, h, qs]
        k_j, v_j, ddk_j, ddv_j = kh[b, h, ks], vh[b, h, ks], ddkh[b, h, ks], ddvh[b, h, ks]
        s = q_i @ k_j.T * scale
        if causal:
            s = np.where(np.arange(qs.start, qs.stop)[:, None] >= np.arange(ks.start, ks.stop)[None, :], s, -np.inf)
        p = np.exp(s - lse[b, h, qs][:, None])
        dp = do_i @ v_j.T
        dds = (ddq_i @ k_j.T + q_i @ ddk_j.T) * scale
        dp2 = None
        if dd_i is not None:
            dp2 = do_i @ ddv_j.T - dp * dd_i[:, None] - dds * d_i[:, None] + dp * dds
        return p, dp, dds, dp2

    def k_tiles_for(qt):
        if not causal:
            return range(0, -(-nk // tile_k))
        last_row = min((qt + 1) * tile_q, nq) - 1
        return range(0, min(last_row // tile_k + 1, -(-nk // tile_k)))

    for b in range(nb):
        for h in range(nh):
            for qt in range(-(-nq // tile_q)):
                qs = slice(qt * tile_q, min((qt + 1) * tile_q, nq))
                d_i = dvec[b, h, qs]
                dd_i = np.zeros(qs.stop - qs.start)
                for kt in k_tiles_for(qt):  # sweep 1: dD
                    ks = slice(kt * tile_k, min((kt + 1) * tile_k, nk))
                    p, _, dds, _ = tile_terms(b, h, qs, ks, d_i, None)
                    dd_i += (dds * p).sum(1)
                b_i = np.zeros_like(dd_i)
                for kt in k_tiles_for(qt):  # sweep 2: B
                    ks = slice(kt * tile_k, min((kt + 1) * tile_k, nk))
                    p, _, _, dp2 = tile_terms(b, h, qs, ks, d_i, dd_i)
                    b_i += (dp2 * p).sum(1)
                for kt in k_tiles_for(qt):  # sweep 3: dQ', ddO
                    ks = slice(kt * tile_k, min((kt + 1) * tile_k, nk))
                    p, dp, dds, dp2 = tile_terms(b, h, qs, ks, d_i, dd_i)
                    ds2 = p * (dp2 - b_i[:, None]) * scale
                    ds = scale * p * (dp - d_i[:, None])
                    ddp = p * (dds - dd_i[:, None])
                    dq2[b, h, qs] += ds @ ddkh[b, h, ks] + ds2 @ kh[b, h, ks]
                    ddo[b, h, qs] += ddp @ vh[b, h, ks] + p @ ddvh[b, h, ks]
                ddvec[b, h, qs] = dd_i
                bvec[b, h, qs] = b_i
            for kt in range(-(-nk // tile_k)):  # stage 2: dK', dV'
                ks = slice(kt * tile_k, min((kt + 1) * tile_k, nk))
                first_q = (kt * tile_k) // tile_q if causal else 0
                for qt in range(first_q, -(-nq // tile_q)):
                    qs = slice(qt * tile_q, min((qt + 1) * tile_q, nq))
                    d_i, dd_i, b_i = dvec[b, h, qs], ddvec[b, h, qs], bvec[b, h, qs]
                    p, dp, dds, dp2 = tile_terms(b, h, qs, ks, d_i, dd_i)
                    ds2 = p * (dp2 - b_i[:, None]) * scale
                    ds = scale * p * (dp - d_i[:, None])
                    ddp = p * (dds - dd_i[:, None])
                    dv2[b, h, ks] += ddp.T @ doh[b, h, qs]
                    dk2[b, h, ks] += ds.T @ ddqh[b, h, qs] + ds2.T @ qh[b, h, qs]
    return (_btnh(dq2), _btnh(dk2), _btnh(dv2), _btnh(ddo)), (dvec, ddvec, bvec)


# --------------------------------------------------------------------------------------
# double backward: autodiff of naive attention (the "XLA reference" analogue)
# --------------------------------------------------------------------------------------

def _torch_attention(q, k, v, scale, causal, window=0):
    """Naive attention in torch ops (every query must see at least one key)."""
    group = q.shape[2] // k.shape[2]
    if group > 1:  # query head n uses key head n // group; autograd sums the group
        k, v = k.repeat_interleave(group, dim=2), v.repeat_interleave(group, dim=2)
    s = torch.einsum("bqhd,bkhd->bhqk", q, k) * scale
    if causal:
        keep = torch.from_numpy(causal_mask(q.shape[1], k.shape[1], causal, window)).to(s.device)
        s = s.masked_fill(~keep, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("bhqk,bkhd->bqhd", p, v)


def autograd_all(q, k, v, do, ddq, ddk, ddv, scale=None, causal=False, window=0):
    """vjp-of-vjp of naive softmax attention, by torch autograd on the CPU.

    The analogue of the reference test oracle ``make_reference_dpa_bwd_bwd``
    (``tests/test_jax_fhog.py:18-34``): XLA autodiff of
    ``jax.nn.dot_product_attention(implementation="xla")`` differentiated
    twice. Inputs are torch tensors (BTNH) in the compute dtype; returns
    ``dict(o, dq, dk, dv, dq2, dk2, dv2, ddo)``. The second-order outputs are
    the cotangents of (Q, K, V, dO) for the cotangent (ddQ, ddK, ddV) on the
    first-order outputs (dQ, dK, dV).
    """
    scale = default_scale(q.shape[-1]) if scale is None else scale
    q, k, v, do = (t.detach().clone().requires_grad_(True) for t in (q, k, v, do))
    with torch.enable_grad():
        o = _torch_attention(q, k, v, scale, causal, window)
        dq, dk, dv = torch.autograd.grad(o, (q, k, v), do, create_graph=True)
        dq2, dk2, dv2, ddo = torch.autograd.grad((dq, dk, dv), (q, k, v, do), (ddq, ddk, ddv))
    return dict(o=o.detach(), dq=dq.detach(), dk=dk.detach(), dv=dv.detach(),
                dq2=dq2, dk2=dk2, dv2=dv2, ddo=ddo)


# --------------------------------------------------------------------------------------
# forward mode: jvp of the forward and of the first-order backward
# --------------------------------------------------------------------------------------

def jvp_fwd(q, k, v, o, lse, tq, tk, tv, scale=None, causal=False, window=0):
    """Forward tangents (tO, tL) of (O, L) along (tQ, tK, tV), in float64.

    No counterpart in the reference (reverse-mode rules only,
    ``flash_hog/jax/attention.py:52-60``). With tS = scale (tQ K^T + Q tK^T):
    tL = rowsum(P o tS), tP = P o (tS - tL), tO = tP V + P tV -- the ddO and dD
    of ``bwdbwd_stats`` with (ddQ, ddK, ddV) = (tQ, tK, tV), which do not
    depend on dO.
    """
    zero = np.zeros_like(np.asarray(q, np.float64))
    (_, _, _, to), (_, tl, _) = bwdbwd_stats(q, k, v, o, lse, zero, tq, tk, tv, scale=scale, causal=causal,
                                              return_stats=True, window=window)
    return to, tl


def jvp_bwd(q, k, v, o, lse, do, tq, tk, tv, tdo=None, scale=None, causal=False, window=0):
    """Forward-mode derivative (tdQ, tdK, tdV) of the first-order backward, float64.

    The backward is grad_{Q,K,V} phi with phi = <O(Q, K, V), dO>, so
        jvp(tQ, tK, tV, tdO) = Hess(phi) (tQ, tK, tV) + J_O^T tdO,
    and Hess(phi) being symmetric, its product with the tangent is the double
    backward (``bwdbwd_stats``) with (ddQ, ddK, ddV) = (tQ, tK, tV); J_O^T tdO
    is the first-order backward (``attention_bwd``) of tdO.
    """
    dq2, dk2, dv2, _ = bwdbwd_stats(q, k, v, o, lse, do, tq, tk, tv, scale=scale, causal=causal, window=window)
    if tdo is None:
        return dq2, dk2, dv2
    dq, dk, dv = attention_bwd(q, k, v, o, lse, tdo, scale=scale, causal=causal, window=window)
    return dq2 + dq, dk2 + dk, dv2 + dv


def autograd_jvp(q, k, v, do, tq, tk, tv, tdo, scale=None, causal=False, window=0):
    """Forward-over-reverse derivatives of naive softmax attention by ``torch.func``
    (an independent statement of ``jvp_fwd`` / ``jvp_bwd``): returns
    ``dict(o, to, tlse, dq, dk, dv, tdq, tdk, tdv)`` for torch inputs (BTNH)."""
    import torch.func as tf

    scale = default_scale(q.shape[-1]) if scale is None else scale

    def attn(q_, k_, v_):
        return _torch_attention(q_, k_, v_, scale, causal, window)

    def lse_fn(q_, k_):
        group = q_.shape[2] // k_.shape[2]
        kk = k_.repeat_interleave(group, dim=2) if group > 1 else k_
        s = torch.einsum("bqhd,bkhd->bhqk", q_, kk) * scale
        if causal:
            keep = torch.from_numpy(causal_mask(q_.shape[1], kk.shape[1], causal, window))
            s = s.masked_fill(~keep, float("-inf"))
        return torch.logsumexp(s, dim=-1)

    def bwd(q_, k_, v_, do_):
        _, vjp = tf.vjp(attn, q_, k_, v_)
        return vjp(do_)

    o, to = tf.jvp(attn, (q, k, v), (tq, tk, tv))
    _, tlse = tf.jvp(lse_fn, (q, k), (tq, tk))
    (dq, dk, dv), (tdq, tdk, tdv) = tf.jvp(bwd, (q, k, v, do), (tq, tk, tv, tdo))
    return dict(o=o, to=to, tlse=tlse, dq=dq, dk=dk, dv=dv, tdq=tdq, tdk=tdk, tdv=tdv)


# --------------------------------------------------------------------------------------
# seeded inputs and credited work
# --------------------------------------------------------------------------------------

def make_inputs(batch, heads, seq_q, seq_k, head_dim, seed=0, dtype=None, kv_heads=None):
    """Seeded N(0,1) Q, K, V, dO, ddQ, ddK, ddV (BTNH) as torch tensors.

    Draw order and shapes follow the reference tests
    (``tests/test_jax_fhog.py:125-132``: q, k, v, do, ddq, ddk, ddv); the
    generator is torch's, seeded with ``seed``. ``dtype`` defaults to bf16;
    ``kv_heads`` (default ``heads``) sets the key-side head count.
    """
    dtype = torch.bfloat16 if dtype is None else dtype
    g = torch.Generator().manual_seed(seed)
    qs = (batch, seq_q, heads, head_dim)
    ks = (batch, seq_k, heads if kv_heads is None else kv_heads, head_dim)
    shapes = dict(q=qs, k=ks, v=ks, do=qs, ddq=qs, ddk=ks, ddv=ks)
    return {n: torch.randn(s, generator=g, dtype=torch.float32).to(dtype) for n, s in shapes.items()}


def causal_pairs(batch, heads, seq_q, seq_k, causal):
    """(query, key) pairs the mask keeps, summed over batch and heads."""
    if not causal:
        return batch * heads * seq_q * seq_k
    per_head = sum(min(i + 1, seq_k) for i in range(seq_q))
    return batch * heads * per_head


def bwdbwd_flops(batch, heads, seq_q, seq_k, head_dim, causal, gemms=22):
    """Credited double-backward FLOPs: ``gemms * 2 * D`` per kept (q, k) pair.

    22 GEMM-equivalents per pair is the atomic-free, no-(Nq,Nk)-intermediate
    schedule (14 in the query-tiled pass, 8 in the key-tiled pass), the count
    of the reference's fastest kernels (``csrc/tk_bwdbwd/stage1.cuh:173-177,219-222``,
    ``stage2.cuh:172-176,215-217``).
    """
    return gemms * 2 * head_dim * causal_pairs(batch, heads, seq_q, seq_k, causal)


def rel_err(a, b) -> float:
    """max|a-b| / max|b| -- the parity metric used by the tests."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = max(float(np.abs(b).max()), 1e-30)
    return float(np.abs(a - b).max()) / den


def max_abs(a, b) -> float:
    return float(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64)).max())
