"""Helpers shared by the parity tests: seeded inputs, oracle evaluation, tolerances."""

from __future__ import annotations

import numpy as np
import torch

from oracle import attention_oracle as ora

# Parity bar for bf16 inputs (fp32 accumulation): max|gpu - oracle| / max|oracle|.
BF16_REL_TOL = 2e-2


def np64(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy().astype(np.float64)


def case_inputs(b, h, tq, tk, d=64, seed=0, causal=False, kv_heads=None):
    """Seeded bf16 inputs plus the oracle forward (O rounded to bf16, L fp32)."""
    x = ora.make_inputs(b, h, tq, tk, d, seed=seed, kv_heads=kv_heads)
    o, lse = ora.attention_fwd(np64(x["q"]), np64(x["k"]), np64(x["v"]), causal=causal)
    x["o"] = torch.from_numpy(o).to(torch.bfloat16)
    x["lse"] = torch.from_numpy(lse).float()
    return x


def oracle_bwdbwd(x, causal, scale=None, heads=None):
    """Oracle double backward (and its stats) on the bf16 values of `x`.

    `heads` optionally restricts to a list of (b, h) pairs (full-size tests)."""
    names = ["q", "k", "v", "o", "lse", "do", "ddq", "ddk", "ddv"]
    arrs = {n: np64(x[n]) for n in names}
    if heads is not None:
        sel = {}
        for n in names:
            if n == "lse":
                sel[n] = np.stack([arrs[n][b, h] for b, h in heads])[None]
            else:
                sel[n] = np.stack([arrs[n][b, :, h] for b, h in heads], axis=1)[None]
        arrs = sel
    return ora.bwdbwd_stats(arrs["q"], arrs["k"], arrs["v"], arrs["o"], arrs["lse"], arrs["do"], arrs["ddq"],
                            arrs["ddk"], arrs["ddv"], scale=scale, causal=causal, return_stats=True)


def select_heads(t: torch.Tensor, heads, stat=False) -> np.ndarray:
    a = np64(t)
    if stat:
        return np.stack([a[b, h] for b, h in heads])[None]
    return np.stack([a[b, :, h] for b, h in heads], axis=1)[None]


def assert_close(name, got, ref, tol=BF16_REL_TOL):
    err = ora.rel_err(got, ref)
    assert np.isfinite(np.asarray(got)).all(), f"{name}: non-finite values"
    assert err <= tol, f"{name}: rel err {err:.3e} > {tol:.1e} (max abs {ora.max_abs(got, ref):.3e})"
    return err


# Per-element bound beside the max-normalised one: every element must satisfy
# |gpu - oracle| <= ELEM_ATOL * max|oracle| + ELEM_RTOL * |oracle|, so elements of
# small magnitude (rows near the causal diagonal, keys few queries see) are held
# to the bar relative to the tensor's scale rather than hidden under its maximum.
ELEM_RTOL = 2e-2
ELEM_ATOL = 5e-3


def elementwise_excess(got, ref, rtol=ELEM_RTOL) -> float:
    """Smallest atol (as a fraction of max|ref|) for which every element passes
    |got - ref| <= atol * max|ref| + rtol * |ref|."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    den = max(float(np.abs(ref).max()), 1e-30)
    return max(float((np.abs(got - ref) - rtol * np.abs(ref)).max()) / den, 0.0)


def assert_elementwise(name, got, ref, rtol=ELEM_RTOL, atol=ELEM_ATOL):
    ex = elementwise_excess(got, ref, rtol)
    assert ex <= atol, (f"{name}: an element exceeds {atol:.0e} * max|ref| + {rtol:.0e} * |ref| "
                        f"(needs atol {ex:.2e})")
    return ex
