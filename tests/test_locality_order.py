"""Every tile is computed under the locality-grouped launch order.

When the per-head tiles that a kernel's CTAs share (K and V for query tiles; Q and dO
for key tiles) are larger together than L2 holds, the attention kernels launch their
(head, batch) pairs in groups, each group heaviest tile first (``grouped_order`` in
``csrc/attn_common.cuh``). These shapes make the forward, both first-order passes and
both double-backward passes group their pairs, each with a last group smaller than the
others. Every output is pre-filled with NaN, so a tile that the order skipped would
show; sampled heads from the first, a middle and the last group are checked against
the oracle.
"""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from parity_util import assert_close, assert_elementwise, np64

pytestmark = pytest.mark.gpu

CASES = [
    # b, q heads, kv heads, t, d (causal). At t=2048, d=128 the shared tiles of 104
    # key heads take 104-208 MB: groups of 32 / 16 / 21 pairs (forward and first-order
    # passes / double-backward query pass / key pass), last groups of 8, 8 and 20.
    (1, 104, 104, 2048, 128),
    # GQA, two query heads per key head, so groups hold whole query-head groups:
    # forward and dQ pass 64 pairs (last 16), dK/dV pass 16 (last 8), double-backward
    # query pass 32 (last 16), key pass 10 (last 4).
    (1, 208, 104, 2048, 128),
    # head_dim 64 (the two-CTA-per-SM layouts): 208 heads of 0.5-1 MB -> groups of
    # 64 / 32 / 42 pairs, last groups of 16, 16 and 40.
    (1, 208, 208, 2048, 64),
]


def _nan_like(t, dtype=None):
    return torch.full_like(t, float("nan"), dtype=dtype or t.dtype)


def _stats(b, h, t, device):
    return torch.full((b, h, t), float("nan"), dtype=torch.float32, device=device)


@pytest.mark.parametrize("b,h,hk,t,d", CASES)
def test_grouped_launch_order_covers_every_tile(b, h, hk, t, d):
    from flash_hog_b200 import _capi
    from flash_hog_b200._capi import device_status

    x = ora.make_inputs(b, h, t, t, d, seed=11 + h, kv_heads=hk)
    g = {n: x[n].cuda() for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")}
    scale = d ** -0.5
    dev = g["q"].device

    o, lse = _nan_like(g["q"]), _stats(b, h, t, dev)
    _capi.attn_fwd(g["q"], g["k"], g["v"], o, lse, scale, 1)
    dq, dk, dv, delta = _nan_like(g["q"]), _nan_like(g["k"]), _nan_like(g["v"]), _stats(b, h, t, dev)
    _capi.attn_bwd(g["q"], g["k"], g["v"], o, g["do"], lse, dq, dk, dv, delta, scale, 1)
    dq2, ddo, dk2, dv2 = _nan_like(g["q"]), _nan_like(g["q"]), _nan_like(g["k"]), _nan_like(g["v"])
    delta2, dd, bv = _stats(b, h, t, dev), _stats(b, h, t, dev), _stats(b, h, t, dev)
    _capi.attn_bwdbwd_o(g["q"], g["k"], g["v"], o, g["do"], g["ddq"], g["ddk"], g["ddv"], lse, dq2, ddo, dk2, dv2,
                        delta2, dd, bv, scale, 1)
    torch.cuda.synchronize()
    assert device_status() == 0
    for name, out in (("O", o), ("L", lse), ("dQ", dq), ("dK", dk), ("dV", dv), ("D", delta), ("dQ2", dq2),
                      ("ddO", ddo), ("dK2", dk2), ("dV2", dv2), ("dD", dd), ("B", bv)):
        assert torch.isfinite(out).all(), f"{name}: rows left unwritten under the grouped order"

    grp = h // hk
    kheads = [0, hk // 2 + 3, hk - 1]  # first, a middle and the last group of every kernel
    qheads = [kh * grp + i for kh in kheads for i in range(grp)]
    qs = lambda a: np64(a)[:, :, qheads]
    ks = lambda a: np64(a)[:, :, kheads]
    st = lambda a: np64(a)[:, qheads]
    q, k, v, do = qs(g["q"]), ks(g["k"]), ks(g["v"]), qs(g["do"])

    ro, rl = ora.attention_fwd(q, k, v, scale=scale, causal=True)
    assert_close("O", qs(o), ro)
    assert ora.max_abs(st(lse), rl) <= 2e-3
    o_s, l_s = qs(o), st(lse)
    for name, got, ref in zip(("dQ", "dK", "dV"), (qs(dq), ks(dk), ks(dv)),
                              ora.attention_bwd(q, k, v, o_s, l_s, do, scale=scale, causal=True)):
        assert_close(name, got, ref)
    want, (wd, wdd, wb) = ora.bwdbwd_stats_rows(q, k, v, o_s, l_s, do, qs(g["ddq"]), ks(g["ddk"]), ks(g["ddv"]),
                                                scale=scale, causal=True)
    for name, got, ref in zip(("dQ2", "dK2", "dV2", "ddO"), (qs(dq2), ks(dk2), ks(dv2), qs(ddo)), want):
        assert_close(name, got, ref)
        assert_elementwise(name, got, ref)
    for name, got, ref in (("D", st(delta2), wd), ("dD", st(dd), wdd), ("B", st(bv), wb)):
        assert_close(name, got, ref)
    assert np.array_equal(np64(delta2), np64(delta)) or ora.rel_err(np64(delta2), np64(delta)) <= 1e-5
