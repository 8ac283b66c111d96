"""Full-size parity of the double backward on BASELINE's long-sequence and
cross-attention configurations (through the public ``flash_bwdbwd`` and the C ABI).

* configuration 3: causal B2 H32 S8192 D128;
* configuration 4: non-causal B8 H16 Sq4096 Sk2048 D128 (cross attention with more
  queries than keys -- the Pallas rule's non-causal branch,
  ``flash_hog/jax/_pallas_gpu_kernel.py:85-101,309-416``).

Both run on the whole batch on the GPU. The oracle (float64 explicit formulas,
evaluated over query-row chunks) checks sampled (batch, head) pairs: the
query-side outputs of a head depend only on that head, and the key-side outputs
of a head only on the query heads of its group, so a sampled head is checked
exactly. Bar: the bf16 tolerance, max-normalised and per element.
"""

import numpy as np
import pytest
import torch

from oracle import attention_oracle as ora
from parity_util import assert_close, assert_elementwise, np64, select_heads

pytestmark = pytest.mark.gpu


def _full_size(b, h, sq, sk, d, causal, heads, seed):
    from flash_hog_b200 import MaskType, flash_bwdbwd
    from flash_hog_b200 import _attention_impl as impl
    from flash_hog_b200._capi import device_status

    x = ora.make_inputs(b, h, sq, sk, d, seed=seed)
    g = {k: v.cuda() for k, v in x.items()}
    mask = MaskType.CAUSAL if causal else MaskType.NO_MASK
    o, lse = impl.cuda_dot_product_attention(g["q"], g["k"], g["v"], mask, d ** -0.5, return_residual=True)
    (dq2, dk2, dv2, ddo), (dl, dd, bv) = flash_bwdbwd(g["q"], g["k"], g["v"], o, g["do"], g["ddq"], g["ddk"],
                                                      g["ddv"], lse, mask_type=mask, return_stats=True)
    torch.cuda.synchronize()
    assert device_status() == 0
    for t in (dq2, dk2, dv2, ddo):
        assert torch.isfinite(t).all()
    sel = lambda t: select_heads(t, heads)
    arrs = {n: sel(x[n]) for n in ("q", "k", "v", "do", "ddq", "ddk", "ddv")}
    arrs["o"], lse_s = sel(o), select_heads(lse, heads, stat=True)
    want, (wd, wdd, wb) = ora.bwdbwd_stats_rows(arrs["q"], arrs["k"], arrs["v"], arrs["o"], lse_s, arrs["do"],
                                                arrs["ddq"], arrs["ddk"], arrs["ddv"], causal=causal)
    report = {}
    for name, got, ref in zip(("dQ2", "dK2", "dV2", "ddO"), (dq2, dk2, dv2, ddo), want):
        got = sel(got)
        report[name] = (assert_close(name, got, ref), assert_elementwise(name, got, ref))
    for name, got, ref in (("D", dl, wd), ("dD", dd, wdd), ("B", bv, wb)):
        report[name] = (assert_close(name, select_heads(got, heads, stat=True), ref),)
    print({k: tuple(float(f"{e:.2e}") for e in v) for k, v in report.items()})


def test_cfg3_causal_b2_h32_s8192_d128_full_size():
    _full_size(2, 32, 8192, 8192, 128, True, [(0, 0), (1, 31), (0, 17)], seed=3)


def test_cfg4_noncausal_b8_h16_sq4096_sk2048_d128_full_size():
    _full_size(8, 16, 4096, 2048, 128, False, [(0, 0), (7, 15), (3, 9), (5, 2)], seed=4)
