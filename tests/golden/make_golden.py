"""Regenerate ``kat_bwdbwd.npz`` from the reference's known-answer archive.

The reference ships ``test_data.zip`` at the root of its checkout. It holds the
pickled fp32 tensors written by ``flash_hog/_jax_refs/jax_impl.py:404-477``
(``scuffed_save_bwd_bwd``, driven from ``jax_impl.py:594-654``):

* ``input_items/{q,k,v,o,do,ddq,ddk,ddv,L}.pt`` -- one unbatched head, Nq=128,
  Nk=256, D=64, non-causal, softmax scale 1/8;
* ``output_items/{dq2,dk2,dv2,ddo}.pt`` -- the double-backward outputs.

q, k, v, do, ddq, ddk and ddv are bf16 values stored as fp32 (they were drawn
as bf16), so they are kept here as raw bf16 bit patterns (uint16) to halve the
fixture. o, L and the four outputs are kept as fp32.

Usage::

    python tests/golden/make_golden.py <reference checkout>/test_data.zip

The archive is read once, here; nothing at test time reads the reference.
"""

import io
import sys
import zipfile
from pathlib import Path

import numpy as np
import torch

BF16_INPUTS = ("q", "k", "v", "do", "ddq", "ddk", "ddv")
F32_INPUTS = ("o", "L")
OUTPUTS = ("dq2", "dk2", "dv2", "ddo")


def bf16_bits(t: torch.Tensor) -> np.ndarray:
    b = t.to(torch.bfloat16)
    assert torch.equal(b.float(), t), "expected a bf16-representable tensor"
    return b.view(torch.int16).numpy().view(np.uint16)


def main(zip_path: str) -> None:
    z = zipfile.ZipFile(zip_path)

    def load(kind: str, name: str) -> torch.Tensor:
        return torch.load(io.BytesIO(z.read(f"test_data/{kind}/{name}.pt")), weights_only=True)

    arrays = {}
    for n in BF16_INPUTS:
        arrays[n + "_bf16"] = bf16_bits(load("input_items", n))
    for n in F32_INPUTS:
        arrays[n] = load("input_items", n).numpy().astype(np.float32)
    for n in OUTPUTS:
        arrays[n] = load("output_items", n).numpy().astype(np.float32)
    arrays["scale"] = np.float32(0.125)
    arrays["causal"] = np.int32(0)
    out = Path(__file__).with_name("kat_bwdbwd.npz")
    np.savez_compressed(out, **arrays)
    print(f"wrote {out} ({out.stat().st_size} bytes)")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
