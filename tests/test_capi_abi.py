"""The C ABI library loads, exports every symbol the header declares, and
rejects bad arguments with the documented status codes -- all without a GPU
(validation precedes any CUDA call)."""

import ctypes
import os
import re
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "flash_hog_b200.h")


def _declared():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^\s*(?:int|const char\*|unsigned long long|long long)\s+(fh_\w+)\s*\(", text,
                                 re.M)))


def test_header_declares_the_binding_symbols():
    from flash_hog_b200 import _capi

    assert _declared() == sorted(_capi.EXPORTED_SYMBOLS)


def test_library_exports_every_declared_symbol():
    from flash_hog_b200 import _capi

    lib = ctypes.CDLL(_capi.library_path())
    for name in _declared():
        assert hasattr(lib, name), name
    h = _capi.lib()
    assert h.fh_abi_version() == _capi.ABI_VERSION
    assert h.fh_status_string(0) == b"ok"
    assert h.fh_status_string(5) == b"injected error"


def _arities():
    """Parameter count of every function the header declares."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    out = {}
    for name, params in re.findall(r"(fh_\w+)\s*\(([^)]*)\)\s*;", text):
        params = params.strip()
        out[name] = 0 if params in ("", "void") else params.count(",") + 1
    return out


def test_binding_argtypes_match_the_header():
    from flash_hog_b200 import _capi

    h = _capi.lib()
    arities = _arities()
    assert sorted(arities) == sorted(_capi.EXPORTED_SYMBOLS)
    for name, n in arities.items():
        assert len(getattr(h, name).argtypes) == n, f"{name}: binding has {len(getattr(h, name).argtypes)}, header {n}"


def _dims(**kw):
    from flash_hog_b200._capi import FhAttnDims, FhStrides

    d = dict(batch=1, heads=2, seq_q=128, seq_k=128, head_dim=64)
    d.update(kw)
    st = FhStrides(128 * 2 * 64, 2 * 64, 64)
    return FhAttnDims(d["batch"], d["heads"], d["seq_q"], d["seq_k"], d["head_dim"], st, st, 0, d.get("window", 0))


def _fwd(dims, ptr=64, causal=1):
    from flash_hog_b200._capi import lib

    p = ctypes.c_void_p(ptr)
    return lib().fh_attn_fwd(None, ctypes.byref(dims) if dims is not None else None, p, p, p, p, p, 0.125, causal)


def test_argument_validation_codes():
    assert _fwd(None) == 1                      # null dims
    assert _fwd(_dims(), causal=3) == 1         # causal code outside 0..2
    assert _fwd(_dims(window=-1)) == 1          # negative window
    assert _fwd(_dims(window=8), causal=0) == 1  # a window needs a causal mask
    assert _fwd(_dims(head_dim=32)) == 2        # unsupported head_dim
    assert _fwd(_dims(seq_q=0)) == 1            # empty sequence
    assert _fwd(_dims(batch=0)) == 1
    assert _fwd(_dims(), ptr=8) == 1            # pointers not 16-byte aligned
    d = _dims()
    d.q.seq = 12                                # stride not a multiple of 8 elements
    assert _fwd(d) == 1


def test_f32_entry_points_validate_like_the_bf16_ones():
    """The fp32 entries share the dims/mask/alignment checks (all before any CUDA call)."""
    from flash_hog_b200._capi import lib

    h = lib()
    p = ctypes.c_void_p(64)

    def fwd(dims, ptr=64, causal=1):
        q = ctypes.c_void_p(ptr)
        return h.fh_attn_fwd_f32(None, ctypes.byref(dims), q, q, q, q, q, 0.125, causal)

    assert fwd(_dims(), causal=3) == 1
    assert fwd(_dims(head_dim=96)) == 2
    assert fwd(_dims(window=8), causal=0) == 1
    assert fwd(_dims(), ptr=8) == 1
    assert h.fh_attn_bwd_f32(None, ctypes.byref(_dims()), p, p, p, p, p, None, p, p, p, p, 0.125, 1) == 1  # no lse
    bb = lambda passes, dq2=p, o=p: h.fh_attn_bwdbwd_f32(None, ctypes.byref(_dims()), p, p, p, o, p, p, p, p, p,
                                                        dq2, p, p, p, p, p, p, 0.125, 1, passes)
    assert bb(0) == 1 and bb(4) == 1            # passes outside 1..3
    assert bb(1, o=None) == 1                   # the query pass needs o (it computes D)
    assert bb(1, dq2=ctypes.c_void_p(8)) == 1   # dq2 may be NULL, but not misaligned
    assert h.fh_attn_jvp_bwd_f32(None, ctypes.byref(_dims()), *([p] * 9), ctypes.c_void_p(8), *([p] * 7), 0.125,
                                 1) == 1        # misaligned tdO


def test_error_injection_is_host_side():
    """FLASH_HOG_B200_INJECT_ERROR makes the named entry return FH_ERR_INJECTED
    before any validation or CUDA call (checked in a fresh process)."""
    code = (
        "import ctypes,sys; sys.path.insert(0, %r)\n"
        "from flash_hog_b200 import _capi\n"
        "h=_capi.lib(); d=_capi.FhAttnDims()\n"
        "p=ctypes.c_void_p(0)\n"
        "print(h.fh_attn_bwdbwd(None, ctypes.byref(d), *([p]*15), 0.1, 1), h.fh_attn_fwd(None, None, p,p,p,p,p, 0.1, 0))\n"
    ) % ROOT
    env = dict(os.environ, FLASH_HOG_B200_INJECT_ERROR="fh_attn_bwdbwd")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    assert out.stdout.split() == ["5", "1"]


def test_python_errors_are_loud():
    import torch

    import flash_hog_b200 as fhb
    from flash_hog_b200._capi import FlashHogError

    q = torch.zeros(1, 128, 2, 64)
    with pytest.raises(ValueError):
        fhb.dot_product_attention(q, q, q)      # CPU tensors: no CPU fallback
    assert issubclass(FlashHogError, RuntimeError)
