"""The C-ABI library: it loads, exports every symbol include/*.h declares, and
rejects bad arguments before touching a GPU."""
import ctypes
import glob
import os
import re

import pytest

from test_speed_scalesweep_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
        names.update(re.findall(r"\b(ssw_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "ssw_scalesweep_mse_nvfp4_quant_out" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol(built_library):
    h = ctypes.CDLL(built_library)
    missing = [n for n in declared_symbols() if not hasattr(h, n)]
    assert not missing, missing


def test_python_binding_covers_every_declared_symbol(built_library):
    assert set(declared_symbols()) <= set(_lib._SIGNATURES)


def test_abi_version(built_library):
    assert _lib.lib().ssw_abi_version() == _lib.ABI_VERSION


def _call(fn, *, dtype=0, m=4, n=64, pn=64, scale=1, out=1, osc=1, swz=1, inp=1):
    p = lambda v: ctypes.c_void_p(0x1000 * v) if v else None  # never dereferenced
    return fn(p(inp), dtype, m, n, pn, p(scale), p(out), p(osc), swz, None)


@pytest.mark.parametrize("kwargs,needle", [
    (dict(dtype=7), "dtype"),
    (dict(n=40, pn=40), "multiple of 16"),
    (dict(pn=72), "multiple of 16"),
    (dict(pn=48), "must be >= n"),
    (dict(m=-1), "negative"),
    (dict(out=0), "null"),
    (dict(scale=0), "null"),
])
def test_invalid_arguments_are_rejected_without_a_gpu(built_library, kwargs, needle):
    h = _lib.lib()
    st = _call(h.ssw_scalesweep_mse_nvfp4_quant_out, **kwargs)
    assert st == _lib.SSW_ERR_INVALID_ARGUMENT
    assert needle in h.ssw_last_error().decode()
    with pytest.raises(ValueError, match=needle):
        _lib.check(st)


def test_reference_variant_rejects_padded_n(built_library):
    h = _lib.lib()
    st = _call(h.ssw_scalesweep_mse_reference_nvfp4_quant_out, pn=96)
    assert st == _lib.SSW_ERR_INVALID_ARGUMENT
    assert "does not support padded_n" in h.ssw_last_error().decode()


def test_empty_problem_is_a_no_op(built_library):
    h = _lib.lib()
    assert _call(h.ssw_scalesweep_mse_nvfp4_quant_out, m=0, out=0, osc=0, scale=0, inp=0) == 0
    assert _call(h.ssw_rtn_nvfp4_quant_out, n=0, pn=0) == 0


def test_amax_rejects_empty_and_null(built_library):
    h = _lib.lib()
    ws = ctypes.c_void_p(0x1000)
    assert h.ssw_absmax(ctypes.c_void_p(0x1000), 0, 0, ctypes.c_void_p(0x2000), ws, None) == 1
    assert h.ssw_absmax(None, 0, 16, ctypes.c_void_p(0x2000), ws, None) == 1
    assert h.ssw_global_scale_inv(ctypes.c_void_p(0x1000), 0, 16, 448.0, None, None, ws, None) == 1
    assert h.ssw_absmax_workspace_bytes() >= 8
