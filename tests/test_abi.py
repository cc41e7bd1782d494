"""The C ABI without a GPU: the library loads, exports every entry point its header declares,
and rejects bad arguments with the reference's fail-fast statuses before touching a device."""

import ctypes
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

import jitcast_b200
from jitcast_b200 import _lib
from jitcast_b200 import chronos2, timestral, tirex2  # noqa: F401  (their entry points' ctypes prototypes)

HEADERS = sorted((Path(__file__).resolve().parent.parent / "include").glob("*.h"))


def declared_symbols():
    names = set()
    for h in HEADERS:
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(jc_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    assert "jc_linear" in declared_symbols()


@pytest.mark.parametrize("name", declared_symbols())
def test_library_exports(name):
    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_prototypes_cover_header():
    missing = [n for n in declared_symbols() if n not in _lib.PROTOTYPES]
    assert not missing, f"no ctypes prototype for {missing}"


def test_version():
    assert "sm_100a" in jitcast_b200.version()


def _call_linear(**kw):
    a = np.ones((4, 8), np.float32)
    w = np.ones((3, 8), np.float32)
    c = np.zeros((4, 3), np.float32)
    args = dict(device=0, precision=_lib.BF16, a=a.ctypes.data, w=w.ctypes.data, bias=None, c=c.ctypes.data,
                m=4, n=3, k=8, flags=0)
    args.update(kw)
    return _lib.lib().jc_linear(*args.values())


@pytest.mark.parametrize("kw,status", [
    (dict(m=0), _lib.ERR_INVALID_ARG),
    (dict(k=-1), _lib.ERR_INVALID_ARG),
    (dict(precision=9), _lib.ERR_INVALID_ARG),
    (dict(flags=_lib.BIAS), _lib.ERR_INVALID_ARG),        # bias flag without a bias
    (dict(flags=_lib.TWIN_ONLY), _lib.ERR_INVALID_ARG),
    (dict(flags=1 << 10), _lib.ERR_INVALID_ARG),
    (dict(flags=_lib.GELU | _lib.SILU), _lib.ERR_INVALID_ARG),
    (dict(a=None), _lib.ERR_INVALID_ARG),
])
def test_invalid_arguments(kw, status):
    assert _call_linear(**kw) == status
    assert _lib.last_error()


def test_argument_errors_raise_value_error():
    with pytest.raises(ValueError):
        jitcast_b200.ops.gemm(np.ones((2, 3)), np.ones((4, 5)), None, None, 0)
    with pytest.raises(jitcast_b200.JcArgumentError):
        jitcast_b200.ops.gemm(np.ones((2, 3)), np.ones((4, 3)), None, None, _lib.TWIN_ONLY)


def test_no_device_is_reported():
    if _lib.lib().jc_device_count() > 0:
        pytest.skip("a device is present")
    st = _call_linear()
    assert st == _lib.ERR_NO_DEVICE
    assert "device" in _lib.last_error().lower()


@pytest.mark.parametrize("name", ["jc_forecast_timestral", "jc_forecast_chronos2", "jc_forward_timestral",
                                  "jc_forward_chronos2", "jc_forward_tirex2"])
def test_model_forwards_reject_a_null_engine(name):
    # the reference's fail-fast contract: a bad handle is an argument error, reported before any device work
    assert getattr(_lib.lib(), name)(None, None, None) == _lib.ERR_INVALID_ARG
    assert "engine" in _lib.last_error()


@pytest.mark.parametrize("name", ["jc_forecast_timestral_device", "jc_forecast_chronos2_device"])
def test_device_forecasts_reject_a_null_engine(name):
    assert getattr(_lib.lib(), name)(None, 0, None, None, None) == _lib.ERR_INVALID_ARG
    assert "engine" in _lib.last_error()


# every ctypes mirror of a header struct: (C struct, Python class) — sizes and field offsets must agree
_STRUCTS = [("jc_tensor_view", "timestral._TensorView"), ("jc_timestral_desc", "timestral._Desc"),
            ("jc_timestral_block", "timestral.Block"), ("jc_timestral_window", "timestral.Window"),
            ("jc_chronos2_desc", "chronos2._Desc"), ("jc_chronos2_block", "chronos2.Block"),
            ("jc_chronos2_window", "chronos2.Window"), ("jc_tirex2_desc", "tirex2._Desc"),
            ("jc_tirex2_batch", "tirex2.Batch"), ("jc_gemm_problem", "ops.GemmProblem")]


def test_struct_layouts_match_the_header(tmp_path):
    # the C compiler's sizeof/offsetof for each struct of include/jitcast_b200.h against the Python mirrors
    import importlib
    import shutil

    if not shutil.which("gcc"):
        pytest.skip("no C compiler")
    classes = {c: getattr(importlib.import_module(f"jitcast_b200.{p.split('.')[0]}"), p.split(".")[1])
               for c, p in _STRUCTS}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "jitcast_b200.h"', "int main(void) {"]
    for c, cls in classes.items():
        lines.append(f'  printf("{c} size %zu\\n", sizeof({c}));')
        for name, _ in cls._fields_:
            lines.append(f'  printf("{c} {name} %zu\\n", offsetof({c}, {name}));')
    lines += ["  return 0;", "}"]
    src = tmp_path / "layouts.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layouts"
    inc = Path(__file__).resolve().parent.parent / "include"
    r = subprocess.run(["gcc", "-std=c11", "-I", str(inc), str(src), "-o", str(exe)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    got = {tuple(l.split()[:2]): int(l.split()[2]) for l in out if l}
    for c, cls in classes.items():
        assert got[(c, "size")] == ctypes.sizeof(cls), c
        for name, _ in cls._fields_:
            assert got[(c, name)] == getattr(cls, name).offset, f"{c}.{name}"


def test_gemm_group_rejects_bad_groups():
    # argument errors come back before any device work (no GPU needed)
    from jitcast_b200 import ops

    L = _lib.lib()
    a = np.ones((64, 64), np.float32)
    c = np.zeros((64, 64), np.float32)
    good = ops.GemmProblem(a.ctypes.data, None, 64, a.ctypes.data, None, 64, None, c.ctypes.data, 64, 64, 64, 64, 0)
    arr = (ops.GemmProblem * 5)(*([good] * 5))
    assert L.jc_gemm_group_device(0, _lib.BF16, arr, 0, None) == _lib.ERR_INVALID_ARG
    assert L.jc_gemm_group_device(0, _lib.BF16, arr, 5, None) == _lib.ERR_INVALID_ARG
    assert L.jc_gemm_group_device(0, _lib.BF16, None, 1, None) == _lib.ERR_INVALID_ARG
    bad = (ops.GemmProblem * 2)(good, ops.GemmProblem(a.ctypes.data, None, 64, a.ctypes.data, None, 64, None,
                                                      c.ctypes.data, 64, 64, 64, 0, 0))
    assert L.jc_gemm_group_device(0, _lib.BF16, bad, 2, None) == _lib.ERR_INVALID_ARG
    assert "problem 1" in _lib.last_error()
    flagged = (ops.GemmProblem * 1)(ops.GemmProblem(a.ctypes.data, None, 64, a.ctypes.data, None, 64, None,
                                                    c.ctypes.data, 64, 64, 64, 64, _lib.BIAS))
    assert L.jc_gemm_group_device(0, _lib.BF16, flagged, 1, None) == _lib.ERR_INVALID_ARG


def test_wait_selftest_arguments():
    assert _lib.lib().jc_device_wait_selftest(0, 0) == _lib.ERR_INVALID_ARG
    assert _lib.lib().jc_device_wait_selftest(0, 2_000_000) == _lib.ERR_INVALID_ARG
    if _lib.lib().jc_device_count() == 0:
        assert _lib.lib().jc_device_wait_selftest(0, 1000) == _lib.ERR_NO_DEVICE
