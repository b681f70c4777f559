"""CPU tests of the C ABI: the library loads, exports every declared symbol, and refuses bad
arguments with the documented codes and messages before touching a device."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT


def _declared():
    text = open(os.path.join(ROOT, "include", "ptts_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(ptts_b200_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol(ptts):
    lib = ptts.lib()
    names = _declared()
    assert len(names) >= 15
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    assert set(names) == set(ptts.EXPORTS)


def test_version_and_empty_last_error(ptts):
    assert ptts.version().startswith("ptts_b200")
    assert ptts.lib().ptts_b200_last_error() is not None


def test_bad_shapes_are_refused_before_any_device_work(ptts):
    lib = ptts.lib()
    out = ctypes.c_void_p()
    rc = lib.ptts_b200_kv_create(0, 1, 1, 16, 4, 32, ptts.BF16, ctypes.byref(out))
    assert rc == ptts.ERR_UNSUPPORTED
    assert "head_dim 64" in lib.ptts_b200_last_error().decode()
    rc = lib.ptts_b200_kv_create(0, 1, 0, 16, 8, 64, ptts.BF16, ctypes.byref(out))
    assert rc == ptts.ERR_ARG
    assert lib.ptts_b200_kv_create(0, 1, 1, 16, 8, 64, 7, ctypes.byref(out)) == ptts.ERR_ARG
    assert lib.ptts_b200_kv_create(0, 1, 1, 16, 8, 64, ptts.BF16, None) == ptts.ERR_ARG


@pytest.mark.parametrize("kv_heads", [0, 3])
def test_kv_heads_that_do_not_divide_the_heads_are_an_error(ptts, kv_heads):
    """bad_config_tests (transformer.rs:1258-1266): the message names key/value heads."""
    cfg = ptts.FlowLMConfig(num_kv_heads=kv_heads).c_struct()
    out = ctypes.c_void_p()
    rc = ptts.lib().ptts_b200_model_create(0, ctypes.byref(cfg), ctypes.byref(out))
    assert rc == ptts.ERR_ARG
    assert "key/value heads" in ptts.lib().ptts_b200_last_error().decode()


@pytest.mark.parametrize("heads", [0, 3])
def test_heads_that_do_not_divide_the_width_are_an_error(ptts, heads):
    """bad_config_tests (transformer.rs:1250-1256): the message names the heads."""
    cfg = ptts.FlowLMConfig(num_heads=heads, num_kv_heads=1).c_struct()
    out = ctypes.c_void_p()
    rc = ptts.lib().ptts_b200_model_create(0, ctypes.byref(cfg), ctypes.byref(out))
    assert rc in (ptts.ERR_ARG, ptts.ERR_UNSUPPORTED)
    assert "heads" in ptts.lib().ptts_b200_last_error().decode()


def test_null_handles_are_refused(ptts):
    lib = ptts.lib()
    n = (ctypes.c_int32 * 4)()
    assert lib.ptts_b200_kv_lengths(None, n) == ptts.ERR_ARG
    assert "kv is NULL" in lib.ptts_b200_last_error().decode()
    assert lib.ptts_b200_forward(None, None, None, n, n, 1, None, None) == ptts.ERR_ARG
    lib.ptts_b200_kv_destroy(None)
    lib.ptts_b200_model_destroy(None)


def test_no_cpu_fallback_without_the_library(ptts, monkeypatch, tmp_path):
    """The product path fails loudly when the CUDA library is missing."""
    monkeypatch.setattr(ptts, "LIB_PATH", str(tmp_path / "missing.so"))
    monkeypatch.setattr(ptts, "_lib", None)
    with pytest.raises(ptts.PttsError):
        ptts.lib()
