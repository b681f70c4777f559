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


@pytest.mark.parametrize("heads", [4, 12])
def test_head_counts_other_than_multiples_of_8_are_unsupported(ptts, heads):
    """Heads come in groups of 8 (the cache's blocks): 4 or 12 heads of 64 are refused before any
    device work, for the cache and for the model, naming the rule."""
    lib = ptts.lib()
    out = ctypes.c_void_p()
    assert lib.ptts_b200_kv_create(0, 1, 1, 16, heads, 64, ptts.BF16, ctypes.byref(out)) == ptts.ERR_UNSUPPORTED
    assert "multiple of 8 heads" in lib.ptts_b200_last_error().decode()
    cfg = ptts.FlowLMConfig(d_model=64 * heads, num_heads=heads, num_kv_heads=heads).c_struct()
    assert lib.ptts_b200_model_create(0, ctypes.byref(cfg), ctypes.byref(out)) == ptts.ERR_UNSUPPORTED
    assert "multiple of 8 heads" in lib.ptts_b200_last_error().decode()


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


def test_header_is_plain_c_and_links(ptts, tmp_path):
    """The header compiles as C99 (no C++ in the boundary), every declared entry point links
    against the built library, and a C host gets the version and an error message without a
    GPU (a NULL handle is refused before any device work)."""
    import shutil
    import subprocess
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    names = _declared()
    src = tmp_path / "abi_check.c"
    src.write_text(
        "#include <stdio.h>\n#include <string.h>\n#include \"ptts_b200.h\"\n"
        "typedef void (*any_fn)(void);\n"
        "static any_fn table[] = {\n" + "".join(f"    (any_fn){n},\n" for n in names) + "};\n"
        "int main(void) {\n"
        "    size_t n = sizeof(table) / sizeof(table[0]);\n"
        "    for (size_t i = 0; i < n; ++i) if (!table[i]) return 2;\n"
        "    if (strncmp(ptts_b200_version(), \"ptts_b200\", 9) != 0) return 3;\n"
        "    if (ptts_b200_kv_create(0, 1, 1, 1, 8, 64, 1, NULL) == 0) return 4;\n"
        "    if (strlen(ptts_b200_last_error()) == 0) return 5;\n"
        "    printf(\"%zu entry points; last error: %s\\n\", n, ptts_b200_last_error());\n"
        "    return 0;\n}\n")
    lib = os.path.abspath(ptts.lib()._name)
    exe = tmp_path / "abi_check"
    r = subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"), str(src),
                        "-o", str(exe), lib, "-Wl,-rpath," + os.path.dirname(lib)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, (r.returncode, r.stdout, r.stderr)
    assert "entry points" in r.stdout
