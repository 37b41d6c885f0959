"""The C-ABI library loads and exports every symbol include/spk.h declares.
No compute call is made, so this runs without a GPU."""
import os
import re
import subprocess

import pytest

import spk

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "spk.h")


def declared_symbols():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b((?:vqg|spk)_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert set(declared_symbols()) == set(spk.exported_symbols())


def test_library_exports_every_declared_symbol():
    if not os.path.exists(spk.LIB_PATH):
        pytest.skip("libspk.so not built")
    out = subprocess.run(["nm", "-D", "--defined-only", spk.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\s[TW]\s+(\S+)", out))
    missing = [s for s in declared_symbols() if s not in exported]
    assert not missing, missing


def test_library_loads_and_binds():
    if not os.path.exists(spk.LIB_PATH):
        pytest.skip("libspk.so not built")
    L = spk.lib()
    for s in declared_symbols():
        assert getattr(L, s) is not None


def test_no_cpu_fallback_symbols():
    """The product exports only the ABI: no internal kernel or oracle name leaks out."""
    if not os.path.exists(spk.LIB_PATH):
        pytest.skip("libspk.so not built")
    out = subprocess.run(["nm", "-D", "--defined-only", spk.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\s[TW]\s+(\S+)", out))
    ours = {s for s in exported if s.startswith(("vqg_", "spk_", "orc_"))}
    assert not any(s.startswith("orc_") for s in ours)
    assert ours == set(declared_symbols())


def test_header_compiles_clean_as_c_and_cpp(tmp_path):
    """include/spk.h is the drop-in boundary for C and C++ callers: it compiles on its own
    with warnings as errors in both languages, and a caller's pointers match its prototypes."""
    import shutil
    import subprocess

    inc = os.path.join(ROOT, "include")
    src = tmp_path / "use.c"
    src.write_text('#include "spk.h"\n'
                   "int use(spk_model *m, spk_vqprof *p) { return spk_model_use_profile(m, p); }\n"
                   "int find(const spk_vqprof *p) { return spk_vqprof_find(p, 0, 4, 4096, 10240, 2560, 1); }\n")
    for cc, lang in (("gcc", "c"), ("g++", "c++")):
        if shutil.which(cc) is None:
            pytest.skip(f"{cc} is not installed")
        subprocess.run([cc, "-x", lang, "-std=" + ("c99" if lang == "c" else "c++17"), "-Wall", "-Wextra", "-Werror",
                        "-c", "-I", inc, str(src), "-o", str(tmp_path / f"use_{lang}.o")], check=True)
