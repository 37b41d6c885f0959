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
