"""The C-ABI library loads and exports every entry point include/apeiron_cuda.h declares
(CPU only: no compute call, no device needed)."""
import ctypes
import os
import re
import subprocess

import pytest

from apeiron_b200 import _abi, build

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_symbols():
    text = open(os.path.join(ROOT, "include", "apeiron_cuda.h")).read()
    return sorted(set(re.findall(r"^APX_API [^(]*?\b(apx_\w+)\(", text, flags=re.M)))


@pytest.fixture(scope="module")
def libpath():
    return build.build()


def test_header_and_binding_agree():
    assert header_symbols() == sorted(_abi.EXPORTS)


def test_library_exports_every_declared_symbol(libpath):
    out = subprocess.run(["nm", "-D", "--defined-only", libpath], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r"\b(apx_\w+)\b", out))
    missing = [s for s in header_symbols() if s not in exported]
    assert not missing, missing
    # nothing but the declared C ABI leaks out under the apx_ prefix
    assert exported == set(header_symbols())


def test_library_loads_without_a_device(libpath):
    lib = _abi.load(libpath)
    assert lib.apx_version().startswith(b"apeiron_b200")
    assert lib.apx_act_padded_len(896) == 1024
    assert lib.apx_act_padded_len(0) == 0
