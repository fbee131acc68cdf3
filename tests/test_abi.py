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


def test_gather_desc_layout_matches_header(tmp_path):
    """The ctypes mirror of apx_gather_desc has the C struct's size and field offsets (the
    descriptor crosses the ABI by pointer, field for field)."""
    import ctypes as C
    import shutil
    import subprocess

    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    fields = [f for f, _ in _abi.GatherDesc._fields_]
    src = tmp_path / "probe.c"
    src.write_text("#include <stddef.h>\n#include <stdio.h>\n#include \"apeiron_cuda.h\"\n"
                   "int main(void) {\n  printf(\"%zu\\n\", sizeof(apx_gather_desc));\n" +
                   "".join(f"  printf(\"%zu\\n\", offsetof(apx_gather_desc, {f}));\n"
                           for f in fields) + "  return 0;\n}\n")
    exe = tmp_path / "probe"
    inc = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include")
    subprocess.run([cc, "-I", inc, str(src), "-o", str(exe)], check=True)
    out = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    assert out[0] == C.sizeof(_abi.GatherDesc)
    assert out[1:] == [getattr(_abi.GatherDesc, f).offset for f in fields]


def test_ffn_status_decode_without_a_device(libpath):
    """apx_ffn_status_decode is host-only: all ones is OK; a SwiGLU refusal word carries the
    lane in the row field and the FfnError kind (3 = Overflow) in the low bits."""
    lib = _abi.load(libpath)
    err = _abi.ApxErr()
    ok = _abi.CallStatus((1 << 64) - 1, 0)
    assert lib.apx_ffn_status_decode(ctypes.byref(ok), ctypes.byref(err)) == _abi.APX_OK
    word = (1234 << 24) | (_abi.APX_ERR_SWIGLU_REFUSED << 16) | 3
    st = _abi.CallStatus(word, 0)
    assert lib.apx_ffn_status_decode(ctypes.byref(st), ctypes.byref(err)) == _abi.APX_ERR_SWIGLU_REFUSED
    assert (err.code, err.row, err.bits) == (_abi.APX_ERR_SWIGLU_REFUSED, 1234, 3)
    assert lib.apx_ffn_status_decode(None, ctypes.byref(err)) == _abi.APX_ERR_INVALID_ARGUMENT
