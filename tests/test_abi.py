"""The C-ABI library on a machine without a GPU (CPU): it loads, exports exactly what include/*.h declares, its
struct layouts match the ctypes mirror, and every call fails with a status code instead of crashing."""
import ctypes
import re
import subprocess
import tempfile
from pathlib import Path

import numpy as np
import pytest

from anvil.runtime import cuda as C

ROOT = Path(__file__).resolve().parents[1]


def _declared():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        names |= set(re.findall(r"ANVIL_API\s+[\w\s\*]*?\b(anvil_\w+)\s*\(", h.read_text()))
    return names


def test_library_exports_every_declared_symbol():
    lib = C.load_library()
    declared = _declared()
    assert declared >= set(C.EXPORTS)
    for name in declared:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", str(C.LIB_PATH)], capture_output=True, text=True).stdout
    exported = set(re.findall(r" T (anvil_\w+)", out))
    assert exported == declared


def test_struct_layout_matches_header(tmp_path):
    src = tmp_path / "sz.c"
    src.write_text('#include <stdio.h>\n#include <stddef.h>\n#include "anvil_cuda.h"\n'
                   'int main(void){printf("%zu %zu %zu %zu %zu %zu\\n", sizeof(anvil_op), offsetof(anvil_op, dims),'
                   ' offsetof(anvil_op, off), offsetof(anvil_op, mult), offsetof(anvil_op, shift2),'
                   ' sizeof(anvil_io));return 0;}\n')
    exe = tmp_path / "sz"
    subprocess.run(["gcc", "-I", str(ROOT / "include"), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True).stdout.split()]
    want = [ctypes.sizeof(C.AnvilOp), C.AnvilOp.dims.offset, C.AnvilOp.off.offset, C.AnvilOp.mult.offset,
            C.AnvilOp.shift2.offset, ctypes.sizeof(C.AnvilIO)]
    assert got == want


def test_calls_fail_cleanly_without_a_device():
    lib = C.load_library()
    assert lib.anvil_abi_version() == C.ABI_VERSION
    if C.device_count() > 0:
        pytest.skip("a GPU is visible")
    h = ctypes.c_void_p()
    rc = lib.anvil_model_create(0, None, 0, ctypes.byref(h))
    assert rc == -7 and not h.value
    assert b"not available" in lib.anvil_last_error()
    with pytest.raises(NotImplementedError):
        C.DeviceModel(0, np.zeros(0, dtype=np.uint8))
    assert lib.anvil_model_prepare(None, None, 0, 0) == -1
