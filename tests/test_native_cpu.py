"""CPU-side checks of the C ABI library: it loads, exports every function
include/exl3b200.h declares, its host-only code tables match the oracle, and
argument validation rejects bad requests before touching a device."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import REPO


def _declared_functions():
    names = []
    for h in sorted(os.listdir(os.path.join(REPO, "include"))):
        if not h.endswith(".h"):
            continue
        src = open(os.path.join(REPO, "include", h)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"^[A-Za-z_][\w\s\*]*?\b([a-z_][a-z0-9_]*)\s*\(", src, re.M):
            if not m.group(0).lstrip().startswith("#"):
                names.append(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    from exl3b import native
    L = native.lib()
    names = _declared_functions()
    assert len(names) >= 8
    for n in names:
        assert hasattr(L, n), f"missing export {n}"
        assert n in native.SIGNATURES, f"no ctypes signature for {n}"
    assert L.exl3b_abi_version() == 1


@pytest.mark.parametrize("code,cid", [("exl3_mul1", 0), ("exl3_3inst", 1), ("exl3_mcg", 2)])
def test_code_tables_match_oracle(oracle, code, cid):
    from exl3b import native
    out = np.empty(65536, dtype=np.float32)
    native.call("exl3b_code_lut", cid, out.ctypes.data_as(ctypes.c_void_p))
    assert np.array_equal(out, oracle.code_lut(code))
    # every decode value is exact in fp16 (the encoder holds them packed)
    assert np.array_equal(out.astype(np.float16).astype(np.float32), out)


def test_argument_validation_without_device():
    from exl3b import native
    L = native.lib()
    assert L.exl3b_code_lut(7, None) == 7
    rc = L.exl3b_tailbite(None, 4, 9, 0, 0, 0, None, None, 0, None)
    assert rc == 8 and "K=9" in native.last_error()
    rc = L.exl3b_tailbite(None, 0, 4, 0, 0, 0, None, None, 0, None)
    assert rc == 6
    rc = L.exl3b_tailbite(None, 4, 4, 5, 0, 0, None, None, 0, None)
    assert rc == 7
    rc = L.exl3b_tailbite(None, 4, 4, 0, 256, 0, None, None, 0, None)
    assert rc == 7
    assert L.exl3b_tailbite_workspace_bytes(10, 1) == 0
