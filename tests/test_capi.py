"""The C-ABI library loads and exports every function include/bpdecode_b200.h
declares (CPU only: no kernel is launched)."""

from __future__ import annotations

import ctypes as C
import os
import subprocess


from conftest import ROOT


def test_library_exports_every_header_symbol() -> None:
    from bpdecode_b200 import _capi

    declared = _capi.header_symbols()
    assert len(declared) >= 20
    dll = C.CDLL(_capi.LIB_PATH)
    missing = [s for s in declared if not hasattr(dll, s)]
    assert not missing, missing
    # the Python binding declares a signature for every exported entry point
    assert set(declared) == set(_capi._SIGNATURES)


def test_host_only_entry_points() -> None:
    from bpdecode_b200 import _capi

    L = _capi.lib()
    assert L.bpd_version().startswith(b"bpdecode_b200")
    assert L.bpd_pda_memo_bytes(4096, 128_256) > 4096 * (128_256 // 8)
    assert L.bpd_pda_workspace_bytes(256, 128_256) >= 256 * 4008 * 4
    assert L.bpd_soft_workspace_bytes(194) >= 2 * 194 * 4
    # argument checks fail before anything touches a device
    assert L.bpd_dense_apply_mask(None, 0, 10, 1, 10, None, None, None, 1, 1, 0.0, None) == 1
    assert b"null pointer" in L.bpd_last_error()
    assert L.bpd_dense_step_greedy(None, 0, 10, 1, 10, None, None, None, 1, None, 1, 0.0, None,
                                   None, 3, None, None) == 1
    assert L.bpd_step_scratch_bytes(1024) >= 12 * 1024
    assert L.bpd_step_scratch_bytes(1024) % 256 == 0


def test_header_compiles_as_c() -> None:
    src = os.path.join(ROOT, "include", "bpdecode_b200.h")
    r = subprocess.run(["gcc", "-std=c99", "-fsyntax-only", "-x", "c", src], capture_output=True,
                       text=True)
    assert r.returncode == 0, r.stderr
