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


def test_serving_and_row_count_entry_points_check_arguments() -> None:
    """The device-turnover and device-row-count entry points reject bad
    arguments before anything is enqueued (no device needed)."""
    from bpdecode_b200 import _capi

    L = _capi.lib()
    fake = 256  # a non-null pointer value: never dereferenced on these paths
    args = [8, 1, fake, 0.1, 0.5, 0.3, 8, 8] + [fake] * 10 + [None]
    bad_prob = list(args)
    bad_prob[3] = 1.5
    assert L.bpd_serving_turnover(*bad_prob) == 1
    assert b"probabilities" in L.bpd_last_error()
    bad_mix = list(args)
    bad_mix[4], bad_mix[5] = 0.8, 0.4
    assert L.bpd_serving_turnover(*bad_mix) == 1
    no_regex = list(args)
    no_regex[6] = 0
    assert L.bpd_serving_turnover(*no_regex) == 1
    assert b"n_regex" in L.bpd_last_error()
    null_ptr = list(args)
    null_ptr[10] = None
    assert L.bpd_serving_turnover(*null_ptr) == 1
    assert b"null pointer" in L.bpd_last_error()
    assert L.bpd_serving_turnover(0, 1, None, 0.1, 0.5, 0.3, 8, 8, *([None] * 11)) == 0
    assert L.bpd_serving_gather_tokens(4, None, fake, fake, fake, fake, fake, None) == 1
    assert L.bpd_serving_gather_tokens(0, None, None, None, None, None, None, None) == 0
    # the *_from_n steps need their device row count
    assert L.bpd_soft_step_greedy_from_n(fake, 0, 16, None, None, 0, 4, None, 16, fake, None,
                                         fake, fake, 4, fake, 2, 1.0, fake, None, 0, fake,
                                         None) == 1
    assert b"row count" in L.bpd_last_error()
    g = _capi.PdaGrammar()
    assert L.bpd_pda_step_greedy_from_n(C.byref(g), fake, 0, 16, None, None, 0, fake, None,
                                        None, 4, None, None, 0, fake, 0.0, fake, None, 0,
                                        None) == 1
    assert b"row count" in L.bpd_last_error()
