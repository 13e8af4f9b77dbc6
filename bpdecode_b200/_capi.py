"""ctypes binding of ``libbpdecode_b200.so`` (the C ABI of
``include/bpdecode_b200.h``).

This is the only place Python touches the native library. It fails loudly:
importing the package on a machine where the library is missing raises
``ImportError`` -- there is no CPU or pure-torch fallback for the device path.
A non-zero ``bpd_status`` becomes ``RuntimeError`` carrying
``bpd_last_error()``, mirroring the reference's ``TORCH_CHECK`` errors.
"""

from __future__ import annotations

import ctypes as C
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libbpdecode_b200.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "bpdecode_b200.h")

_P = C.c_void_p
_I32 = C.c_int32
_I64 = C.c_int64
_F = C.c_float
_S = C.c_size_t

F32, BF16, F16 = 0, 1, 2
PDA_CONFIG_INTS = 266


class PdaGrammar(C.Structure):
    """``bpd_pda_grammar``: device pointers of a flattened PDA grammar."""

    _fields_ = [
        ("num_states", _I32), ("num_edges", _I32), ("root_start", _I32), ("root_accept", _I32),
        ("accept", _P), ("live", _P), ("edge_offsets", _P), ("edge_kind", _P),
        ("edge_lo", _P), ("edge_hi", _P), ("edge_dst", _P), ("edge_callee", _P),
        ("vocab_size", _I32), ("eos_id", _I32), ("tok_offsets", _P), ("tok_bytes", _P),
    ]


_SIGNATURES: dict[str, tuple[object, list]] = {
    "bpd_version": (C.c_char_p, []),
    "bpd_last_error": (C.c_char_p, []),
    "bpd_dense_build_tok_next": (_I32, [_P, _I32, _I32, _P, _P, _I32, _P, _P, _I32, _I32, _P,
                                        _I32, _P, _P]),
    "bpd_dense_build_allow_bits": (_I32, [_P, _I32, _I32, _P, _I32, _P]),
    "bpd_dense_apply_mask": (_I32, [_P, _I32, _I64, _I32, _I32, _P, _P, _P, _I32, _I32, _F, _P]),
    "bpd_dense_advance": (_I32, [_P, _P, _I32, _P, _I32, _P, _I32, _I32, _P, _I32, _P]),
    "bpd_dense_mask_bits": (_I32, [_P, _P, _I32, _P, _I32, _I32, _I32, _P, _P]),
    "bpd_step_scratch_bytes": (C.c_size_t, [_I32]),
    "bpd_dense_step_greedy": (_I32, [_P, _I32, _I64, _I32, _I32, _P, _P, _P, _I32, _P, _I32, _F,
                                     _P, _P, _I32, _P, _P]),
    "bpd_walk_apply_mask": (_I32, [_P, _I32, _I64, _I32, _P, _I32, _I32, _P, _P, _I32, _P, _P,
                                   _I32, _I32, _P, _F, _P]),
    "bpd_walk_mask_bits": (_I32, [_P, _I32, _I32, _P, _P, _I32, _P, _P, _I32, _I32, _P, _I32, _P,
                                  _P]),
    "bpd_walk_advance": (_I32, [_P, _I32, _I32, _P, _P, _I32, _P, _P, _I32, _I32, _P, _P, _I32,
                                _I32, _P, _P]),
    "bpd_soft_workspace_bytes": (_S, [_I32]),
    "bpd_soft_build_lookahead": (_I32, [_P, _I32, _I32, _P, _P, _I32, _I32, _P, _P, _P]),
    "bpd_soft_apply": (_I32, [_P, _I32, _I64, _I32, _I32, _P, _P, _P, _P, _I32, _I32, _F, _P]),
    "bpd_soft_step_greedy": (_I32, [_P, _I32, _I64, _I32, _I32, _P, _P, _P, _P, _I32, _P, _I32,
                                    _F, _P, _P, _I32, _P, _P]),
    "bpd_dense_step_greedy_from": (_I32, [_P, _I32, _I64, _P, _P, _I64, _I32, _I32, _P, _P, _P,
                                          _I32, _P, _I32, _F, _P, _P, _I32, _P, _P]),
    "bpd_soft_step_greedy_from": (_I32, [_P, _I32, _I64, _P, _P, _I64, _I32, _I32, _P, _P, _P,
                                         _P, _I32, _P, _I32, _F, _P, _P, _I32, _P, _P]),
    "bpd_pda_step_greedy_from": (_I32, [C.POINTER(PdaGrammar), _P, _I32, _I64, _P, _P, _I64, _P,
                                        _P, _P, _I32, _P, _I32, _P, _F, _P, _P, _I32, _P]),
    "bpd_soft_step_greedy_from_n": (_I32, [_P, _I32, _I64, _P, _P, _I64, _I32, _P, _I32, _P, _P,
                                           _P, _P, _I32, _P, _I32, _F, _P, _P, _I32, _P, _P]),
    "bpd_pda_step_greedy_from_n": (_I32, [C.POINTER(PdaGrammar), _P, _I32, _I64, _P, _P, _I64,
                                          _P, _P, _P, _I32, _P, _P, _I32, _P, _F, _P, _P, _I32,
                                          _P]),
    "bpd_serving_turnover": (_I32, [_I32, C.c_uint64, _P, _F, _F, _F, _I32, _I32, _P, _P, _P, _P,
                                    _P, _P, _P, _P, _P, _P, _P]),
    "bpd_serving_gather_tokens": (_I32, [_I32, _P, _P, _P, _P, _P, _P, _P]),
    "bpd_pda_init": (_I32, [C.POINTER(PdaGrammar), _P, _P]),
    "bpd_pda_memo_bytes": (_S, [_I32, _I32]),
    "bpd_pda_memo_reset": (_I32, [_P, _I32, _I32, _P]),
    "bpd_pda_workspace_bytes": (_S, [_I32, _I32]),
    "bpd_pda_mask_bits": (_I32, [C.POINTER(PdaGrammar), _P, _P, _P, _I32, _P, _I32, _P, _P, _P]),
    "bpd_pda_apply_mask": (_I32, [C.POINTER(PdaGrammar), _P, _I32, _I64, _P, _P, _P, _I32, _P,
                                  _I32, _P, _F, _P]),
    "bpd_pda_apply_mask_noalloc": (_I32, [C.POINTER(PdaGrammar), _P, _I32, _I64, _P, _P, _P,
                                          _I32, _P, _I32, _F, _P]),
    "bpd_pda_step_greedy": (_I32, [C.POINTER(PdaGrammar), _P, _I32, _I64, _P, _P, _P, _I32, _P,
                                   _I32, _P, _F, _P, _P, _I32, _P]),
    "bpd_pda_advance": (_I32, [C.POINTER(PdaGrammar), _P, _P, _I32, _P, _I32, _P, _P, _P, _P]),
    "bpd_pda_is_complete": (_I32, [C.POINTER(PdaGrammar), _P, _P, _P, _I32, _P, _P]),
}


def header_symbols() -> list[str]:
    """Every function the C header declares."""
    with open(HEADER) as f:
        text = f.read()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(bpd_\w+)\s*\(", text, re.M)))


class _Lib:
    def __init__(self) -> None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"bpdecode_b200: native library {LIB_PATH} is not built; run "
                "`python -m bpdecode_b200.build` (needs nvcc). There is no CPU fallback.")
        self.dll = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGNATURES.items():
            fn = getattr(self.dll, name)
            fn.restype = res
            fn.argtypes = args
            setattr(self, name, fn)

    def check(self, status: int) -> None:
        if status != 0:
            msg = self.bpd_last_error().decode(errors="replace")
            raise RuntimeError(f"bpdecode_b200: {msg}")


_LIB: _Lib | None = None


def lib() -> _Lib:
    global _LIB
    if _LIB is None:
        _LIB = _Lib()
    return _LIB
