"""TEST INFRASTRUCTURE ONLY -- ctypes access to the CPU checkers.

* :class:`Oracle` wraps ``_build/libbpd_oracle.so``, the plain-C restatement of
  bpdecode's step (``bpd_oracle.c``).
* :class:`RefLib` wraps ``_ref/libbpdref.so``, the reference's own CPU sources
  (``csrc/src/mask_cpu.cpp``, ``csrc/src/pda_cpu.cpp``) compiled unchanged.

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of
``bench.py`` import this module; the product never does. Arrays are numpy.
"""

from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libbpd_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libbpdref.so")
REF_CUDA_SO = os.path.join(HERE, "_ref", "libbpdref_cuda.so")

NCFG = 266

_P = C.c_void_p
_I = C.c_int32
_L = C.c_int64
_F = C.c_float


def _ptr(a: np.ndarray | None) -> C.c_void_p | None:
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "oracle arrays must be contiguous"
    return C.c_void_p(a.ctypes.data)


class PdaGrammarStruct(C.Structure):
    """Field layout shared by orc_pda_grammar, the shim's PdaArgs and
    bpd_pda_grammar."""

    _fields_ = [
        ("num_states", _I), ("num_edges", _I), ("root_start", _I), ("root_accept", _I),
        ("accept", _P), ("live", _P), ("edge_offsets", _P), ("edge_kind", _P),
        ("edge_lo", _P), ("edge_hi", _P), ("edge_dst", _P), ("edge_callee", _P),
        ("vocab_size", _I), ("eos_id", _I), ("tok_offsets", _P), ("tok_bytes", _P),
    ]


class HostPda:
    """Host (numpy) copy of a flattened PDA grammar + vocabulary bytes."""

    def __init__(self, arrays: dict, tok_offsets: np.ndarray, tok_bytes: np.ndarray,
                 eos_id: int) -> None:
        self.a = {k: (v if np.isscalar(v) else np.ascontiguousarray(v))
                  for k, v in arrays.items()}
        self.tok_offsets = np.ascontiguousarray(tok_offsets, dtype=np.int32)
        self.tok_bytes = np.ascontiguousarray(tok_bytes, dtype=np.uint8)
        if self.tok_bytes.size == 0:
            self.tok_bytes = np.zeros(1, np.uint8)
        self.vocab_size = int(self.tok_offsets.size - 1)
        self.eos_id = int(eos_id)
        a = self.a
        self.struct = PdaGrammarStruct(
            int(a["accept"].size), int(a["edge_kind"].size), int(a["root_start"]),
            int(a["root_accept"]), _ptr(a["accept"]), _ptr(a["live"]),
            _ptr(a["edge_offsets"]), _ptr(a["edge_kind"]), _ptr(a["edge_lo"]),
            _ptr(a["edge_hi"]), _ptr(a["edge_dst"]), _ptr(a["edge_callee"]),
            self.vocab_size, self.eos_id, _ptr(self.tok_offsets), _ptr(self.tok_bytes),
        )


def _load(path: str) -> C.CDLL:
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} is not built (run `make -C oracle`)")
    return C.CDLL(path)


class Oracle:
    """The plain-C restatement."""

    def __init__(self) -> None:
        lib = self.lib = _load(ORACLE_SO)
        lib.orc_step.restype = _I
        lib.orc_step.argtypes = [_P, _I, _P, _P, _I, _P, _P, _I, _I, _I]
        lib.orc_pda_is_complete.restype = C.c_int
        lib.orc_pda_try_token.restype = C.c_int
        lib.orc_pda_advance_byte.restype = C.c_int

    # --- dense ---------------------------------------------------------
    def build_tok_next(self, f: dict, offsets: np.ndarray, symbols: np.ndarray, eos_id: int,
                       ) -> np.ndarray:
        S = int(f["accept"].size)
        V = int(offsets.size - 1)
        out = np.empty((S, V), np.int32)
        sym = symbols if symbols.size else np.zeros(1, np.int32)
        self.lib.orc_build_tok_next(
            _ptr(f["trans"]), _I(S), _I(f["num_symbols"]), _ptr(f["accept"]), _ptr(f["live"]),
            _I(f["dead"]), _ptr(offsets), _ptr(sym), _I(V), _I(eos_id), _ptr(out))
        return out

    def allow_bits(self, tok_next: np.ndarray, words_stride: int | None = None) -> np.ndarray:
        S, V = tok_next.shape
        W = words_stride or (V + 31) // 32
        out = np.empty((S, W), np.uint32)
        self.lib.orc_allow_bits(_ptr(tok_next), _I(S), _I(V), _I(W), _ptr(out))
        return out

    def dense_apply_mask(self, logits: np.ndarray, tok_next: np.ndarray, states: np.ndarray,
                         neg_inf_bits: int | float) -> None:
        """In place on a [B, V] float32 array, or a uint16 array holding bf16 /
        fp16 bit patterns (then ``neg_inf_bits`` is the 16-bit fill pattern)."""
        S, V = tok_next.shape
        B = logits.shape[0]
        st = np.ascontiguousarray(states, np.int32)
        if logits.dtype == np.float32:
            self.lib.orc_dense_apply_mask_f32(_ptr(logits), _L(logits.shape[1]), _I(B), _I(V),
                                              _ptr(tok_next), _I(S), _ptr(st), _F(neg_inf_bits))
        else:
            assert logits.dtype == np.uint16
            self.lib.orc_dense_apply_mask_u16(_ptr(logits), _L(logits.shape[1]), _I(B), _I(V),
                                              _ptr(tok_next), _I(S), _ptr(st),
                                              C.c_uint16(int(neg_inf_bits)))

    def dense_advance(self, tok_next: np.ndarray, states: np.ndarray, tokens: np.ndarray,
                      ) -> np.ndarray:
        S, V = tok_next.shape
        st = np.ascontiguousarray(states, np.int32)
        tk = np.ascontiguousarray(tokens, np.int64)
        out = np.empty(st.size, np.int32)
        self.lib.orc_dense_advance(_ptr(tok_next), _I(S), _I(V), _ptr(st), _ptr(tk),
                                   _I(st.size), _ptr(out))
        return out

    def dense_mask_bits(self, tok_next: np.ndarray, states: np.ndarray) -> np.ndarray:
        S, V = tok_next.shape
        st = np.ascontiguousarray(states, np.int32)
        out = np.empty((st.size, (V + 31) // 32), np.uint32)
        self.lib.orc_dense_mask_bits(_ptr(tok_next), _I(S), _I(V), _ptr(st), _I(st.size),
                                     _ptr(out))
        return out

    # --- soft ----------------------------------------------------------
    def build_lookahead(self, tok_next: np.ndarray, accept: np.ndarray, live: np.ndarray,
                        eos_id: int, k: int) -> np.ndarray:
        S, V = tok_next.shape
        out = np.empty((S, V), np.float64)
        w1 = np.empty(S, np.float64)
        w2 = np.empty(S, np.float64)
        self.lib.orc_build_lookahead(_ptr(tok_next), _I(S), _I(V), _ptr(accept), _ptr(live),
                                     _I(eos_id), _I(k), _ptr(w1), _ptr(w2), _ptr(out))
        return out

    def apply_soft(self, logits: np.ndarray, lookahead: np.ndarray, states: np.ndarray,
                   alpha: float) -> None:
        S, V = lookahead.shape
        st = np.ascontiguousarray(states, np.int32)
        self.lib.orc_apply_soft_f32(_ptr(logits), _L(logits.shape[1]), _I(logits.shape[0]),
                                    _I(V), _ptr(lookahead), _I(S), _ptr(st), _F(alpha))

    # --- pda -----------------------------------------------------------
    def pda_init(self, g: HostPda) -> np.ndarray:
        out = np.empty(NCFG, np.int32)
        self.lib.orc_pda_init(C.byref(g.struct), _ptr(out))
        return out

    def pda_is_complete(self, g: HostPda, cfg: np.ndarray) -> bool:
        return bool(self.lib.orc_pda_is_complete(C.byref(g.struct), _ptr(cfg)))

    def pda_try_token(self, g: HostPda, cfg: np.ndarray, tok: int) -> bool:
        return bool(self.lib.orc_pda_try_token(C.byref(g.struct), _ptr(cfg), _I(tok)))

    def pda_advance_byte(self, g: HostPda, cfg: np.ndarray, byte: int) -> bool:
        return bool(self.lib.orc_pda_advance_byte(C.byref(g.struct), _ptr(cfg), _I(byte)))

    def pda_mask_bits(self, g: HostPda, cfgs: np.ndarray) -> np.ndarray:
        cfgs = np.ascontiguousarray(cfgs, np.int32).reshape(-1, NCFG)
        out = np.empty((cfgs.shape[0], (g.vocab_size + 31) // 32), np.uint32)
        self.lib.orc_pda_mask_bits(C.byref(g.struct), _ptr(cfgs), _I(cfgs.shape[0]), _ptr(out))
        return out

    def pda_apply_mask(self, g: HostPda, cfgs: np.ndarray, logits: np.ndarray,
                       neg_inf: float) -> None:
        cfgs = np.ascontiguousarray(cfgs, np.int32).reshape(-1, NCFG)
        self.lib.orc_pda_apply_mask_f32(C.byref(g.struct), _ptr(cfgs), _I(cfgs.shape[0]),
                                        _ptr(logits), _L(logits.shape[1]), _F(neg_inf))

    def pda_advance(self, g: HostPda, cfgs: np.ndarray, tokens: np.ndarray) -> np.ndarray:
        """In place on cfgs [B, 266]; returns ok uint8 [B]."""
        assert cfgs.flags["C_CONTIGUOUS"] and cfgs.dtype == np.int32
        tk = np.ascontiguousarray(tokens, np.int64)
        ok = np.empty(tk.size, np.uint8)
        self.lib.orc_pda_advance(C.byref(g.struct), _ptr(cfgs), _ptr(tk), _I(tk.size), _ptr(ok))
        return ok


class RefLib:
    """The reference's own CPU implementation, compiled from its sources."""

    def __init__(self) -> None:
        lib = self.lib = _load(REF_SO)
        lib.ref_pda_is_complete.restype = _I
        lib.ref_pda_advance_byte.restype = _I

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_SO)

    def build_reachability(self, trans: np.ndarray, num_symbols: int, accept: np.ndarray,
                           ) -> np.ndarray:
        S = int(accept.size)
        out = np.empty(S, np.uint8)
        self.lib.ref_build_reachability(_ptr(trans), _I(S), _I(num_symbols), _ptr(accept),
                                        _ptr(out))
        return out

    def _fsa_args(self, f: dict, offsets: np.ndarray, symbols: np.ndarray, eos_id: int):
        V = int(offsets.size - 1)
        sym = symbols if symbols.size else np.zeros(1, np.int32)
        return (_ptr(f["trans"]), _I(int(f["accept"].size)), _I(f["num_symbols"]),
                _ptr(f["accept"]), _ptr(f["live"]), _I(f["dead"]), _ptr(offsets), _ptr(sym),
                _I(V), _I(eos_id)), V

    def compute_mask_batch(self, f, offsets, symbols, eos_id, states) -> np.ndarray:
        args, V = self._fsa_args(f, offsets, symbols, eos_id)
        st = np.ascontiguousarray(states, np.int32)
        out = np.empty((st.size, (V + 31) // 32), np.uint32)
        self.lib.ref_compute_mask_batch(*args, _ptr(st), _I(st.size), _ptr(out))
        return out

    def advance_state_batch(self, f, offsets, symbols, eos_id, states, tokens) -> np.ndarray:
        args, V = self._fsa_args(f, offsets, symbols, eos_id)
        st = np.ascontiguousarray(states, np.int32)
        tk = np.ascontiguousarray(tokens, np.int32)
        out = np.empty(st.size, np.int32)
        self.lib.ref_advance_state_batch(*args, _ptr(st), _ptr(tk), _I(st.size), _ptr(out))
        return out

    def apply_mask_batch(self, f, offsets, symbols, eos_id, states, logits, neg_inf) -> None:
        args, V = self._fsa_args(f, offsets, symbols, eos_id)
        st = np.ascontiguousarray(states, np.int32)
        assert logits.dtype == np.float32 and logits.flags["C_CONTIGUOUS"]
        self.lib.ref_apply_mask_batch(*args, _ptr(st), _I(st.size), _ptr(logits), _F(neg_inf))

    def pda_init(self, g: HostPda) -> np.ndarray:
        out = np.empty(NCFG, np.int32)
        self.lib.ref_pda_init(C.byref(g.struct), _ptr(out))
        return out

    def pda_is_complete(self, g: HostPda, cfg: np.ndarray) -> bool:
        return bool(self.lib.ref_pda_is_complete(C.byref(g.struct), _ptr(cfg)))

    def pda_advance_byte(self, g: HostPda, cfg: np.ndarray, byte: int) -> bool:
        return bool(self.lib.ref_pda_advance_byte(C.byref(g.struct), _ptr(cfg), _I(byte)))

    def pda_mask_bits(self, g: HostPda, cfgs: np.ndarray) -> np.ndarray:
        cfgs = np.ascontiguousarray(cfgs, np.int32).reshape(-1, NCFG)
        out = np.empty((cfgs.shape[0], (g.vocab_size + 31) // 32), np.uint32)
        self.lib.ref_pda_mask_bits(C.byref(g.struct), _ptr(cfgs), _I(cfgs.shape[0]), _ptr(out))
        return out

    def pda_apply_mask(self, g: HostPda, cfgs: np.ndarray, logits: np.ndarray,
                       neg_inf: float) -> None:
        cfgs = np.ascontiguousarray(cfgs, np.int32).reshape(-1, NCFG)
        assert logits.flags["C_CONTIGUOUS"]
        self.lib.ref_pda_apply_mask(C.byref(g.struct), _ptr(cfgs), _I(cfgs.shape[0]),
                                    _ptr(logits), _F(neg_inf))

    def pda_advance(self, g: HostPda, cfgs: np.ndarray, tokens: np.ndarray) -> np.ndarray:
        assert cfgs.flags["C_CONTIGUOUS"] and cfgs.dtype == np.int32
        tk = np.ascontiguousarray(tokens, np.int32)
        ok = np.empty(tk.size, np.uint8)
        self.lib.ref_pda_advance(C.byref(g.struct), _ptr(cfgs), _ptr(tk), _I(tk.size), _ptr(ok))
        return ok


# --- helpers shared by tests and the CPU baseline ---------------------------

def dfa_with_vocab(dfa: dict, token_bytes: tuple[bytes, ...]) -> tuple[np.ndarray, np.ndarray]:
    """Token symbol sequences of a vocabulary through a DFA's byte -> class
    table (fsa.py:133-152, token_symbols)."""
    lut = np.asarray(dfa["lut"], np.int32)
    offsets = np.zeros(len(token_bytes) + 1, np.int32)
    np.cumsum([len(t) for t in token_bytes], out=offsets[1:])
    flat = np.frombuffer(b"".join(token_bytes), np.uint8)
    return offsets, lut[flat].astype(np.int32)


class _RefPdaStruct(C.Structure):
    """ref_cuda_shim.cu's RefPda."""

    _fields_ = [
        ("num_states", _I), ("root_start", _I), ("root_accept", _I),
        ("accept", _P), ("live", _P), ("edge_offsets", _P), ("edge_kind", _P),
        ("edge_lo", _P), ("edge_hi", _P), ("edge_dst", _P), ("edge_callee", _P),
        ("vocab_size", _I), ("eos_id", _I), ("tok_offsets", _P), ("tok_bytes", _P),
    ]


class RefCudaLib:
    """The reference's own CUDA implementation (mask_cuda.cu, pda_cuda.cu),
    compiled from its sources for sm_100a. Takes and returns torch CUDA
    tensors; launches on the current stream without synchronising."""

    def __init__(self) -> None:
        lib = self.lib = _load(REF_CUDA_SO)
        lib.bpdref_cuda_config_bytes.restype = _I
        assert lib.bpdref_cuda_config_bytes() == NCFG * 4

    @staticmethod
    def available() -> bool:
        return os.path.exists(REF_CUDA_SO)

    @staticmethod
    def _stream():
        import torch

        return C.c_void_p(torch.cuda.current_stream().cuda_stream)

    @staticmethod
    def _pda(g) -> _RefPdaStruct:
        nedges = int(g.edge_kind.numel())
        p = lambda t, n: C.c_void_p(t.data_ptr() if n else 0)  # noqa: E731
        return _RefPdaStruct(
            g.num_states, g.root_start, g.root_accept, p(g.accept, 1), p(g.live, 1),
            p(g.edge_offsets, 1), p(g.edge_kind, nedges), p(g.edge_lo, nedges),
            p(g.edge_hi, nedges), p(g.edge_dst, nedges), p(g.edge_callee, nedges),
            g.vocab_size, g.eos_id, p(g.tok_offsets, 1), p(g.tok_bytes, 1))

    def pda_mask(self, g, configs):
        """Packed allow bits int32 [B, ceil(V/32)] (compute_mask_pda_batch_cuda)."""
        import torch

        B = int(configs.shape[0])
        out = torch.empty((B, (g.vocab_size + 31) // 32), dtype=torch.int32,
                          device=configs.device)
        gs = self._pda(g)
        self.lib.bpdref_cuda_pda_mask(C.byref(gs), C.c_void_p(configs.data_ptr()), _I(B),
                                      C.c_void_p(out.data_ptr()), self._stream())
        return out

    def pda_apply_mask(self, g, configs, logits, neg_inf: float = float("-inf")) -> None:
        """In place on fp32 logits [B, V] (apply_mask_pda_batch_cuda)."""
        gs = self._pda(g)
        self.lib.bpdref_cuda_pda_apply_mask(C.byref(gs), C.c_void_p(configs.data_ptr()),
                                            _I(int(configs.shape[0])),
                                            C.c_void_p(logits.data_ptr()), _F(neg_inf),
                                            self._stream())

    def pda_advance(self, g, configs, tokens):
        """Advance configs [B, 266] in place by int32 tokens; uint8 ok [B]."""
        import torch

        B = int(configs.shape[0])
        ok = torch.empty(B, dtype=torch.uint8, device=configs.device)
        gs = self._pda(g)
        self.lib.bpdref_cuda_pda_advance(C.byref(gs), C.c_void_p(configs.data_ptr()),
                                         C.c_void_p(tokens.data_ptr()), _I(B),
                                         C.c_void_p(ok.data_ptr()), self._stream())
        return ok

    def _fsa(self, f):
        sym = f.symbols if f.symbols.numel() else f.offsets  # never read when empty
        return (_I(int(f.accept.numel())), _I(f.num_symbols), C.c_void_p(f.trans.data_ptr()),
                C.c_void_p(f.accept.data_ptr()), C.c_void_p(f.live.data_ptr()), _I(f.dead),
                C.c_void_p(f.offsets.data_ptr()), C.c_void_p(sym.data_ptr()),
                _I(int(f.offsets.numel()) - 1), _I(f.eos_id))

    def compute_mask(self, f, states):
        """Packed allow bits int32 [B, ceil(V/32)] of a byte-walk FSA
        (compute_mask_batch_cuda); `f` an FsaTensors on the device."""
        import torch

        B = int(states.numel())
        V = int(f.offsets.numel()) - 1
        out = torch.empty((B, (V + 31) // 32), dtype=torch.int32, device=states.device)
        self.lib.bpdref_cuda_compute_mask(*self._fsa(f), C.c_void_p(states.data_ptr()), _I(B),
                                          C.c_void_p(out.data_ptr()), self._stream())
        return out

    def advance_state(self, f, states, tokens):
        """Next states int32 [B] (advance_state_batch_cuda)."""
        import torch

        B = int(states.numel())
        out = torch.empty(B, dtype=torch.int32, device=states.device)
        self.lib.bpdref_cuda_advance_state(*self._fsa(f), C.c_void_p(states.data_ptr()),
                                           C.c_void_p(tokens.data_ptr()), _I(B),
                                           C.c_void_p(out.data_ptr()), self._stream())
        return out
