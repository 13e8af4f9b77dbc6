"""Per-step device ops of the dense regular path and the soft lookahead.

Drop-in for bpdecode's ``ops.py`` (``src/bpdecode/ops.py``): the same
:class:`FsaTensors` bundle (same fields, in the same order) and the same
``apply_mask_`` / ``compute_mask`` / ``advance_state`` / ``apply_soft_`` /
``build_token_transitions`` / ``build_lookahead`` signatures. The per-step
functions run hand-written sm_100a kernels through the C ABI
(``include/bpdecode_b200.h``); they accept CUDA tensors only and raise on CPU
tensors -- there is no CPU fallback on the device path.

Differences from the reference, all additive:

* ``FsaTensors.allow_bits`` -- the packed allow bits of every state (one bit
  per token, 32x smaller than ``tok_next``), built on the device the first time
  a per-step op needs it. The mask kernels read these bits instead of
  gathering an int32 ``tok_next`` row per logit row.
* a bundle without ``tok_next`` runs the byte-walk kernels on the raw DFA, as
  the reference's native ops do; :class:`~bpdecode_b200.batch.ConstraintBatch`
  densifies its grammars on the device (B200's HBM holds tables far past the
  reference's 32 M-entry auto-dense threshold).
* :func:`step_greedy_` -- mask + argmax + commit fused into one launch.
"""

from __future__ import annotations

from dataclasses import dataclass, replace

import numpy as np
from collections.abc import Sequence

import torch

from . import _capi
from .tokenizer import Vocabulary, as_vocabulary

_DTYPE_CODE = {torch.float32: _capi.F32, torch.bfloat16: _capi.BF16, torch.float16: _capi.F16}

# The reference's auto-dense threshold (ops.py:138), kept for `build(dense="auto")`.
DENSE_AUTO_LIMIT = 32_000_000


def words_stride(vocab_size: int) -> int:
    """Row stride (in 32-bit words) of a packed allow row: ceil(V/32) rounded
    up to a multiple of 4 so rows start on 16-byte boundaries."""
    return (((vocab_size + 31) // 32) + 3) // 4 * 4


_RAW_STREAM = getattr(torch._C, "_cuda_getCurrentRawStream", None)


def _stream(t: torch.Tensor) -> int:
    """torch's current CUDA stream on ``t``'s device, as the raw handle the C
    ABI takes (the direct accessor when torch has it: a tenth of the cost of
    building a Stream object every call)."""
    if _RAW_STREAM is not None and t.device.index is not None:
        return _RAW_STREAM(t.device.index)
    return torch.cuda.current_stream(t.device).cuda_stream


def _require_cuda(t: torch.Tensor, what: str) -> None:
    if t.device.type != "cuda":
        raise RuntimeError(
            f"bpdecode_b200: {what} must be a CUDA tensor (the device path has no CPU "
            "implementation)")


def _check_logits(logits: torch.Tensor, vocab: int) -> int:
    _require_cuda(logits, "logits")
    if logits.dim() != 2 or logits.shape[1] != vocab:
        raise RuntimeError(
            f"bpdecode_b200: logits must be [batch, {vocab}], got {tuple(logits.shape)}")
    if logits.dtype not in _DTYPE_CODE:
        raise RuntimeError(f"bpdecode_b200: unsupported logits dtype {logits.dtype}")
    if logits.shape[0] > 1 and logits.stride(0) < vocab or logits.stride(1) != 1:
        raise RuntimeError(
            "bpdecode_b200: logits columns must be contiguous and rows must not overlap "
            f"(strides {logits.stride()})")
    return _DTYPE_CODE[logits.dtype]


def _source_args(src: torch.Tensor, vocab: int, batch: int, src_rows: torch.Tensor | None,
                 out: torch.Tensor | None, device: torch.device) -> tuple:
    """(src code, row map, out) of the ``*_from`` steps: ``src`` [N, >= vocab]
    any float dtype on the device (columns contiguous); ``src_rows`` int64
    [batch] row indices into it, or None for rows 0..batch-1; ``out`` None or
    fp32 [batch, >= vocab]."""
    _require_cuda(src, "src")
    if src.dim() != 2 or src.shape[1] < vocab or src.stride(1) != 1:
        raise RuntimeError(f"bpdecode_b200: src must be [rows, >= {vocab}] with contiguous "
                           f"columns, got {tuple(src.shape)} strides {src.stride()}")
    if src.dtype not in _DTYPE_CODE:
        raise RuntimeError(f"bpdecode_b200: unsupported src dtype {src.dtype}")
    if src_rows is None:
        if src.shape[0] < batch:
            raise RuntimeError("bpdecode_b200: src has fewer rows than the batch")
    else:
        if (src_rows.dtype != torch.int64 or src_rows.numel() != batch
                or src_rows.device != device):
            raise RuntimeError("bpdecode_b200: src_rows must be int64 [batch] on the device")
        src_rows = src_rows.contiguous()
    if out is not None:
        _require_cuda(out, "out")
        if (out.dtype != torch.float32 or out.dim() != 2 or out.shape[0] != batch
                or out.shape[1] < vocab or out.stride(1) != 1):
            raise RuntimeError(f"bpdecode_b200: out must be fp32 [batch, >= {vocab}]")
    return _DTYPE_CODE[src.dtype], src_rows, out


def _as_i32(states: torch.Tensor, n: int, device: torch.device) -> torch.Tensor:
    _require_cuda(states, "states")
    if states.device != device:
        raise RuntimeError("bpdecode_b200: states and tables live on different devices")
    s = states.reshape(-1)
    if s.numel() != n:
        raise RuntimeError(f"bpdecode_b200: one state per logits row ({s.numel()} != {n})")
    if s.dtype != torch.int32:
        s = s.to(torch.int32)
    return s.contiguous()


def _upload(values: Sequence[int], dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A small host list as a device tensor without a host synchronisation:
    staged through page-locked memory (torch's caching host allocator) and
    copied asynchronously on the current stream -- a copy from pageable
    memory would wait for the work already queued on the GPU."""
    host = torch.tensor(list(values), dtype=dtype)
    if device.type != "cuda":
        return host.to(device)
    return host.pin_memory().to(device, non_blocking=True)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


@dataclass
class FsaTensors:
    """The FSA + token tables as tensors (ops.py:44-140, same fields and order)."""

    trans: torch.Tensor  # int32 [num_states * num_symbols]
    accept: torch.Tensor  # uint8 [num_states]
    live: torch.Tensor  # uint8 [num_states]
    num_symbols: int
    dead: int
    offsets: torch.Tensor  # int32 [vocab_size + 1]
    symbols: torch.Tensor  # int32 [offsets[-1]]
    eos_id: int
    start: int = 0
    accepting: frozenset[int] = frozenset()
    tok_next: torch.Tensor | None = None  # int32 [num_states, vocab]
    lookahead: torch.Tensor | None = None  # float32 [num_states, vocab]
    allow_bits: torch.Tensor | None = None  # int32 [num_states, words_stride(vocab)]

    @property
    def device(self) -> torch.device:
        return self.trans.device

    @property
    def num_states(self) -> int:
        return int(self.accept.numel())

    @property
    def vocab_size(self) -> int:
        return int(self.offsets.numel() - 1)

    def to(self, device: torch.device | str) -> FsaTensors:
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if self.trans.device == device:
            return self

        def mv(t: torch.Tensor | None) -> torch.Tensor | None:
            return None if t is None else t.to(device)

        return replace(
            self, trans=mv(self.trans), accept=mv(self.accept), live=mv(self.live),
            offsets=mv(self.offsets), symbols=mv(self.symbols), tok_next=mv(self.tok_next),
            lookahead=mv(self.lookahead), allow_bits=mv(self.allow_bits))

    def densify(self) -> FsaTensors:
        """Return a copy carrying the precomputed ``tok_next`` table."""
        if self.tok_next is not None:
            return self
        return replace(self, tok_next=build_token_transitions(self))

    def with_lookahead(self, k: int = 3) -> FsaTensors:
        """Return a copy carrying the ``k``-step soft-lookahead bias table."""
        base = self.densify()
        return replace(base, lookahead=build_lookahead(base, k))

    def _memo_empty_symbols(self) -> torch.Tensor:
        # a vocabulary of empty tokens has no symbols; kernels still need a pointer
        return torch.zeros(1, dtype=torch.int32, device=self.device)

    def dense_tables(self) -> tuple[torch.Tensor, torch.Tensor]:
        """(tok_next, allow_bits) on this bundle's CUDA device, built on first use
        and kept on the bundle."""
        _require_cuda(self.trans, "FsaTensors")
        if self.tok_next is None:
            self.tok_next = build_token_transitions(self)
        if self.allow_bits is None:
            self.allow_bits = build_allow_bits(self.tok_next)
        return self.tok_next, self.allow_bits

    @classmethod
    def from_tables(cls, fsa: object, toks: object) -> FsaTensors:
        """From bpdecode's host ``FsaTable`` / ``TokenSymbols`` (or anything with
        the same attributes, fsa.py:32-66)."""
        accept = list(fsa.accept)
        return cls(
            trans=torch.tensor(list(fsa.trans), dtype=torch.int32),
            accept=torch.tensor(accept, dtype=torch.uint8),
            live=torch.tensor(list(fsa.live), dtype=torch.uint8),
            num_symbols=int(fsa.num_symbols),
            dead=int(fsa.dead),
            offsets=torch.tensor(list(toks.offsets), dtype=torch.int32),
            symbols=torch.frombuffer(bytearray(bytes(toks.symbols) or b"\x00"),
                                     dtype=torch.uint8).to(torch.int32)[: len(toks.symbols)],
            eos_id=int(toks.eos_id),
            start=int(fsa.start),
            accepting=frozenset(i for i, a in enumerate(accept) if a),
        )

    @classmethod
    def from_arrays(cls, dfa: dict, vocab: object) -> FsaTensors:
        """From flattened DFA arrays (``trans``, ``accept``, ``live``,
        ``num_symbols``, ``dead``, ``start``, ``lut`` -- the 256-entry byte ->
        symbol-class table) and a vocabulary."""
        v = as_vocabulary(vocab)
        lut = np.asarray(dfa["lut"], dtype=np.int32)
        lengths = np.fromiter((len(t) for t in v.token_bytes), dtype=np.int64, count=v.size)
        offsets = np.zeros(v.size + 1, dtype=np.int32)
        np.cumsum(lengths, out=offsets[1:])
        flat = np.frombuffer(b"".join(v.token_bytes), dtype=np.uint8)
        symbols = lut[flat].astype(np.int32) if flat.size else np.zeros(0, np.int32)
        accept = np.asarray(dfa["accept"], dtype=np.uint8)
        return cls(
            trans=torch.from_numpy(np.asarray(dfa["trans"], dtype=np.int32).copy()),
            accept=torch.from_numpy(accept.copy()),
            live=torch.from_numpy(np.asarray(dfa["live"], dtype=np.uint8).copy()),
            num_symbols=int(dfa["num_symbols"]),
            dead=int(dfa["dead"]),
            offsets=torch.from_numpy(offsets),
            symbols=torch.from_numpy(symbols),
            eos_id=v.eos_id if v.eos_id is not None else -1,
            start=int(dfa["start"]),
            accepting=frozenset(int(i) for i in np.nonzero(accept)[0]),
        )

    @classmethod
    def build(cls, pattern: object, vocab: object, *, dense: bool | str = "auto") -> FsaTensors:
        """Compile ``pattern`` (a regex string or a compiled DFA) against ``vocab``.

        Regex compilation is bpdecode's front-end (``regex/compile.py``), used as
        is; this package rebuilds the per-step device path, not the compiler.
        """
        bundle = cls.from_arrays(dfa_arrays(pattern), vocab)
        want = dense is True or (
            dense == "auto" and bundle.num_states * bundle.vocab_size <= DENSE_AUTO_LIMIT)
        return bundle.densify() if want else bundle


def dfa_arrays(pattern: object) -> dict:
    """Flattened arrays of a DFA (a bpdecode ``DFA`` object, or a regex string
    compiled by bpdecode's front-end): dense ``trans`` over symbol classes,
    ``accept``, backward-reachability ``live`` (fsa.py:70-130) and the byte ->
    class table."""
    if isinstance(pattern, str):
        try:
            from bpdecode.regex import compile_regex  # type: ignore
        except ImportError as exc:
            raise ImportError(
                "compiling a regex string needs bpdecode's front-end (bpdecode.regex); "
                "pass a compiled DFA or use FsaTensors.from_arrays") from exc
        pattern = compile_regex(pattern)
    dfa = pattern
    num_states = len(dfa.trans)
    num_symbols = len(dfa.symbols)
    trans = np.asarray([x for row in dfa.trans for x in row], dtype=np.int32)
    accept = np.zeros(num_states, dtype=np.uint8)
    accept[list(dfa.accept)] = 1
    # live[s]: some accepting state is reachable from s (reverse BFS)
    preds: list[list[int]] = [[] for _ in range(num_states)]
    for s in range(num_states):
        for t in dfa.trans[s]:
            if 0 <= t < num_states:
                preds[t].append(s)
    live = accept.copy()
    work = [int(s) for s in np.nonzero(accept)[0]]
    while work:
        for p in preds[work.pop()]:
            if not live[p]:
                live[p] = 1
                work.append(p)
    return {
        "trans": trans, "accept": accept, "live": live, "num_symbols": num_symbols,
        "dead": int(dfa.dead), "start": int(dfa.start),
        "lut": np.asarray([dfa.symbol_of(b) for b in range(256)], dtype=np.int32),
    }


# --- table construction (compile time) ---------------------------------------

def build_token_transitions(
    fsa: FsaTensors, rows: torch.Tensor | list[int] | None = None
) -> torch.Tensor:
    """Dense ``[num_states, vocab]`` int32 next-state table (ops.py:143-197):
    the state after emitting token ``t`` from state ``s``, ``-1`` if rejected;
    EOS column ``s`` if ``s`` accepts, else ``-1``. On CUDA one thread walks one
    (state, token) pair; on CPU (compile time only) a vectorised torch walk."""
    if fsa.device.type == "cuda":
        return _build_tok_next_cuda(fsa, rows)
    return _build_tok_next_host(fsa, rows)


def _build_tok_next_cuda(fsa: FsaTensors, rows) -> torch.Tensor:
    dev = fsa.device
    S, V = fsa.num_states, fsa.vocab_size
    row_t = None
    if rows is not None:
        row_t = torch.as_tensor(rows, dtype=torch.int32, device=dev).contiguous()
    R = S if row_t is None else int(row_t.numel())
    out = torch.empty((R, V), dtype=torch.int32, device=dev)
    sym = fsa.symbols if fsa.symbols.numel() else torch.zeros(1, dtype=torch.int32, device=dev)
    trans, accept, live = (fsa.trans.contiguous(), fsa.accept.contiguous(),
                           fsa.live.contiguous())
    offsets, sym = fsa.offsets.contiguous(), sym.to(torch.int32).contiguous()
    L = _capi.lib()
    with torch.cuda.device(dev):
        L.check(L.bpd_dense_build_tok_next(
            trans.data_ptr(), S, fsa.num_symbols, accept.data_ptr(), live.data_ptr(), fsa.dead,
            offsets.data_ptr(), sym.data_ptr(), V, fsa.eos_id, _ptr(row_t), R, out.data_ptr(),
            _stream(out)))
    return out


def _build_tok_next_host(fsa: FsaTensors, rows) -> torch.Tensor:
    S, M, V = fsa.num_states, fsa.num_symbols, fsa.vocab_size
    trans = fsa.trans.to(torch.long)
    offsets = fsa.offsets.to(torch.long)
    lengths = offsets[1:] - offsets[:-1]
    row_states = (torch.arange(S) if rows is None
                  else torch.as_tensor(rows, dtype=torch.long))
    R = int(row_states.numel())
    cur = row_states.view(R, 1).expand(R, V).clone()
    sym = fsa.symbols.to(torch.long)
    bad = torch.zeros(V, dtype=torch.bool)
    L = int(lengths.max()) if V else 0
    for k in range(L):
        has = lengths > k
        idx = (offsets[:-1] + k).clamp(max=max(int(sym.numel()) - 1, 0))
        sk = sym[idx] if sym.numel() else torch.zeros(V, dtype=torch.long)
        bad |= has & ((sk < 0) | (sk >= M))
        nxt = trans[cur * M + sk.clamp(0, M - 1)]
        cur = torch.where(has.view(1, V), nxt, cur)
    live = fsa.live.to(torch.bool)
    out = torch.where(live[cur] & ~bad.view(1, V), cur, torch.full_like(cur, -1)).to(torch.int32)
    if fsa.eos_id is not None and 0 <= fsa.eos_id < V:
        acc = fsa.accept.to(torch.bool)[row_states]
        out[:, fsa.eos_id] = torch.where(acc, row_states.to(torch.int32),
                                         torch.full((R,), -1, dtype=torch.int32))
    return out


def build_allow_bits(tok_next: torch.Tensor) -> torch.Tensor:
    """Packed allow rows ``[S, words_stride(V)]`` (int32 storage of uint32
    words, LSB first) of a CUDA ``tok_next``."""
    _require_cuda(tok_next, "tok_next")
    S, V = tok_next.shape
    ws = words_stride(V)
    tn = tok_next.contiguous()
    out = torch.empty((S, ws), dtype=torch.int32, device=tn.device)
    L = _capi.lib()
    with torch.cuda.device(tn.device):
        L.check(L.bpd_dense_build_allow_bits(tn.data_ptr(), S, V, out.data_ptr(), ws,
                                             _stream(out)))
    return out


def build_lookahead(fsa: FsaTensors, k: int) -> torch.Tensor:
    """Soft-lookahead bias table ``[num_states, vocab]`` float32 (ops.py:200-236):
    ``out[s, t] = log Z_{k-1}(delta(s, t))``, ``-inf`` where ``t`` is not
    allowed. Built on the CUDA device (a CPU bundle is built on the current
    CUDA device and copied back)."""
    if fsa.tok_next is None:
        fsa = fsa.densify()
    if fsa.device.type != "cuda":
        if not torch.cuda.is_available():
            raise RuntimeError("bpdecode_b200: build_lookahead runs on a CUDA device")
        return build_lookahead(fsa.to("cuda"), k).to(fsa.device)
    tn = fsa.tok_next.contiguous()
    S, V = tn.shape
    L = _capi.lib()
    out = torch.empty((S, V), dtype=torch.float32, device=tn.device)
    ws = torch.empty(L.bpd_soft_workspace_bytes(S), dtype=torch.uint8, device=tn.device)
    accept, live = fsa.accept.contiguous(), fsa.live.contiguous()
    with torch.cuda.device(tn.device):
        L.check(L.bpd_soft_build_lookahead(
            tn.data_ptr(), S, V, accept.data_ptr(), live.data_ptr(), fsa.eos_id, int(k),
            out.data_ptr(), ws.data_ptr(), _stream(out)))
    return out


# --- per-step ops --------------------------------------------------------------

def apply_mask_(
    logits: torch.Tensor,
    fsa: FsaTensors,
    states: torch.Tensor,
    neg_inf: float = float("-inf"),
) -> torch.Tensor:
    """In place: every disallowed logit of ``logits`` [batch, vocab] becomes
    ``neg_inf``, one grammar state per row; rows with a negative state (BROKEN /
    FREE) are fully masked (ops.py:262-281)."""
    B = int(logits.shape[0])
    code = _check_logits(logits, fsa.vocab_size)
    st = _as_i32(states, B, fsa.device)
    L = _capi.lib()
    if fsa.tok_next is None:
        L.check(L.bpd_walk_apply_mask(
            logits.data_ptr(), code, logits.stride(0), B, *_walk_args(fsa), st.data_ptr(),
            float(neg_inf), _stream(logits)))
        return logits
    tok_next, bits = fsa.dense_tables()
    L.check(L.bpd_dense_apply_mask(
        logits.data_ptr(), code, logits.stride(0), B, fsa.vocab_size, st.data_ptr(), None,
        bits.data_ptr(), bits.shape[1], fsa.num_states, float(neg_inf), _stream(logits)))
    return logits


def compute_mask(fsa: FsaTensors, states: torch.Tensor) -> torch.Tensor:
    """Packed allow-mask, uint32 bits in an int32 tensor [batch, ceil(vocab/32)]
    (LSB first), one state per row (ops.py:284-292)."""
    B = int(states.numel())
    st = _as_i32(states, B, fsa.device)
    W = (fsa.vocab_size + 31) // 32
    out = torch.empty((B, W), dtype=torch.int32, device=fsa.device)
    L = _capi.lib()
    if fsa.tok_next is None:
        L.check(L.bpd_walk_mask_bits(*_walk_args(fsa), st.data_ptr(), B, out.data_ptr(),
                                     _stream(out)))
        return out
    _, bits = fsa.dense_tables()
    L.check(L.bpd_dense_mask_bits(st.data_ptr(), None, B, bits.data_ptr(), bits.shape[1],
                                  fsa.num_states, fsa.vocab_size, out.data_ptr(), _stream(out)))
    return out


def advance_state(fsa: FsaTensors, states: torch.Tensor, token_ids: torch.Tensor) -> torch.Tensor:
    """Next state per row after emitting ``token_ids``; ``-1`` if the token was
    off a valid path or the row was already broken (ops.py:295-310)."""
    B = int(states.numel())
    st = _as_i32(states, B, fsa.device)
    tk = _tokens(token_ids, B, fsa.device)
    out = torch.empty(B, dtype=torch.int32, device=fsa.device)
    L = _capi.lib()
    if fsa.tok_next is None:
        L.check(L.bpd_walk_advance(*_walk_args(fsa), st.data_ptr(), tk.data_ptr(),
                                   int(tk.dtype == torch.int64), B, out.data_ptr(),
                                   _stream(out)))
        return out
    tok_next, _ = fsa.dense_tables()
    L.check(L.bpd_dense_advance(st.data_ptr(), None, B, tk.data_ptr(),
                                int(tk.dtype == torch.int64), tok_next.data_ptr(),
                                fsa.num_states, fsa.vocab_size, out.data_ptr(), 0, _stream(out)))
    return out


def _walk_args(fsa: FsaTensors) -> tuple:
    """(trans, S, M, accept, live, dead, offsets, symbols, V, eos) pointers of
    the byte-walk entry points; the tensors must already be contiguous int32 /
    uint8 on the device (FsaTensors keeps them so)."""
    _require_cuda(fsa.trans, "FsaTensors")
    sym = fsa.symbols
    if sym.numel() == 0:
        sym = fsa._memo_empty_symbols()
    return (fsa.trans.data_ptr(), fsa.num_states, fsa.num_symbols, fsa.accept.data_ptr(),
            fsa.live.data_ptr(), fsa.dead, fsa.offsets.data_ptr(), sym.data_ptr(),
            fsa.vocab_size, fsa.eos_id)


def _tokens(token_ids: torch.Tensor, n: int, device: torch.device) -> torch.Tensor:
    _require_cuda(token_ids, "token_ids")
    t = token_ids.reshape(-1)
    if t.numel() != n:
        raise RuntimeError(f"bpdecode_b200: one token per row ({t.numel()} != {n})")
    if t.device != device:
        t = t.to(device)
    if t.dtype not in (torch.int32, torch.int64):
        t = t.to(torch.int64)
    return t.contiguous()


def apply_soft_(
    logits: torch.Tensor,
    fsa: FsaTensors,
    states: torch.Tensor,
    alpha: float = 1.0,
) -> torch.Tensor:
    """In place: ``logits += alpha * lookahead[states]`` on allowed entries and
    ``-inf`` on disallowed ones; ``alpha = 0`` is exactly hard masking
    (ops.py:239-259)."""
    if fsa.lookahead is None:
        raise ValueError("fsa has no lookahead table; build with dense + with_lookahead")
    _require_cuda(fsa.lookahead, "lookahead")
    B = int(logits.shape[0])
    code = _check_logits(logits, fsa.vocab_size)
    st = _as_i32(states, B, fsa.device)
    la = fsa.lookahead.contiguous()
    bits = fsa.dense_tables()[1]
    L = _capi.lib()
    L.check(L.bpd_soft_apply(logits.data_ptr(), code, logits.stride(0), B, fsa.vocab_size,
                             st.data_ptr(), None, la.data_ptr(), bits.data_ptr(), bits.shape[1],
                             fsa.num_states, float(alpha), _stream(logits)))
    return logits


_SCRATCH: dict[tuple[int, int], torch.Tensor] = {}


def step_scratch(batch: int, device: torch.device) -> torch.Tensor:
    """Zeroed device scratch of the fused steps for ``batch`` rows
    (``bpd_step_scratch_bytes``), cached per device and grown on demand; the
    kernels leave it zero, so one buffer serves every call on a stream."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    key = (idx, 0)
    need = int(_capi.lib().bpd_step_scratch_bytes(max(int(batch), 1)))
    buf = _SCRATCH.get(key)
    if buf is None or buf.numel() < need:
        buf = torch.zeros(need, dtype=torch.uint8, device=torch.device("cuda", idx))
        _SCRATCH[key] = buf
    return buf


def step_greedy_(
    logits: torch.Tensor,
    fsa: FsaTensors,
    state_pool: torch.Tensor,
    slots: torch.Tensor | None = None,
    neg_inf: float = float("-inf"),
    chunks_per_row: int = 0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """NEW, fused: mask ``logits`` in place, take the first maximal token of
    every masked row (``torch.argmax`` semantics) and commit it into
    ``state_pool[slots[b]]``. Returns (tokens int64 [B], next states int32 [B]).
    Identical results to ``apply_mask_`` + ``logits.argmax(-1)`` +
    ``advance_state``, in one launch."""
    tok_next, bits = fsa.dense_tables()
    B = int(logits.shape[0])
    code = _check_logits(logits, fsa.vocab_size)
    _require_cuda(state_pool, "state_pool")
    if state_pool.dtype != torch.int32 or not state_pool.is_contiguous():
        raise RuntimeError("bpdecode_b200: state_pool must be a contiguous int32 tensor")
    if slots is not None and (slots.dtype != torch.int64 or slots.numel() != B):
        raise RuntimeError("bpdecode_b200: slots must be int64 [batch]")
    tokens = torch.empty(B, dtype=torch.int64, device=logits.device)
    nxt = torch.empty(B, dtype=torch.int32, device=logits.device)
    L = _capi.lib()
    L.check(L.bpd_dense_step_greedy(
        logits.data_ptr(), code, logits.stride(0), B, fsa.vocab_size, state_pool.data_ptr(),
        _ptr(slots), bits.data_ptr(), bits.shape[1], tok_next.data_ptr(), fsa.num_states,
        float(neg_inf), tokens.data_ptr(), nxt.data_ptr(), int(chunks_per_row),
        step_scratch(B, logits.device).data_ptr(), _stream(logits)))
    return tokens, nxt


def soft_step_greedy_(
    logits: torch.Tensor,
    fsa: FsaTensors,
    state_pool: torch.Tensor,
    slots: torch.Tensor | None = None,
    alpha: float = 1.0,
    chunks_per_row: int = 0,
) -> tuple[torch.Tensor, torch.Tensor]:
    """NEW, fused: ``apply_soft_`` in place, the first maximal token of every
    biased row, and its commit into ``state_pool[slots[b]]``. Returns
    (tokens int64 [B], next states int32 [B]); identical to ``apply_soft_`` +
    ``logits.argmax(-1)`` + ``advance_state``, in one launch."""
    if fsa.lookahead is None or fsa.tok_next is None:
        raise ValueError("fsa has no lookahead table; build with dense + with_lookahead")
    B = int(logits.shape[0])
    code = _check_logits(logits, fsa.vocab_size)
    _require_cuda(state_pool, "state_pool")
    if state_pool.dtype != torch.int32 or not state_pool.is_contiguous():
        raise RuntimeError("bpdecode_b200: state_pool must be a contiguous int32 tensor")
    if slots is not None and (slots.dtype != torch.int64 or slots.numel() != B):
        raise RuntimeError("bpdecode_b200: slots must be int64 [batch]")
    la = fsa.lookahead.contiguous()
    tok_next, bits = fsa.dense_tables()
    tokens = torch.empty(B, dtype=torch.int64, device=logits.device)
    nxt = torch.empty(B, dtype=torch.int32, device=logits.device)
    L = _capi.lib()
    L.check(L.bpd_soft_step_greedy(
        logits.data_ptr(), code, logits.stride(0), B, fsa.vocab_size, state_pool.data_ptr(),
        _ptr(slots), la.data_ptr(), bits.data_ptr(), bits.shape[1], tok_next.data_ptr(),
        fsa.num_states, float(alpha), tokens.data_ptr(), nxt.data_ptr(), int(chunks_per_row),
        step_scratch(B, logits.device).data_ptr(), _stream(logits)))
    return tokens, nxt


__all__ = [
    "DENSE_AUTO_LIMIT", "FsaTensors", "Vocabulary", "advance_state", "apply_mask_",
    "apply_soft_", "build_allow_bits", "build_lookahead", "build_token_transitions",
    "compute_mask", "dfa_arrays", "soft_step_greedy_", "step_greedy_", "step_scratch",
    "words_stride",
]
