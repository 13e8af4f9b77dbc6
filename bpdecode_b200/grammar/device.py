"""Pushdown-automaton (context-free grammar) path on the device.

Drop-in for bpdecode's ``grammar/device.py``: :class:`PdaTensors`,
:func:`build_pda_tensors`, :func:`pda_apply_mask_`, :func:`pda_advance_state`,
:class:`CFGConstraintBatch` and the ``PDA_*`` constants keep their names,
layouts and semantics (config rows of 266 int32: ``num_configs``,
``saturated``, ``depth[8]``, ``stack[8][32]``). The kernels behind them are the
sm_100a ones of ``csrc/pda.cu`` through the C ABI; what changes:

* :meth:`PdaTensors.init_config` runs the closure on the device (the
  reference's ``pda_init`` op computes it on the host and copies it over);
* every mask call consults a per-grammar mask memo held in HBM, so a
  config-set whose mask was computed before is applied like a dense row;
* :class:`CFGConstraintBatch` masks and commits its pool rows in place through
  the slot tensor and masks broken rows inside the same launch sequence -- no
  gather copies and no host sync per step (the reference syncs on
  ``bool(broken.any())`` every step, grammar/device.py:263-265).
"""

from __future__ import annotations

import ctypes as C
import os
from collections import OrderedDict
from collections.abc import Hashable, Sequence
from dataclasses import dataclass, field, replace

import numpy as np
import torch

from .. import _capi
from ..ops import _check_logits, _require_cuda, _stream, _tokens, _upload
from ..tokenizer import as_vocabulary

# Must match the C ABI (BPD_PDA_MAX_CONFIGS / BPD_PDA_MAX_DEPTH / ..._INTS) and
# the reference's pda.hpp:35-36.
PDA_MAX_CONFIGS = 8
PDA_MAX_DEPTH = 32
PDA_CONFIG_FLAT = 2 + PDA_MAX_CONFIGS + PDA_MAX_CONFIGS * PDA_MAX_DEPTH

_EPS, _BYTE, _CALL = 0, 1, 2

# Mask-memo entries per grammar (power of two); each entry holds one packed
# allow row (V/8 bytes) plus a 1 KB key. Override with BPDECODE_PDA_MEMO.
DEFAULT_MEMO_CAPACITY = int(os.environ.get("BPDECODE_PDA_MEMO", "4096"))

_GRAMMAR_FIELDS = ("accept", "live", "edge_offsets", "edge_kind", "edge_lo", "edge_hi",
                   "edge_dst", "edge_callee", "tok_offsets", "tok_bytes")


@dataclass
class PdaTensors:
    """Flattened grammar + token bytes (grammar/device.py:33-76, same fields)."""

    num_states: int
    root_start: int
    root_accept: int
    accept: torch.Tensor  # uint8 [num_states]
    live: torch.Tensor  # uint8 [num_states]
    edge_offsets: torch.Tensor  # int32 [num_states + 1]
    edge_kind: torch.Tensor  # int32 [nnz]
    edge_lo: torch.Tensor  # int32 [nnz]
    edge_hi: torch.Tensor  # int32 [nnz]
    edge_dst: torch.Tensor  # int32 [nnz]
    edge_callee: torch.Tensor  # int32 [nnz]
    tok_offsets: torch.Tensor  # int32 [vocab_size + 1]
    tok_bytes: torch.Tensor  # uint8 [tok_offsets[-1]]
    vocab_size: int
    eos_id: int
    _memo: dict = field(default_factory=dict, repr=False, compare=False)

    @property
    def device(self) -> torch.device:
        return self.accept.device

    def to(self, device: torch.device | str) -> PdaTensors:
        device = torch.device(device)
        if device.type == "cuda" and device.index is None:
            device = torch.device("cuda", torch.cuda.current_device())
        if self.accept.device == device:
            return self
        return replace(self, _memo={}, **{f: getattr(self, f).to(device)
                                          for f in _GRAMMAR_FIELDS})

    # --- device view ---------------------------------------------------
    def _struct(self) -> _capi.PdaGrammar:
        """The C ABI grammar struct (device pointers); built once per bundle."""
        s = self._memo.get("struct")
        if s is None:
            _require_cuda(self.accept, "PdaTensors")
            keep = {f: getattr(self, f).contiguous() for f in _GRAMMAR_FIELDS}
            if keep["tok_bytes"].numel() == 0:
                keep["tok_bytes"] = torch.zeros(1, dtype=torch.uint8, device=self.device)
            for f in ("edge_kind", "edge_lo", "edge_hi", "edge_dst", "edge_callee"):
                if keep[f].numel() == 0:
                    keep[f] = torch.zeros(1, dtype=torch.int32, device=self.device)
            s = _capi.PdaGrammar(
                self.num_states, int(self.edge_kind.numel()), self.root_start, self.root_accept,
                *(keep[f].data_ptr() for f in _GRAMMAR_FIELDS[:8]),
                self.vocab_size, self.eos_id, keep["tok_offsets"].data_ptr(),
                keep["tok_bytes"].data_ptr())
            self._memo["struct"] = s
            self._memo["keep"] = keep
        return s

    def mask_memo(self) -> tuple[torch.Tensor, int]:
        """(memo buffer, capacity) of this grammar on its device (created and
        cleared on first use)."""
        m = self._memo.get("memo")
        if m is None:
            cap = DEFAULT_MEMO_CAPACITY
            L = _capi.lib()
            buf = torch.empty(L.bpd_pda_memo_bytes(cap, self.vocab_size), dtype=torch.uint8,
                              device=self.device)
            L.check(L.bpd_pda_memo_reset(buf.data_ptr(), cap, self.vocab_size, _stream(buf)))
            m = (buf, cap)
            self._memo["memo"] = m
        return m

    def clear_memo(self) -> None:
        """Forget every cached mask (the next mask call recomputes)."""
        if "memo" in self._memo:
            buf, cap = self._memo["memo"]
            L = _capi.lib()
            L.check(L.bpd_pda_memo_reset(buf.data_ptr(), cap, self.vocab_size, _stream(buf)))

    def workspace(self, batch: int) -> torch.Tensor:
        L = _capi.lib()
        need = int(L.bpd_pda_workspace_bytes(max(batch, 1), self.vocab_size))
        ws = self._memo.get("workspace")
        if ws is None or ws.numel() < need:
            ws = torch.empty(need, dtype=torch.uint8, device=self.device)
            self._memo["workspace"] = ws
        return ws

    def init_config(self) -> torch.Tensor:
        """One freshly initialised config-set, ``[PDA_CONFIG_FLAT]`` int32
        (pda.hpp:200-207), computed on the device."""
        hit = self._memo.get("init")
        if hit is None:
            hit = torch.empty(PDA_CONFIG_FLAT, dtype=torch.int32, device=self.device)
            L = _capi.lib()
            L.check(L.bpd_pda_init(C.byref(self._struct()), hit.data_ptr(), _stream(hit)))
            self._memo["init"] = hit
        return hit.clone()

    def init_batch(self, batch: int) -> torch.Tensor:
        """``batch`` copies of the initial config-set, ``[batch, PDA_CONFIG_FLAT]``."""
        return self.init_config().unsqueeze(0).expand(batch, -1).contiguous()

    @classmethod
    def from_arrays(cls, grammar: dict, vocab: object, device: torch.device | str = "cpu",
                    ) -> PdaTensors:
        """From flattened grammar arrays (``accept``, ``live``, ``edge_*``,
        ``num_states``, ``root_start``, ``root_accept``) and a vocabulary."""
        v = as_vocabulary(vocab)
        offs = np.zeros(v.size + 1, np.int32)
        np.cumsum([len(t) for t in v.token_bytes], out=offs[1:])
        flat = np.frombuffer(b"".join(v.token_bytes), np.uint8).copy()

        def t(name: str, dtype: torch.dtype) -> torch.Tensor:
            return torch.as_tensor(np.asarray(grammar[name]), dtype=dtype).to(device)

        return cls(
            num_states=int(grammar["num_states"]), root_start=int(grammar["root_start"]),
            root_accept=int(grammar["root_accept"]),
            accept=t("accept", torch.uint8), live=t("live", torch.uint8),
            edge_offsets=t("edge_offsets", torch.int32), edge_kind=t("edge_kind", torch.int32),
            edge_lo=t("edge_lo", torch.int32), edge_hi=t("edge_hi", torch.int32),
            edge_dst=t("edge_dst", torch.int32), edge_callee=t("edge_callee", torch.int32),
            tok_offsets=torch.from_numpy(offs).to(device),
            tok_bytes=torch.from_numpy(flat).to(device),
            vocab_size=v.size, eos_id=v.eos_id if v.eos_id is not None else -1,
        )


def build_pda_tensors(compiled: object, vocab: object, device: torch.device | str = "cpu",
                      ) -> PdaTensors:
    """Flatten a compiled grammar into one global state space with a CSR edge
    list (grammar/device.py:79-158): rule NFAs concatenated in rule order,
    edges in each state's ``out()`` order (which fixes the closure's push
    order), a call edge as (return state, callee start state).

    ``compiled`` is bpdecode's ``CompiledGrammar`` (the grammar front-end is
    used as is): ``rules`` (name -> NFA with ``num_states``, ``start``,
    ``accept``, ``out(s)``), ``root`` and ``coreachable``.
    """
    order = list(compiled.rules)
    offset: dict[str, int] = {}
    total = 0
    for name in order:
        offset[name] = total
        total += compiled.rules[name].num_states
    accept = np.zeros(total, np.uint8)
    live = np.zeros(total, np.uint8)
    offsets = np.zeros(total + 1, np.int32)
    kind: list[int] = []
    lo: list[int] = []
    hi: list[int] = []
    dst: list[int] = []
    callee: list[int] = []
    for name in order:
        nfa = compiled.rules[name]
        base = offset[name]
        accept[base + nfa.accept] = 1
        for s in compiled.coreachable[name]:
            live[base + s] = 1
        for s in range(nfa.num_states):
            offsets[base + s] = len(kind)
            for label, d in nfa.out(s):
                if label is None:
                    kind.append(_EPS), lo.append(0), hi.append(0), callee.append(-1)
                elif label[0] == "byte":
                    kind.append(_BYTE), lo.append(label[1]), hi.append(label[2]), callee.append(-1)
                else:
                    c = label[1]
                    kind.append(_CALL), lo.append(0), hi.append(0)
                    callee.append(offset[c] + compiled.rules[c].start)
                dst.append(base + d)
    offsets[total] = len(kind)
    root = compiled.rules[compiled.root]
    arrays = {
        "num_states": total, "root_start": offset[compiled.root] + root.start,
        "root_accept": offset[compiled.root] + root.accept, "accept": accept, "live": live,
        "edge_offsets": offsets, "edge_kind": np.asarray(kind, np.int32),
        "edge_lo": np.asarray(lo, np.int32), "edge_hi": np.asarray(hi, np.int32),
        "edge_dst": np.asarray(dst, np.int32), "edge_callee": np.asarray(callee, np.int32),
    }
    return PdaTensors.from_arrays(arrays, vocab, device)


def pda_apply_mask_(
    logits: torch.Tensor, g: PdaTensors, configs: torch.Tensor,
    neg_inf: float = float("-inf"), *, slots: torch.Tensor | None = None,
    broken: torch.Tensor | None = None, memo: bool = True,
) -> torch.Tensor:
    """In place: ``neg_inf`` on every token rejected from each row's config-set
    (the pda_apply_mask_ op, bindings/torch_ops.cpp:326-376). Any float logits
    dtype. Keyword extensions: ``slots`` (row b uses ``configs[slots[b]]``),
    ``broken`` (uint8/bool per pool row: such rows are fully masked) and
    ``memo`` (use the grammar's HBM mask memo)."""
    B = int(logits.shape[0])
    code = _check_logits(logits, g.vocab_size)
    cfg = _check_configs(configs, g)
    if slots is None and cfg.shape[0] != B:
        raise RuntimeError("bpdecode_b200: one config-set per logits row")
    mbuf, cap = g.mask_memo() if memo else (None, 0)
    ws = g.workspace(B)
    L = _capi.lib()
    L.check(L.bpd_pda_apply_mask(
        C.byref(g._struct()), logits.data_ptr(), code, logits.stride(0), cfg.data_ptr(),
        None if slots is None else slots.data_ptr(),
        None if broken is None else _u8(broken).data_ptr(), B,
        None if mbuf is None else mbuf.data_ptr(), cap, ws.data_ptr(), float(neg_inf),
        _stream(logits)))
    return logits


def pda_compute_mask(g: PdaTensors, configs: torch.Tensor, *, memo: bool = True) -> torch.Tensor:
    """Packed allow bits, int32 ``[batch, ceil(vocab/32)]`` LSB first
    (compute_mask_pda_batch, pda_cpu.cpp:7-21)."""
    cfg = _check_configs(configs, g)
    B = int(cfg.shape[0])
    out = torch.empty((B, (g.vocab_size + 31) // 32), dtype=torch.int32, device=g.device)
    mbuf, cap = g.mask_memo() if memo else (None, 0)
    ws = g.workspace(B)
    L = _capi.lib()
    L.check(L.bpd_pda_mask_bits(
        C.byref(g._struct()), cfg.data_ptr(), None, None, B,
        None if mbuf is None else mbuf.data_ptr(), cap, ws.data_ptr(), out.data_ptr(),
        _stream(out)))
    return out


def pda_advance_state(configs: torch.Tensor, g: PdaTensors, token_ids: torch.Tensor,
                      ) -> torch.Tensor:
    """Advance each config-set by its token in place; returns uint8 ``ok``
    (0 where the token was off a valid path -- that config-set is left
    unchanged), grammar/device.py:172-183."""
    cfg = _check_configs(configs, g)
    B = int(cfg.shape[0])
    tk = _tokens(token_ids, B, g.device)
    ok = torch.empty(B, dtype=torch.uint8, device=g.device)
    L = _capi.lib()
    L.check(L.bpd_pda_advance(C.byref(g._struct()), cfg.data_ptr(), None, B, tk.data_ptr(),
                              int(tk.dtype == torch.int64), ok.data_ptr(), None, None,
                              _stream(ok)))
    return ok


def _check_configs(configs: torch.Tensor, g: PdaTensors) -> torch.Tensor:
    _require_cuda(configs, "configs")
    if configs.dtype != torch.int32:
        raise RuntimeError("bpdecode_b200: configs must be int32")
    if configs.dim() != 2 or configs.shape[1] != PDA_CONFIG_FLAT:
        raise RuntimeError(f"bpdecode_b200: configs must be [batch, {PDA_CONFIG_FLAT}]")
    if not configs.is_contiguous():
        raise RuntimeError("bpdecode_b200: configs must be contiguous")
    if configs.device != g.device:
        raise RuntimeError("bpdecode_b200: configs and grammar live on different devices")
    return configs


def _u8(t: torch.Tensor) -> torch.Tensor:
    if t.dtype == torch.bool:
        return t.view(torch.uint8)
    if t.dtype != torch.uint8:
        raise RuntimeError("bpdecode_b200: broken flags must be bool or uint8")
    return t


_BROKEN = -1  # status of a row whose token left the grammar (ConstraintBatch.BROKEN)


class CFGConstraintBatch:
    """Fixed-capacity pool of PDA config-sets sharing one :class:`PdaTensors`
    (grammar/device.py:189-300): one masked/committed row per ``seq_ids``
    entry, masks memoised per config-set in HBM."""

    _SLOT_CACHE = 8

    def __init__(self, g: PdaTensors, capacity: int, device: torch.device | str | None = None,
                 ) -> None:
        self.g = g if device is None else g.to(device)
        self.device = self.g.device
        _require_cuda(self.g.accept, "CFGConstraintBatch tables")
        self.capacity = capacity
        self._configs = self.g.init_batch(capacity)
        self._broken = torch.zeros(capacity, dtype=torch.bool, device=self.device)
        self._slot_of: dict[Hashable, int] = {}
        self._free: list[int] = list(reversed(range(capacity)))
        self._slot_cache: OrderedDict[tuple, torch.Tensor] = OrderedDict()

    # --- lifecycle -------------------------------------------------------
    def add(self, seq_id: Hashable) -> int:
        if seq_id in self._slot_of:
            raise KeyError(f"sequence {seq_id!r} already in the batch")
        if not self._free:
            raise RuntimeError("CFGConstraintBatch is at capacity")
        slot = self._free.pop()
        self._slot_of[seq_id] = slot
        self._configs[slot] = self.g.init_config()
        self._broken[slot] = False
        self._slot_cache.clear()
        return slot

    def evict(self, seq_id: Hashable) -> None:
        slot = self._slot_of.pop(seq_id)
        self._free.append(slot)
        self._slot_cache.clear()

    def reset(self, seq_id: Hashable) -> None:
        slot = self._slot_of[seq_id]
        self._configs[slot] = self.g.init_config()
        self._broken[slot] = False

    def add_many(self, seq_ids: Sequence[Hashable]) -> list[int]:
        """NEW: :meth:`add` of every id with one device write per pool."""
        slots = self._add_host(seq_ids)
        if slots:
            self._init_slots(_upload(slots, torch.int64, self.device))
        return slots

    def _add_host(self, seq_ids: Sequence[Hashable]) -> list[int]:
        """The bookkeeping of :meth:`add_many` without the device write (the
        slots returned must get :meth:`_init_slots`)."""
        ids = set(seq_ids)
        if len(ids) != len(seq_ids) or not self._slot_of.keys().isdisjoint(ids):
            raise KeyError("add_many: ids must be distinct and new")
        if len(seq_ids) > len(self._free):
            raise RuntimeError("CFGConstraintBatch is at capacity")
        slots = [self._free.pop() for _ in seq_ids]
        for sid, slot in zip(seq_ids, slots):
            self._slot_of[sid] = slot
        self._slot_cache.clear()
        return slots

    def _init_slots(self, idx: torch.Tensor) -> None:
        """Fresh initial config-sets and cleared broken flags at device slot
        indices ``idx`` (int64)."""
        n = int(idx.numel())
        self._configs.index_copy_(0, idx, self.g.init_config().unsqueeze(0).expand(n, -1))
        self._broken.index_fill_(0, idx, False)

    def evict_many(self, seq_ids: Sequence[Hashable]) -> None:
        """NEW: :meth:`evict` of every id (host bookkeeping only)."""
        for s in seq_ids:
            self._free.append(self._slot_of.pop(s))
        self._slot_cache.clear()

    # --- checkpoint / resume ------------------------------------------
    def state_dict(self) -> dict:
        """NEW: the config-set pool ([capacity, 266] int32), the broken flags
        and the slot bookkeeping, as host copies; the grammar tables and the
        mask memo (a cache) are not included."""
        return {"kind": "pda", "capacity": self.capacity, "num_states": self.g.num_states,
                "configs": self._configs.cpu().clone(), "broken": self._broken.cpu().clone(),
                "slot_of": dict(self._slot_of), "free": list(self._free)}

    def load_state_dict(self, sd: dict) -> None:
        """NEW: restore what :meth:`state_dict` saved (same capacity and
        grammar), replacing every sequence of this batch."""
        if sd.get("kind") != "pda" or sd["capacity"] != self.capacity:
            raise ValueError("state_dict is not from a CFGConstraintBatch of this capacity")
        if sd["num_states"] != self.g.num_states:
            raise ValueError("state_dict was saved over a different grammar")
        self._configs.copy_(sd["configs"].to(device=self.device, dtype=torch.int32))
        self._broken.copy_(sd["broken"].to(device=self.device, dtype=torch.bool))
        self._slot_of = dict(sd["slot_of"])
        self._free = list(sd["free"])
        self._slot_cache.clear()

    def __len__(self) -> int:
        return len(self._slot_of)

    def __contains__(self, seq_id: Hashable) -> bool:
        return seq_id in self._slot_of

    # --- per-step ------------------------------------------------------
    def _slots(self, seq_ids: Sequence[Hashable]) -> torch.Tensor:
        return self._slots_arg(seq_ids)[0]

    def _slots_arg(self, seq_ids: Sequence[Hashable]) -> tuple[torch.Tensor, int | None]:
        """The device slot tensor of ``seq_ids`` and the pointer the kernels
        get for it: None when row b is slot b for every row (the kernels then
        skip the slot load)."""
        key = seq_ids if isinstance(seq_ids, tuple) else tuple(seq_ids)
        hit = self._slot_cache.get(key)
        if hit is not None:
            self._slot_cache.move_to_end(key)
            return hit
        host = [self._slot_of[s] for s in key]
        slots = _upload(host, torch.int64, self.device)
        hit = (slots, None if all(s == i for i, s in enumerate(host)) else slots.data_ptr())
        self._slot_cache[key] = hit
        if len(self._slot_cache) > self._SLOT_CACHE:
            self._slot_cache.popitem(last=False)
        return hit

    def apply_mask(self, seq_ids: Sequence[Hashable], logits: torch.Tensor,
                   neg_inf: float = float("-inf")) -> torch.Tensor:
        """In place: push every grammar-disallowed logit in ``logits``
        ``[len(seq_ids), vocab]`` to ``neg_inf``; broken rows are fully masked."""
        slots = self._slots(seq_ids)
        if int(logits.shape[0]) != int(slots.numel()):
            raise RuntimeError("bpdecode_b200: one logits row per seq_id")
        return pda_apply_mask_(logits, self.g, self._configs, neg_inf, slots=slots,
                               broken=self._broken)

    def commit(self, seq_ids: Sequence[Hashable], tokens: torch.Tensor) -> torch.Tensor:
        """Advance each named sequence by its sampled token. Returns int32
        status per sequence: 1, or ``-1`` if the token was off a valid path now
        or earlier (the config-set is then left unchanged; sticky until
        :meth:`reset`)."""
        slots = self._slots(seq_ids)
        B = int(slots.numel())
        tk = _tokens(tokens, B, self.device)
        status = torch.empty(B, dtype=torch.int32, device=self.device)
        L = _capi.lib()
        L.check(L.bpd_pda_advance(
            C.byref(self.g._struct()), self._configs.data_ptr(), slots.data_ptr(), B,
            tk.data_ptr(), int(tk.dtype == torch.int64), None,
            self._broken.view(torch.uint8).data_ptr(), status.data_ptr(), _stream(status)))
        return status

    def step_greedy(self, seq_ids: Sequence[Hashable], logits: torch.Tensor,
                    neg_inf: float = float("-inf"), chunks_per_row: int = 0) -> torch.Tensor:
        """NEW: ``apply_mask`` + ``logits.argmax(-1)`` + ``commit`` with the
        argmax fused into the masking pass. Masks ``logits`` in place, commits
        the first maximal token of every row and returns those tokens (int64);
        the per-row commit status is kept in ``last_status``."""
        slots, slot_ptr = self._slots_arg(seq_ids)
        B = int(slots.numel())
        if int(logits.shape[0]) != B:
            raise RuntimeError("bpdecode_b200: one logits row per seq_id")
        code = _check_logits(logits, self.g.vocab_size)
        tokens = torch.empty(B, dtype=torch.int64, device=self.device)
        status = torch.empty(B, dtype=torch.int32, device=self.device)
        mbuf, cap = self.g.mask_memo()
        ws = self.g.workspace(B)
        L = _capi.lib()
        L.check(L.bpd_pda_step_greedy(
            C.byref(self.g._struct()), logits.data_ptr(), code, logits.stride(0),
            self._configs.data_ptr(), slot_ptr, self._broken.view(torch.uint8).data_ptr(),
            B, mbuf.data_ptr(), cap, ws.data_ptr(), float(neg_inf), tokens.data_ptr(),
            status.data_ptr(), int(chunks_per_row), _stream(logits)))
        self.last_status = status
        return tokens

    def step_greedy_from(self, seq_ids: Sequence[Hashable], src: torch.Tensor,
                         src_rows: torch.Tensor | None = None, out: torch.Tensor | None = None,
                         neg_inf: float = float("-inf"), chunks_per_row: int = 0,
                         ) -> torch.Tensor:
        """NEW: :meth:`step_greedy` on an fp32 working copy of the rows without
        making the copy: row b reads ``src[src_rows[b]]`` (any float dtype;
        rows 0..B-1 when ``src_rows`` is None), the masked fp32 row goes to
        ``out[b]`` (None: nowhere), ``src`` is not modified."""
        return self._step_from_slots(self._slots(seq_ids), src, src_rows, out, neg_inf,
                                     chunks_per_row)

    def _step_from_slots(self, slots: torch.Tensor, src: torch.Tensor,
                         src_rows: torch.Tensor | None, out: torch.Tensor | None,
                         neg_inf: float = float("-inf"), chunks_per_row: int = 0,
                         ) -> torch.Tensor:
        """:meth:`step_greedy_from` on device slot indices (int64)."""
        from ..ops import _ptr, _source_args

        B = int(slots.numel())
        code, rows, out = _source_args(src, self.g.vocab_size, B, src_rows, out, self.device)
        tokens = torch.empty(B, dtype=torch.int64, device=self.device)
        status = torch.empty(B, dtype=torch.int32, device=self.device)
        mbuf, cap = self.g.mask_memo()
        ws = self.g.workspace(B)
        L = _capi.lib()
        L.check(L.bpd_pda_step_greedy_from(
            C.byref(self.g._struct()), src.data_ptr(), code, src.stride(0), _ptr(rows), _ptr(out),
            out.stride(0) if out is not None else 0, self._configs.data_ptr(), slots.data_ptr(),
            self._broken.view(torch.uint8).data_ptr(), B, mbuf.data_ptr(), cap, ws.data_ptr(),
            float(neg_inf), tokens.data_ptr(), status.data_ptr(), int(chunks_per_row),
            _stream(src)))
        self.last_status = status
        return tokens

    # --- queries ------------------------------------------------------
    def is_complete(self, seq_id: Hashable) -> bool:
        """True when the string so far is a full match (EOS is allowed)."""
        slot = self._slot_of[seq_id]
        if self.g.eos_id < 0:
            return False
        out = torch.empty(1, dtype=torch.uint8, device=self.device)
        st = torch.tensor([slot], dtype=torch.int64, device=self.device)
        L = _capi.lib()
        L.check(L.bpd_pda_is_complete(
            C.byref(self.g._struct()), self._configs.data_ptr(), st.data_ptr(),
            self._broken.view(torch.uint8).data_ptr(), 1, out.data_ptr(), _stream(out)))
        return bool(out.item())

    def is_broken(self, seq_id: Hashable) -> bool:
        return bool(self._broken[self._slot_of[seq_id]])


__all__ = [
    "PDA_CONFIG_FLAT", "PDA_MAX_CONFIGS", "PDA_MAX_DEPTH", "CFGConstraintBatch", "PdaTensors",
    "build_pda_tensors", "pda_advance_state", "pda_apply_mask_", "pda_compute_mask",
]
