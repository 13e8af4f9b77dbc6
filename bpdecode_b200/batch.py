"""Batched constraint state for continuous-batching serving.

Drop-in for bpdecode's ``batch.py`` (``src/bpdecode/batch.py``):
:class:`ConstraintBatch`, :class:`GrammarCache`, :class:`MaskCache` and the
``FREE`` / ``BROKEN`` sentinels keep their signatures and semantics. What
changes is underneath:

* the per-step kernels index the device-resident state pool through the slot
  tensor themselves, so ``apply_mask`` and ``commit`` are one launch each with
  no gather / scatter copies of the states;
* the slot tensor for a given ``seq_ids`` sequence is built once and reused
  until the batch membership changes (the reference rebuilds and uploads it
  from a Python list on every call, batch.py:171-174);
* :meth:`ConstraintBatch.step_greedy` fuses mask + argmax + commit;
* a batch may mix grammars (NEW): pass a list of :class:`FsaTensors` and
  ``add(seq_id, grammar=i)``; their states are concatenated into one global
  state space so a mixed batch is still one launch per step (the reference is
  single-grammar per batch, batch.py:16-18).
"""

from __future__ import annotations

from collections import OrderedDict
from collections.abc import Hashable, Sequence

import torch

from . import _capi
from .ops import (
    FsaTensors,
    _check_logits,
    _ptr,
    _require_cuda,
    _source_args,
    _stream,
    _upload,
    _tokens,
    apply_mask_,
)

FREE = -2  # slot holds no sequence
BROKEN = -1  # a committed token left the grammar-valid path


_BIT_SHIFTS: dict[torch.device, torch.Tensor] = {}


def _unpack_allow_row(words: torch.Tensor, vocab: int) -> torch.Tensor:
    """Token ids (int64, ascending) whose bit is set in one packed allow row
    (int32 storage of uint32 words, bit t of word t >> 5)."""
    shifts = _BIT_SHIFTS.get(words.device)
    if shifts is None:
        shifts = torch.arange(32, dtype=torch.int32, device=words.device)
        _BIT_SHIFTS[words.device] = shifts
    flags = (words.unsqueeze(1) >> shifts).bitwise_and_(1).reshape(-1)[:vocab]
    return flags.nonzero().reshape(-1)


class MaskCache:
    """Allow-sets of one dense grammar, per DFA state (API of batch.py:35-86).

    On this device path every state's allow-set is already resident as a
    packed bit row (``FsaTensors.allow_bits``), 32x smaller than the id
    list, and masking a batch is one kernel launch whatever the states. So
    this class keeps no copy of the masks: :meth:`apply` is that launch, and
    :meth:`allowed_ids` unpacks one state's row into token ids on demand,
    remembering the ``max_states`` most recently requested lists. States that
    :meth:`apply` masks with count as held (``len``) from the next query on;
    :meth:`apply` itself does not synchronise with the device.
    """

    def __init__(self, fsa: FsaTensors, max_states: int = 512) -> None:
        self._fsa = fsa
        self._max = max_states
        # state -> unpacked ids (None until asked for); dict order = recency
        self._allowed: dict[int, torch.Tensor | None] = {}
        self._pending: list[torch.Tensor] = []  # state tensors of apply() calls

    def _remember(self, state: int, ids: torch.Tensor | None) -> None:
        known = self._allowed.pop(state, None)
        self._allowed[state] = ids if ids is not None else known
        while len(self._allowed) > self._max:
            del self._allowed[next(iter(self._allowed))]

    def _settle(self) -> None:
        """Fold the states of earlier apply() calls into the recency order."""
        pending, self._pending = self._pending, []
        for st in pending:
            for s in torch.unique(st).tolist():
                self._remember(int(s), None)

    def allowed_ids(self, state: int) -> torch.Tensor:
        self._settle()
        ids = self._allowed.get(state)
        if ids is None:
            _, bits = self._fsa.dense_tables()
            if 0 <= state < self._fsa.num_states:
                ids = _unpack_allow_row(bits[state], self._fsa.vocab_size)
            else:
                ids = torch.zeros(0, dtype=torch.long, device=bits.device)
        self._remember(state, ids)
        return ids

    def __len__(self) -> int:
        self._settle()
        return len(self._allowed)

    def apply(
        self, states: torch.Tensor, logits: torch.Tensor, neg_inf: float = float("-inf")
    ) -> torch.Tensor:
        """In place: mask ``logits`` [n, vocab] given one state per row (one
        ``bpd_dense_apply_mask`` launch)."""
        apply_mask_(logits, self._fsa, states, neg_inf)
        self._pending.append(states.detach().reshape(-1))
        return logits


class GrammarCache:
    """Compiled grammars for one tokenizer and device, shared by every
    request that names the same pattern (API of batch.py:89-115).

    ``get`` compiles a pattern (a regex string or a compiled DFA) the first
    time it is asked for and returns the same :class:`FsaTensors` -- tables
    already on ``device`` -- every later time; the ``max_size`` most recently
    used grammars are kept.
    """

    def __init__(self, vocab: object, device: torch.device | str = "cpu", max_size: int = 128,
                 ) -> None:
        self._vocab = vocab
        self._device = torch.device(device)
        self._max = max_size
        self._cache: dict[Hashable, FsaTensors] = {}  # dict order = recency

    def get(self, pattern: object) -> FsaTensors:
        fsa = self._cache.pop(pattern, None)
        if fsa is None:
            fsa = FsaTensors.build(pattern, self._vocab).to(self._device)
        self._cache[pattern] = fsa
        while len(self._cache) > self._max:
            del self._cache[next(iter(self._cache))]
        return fsa

    def __len__(self) -> int:
        return len(self._cache)


class _Tables:
    """Device tables of the batch's grammars in one global state space."""

    def __init__(self, grammars: list[FsaTensors]) -> None:
        self.offsets: list[int] = []
        total = 0
        for g in grammars:
            self.offsets.append(total)
            total += g.num_states
        self.num_states = total
        self.vocab_size = grammars[0].vocab_size
        if any(g.vocab_size != self.vocab_size for g in grammars):
            raise ValueError("every grammar of a batch must share one vocabulary")
        tables = [g.dense_tables() for g in grammars]
        if len(grammars) == 1:
            self.tok_next, self.allow_bits = tables[0]
        else:
            self.tok_next = torch.cat([
                torch.where(tn >= 0, tn + off, tn) for (tn, _), off in zip(tables, self.offsets)])
            self.allow_bits = torch.cat([b for _, b in tables])
        self.starts = [g.start + off for g, off in zip(grammars, self.offsets)]
        self.accepting = frozenset(
            s + off for g, off in zip(grammars, self.offsets) for s in g.accepting)
        las = [g.lookahead for g in grammars]
        self.lookahead = None
        if all(la is not None for la in las):
            self.lookahead = las[0].contiguous() if len(las) == 1 else torch.cat(las)


class ConstraintBatch:
    """A fixed-capacity pool of grammar states (batch.py:118-226).

    Slots are stable for a sequence's lifetime (``add`` -> ``evict``); the caller
    passes an ordered list of sequence ids each step that lines up with its
    logit rows. ``seq_ids`` of one call must be distinct.
    """

    _SLOT_CACHE = 8

    def __init__(
        self,
        fsa: FsaTensors | Sequence[FsaTensors],
        capacity: int,
        device: torch.device | str | None = None,
        mask_cache: bool | MaskCache = False,
    ) -> None:
        grammars = list(fsa) if isinstance(fsa, (list, tuple)) else [fsa]
        if device is not None:
            grammars = [g.to(device) for g in grammars]
        self.grammars = grammars
        self.fsa = grammars[0]
        self.device = self.fsa.device
        _require_cuda(self.fsa.trans, "ConstraintBatch tables")
        self._t = _Tables(grammars)
        self.capacity = capacity
        self._state = torch.full((capacity,), FREE, dtype=torch.int32, device=self.device)
        # scratch of the fused steps (zero; the kernels leave it zero)
        self._scratch = torch.zeros(_capi.lib().bpd_step_scratch_bytes(max(capacity, 1)),
                                    dtype=torch.uint8, device=self.device)
        self._slot_of: dict[Hashable, int] = {}
        self._grammar_of: dict[Hashable, int] = {}
        self._free: list[int] = list(reversed(range(capacity)))
        self._slot_cache: OrderedDict[tuple, torch.Tensor] = OrderedDict()
        if mask_cache is True:
            if len(grammars) != 1:
                raise ValueError("mask_cache needs a single-grammar batch")
            mask_cache = MaskCache(self.fsa)
        self.cache: MaskCache | None = mask_cache or None

    def add_grammar(self, fsa: FsaTensors) -> int:
        """NEW: append a grammar to the batch and return its index for
        :meth:`add`. States of the grammars already present keep their
        global numbering (the new grammar's states are appended), so running
        sequences are unaffected; the merged tables are rebuilt once."""
        fsa = fsa.to(self.device)
        if fsa.vocab_size != self._t.vocab_size:
            raise ValueError("every grammar of a batch must share one vocabulary")
        self.grammars.append(fsa)
        self._t = _Tables(self.grammars)
        return len(self.grammars) - 1

    # --- lifecycle -------------------------------------------------------
    def add(self, seq_id: Hashable, grammar: int = 0) -> int:
        if seq_id in self._slot_of:
            raise KeyError(f"sequence {seq_id!r} already in the batch")
        if not self._free:
            raise RuntimeError("ConstraintBatch is at capacity")
        slot = self._free.pop()
        self._slot_of[seq_id] = slot
        self._grammar_of[seq_id] = grammar
        self._state[slot] = self._t.starts[grammar]
        self._slot_cache.clear()
        return slot

    def evict(self, seq_id: Hashable) -> None:
        slot = self._slot_of.pop(seq_id)
        self._grammar_of.pop(seq_id, None)
        self._state[slot] = FREE
        self._free.append(slot)
        self._slot_cache.clear()

    def reset(self, seq_id: Hashable) -> None:
        self._state[self._slot_of[seq_id]] = self._t.starts[self._grammar_of[seq_id]]

    def add_many(self, seq_ids: Sequence[Hashable], grammars: Sequence[int] | int = 0,
                 ) -> list[int]:
        """NEW: :meth:`add` of every id (grammar index per id, or one for
        all) with one device write for the whole group."""
        gs = [grammars] * len(seq_ids) if isinstance(grammars, int) else list(grammars)
        slots, starts = self._add_host(seq_ids, gs)
        if slots:
            idx = _upload(slots, torch.int64, self.device)
            val = _upload(starts, torch.int32, self.device)
            self._state.index_copy_(0, idx, val)
        return slots

    def evict_many(self, seq_ids: Sequence[Hashable]) -> None:
        """NEW: :meth:`evict` of every id with one device write."""
        slots = self._evict_host(seq_ids)
        if slots:
            idx = _upload(slots, torch.int64, self.device)
            self._state.index_fill_(0, idx, FREE)

    def _add_host(self, seq_ids: Sequence[Hashable], gs: Sequence[int],
                  ) -> tuple[list[int], list[int]]:
        """The bookkeeping of :meth:`add_many` (slots taken, grammars recorded)
        without the device write: returns the slots and the start state each
        must be given."""
        ids = set(seq_ids)
        if len(gs) != len(seq_ids) or len(ids) != len(seq_ids):
            raise ValueError("add_many: one grammar per id, ids distinct")
        if not self._slot_of.keys().isdisjoint(ids):
            raise KeyError("add_many: a sequence is already in the batch")
        if len(seq_ids) > len(self._free):
            raise RuntimeError("ConstraintBatch is at capacity")
        slots = [self._free.pop() for _ in seq_ids]
        for sid, slot, g in zip(seq_ids, slots, gs):
            self._slot_of[sid] = slot
            self._grammar_of[sid] = g
        self._slot_cache.clear()
        return slots, [self._t.starts[g] for g in gs]

    def _evict_host(self, seq_ids: Sequence[Hashable]) -> list[int]:
        """The bookkeeping of :meth:`evict_many` without the device write:
        returns the freed slots (their state must become FREE)."""
        slots = [self._slot_of.pop(s) for s in seq_ids]
        for s in seq_ids:
            self._grammar_of.pop(s, None)
        self._free.extend(slots)
        self._slot_cache.clear()
        return slots

    def reset_many(self, seq_ids: Sequence[Hashable]) -> None:
        """NEW: :meth:`reset` of every id in ``seq_ids`` as one device write on
        the current stream (no host synchronisation once the id list has been
        seen, as with the per-step calls)."""
        slots = self._slots(seq_ids)
        key = ("starts",) + (seq_ids if isinstance(seq_ids, tuple) else tuple(seq_ids))
        starts = self._slot_cache.get(key)
        if starts is None:
            starts = _upload([self._t.starts[self._grammar_of[s]] for s in key[1:]],
                             torch.int32, self.device)
            self._slot_cache[key] = starts
            if len(self._slot_cache) > self._SLOT_CACHE:
                self._slot_cache.popitem(last=False)
        self._state.index_copy_(0, slots, starts)

    # --- checkpoint / resume ------------------------------------------
    def state_dict(self) -> dict:
        """NEW: everything needed to resume the batch (host copies): the
        per-slot automaton states and the slot / grammar bookkeeping. The
        tables are not included -- restore into a batch built over the same
        grammars (``torch.save`` / ``torch.load`` handle the dict)."""
        return {"kind": "dense", "capacity": self.capacity,
                "num_grammars": len(self.grammars),
                "num_states": [g.num_states for g in self.grammars],
                "state": self._state.cpu().clone(),
                "slot_of": dict(self._slot_of), "grammar_of": dict(self._grammar_of),
                "free": list(self._free)}

    def load_state_dict(self, sd: dict) -> None:
        """NEW: restore what :meth:`state_dict` saved (same capacity and
        grammars), replacing every sequence of this batch."""
        if sd.get("kind") != "dense" or sd["capacity"] != self.capacity:
            raise ValueError("state_dict is not from a ConstraintBatch of this capacity")
        if sd["num_states"] != [g.num_states for g in self.grammars]:
            raise ValueError("state_dict was saved over different grammars")
        self._state.copy_(sd["state"].to(device=self.device, dtype=torch.int32))
        self._slot_of = dict(sd["slot_of"])
        self._grammar_of = dict(sd["grammar_of"])
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
        skip the slot load, one dependent load less per row)."""
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

    def apply_mask(
        self,
        seq_ids: Sequence[Hashable],
        logits: torch.Tensor,
        neg_inf: float = float("-inf"),
    ) -> torch.Tensor:
        """In place: push every grammar-disallowed logit in ``logits``
        ``[len(seq_ids), vocab]`` to ``neg_inf``, one row per ``seq_ids`` entry."""
        slots, slot_ptr = self._slots_arg(seq_ids)
        if self.cache is not None:
            self.cache.apply(self._state[slots], logits, neg_inf)
            return logits
        t = self._t
        B = int(slots.numel())
        if int(logits.shape[0]) != B:
            raise RuntimeError("bpdecode_b200: one logits row per seq_id")
        code = _check_logits(logits, t.vocab_size)
        L = _capi.lib()
        L.check(L.bpd_dense_apply_mask(
            logits.data_ptr(), code, logits.stride(0), B, t.vocab_size, self._state.data_ptr(),
            slot_ptr, t.allow_bits.data_ptr(), t.allow_bits.shape[1], t.num_states,
            float(neg_inf), _stream(logits)))
        return logits

    def apply_soft(
        self,
        seq_ids: Sequence[Hashable],
        logits: torch.Tensor,
        alpha: float = 1.0,
    ) -> torch.Tensor:
        """In place: add ``alpha * lookahead[state]`` per row (and mask, since
        disallowed entries are ``-inf``); every grammar needs a lookahead table
        (:meth:`FsaTensors.with_lookahead`)."""
        t = self._t
        if t.lookahead is None:
            raise ValueError("fsa has no lookahead table; build with dense + with_lookahead")
        slots = self._slots(seq_ids)
        B = int(slots.numel())
        code = _check_logits(logits, t.vocab_size)
        L = _capi.lib()
        L.check(L.bpd_soft_apply(
            logits.data_ptr(), code, logits.stride(0), B, t.vocab_size, self._state.data_ptr(),
            slots.data_ptr(), t.lookahead.data_ptr(), t.allow_bits.data_ptr(),
            t.allow_bits.shape[1], t.num_states, float(alpha), _stream(logits)))
        return logits

    def commit(self, seq_ids: Sequence[Hashable], tokens: torch.Tensor) -> torch.Tensor:
        """Advance each named sequence by the token it sampled. Returns the new
        state per sequence (``BROKEN`` if the token was off a valid path)."""
        slots = self._slots(seq_ids)
        B = int(slots.numel())
        tk = _tokens(tokens, B, self.device)
        nxt = torch.empty(B, dtype=torch.int32, device=self.device)
        t = self._t
        L = _capi.lib()
        L.check(L.bpd_dense_advance(
            self._state.data_ptr(), slots.data_ptr(), B, tk.data_ptr(),
            int(tk.dtype == torch.int64), t.tok_next.data_ptr(), t.num_states, t.vocab_size,
            nxt.data_ptr(), 1, _stream(nxt)))
        return nxt

    def step_greedy(
        self,
        seq_ids: Sequence[Hashable],
        logits: torch.Tensor,
        neg_inf: float = float("-inf"),
        chunks_per_row: int = 0,
    ) -> torch.Tensor:
        """NEW: ``apply_mask`` + ``logits.argmax(-1)`` + ``commit`` in one
        launch. Masks ``logits`` in place and returns the chosen tokens (int64,
        torch.argmax semantics: first maximal index)."""
        slots, slot_ptr = self._slots_arg(seq_ids)
        B = int(slots.numel())
        if int(logits.shape[0]) != B:
            raise RuntimeError("bpdecode_b200: one logits row per seq_id")
        t = self._t
        code = _check_logits(logits, t.vocab_size)
        tokens = torch.empty(B, dtype=torch.int64, device=self.device)
        L = _capi.lib()
        L.check(L.bpd_dense_step_greedy(
            logits.data_ptr(), code, logits.stride(0), B, t.vocab_size, self._state.data_ptr(),
            slot_ptr, t.allow_bits.data_ptr(), t.allow_bits.shape[1],
            t.tok_next.data_ptr(), t.num_states, float(neg_inf), tokens.data_ptr(), None,
            int(chunks_per_row), self._scratch.data_ptr(), _stream(logits)))
        return tokens

    def soft_step_greedy(
        self,
        seq_ids: Sequence[Hashable],
        logits: torch.Tensor,
        alpha: float = 1.0,
        chunks_per_row: int = 0,
    ) -> torch.Tensor:
        """NEW: ``apply_soft`` + ``logits.argmax(-1)`` + ``commit`` in one
        launch. Biases ``logits`` in place and returns the chosen tokens
        (int64, first maximal index)."""
        t = self._t
        if t.lookahead is None:
            raise ValueError("fsa has no lookahead table; build with dense + with_lookahead")
        slots, slot_ptr = self._slots_arg(seq_ids)
        B = int(slots.numel())
        if int(logits.shape[0]) != B:
            raise RuntimeError("bpdecode_b200: one logits row per seq_id")
        code = _check_logits(logits, t.vocab_size)
        tokens = torch.empty(B, dtype=torch.int64, device=self.device)
        L = _capi.lib()
        L.check(L.bpd_soft_step_greedy(
            logits.data_ptr(), code, logits.stride(0), B, t.vocab_size, self._state.data_ptr(),
            slot_ptr, t.lookahead.data_ptr(), t.allow_bits.data_ptr(),
            t.allow_bits.shape[1], t.tok_next.data_ptr(), t.num_states, float(alpha),
            tokens.data_ptr(), None, int(chunks_per_row), self._scratch.data_ptr(),
            _stream(logits)))
        return tokens

    def step_greedy_from(
        self,
        seq_ids: Sequence[Hashable],
        src: torch.Tensor,
        src_rows: torch.Tensor | None = None,
        out: torch.Tensor | None = None,
        neg_inf: float = float("-inf"),
        chunks_per_row: int = 0,
    ) -> torch.Tensor:
        """NEW: :meth:`step_greedy` on an fp32 working copy of the rows
        without making the copy: row b reads ``src[src_rows[b]]`` (any float
        dtype; rows 0..B-1 when ``src_rows`` is None), the masked fp32 row goes
        to ``out[b]`` (None: nowhere), ``src`` is not modified. Returns the
        tokens (int64)."""
        slots, slot_ptr = self._slots_arg(seq_ids)
        B = int(slots.numel())
        t = self._t
        code, rows, out = _source_args(src, t.vocab_size, B, src_rows, out, self.device)
        tokens = torch.empty(B, dtype=torch.int64, device=self.device)
        L = _capi.lib()
        L.check(L.bpd_dense_step_greedy_from(
            src.data_ptr(), code, src.stride(0), _ptr(rows), _ptr(out),
            out.stride(0) if out is not None else 0, B, t.vocab_size, self._state.data_ptr(),
            slot_ptr, t.allow_bits.data_ptr(), t.allow_bits.shape[1],
            t.tok_next.data_ptr(), t.num_states, float(neg_inf), tokens.data_ptr(), None,
            int(chunks_per_row), self._scratch.data_ptr(), _stream(src)))
        return tokens

    def soft_step_greedy_from(
        self,
        seq_ids: Sequence[Hashable],
        src: torch.Tensor,
        src_rows: torch.Tensor | None = None,
        out: torch.Tensor | None = None,
        alpha: float = 1.0,
        chunks_per_row: int = 0,
    ) -> torch.Tensor:
        """NEW: :meth:`soft_step_greedy` on an fp32 working copy of the rows
        without making the copy (the contract of :meth:`step_greedy_from`)."""
        return self._soft_step_from_slots(self._slots(seq_ids), src, src_rows, out, alpha,
                                          chunks_per_row)

    def _soft_step_from_slots(self, slots: torch.Tensor, src: torch.Tensor,
                              src_rows: torch.Tensor | None, out: torch.Tensor | None,
                              alpha: float, chunks_per_row: int = 0) -> torch.Tensor:
        """:meth:`soft_step_greedy_from` on device slot indices (int64)."""
        t = self._t
        if t.lookahead is None:
            raise ValueError("fsa has no lookahead table; build with dense + with_lookahead")
        B = int(slots.numel())
        code, rows, out = _source_args(src, t.vocab_size, B, src_rows, out, self.device)
        tokens = torch.empty(B, dtype=torch.int64, device=self.device)
        L = _capi.lib()
        L.check(L.bpd_soft_step_greedy_from(
            src.data_ptr(), code, src.stride(0), _ptr(rows), _ptr(out),
            out.stride(0) if out is not None else 0, B, t.vocab_size, self._state.data_ptr(),
            slots.data_ptr(), t.lookahead.data_ptr(), t.allow_bits.data_ptr(),
            t.allow_bits.shape[1], t.tok_next.data_ptr(), t.num_states, float(alpha),
            tokens.data_ptr(), None, int(chunks_per_row), self._scratch.data_ptr(),
            _stream(src)))
        return tokens

    # --- queries ------------------------------------------------------
    def state_of(self, seq_id: Hashable) -> int:
        return int(self._state[self._slot_of[seq_id]])

    def is_complete(self, seq_id: Hashable) -> bool:
        """True when the string so far is a full match (EOS is allowed)."""
        return self.state_of(seq_id) in self._t.accepting

    def is_broken(self, seq_id: Hashable) -> bool:
        return self.state_of(seq_id) == BROKEN


__all__ = ["BROKEN", "FREE", "ConstraintBatch", "GrammarCache", "MaskCache"]
