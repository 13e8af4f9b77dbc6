"""vLLM logits-processor adapters over the B200 device path (vllm.py:1-184).

Mirrors bpdecode's module: :class:`RegexLogitsProcessor` is the
request-level processor (vLLM's 2-argument ``(past_token_ids, logits)``
form, one instance per request), :class:`RegexLogitsProcessorFactory` hands
out processors sharing one compiled grammar, and :class:`BatchConstraintState`
is the state machine behind a V1 batch-level processor (``add`` / ``remove``
/ ``move`` / ``advance`` events, then :meth:`~BatchConstraintState.mask` on the
``[num_rows, vocab]`` logits). Like the reference this module never imports
vLLM.

What differs: everything runs on the CUDA kernels (``device="cuda"`` is the
default; there is no CPU path), a batch may mix grammars -- a new pattern is
appended to the running batch (:meth:`ConstraintBatch.add_grammar`) instead
of raising -- ``move`` re-points a slot without touching the device, a whole
step of sampled tokens commits in one launch (:meth:`advance_batch`), and
``mask`` works in place when the managed rows are the leading rows of the
logits. A pattern may be regex source (compiled with bpdecode's front-end
through :class:`GrammarCache`), precompiled :class:`FsaTensors`, or the
dict of DFA arrays :meth:`FsaTensors.from_arrays` takes.
"""

from __future__ import annotations

from collections.abc import Hashable, Sequence

import torch

from .batch import ConstraintBatch, GrammarCache
from .ops import FsaTensors
from .tokenizer import as_vocabulary


def _resolve(pattern: object, vocab: object, cache: GrammarCache | None,
             device: torch.device) -> FsaTensors:
    if isinstance(pattern, FsaTensors):
        return pattern.to(device)
    if isinstance(pattern, dict):
        return FsaTensors.from_arrays(pattern, vocab).to(device)
    if cache is not None:
        return cache.get(pattern)  # type: ignore[arg-type]
    return FsaTensors.build(pattern, vocab).to(device)


def _key(pattern: object) -> Hashable:
    return pattern if isinstance(pattern, str) else id(pattern)


def _mask_padding(logits: torch.Tensor, vocab_size: int, neg_inf: float) -> torch.Tensor:
    # a model may have more logit columns than real tokens (padded lm_head);
    # those can never be valid
    if logits.shape[-1] > vocab_size:
        logits[..., vocab_size:] = neg_inf
    return logits[..., :vocab_size]


class RegexLogitsProcessor:
    """One per request; constrains the generated continuation to ``pattern``
    (vllm.py:48-82)."""

    def __init__(
        self,
        pattern: object,
        tokenizer: object,
        *,
        device: torch.device | str = "cuda",
        neg_inf: float = float("-inf"),
        _fsa: FsaTensors | None = None,
    ) -> None:
        dev = torch.device(device)
        fsa = _fsa if _fsa is not None else _resolve(pattern, as_vocabulary(tokenizer), None, dev)
        self._batch = ConstraintBatch(fsa, capacity=1, device=dev)
        self._batch.add(0)
        self._neg_inf = neg_inf
        self._pos = 0

    def __call__(self, past_token_ids: Sequence[int], logits: torch.Tensor) -> torch.Tensor:
        n = len(past_token_ids)
        if n < self._pos:  # the sequence was rewound: replay it
            self._batch.reset(0)
            self._pos = 0
        if self._pos < n:
            dev = self._batch.device
            for tok in past_token_ids[self._pos:]:
                self._batch.commit([0], torch.tensor([int(tok)], dtype=torch.int32, device=dev))
            self._pos = n
        row = _mask_padding(logits.unsqueeze(0), self._batch.fsa.vocab_size, self._neg_inf)
        self._batch.apply_mask([0], row, self._neg_inf)
        return logits

    @property
    def is_complete(self) -> bool:
        return self._batch.is_complete(0)


class RegexLogitsProcessorFactory:
    """Compile each distinct pattern once; hand out fresh per-request
    processors (vllm.py:84-97)."""

    def __init__(self, tokenizer: object, *, device: torch.device | str = "cuda") -> None:
        self._vocab = as_vocabulary(tokenizer)
        self._device = torch.device(device)
        self._cache = GrammarCache(self._vocab, device=self._device)

    def make(self, pattern: object) -> RegexLogitsProcessor:
        fsa = _resolve(pattern, self._vocab, self._cache, self._device)
        return RegexLogitsProcessor(pattern, None, device=self._device, _fsa=fsa)


class BatchConstraintState:
    """The state machine behind a vLLM V1 batch-level ``LogitsProcessor``
    (vllm.py:100-184): vLLM's persistent batch addresses each running request
    by a row index that is reused and occasionally reshuffled; feed those
    events in and call :meth:`mask` on the ``[num_rows, vocab]`` logits.
    Rows may use different patterns."""

    def __init__(
        self,
        tokenizer: object,
        *,
        device: torch.device | str = "cuda",
        mask_cache: bool = False,
        capacity: int = 256,
    ) -> None:
        self._vocab = as_vocabulary(tokenizer)
        self._device = torch.device(device)
        self._grammars = GrammarCache(self._vocab, device=self._device)
        self._capacity = capacity
        self._batch: ConstraintBatch | None = None
        self._index: dict[Hashable, int] = {}
        self._pos: dict[int, int] = {}
        del mask_cache  # accepted for the reference's signature; the kernels need no cache

    def _grammar(self, pattern: object) -> int:
        key = _key(pattern)
        idx = self._index.get(key)
        if idx is not None:
            return idx
        fsa = _resolve(pattern, self._vocab, self._grammars, self._device)
        if self._batch is None:
            self._batch = ConstraintBatch(fsa, capacity=self._capacity, device=self._device)
            idx = 0
        else:
            idx = self._batch.add_grammar(fsa)
        self._index[key] = idx
        return idx

    def add(self, row: int, pattern: object) -> None:
        g = self._grammar(pattern)
        assert self._batch is not None
        if row in self._pos:
            self._batch.evict(row)
        self._batch.add(row, grammar=g)
        self._pos[row] = 0

    def remove(self, row: int) -> None:
        if row in self._pos:
            self._batch.evict(row)  # type: ignore[union-attr]
            del self._pos[row]

    def move(self, src: int, dst: int) -> None:
        """Row ``src`` is now row ``dst`` (whatever ``dst`` held is gone)."""
        if src not in self._pos or src == dst:
            return
        b = self._batch
        assert b is not None
        if dst in self._pos:
            self.remove(dst)
        b._slot_of[dst] = b._slot_of.pop(src)
        b._grammar_of[dst] = b._grammar_of.pop(src)
        b._slot_cache.clear()
        self._pos[dst] = self._pos.pop(src)

    def advance(self, row: int, generated_ids: Sequence[int]) -> None:
        """``generated_ids`` is the request's full output-token list so far."""
        if row not in self._pos or self._batch is None:
            return
        for tok in generated_ids[self._pos[row]:]:
            self._batch.commit([row], torch.tensor([int(tok)], dtype=torch.int32,
                                                   device=self._device))
        self._pos[row] = len(generated_ids)

    def advance_batch(self, rows: Sequence[int], token_ids: torch.Tensor) -> None:
        """NEW: commit one freshly sampled token per row (``token_ids``
        aligned with ``rows``, on any device) in one launch."""
        rows = [r for r in rows if r in self._pos]
        if not rows or self._batch is None:
            return
        self._batch.commit(rows, token_ids.to(self._device))
        for r in rows:
            self._pos[r] += 1

    def mask(self, logits: torch.Tensor, neg_inf: float = float("-inf")) -> torch.Tensor:
        """Mask the rows this state manages, in place. ``logits`` is
        ``[num_rows, vocab]`` indexed by row; rows not managed are untouched."""
        if not self._pos or self._batch is None:
            return logits
        rows = sorted(self._pos)
        V = self._batch.fsa.vocab_size
        if rows == list(range(len(rows))):
            view = _mask_padding(logits[: len(rows)], V, neg_inf)
            self._batch.apply_mask(rows, view, neg_inf)
            return logits
        idx = torch.tensor(rows, device=logits.device)
        sub = logits.index_select(0, idx)
        self._batch.apply_mask(rows, _mask_padding(sub, V, neg_inf), neg_inf)
        logits[idx] = sub
        return logits

    def is_complete(self, row: int) -> bool:
        return self._batch is not None and row in self._pos and self._batch.is_complete(row)


__all__ = ["BatchConstraintState", "RegexLogitsProcessor", "RegexLogitsProcessorFactory"]
