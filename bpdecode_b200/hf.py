"""Hugging Face ``LogitsProcessor`` adapters over the B200 device path.

Drop-in for bpdecode's ``hf.py``: ``RegexLogitsProcessor`` (a regex, through
:class:`~bpdecode_b200.batch.ConstraintBatch`) and ``GrammarLogitsProcessor``
(a context-free grammar or JSON Schema, through
:class:`~bpdecode_b200.grammar.device.CFGConstraintBatch`), same constructor
arguments and calling convention (``lp(input_ids, scores)`` each step,
``reset()``, ``is_complete(row)``). Greedy and sampling decoding work; beam
search reorders rows and is not supported.

What differs: half-precision scores are masked in place -- the kernels read
bf16 / fp16, compute in fp32 and round once, which is what the reference gets
by upcasting to an fp32 copy and copying back (hf.py:106-113, 253-259) without
the two extra passes. Grammar compilation (GBNF / JSON Schema / regex) is
bpdecode's front-end, used as is; precompiled tables
(:class:`~bpdecode_b200.ops.FsaTensors`,
:class:`~bpdecode_b200.grammar.device.PdaTensors`) are accepted directly.
Only the device backend exists: ``backend="cpu"`` (the reference's per-row
Python oracle) is not part of this package.
"""

from __future__ import annotations

import torch

from .batch import ConstraintBatch
from .grammar.device import CFGConstraintBatch, PdaTensors, build_pda_tensors
from .ops import FsaTensors
from .tokenizer import as_vocabulary


class RegexLogitsProcessor:
    """Constrain generation to ``pattern`` (hf.py:38-119). One instance per
    ``generate`` call. With ``soft_k`` the k-step soft-lookahead bias replaces
    hard masking (``alpha`` scales it; ``alpha=0`` is plain masking)."""

    def __init__(
        self,
        pattern: object,
        tokenizer: object,
        *,
        device: torch.device | str = "cuda",
        neg_inf: float = float("-inf"),
        soft_k: int | None = None,
        alpha: float = 1.0,
    ) -> None:
        if isinstance(pattern, FsaTensors):
            fsa = pattern
        elif isinstance(pattern, dict):
            fsa = FsaTensors.from_arrays(pattern, as_vocabulary(tokenizer))
        else:
            fsa = FsaTensors.build(pattern, as_vocabulary(tokenizer))
        self._soft = soft_k is not None
        self._alpha = alpha
        fsa = fsa.to(device)
        if self._soft:
            fsa = fsa.with_lookahead(soft_k)
        self._fsa: FsaTensors = fsa
        self._neg_inf = neg_inf
        self._batch: ConstraintBatch | None = None
        self._rows: list[int] = []

    def reset(self) -> None:
        """Forget accumulated state so the processor can be reused."""
        self._batch = None
        self._rows = []

    def __call__(self, input_ids: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
        n_rows = scores.shape[0]
        if self._batch is None:
            self._batch = ConstraintBatch(self._fsa, capacity=n_rows, device=scores.device)
            self._rows = list(range(n_rows))
            for r in self._rows:
                self._batch.add(r)
        else:
            if n_rows != len(self._rows):
                raise RuntimeError(
                    "RegexLogitsProcessor: row count changed between steps "
                    "(beam search is not supported); call reset() per generation")
            self._batch.commit(self._rows, input_ids[:, -1])
        v = self._fsa.vocab_size
        # a model may have more logit columns than real tokens (padded lm_head);
        # those extras can never be valid
        if scores.shape[1] > v:
            scores[:, v:] = self._neg_inf
        view = scores[:, :v]
        if self._soft:
            self._batch.apply_soft(self._rows, view, self._alpha)
        else:
            self._batch.apply_mask(self._rows, view, self._neg_inf)
        return scores

    def is_complete(self, row: int = 0) -> bool:
        """True when row ``row`` has reached an accepting state (EOS allowed)."""
        assert self._batch is not None, "call the processor at least once first"
        return self._batch.is_complete(self._rows[row])


class GrammarLogitsProcessor:
    """Constrain generation to a context-free grammar (hf.py:121-264), on the
    device PDA kernels. ``grammar`` is GBNF source or a bpdecode ``Grammar``
    (compiled with bpdecode's front-end), or a precompiled :class:`PdaTensors`.
    """

    def __init__(
        self,
        grammar: object,
        tokenizer: object,
        *,
        root: str = "root",
        neg_inf: float = float("-inf"),
        device: torch.device | str = "cuda",
        backend: str = "auto",
    ) -> None:
        self._device = torch.device(device)
        if backend == "auto":
            backend = "cpu" if self._device.type == "cpu" else "device"
        if backend not in ("cpu", "device"):
            raise ValueError(f"backend must be 'auto', 'cpu' or 'device', got {backend!r}")
        if backend == "cpu":
            raise ValueError(
                "bpdecode_b200 implements the device backend only; pass device='cuda' (the "
                "per-row CPU backend is bpdecode's own GrammarLogitsProcessor)")
        self._backend = backend
        self._vocab = as_vocabulary(tokenizer)
        self._neg_inf = neg_inf
        if isinstance(grammar, PdaTensors):
            self._pda_tensors = grammar.to(self._device)
        else:
            try:
                from bpdecode.grammar.gbnf import parse_gbnf  # type: ignore
                from bpdecode.grammar.ir import Grammar  # type: ignore
                from bpdecode.grammar.pda import CompiledGrammar  # type: ignore
            except ImportError as exc:
                raise ImportError(
                    "compiling GBNF needs bpdecode's grammar front-end; pass PdaTensors "
                    "instead") from exc
            g = grammar if isinstance(grammar, Grammar) else parse_gbnf(grammar, root)
            self._pda_tensors = build_pda_tensors(CompiledGrammar.build(g), self._vocab,
                                                  self._device)
        self._batch: CFGConstraintBatch | None = None
        self._rows: list[int] = []

    @classmethod
    def from_json_schema(cls, schema: object, tokenizer: object, **kw: object,
                         ) -> GrammarLogitsProcessor:
        try:
            from bpdecode.grammar.json_schema import json_schema_to_grammar  # type: ignore
        except ImportError as exc:
            raise ImportError("JSON Schema compilation needs bpdecode's grammar front-end"
                              ) from exc
        return cls(json_schema_to_grammar(schema), tokenizer, **kw)  # type: ignore[arg-type]

    @property
    def backend(self) -> str:
        """The resolved backend (always ``"device"`` here)."""
        return self._backend

    def reset(self) -> None:
        self._batch = None
        self._rows = []

    def __call__(self, input_ids: torch.Tensor, scores: torch.Tensor) -> torch.Tensor:
        n_rows = scores.shape[0]
        if self._batch is None:
            self._batch = CFGConstraintBatch(self._pda_tensors, capacity=n_rows,
                                             device=scores.device)
            self._rows = list(range(n_rows))
            for r in self._rows:
                self._batch.add(r)
        else:
            if n_rows != len(self._rows):
                raise RuntimeError(
                    "GrammarLogitsProcessor: row count changed (beam search "
                    "unsupported); call reset() per generation")
            self._batch.commit(self._rows, input_ids[:, -1])
        v = self._pda_tensors.vocab_size
        if scores.shape[1] > v:
            scores[:, v:] = self._neg_inf
        self._batch.apply_mask(self._rows, scores[:, :v], self._neg_inf)
        return scores

    def is_complete(self, row: int = 0) -> bool:
        return self._batch is not None and self._batch.is_complete(self._rows[row])


__all__ = ["GrammarLogitsProcessor", "RegexLogitsProcessor"]
