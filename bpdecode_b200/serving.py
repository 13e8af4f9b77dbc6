"""Continuous batching over both grammar paths (the whole-box serving loop).

One :class:`MixedServingLoop` owns the rows of one GPU: each row holds a
request constrained by a regex or a non-recursive JSON Schema (dense DFAs,
one :class:`~bpdecode_b200.batch.ConstraintBatch` over all of them, scored
with the soft-lookahead bias on an fp32 working copy of the row's logits, as
bpdecode's HF processor upcasts, hf.py:106-113) or by a recursive grammar
(the PDA path, one :class:`~bpdecode_b200.grammar.device.CFGConstraintBatch`).
A step takes the ``[rows, V]`` model logits, runs the fused soft step on the
dense rows and the fused PDA step on the grammar rows (greedy; both read the
rows of the model's logits straight into fp32 working values -- the same
values an fp32 copy would hold -- and materialise no copy), then retires a
fraction of the requests and admits new ones in their rows -- the eviction
and re-add pattern of a continuous-batching server. Rows never move between
GPUs; several loops (one process per GPU) shard requests with no
communication.

The request mix, the eviction fraction and every random choice come from a
seed, so two loops built alike make identical decisions; ``fused=False``
runs the same loop through the unfused drop-in calls on an fp32 copy
(apply_soft / apply_mask + argmax + commit), the reference's sequence.
"""

from __future__ import annotations

from collections.abc import Sequence

import numpy as np
import torch

from .batch import FREE, ConstraintBatch
from .grammar.device import CFGConstraintBatch, PdaTensors
from .ops import FsaTensors


class MixedServingLoop:
    """Rows ``0..rows-1`` of one device; see the module docstring.

    ``dense`` are the dense grammars (with lookahead tables when ``alpha`` is
    used), ``pda`` the recursive grammar; ``mix`` gives the probabilities of
    (a dense grammar chosen uniformly from ``dense[:n_regex]``, the dense
    grammar ``dense[n_regex]`` when present, the PDA grammar).

    Host work per step is kept to one host-to-device copy: the turnover does
    the batches' slot bookkeeping on the host and stages, in one pinned
    buffer, the device writes of the retired and admitted requests together
    with the next step's row and slot indices."""

    def __init__(
        self,
        rows: int,
        dense: Sequence[FsaTensors],
        pda: PdaTensors,
        *,
        n_regex: int,
        mix: tuple[float, float, float] = (0.5, 0.3, 0.2),
        evict_fraction: float = 0.1,
        alpha: float = 1.0,
        seed: int = 0,
        fused: bool = True,
    ) -> None:
        self.rows = rows
        self.n_regex = n_regex
        self.mix = mix
        self.evict_fraction = evict_fraction
        self.alpha = alpha
        self.fused = fused
        self.rng = np.random.Generator(np.random.PCG64(seed))
        self.dense = ConstraintBatch(list(dense), capacity=rows)
        self.device = self.dense.device
        self.pda = CFGConstraintBatch(pda, capacity=rows, device=self.device)
        self.kind = np.zeros(rows, np.int8)  # 0 dense, 1 pda
        self.req = np.zeros(rows, np.int64)  # request id held by each row
        self.slot = np.zeros(rows, np.int64)  # its slot in the row's batch
        self._next_req = 0
        self._step_args: tuple | None = None
        self._admit(np.arange(rows), [])

    # --- request admission ---------------------------------------------
    def _admit(self, rows: np.ndarray, freed_dense: list[int]) -> None:
        """New requests in ``rows`` (kind and dense grammar drawn from the
        mix); ``freed_dense`` are the dense slots the retired requests gave
        back. Writes the device state of every changed slot and the next
        step's indices with one copy."""
        n = len(rows)
        u = self.rng.random(n)
        regex = self.rng.integers(0, self.n_regex, n)
        has_schema = len(self.dense.grammars) > self.n_regex
        schema = (u >= self.mix[0]) & (u < self.mix[0] + self.mix[1]) & has_schema
        kind = np.where((u < self.mix[0]) | schema, 0, 1).astype(np.int8)
        grammar = np.where(schema, self.n_regex, regex)
        ids = np.arange(self._next_req, self._next_req + n, dtype=np.int64)
        self._next_req += n
        self.kind[rows] = kind
        self.req[rows] = ids
        d = kind == 0
        d_slots, starts = self.dense._add_host(ids[d].tolist(), grammar[d].tolist())
        p_slots = self.pda._add_host(ids[~d].tolist())
        self.slot[rows[d]] = d_slots
        self.slot[rows[~d]] = p_slots
        # dense slot states: a freed slot that no new request took is FREE
        new_state = dict.fromkeys(freed_dense, FREE)
        new_state.update(zip(d_slots, starts))
        self._stage(np.fromiter(new_state.keys(), np.int64, len(new_state)),
                    np.fromiter(new_state.values(), np.int64, len(new_state)),
                    np.asarray(p_slots, np.int64))

    def _stage(self, dense_slots: np.ndarray, dense_states: np.ndarray,
               pda_slots: np.ndarray) -> None:
        d_rows = np.flatnonzero(self.kind == 0)
        p_rows = np.flatnonzero(self.kind == 1)
        # int32 states packed two per int64 word (viewed back on the device)
        st32 = np.zeros(2 * ((len(dense_states) + 1) // 2), np.int32)
        st32[:len(dense_states)] = dense_states
        parts = [dense_slots, st32.view(np.int64), pda_slots, d_rows, self.slot[d_rows], p_rows,
                 self.slot[p_rows]]
        host = torch.from_numpy(np.concatenate(parts).astype(np.int64, copy=False))
        dev = host.pin_memory().to(self.device, non_blocking=True)
        views, o = [], 0
        for x in parts:
            views.append(dev[o:o + len(x)])
            o += len(x)
        u_slots, u_states, p_new, d_idx, d_sl, p_idx, p_sl = views
        if len(u_slots):
            states = u_states.view(torch.int32)[:len(dense_states)]
            self.dense._state.index_copy_(0, u_slots, states)
        if len(p_new):
            self.pda._init_slots(p_new)
        self._step_args = (d_rows, d_idx, d_sl, p_rows, p_idx, p_sl)

    def turnover(self) -> list[int]:
        """Retire a random ``evict_fraction`` of the requests and admit new
        ones in their rows; returns the rows that changed."""
        n = int(round(self.rows * self.evict_fraction))
        rows = np.sort(self.rng.choice(self.rows, n, replace=False))
        old, kind = self.req[rows], self.kind[rows]
        freed = self.dense._evict_host(old[kind == 0].tolist())
        self.pda.evict_many(old[kind == 1].tolist())
        self._admit(rows, freed)
        return rows.tolist()

    # --- one step --------------------------------------------------------
    def step(self, logits: torch.Tensor) -> torch.Tensor:
        """Greedy tokens (int64 ``[rows]``) for one step of ``logits``
        (``[rows, V]``, any float dtype; not modified)."""
        d_rows, d_idx, d_sl, p_rows, p_idx, p_sl = self._step_args
        tokens = torch.empty(self.rows, dtype=torch.int64, device=self.device)
        if len(d_rows):
            if self.fused:
                tok = self.dense._soft_step_from_slots(d_sl, logits, d_idx, None, self.alpha)
            else:
                d_ids = self.req[d_rows].tolist()
                work = logits.index_select(0, d_idx).float()
                self.dense.apply_soft(d_ids, work, self.alpha)
                tok = work.argmax(-1)
                self.dense.commit(d_ids, tok)
            tokens.index_copy_(0, d_idx, tok)
        if len(p_rows):
            if self.fused:
                tok = self.pda._step_from_slots(p_sl, logits, p_idx, None)
            else:
                p_ids = self.req[p_rows].tolist()
                work = logits.index_select(0, p_idx).float()
                self.pda.apply_mask(p_ids, work)
                tok = work.argmax(-1)
                self.pda.commit(p_ids, tok)
            tokens.index_copy_(0, p_idx, tok)
        return tokens

    def states(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(dense state pool, PDA config pool, PDA broken flags) -- for checks."""
        return self.dense._state, self.pda._configs, self.pda._broken


__all__ = ["MixedServingLoop"]
