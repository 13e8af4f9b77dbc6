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

import ctypes as C

from . import _capi
from .batch import FREE, ConstraintBatch
from .grammar.device import CFGConstraintBatch, PdaTensors
from .ops import FsaTensors, _source_args, _stream


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
        if logits.dim() != 2 or int(logits.shape[0]) < self.rows:
            raise RuntimeError(f"bpdecode_b200: logits must be [>= {self.rows}, vocab], got "
                               f"{tuple(logits.shape)}")
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


class DeviceServingLoop:
    """The serving loop of :class:`MixedServingLoop` with its request
    turnover on the device, so that a whole step -- the fused soft step of
    the dense rows, the fused PDA step of the grammar rows, the tokens put
    back in row order, the turnover -- is a fixed sequence of launches that
    can be captured once and replayed from a CUDA graph (:meth:`graph`).

    Row r holds one request and always uses slot r of the dense state pool
    and of the PDA config pool. Device tensors describe the mix: ``kind``
    (int32, 0 dense / 1 PDA), the ascending row lists ``dense_rows`` /
    ``pda_rows`` (int64) and their lengths ``counts`` (int32 [2]), which the
    steps read on the device (``bpd_*_step_greedy_from_n``). Every
    :meth:`turnover` retires each row's request with probability
    ``evict_fraction`` (a seeded counter-based hash of (seed, step, row):
    10 % of the rows per step on average, where :class:`MixedServingLoop`
    retires exactly 10 %) and admits a new one drawn from ``mix`` in its row
    (``bpd_serving_turnover``); ``retired`` (uint8) marks the rows that turned
    over. The host never reads the mix.

    With ``overlap`` (the default) the PDA rows' mask pipeline and step run
    on a second stream, forked from and joined back into the caller's stream
    within :meth:`step`, beside the dense rows' soft step: they read and
    write disjoint rows, states and outputs, and the PDA pipeline's short
    latency-bound launches then hide under the dense step. The second
    stream has the higher priority (config 5 on one box: 138.0 us per step,
    against 143.9 with equal priorities and 150.1 on one stream). A graph
    captured by :meth:`graph` holds both branches.

    :meth:`step` returns ``tokens``, a buffer the next step overwrites.
    """

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
        overlap: bool = True,
    ) -> None:
        self.rows = rows
        self.overlap = overlap
        self.n_regex = n_regex
        self.mix = mix
        self.evict_fraction = evict_fraction
        self.alpha = alpha
        self.seed = seed
        self.dense = ConstraintBatch(list(dense), capacity=rows)
        if self.dense._t.lookahead is None:
            raise ValueError("DeviceServingLoop: every dense grammar needs a lookahead table")
        dev = self.device = self.dense.device
        self.pda = CFGConstraintBatch(pda, capacity=rows, device=dev)
        self.schema = n_regex if len(self.dense.grammars) > n_regex else -1
        i32, i64 = torch.int32, torch.int64
        self.kind = torch.ones(rows, dtype=i32, device=dev)
        self.dense_rows = torch.zeros(rows, dtype=i64, device=dev)
        self.pda_rows = torch.zeros(rows, dtype=i64, device=dev)
        self.counts = torch.zeros(2, dtype=i32, device=dev)
        self.retired = torch.zeros(rows, dtype=torch.uint8, device=dev)
        self.step_counter = torch.zeros(1, dtype=i64, device=dev)
        self.tokens = torch.zeros(rows, dtype=i64, device=dev)
        self._dtok = torch.zeros(rows, dtype=i64, device=dev)
        self._ptok = torch.zeros(rows, dtype=i64, device=dev)
        self._pstatus = torch.zeros(rows, dtype=i32, device=dev)
        self._starts = torch.tensor(self.dense._t.starts, dtype=i32, device=dev)
        self._init = self.pda.g.init_config()
        self.dense._state.fill_(FREE)
        self._memo = self.pda.g.mask_memo()
        self._ws = self.pda.g.workspace(rows)
        # a higher priority than the default stream's: the block scheduler
        # starts the PDA pipeline's blocks as soon as dense-step blocks retire
        self._side = torch.cuda.Stream(device=dev, priority=-1) if overlap else None
        self._turnover(1.0)  # every row admits its first request

    def _turnover(self, prob: float) -> None:
        L = _capi.lib()
        L.check(L.bpd_serving_turnover(
            self.rows, self.seed & 0xFFFFFFFFFFFFFFFF, self.step_counter.data_ptr(), float(prob),
            float(self.mix[0]), float(self.mix[1]), self.n_regex, self.schema,
            self._starts.data_ptr(), self._init.data_ptr(), self.kind.data_ptr(),
            self.dense._state.data_ptr(), self.pda._configs.data_ptr(),
            self.pda._broken.view(torch.uint8).data_ptr(), self.dense_rows.data_ptr(),
            self.pda_rows.data_ptr(), self.counts.data_ptr(), self.retired.data_ptr(),
            _stream(self.kind)))

    def turnover(self) -> None:
        """Retire and admit requests (on the device, nothing read back)."""
        self._turnover(self.evict_fraction)

    def step(self, logits: torch.Tensor) -> torch.Tensor:
        """Greedy tokens (``tokens``, int64 ``[rows]``) for ``logits``
        (``[rows, V]``, any float dtype; not modified)."""
        R = self.rows
        t = self.dense._t
        if logits.dim() != 2 or int(logits.shape[0]) < R:
            raise RuntimeError(f"bpdecode_b200: logits must be [>= {R}, vocab], got "
                               f"{tuple(logits.shape)}")
        code, _, _ = _source_args(logits, t.vocab_size, R, self.dense_rows, None, self.device)
        st = _stream(logits)
        L = _capi.lib()
        main = torch.cuda.current_stream(self.device)
        side = self._side
        if side is not None:
            # the PDA rows' pipeline (short, latency-bound launches, then the
            # step) runs on a second stream beside the dense rows' soft step:
            # the two touch disjoint rows, states and outputs
            side.wait_stream(main)
            pst = side.cuda_stream
        else:
            pst = st
        mbuf, cap = self._memo
        L.check(L.bpd_pda_step_greedy_from_n(
            C.byref(self.pda.g._struct()), logits.data_ptr(), code, logits.stride(0),
            self.pda_rows.data_ptr(), None, 0, self.pda._configs.data_ptr(),
            self.pda_rows.data_ptr(), self.pda._broken.view(torch.uint8).data_ptr(), R,
            self.counts.data_ptr() + 4, mbuf.data_ptr(), cap, self._ws.data_ptr(),
            float("-inf"), self._ptok.data_ptr(), self._pstatus.data_ptr(), 0, pst))
        L.check(L.bpd_soft_step_greedy_from_n(
            logits.data_ptr(), code, logits.stride(0), self.dense_rows.data_ptr(), None, 0, R,
            self.counts.data_ptr(), t.vocab_size, self.dense._state.data_ptr(),
            self.dense_rows.data_ptr(), t.lookahead.data_ptr(), t.allow_bits.data_ptr(),
            t.allow_bits.shape[1], t.tok_next.data_ptr(), t.num_states, float(self.alpha),
            self._dtok.data_ptr(), None, 0, self.dense._scratch.data_ptr(), st))
        if side is not None:
            main.wait_stream(side)
        L.check(L.bpd_serving_gather_tokens(
            R, self.dense_rows.data_ptr(), self.pda_rows.data_ptr(), self.counts.data_ptr(),
            self._dtok.data_ptr(), self._ptok.data_ptr(), self.tokens.data_ptr(), st))
        return self.tokens

    def graph(self, logits: torch.Tensor) -> torch.cuda.CUDAGraph:
        """A CUDA graph of :meth:`step` on ``logits`` (this buffer; refill it
        before each replay) followed by :meth:`turnover`. Call :meth:`step`
        once before the first capture (it loads the kernels and sets their
        shared-memory limits, which a capture cannot)."""
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            self.step(logits)
            self.turnover()
        return g

    def states(self) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(dense state pool, PDA config pool, PDA broken flags) -- row r at index r."""
        return self.dense._state, self.pda._configs, self.pda._broken


__all__ = ["DeviceServingLoop", "MixedServingLoop"]
