"""The allocation-free PDA mask entry point against the regular one.

Some callers of this library cannot allocate device memory at the moment they
mask logits: a serving engine that has reserved (nearly) all of HBM for its
own pool or KV cache, where a raw cudaMalloc would fail or fragment that pool,
or a foreign-language binding with no access to the host framework's caching
allocator. For them ``bpd_pda_apply_mask_noalloc`` keeps its per-call scratch
in a fixed device array built into the library.

This file is collected last on purpose (its name sorts after every other test
file), so a run that stops at the first failure has already run everything
else. It must pass alone in a fresh process and after the other tests.
"""

from __future__ import annotations

import ctypes as C

import pytest
import torch

from conftest import golden_npz

pytestmark = pytest.mark.gpu

MAX_BATCH = 128  # BPD_NOALLOC_MAX_BATCH
MAX_VOCAB = 262144  # BPD_NOALLOC_MAX_VOCAB
CAPACITY_ERROR = 3  # BPD_ERR_CAPACITY


def _grammar(name: str):
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import PdaTensors
    from bpdecode_b200.workloads import vocab_large

    return PdaTensors.from_arrays(tables.load_pda(name), vocab_large(4096), "cuda")


def _regular(L, g, logits, pool, slots, broken):
    """bpd_pda_apply_mask with a workspace allocated here, no memo."""
    ws = torch.empty(L.bpd_pda_workspace_bytes(logits.shape[0], g.vocab_size),
                     dtype=torch.uint8, device="cuda")
    return L.bpd_pda_apply_mask(
        C.byref(g._struct()), logits.data_ptr(), _code(logits), logits.stride(0),
        pool.data_ptr(), slots.data_ptr(), broken.data_ptr(), logits.shape[0], None, 0,
        ws.data_ptr(), float("-inf"), torch.cuda.current_stream().cuda_stream)


def _noalloc(L, g, logits, pool, slots, broken):
    return L.bpd_pda_apply_mask_noalloc(
        C.byref(g._struct()), logits.data_ptr(), _code(logits), logits.stride(0),
        pool.data_ptr(), slots.data_ptr(), broken.data_ptr(), logits.shape[0], None, 0,
        float("-inf"), torch.cuda.current_stream().cuda_stream)


def _code(t: torch.Tensor) -> int:
    return {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}[t.dtype]


def test_noalloc_matches_workspace_entry_point_on_two_calls() -> None:
    """Two calls in a row with different grammars, rows, dtypes and broken
    flags: the shared built-in scratch carries nothing stale from one call to
    the next, and each result equals the workspace entry point's exactly."""
    from bpdecode_b200 import _capi

    L = _capi.lib()
    pda = golden_npz("pda.npz")
    cases = [("schema", "schema_v4096", torch.float32, 72),
             ("jsonvalue", "jsonvalue_v4096", torch.bfloat16, 30)]
    for call, (name, rows_key, dtype, n) in enumerate(cases):
        g = _grammar(name)
        pool = torch.from_numpy(pda[f"{rows_key}/rows"]).cuda()
        slots = torch.randperm(n, generator=torch.Generator().manual_seed(call)).cuda()
        broken = torch.zeros(n, dtype=torch.uint8, device="cuda")
        broken[call::7] = 1
        gen = torch.Generator(device="cuda").manual_seed(10 + call)
        logits = torch.randn(n, g.vocab_size, generator=gen, device="cuda").to(dtype)
        want = logits.clone()
        got = logits.clone()
        assert _regular(L, g, want, pool, slots, broken) == 0, L.bpd_last_error()
        assert _noalloc(L, g, got, pool, slots, broken) == 0, L.bpd_last_error()
        torch.cuda.synchronize()
        assert torch.equal(got, want), f"call {call + 1} differs"
        assert torch.isneginf(got[broken[slots].bool()]).all()  # broken is per pool slot


def test_noalloc_rejects_batches_beyond_its_scratch() -> None:
    from bpdecode_b200 import _capi

    L = _capi.lib()
    g = _grammar("xy")
    n = MAX_BATCH + 1
    pool = g.init_batch(n)
    slots = torch.arange(n, device="cuda")
    broken = torch.zeros(n, dtype=torch.uint8, device="cuda")
    logits = torch.zeros(n, g.vocab_size, device="cuda")
    assert _noalloc(L, g, logits, pool, slots, broken) == CAPACITY_ERROR
    assert b"at most 128 rows" in L.bpd_last_error()
    torch.cuda.synchronize()
    assert (logits == 0).all()  # nothing was enqueued


def test_noalloc_rejects_vocabularies_beyond_its_scratch() -> None:
    """A grammar whose vocabulary is one token past the built-in limit is
    refused before anything is enqueued (the logits stay untouched)."""
    from bpdecode_b200 import _capi

    L = _capi.lib()
    g = _grammar("xy")
    n = 4
    pool = g.init_batch(n)
    slots = torch.arange(n, device="cuda")
    broken = torch.zeros(n, dtype=torch.uint8, device="cuda")
    logits = torch.zeros(n, g.vocab_size, device="cuda")
    big = _capi.PdaGrammar.from_buffer_copy(g._struct())
    big.vocab_size = MAX_VOCAB + 1
    rc = L.bpd_pda_apply_mask_noalloc(
        C.byref(big), logits.data_ptr(), 0, logits.stride(0), pool.data_ptr(),
        slots.data_ptr(), broken.data_ptr(), n, None, 0, float("-inf"),
        torch.cuda.current_stream().cuda_stream)
    assert rc == CAPACITY_ERROR
    assert b"262145" in L.bpd_last_error()
    torch.cuda.synchronize()
    assert (logits == 0).all()  # nothing was enqueued
    # the same call at the real vocabulary size still works afterwards
    assert _noalloc(L, g, logits, pool, slots, broken) == 0, L.bpd_last_error()
    torch.cuda.synchronize()
