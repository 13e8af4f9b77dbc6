"""Pin the CPU oracle before trusting it (no GPU needed).

The plain-C restatement (oracle/bpd_oracle.c) is checked against
* the reference's own C++ known-answer tests, re-expressed as data
  (csrc/tests/test_mask.cpp, csrc/tests/test_pda.cpp),
* golden vectors produced by the reference's Python package (tests/golden/),
* the reference's C++ CPU sources compiled unchanged (oracle/_ref), on the same
  inputs, including full 266-int PDA config rows.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import (
    PDA_VOCAB,
    golden_checksums,
    golden_npz,
    small_cases,
    small_dfa,
    vocab_of,
)
from oracle.oracle import NCFG, HostPda, Oracle, RefLib, dfa_with_vocab

ORC = Oracle()
NINF = float("-inf")


# --- csrc/tests/test_mask.cpp:14-39 fixtures ---------------------------------

def ab_fsa() -> dict:
    return {"trans": np.asarray([1, 3, 3, 2, 3, 3, 3, 3], np.int32),
            "accept": np.asarray([0, 0, 1, 0], np.uint8),
            "live": np.asarray([1, 1, 1, 0], np.uint8), "num_symbols": 2, "dead": 3}


AB_OFFSETS = np.asarray([0, 1, 2, 4, 5, 5], np.int32)
AB_SYMBOLS = np.asarray([0, 1, 0, 1, -1], np.int32)


def ab_step(s: int, t: int) -> int:
    f = ab_fsa()
    return ORC.lib.orc_step(
        f["trans"].ctypes.data, 2, f["accept"].ctypes.data, f["live"].ctypes.data, 3,
        AB_OFFSETS.ctypes.data, AB_SYMBOLS.ctypes.data, 4, s, t)  # argtypes set by Oracle


def test_step_known_answers() -> None:
    # test_mask.cpp:67-80
    assert ab_step(0, 0) == 1
    assert ab_step(0, 1) == -1
    assert ab_step(1, 1) == 2
    assert ab_step(0, 2) == 2
    assert ab_step(0, 3) == -1
    assert ab_step(0, 4) == -1
    assert ab_step(2, 4) == 2


def test_dense_known_answers() -> None:
    f = ab_fsa()
    tn = ORC.build_tok_next(f, AB_OFFSETS, AB_SYMBOLS, 4)
    bits = ORC.dense_mask_bits(tn, np.asarray([0, 2]))
    # test_mask.cpp:82-107
    assert bits[0, 0] & 1 and bits[0, 0] & 4 and not bits[0, 0] & 2 and not bits[0, 0] & 16
    assert bits[1, 0] & 16
    nxt = ORC.dense_advance(tn, np.asarray([0, 1, 2, 0]), np.asarray([0, 1, 4, 1]))
    assert nxt.tolist() == [1, 2, 2, -1]  # test_mask.cpp:109-125
    logits = np.ones((2, 5), np.float32)
    ORC.dense_apply_mask(logits, tn, np.asarray([0, 2]), NINF)
    assert logits[0].tolist() == [1.0, NINF, 1.0, NINF, NINF]  # test_mask.cpp:127-146
    assert logits[1, 4] == 1.0 and logits[1, 0] == NINF


@pytest.mark.skipif(not RefLib.available(), reason="reference C++ not compiled")
def test_dense_matches_reference_cpp_on_known_answers() -> None:
    ref = RefLib()
    f = ab_fsa()
    live = ref.build_reachability(f["trans"], 2, f["accept"])
    assert live.tolist() == [1, 1, 1, 0]  # test_mask.cpp:43-52
    tn = ORC.build_tok_next(f, AB_OFFSETS, AB_SYMBOLS, 4)
    st = np.asarray([0, 1, 2, 3, -1], np.int32)
    assert np.array_equal(ref.compute_mask_batch(f, AB_OFFSETS, AB_SYMBOLS, 4, st)[:, 0],
                          ORC.dense_mask_bits(tn, st)[:, 0])


# --- golden vectors from the reference's Python package --------------------

SMALL = golden_npz("small.npz")


@pytest.mark.parametrize("vname,pi", small_cases())
def test_tok_next_and_mask_match_reference_python(vname: str, pi: int) -> None:
    dfa = small_dfa(SMALL, vname, pi)
    v = vocab_of(vname)
    offsets, symbols = dfa_with_vocab(dfa, v.token_bytes)
    tn = ORC.build_tok_next(dfa, offsets, symbols, v.eos_id)
    want = SMALL[f"{vname}/{pi}/tok_next"]
    assert np.array_equal(tn, want)

    logits = SMALL[f"{vname}/{pi}/logits"].copy()
    ORC.dense_apply_mask(logits, tn, np.arange(tn.shape[0]), NINF)
    assert np.array_equal(logits, SMALL[f"{vname}/{pi}/masked"])


@pytest.mark.parametrize("vname,pi", small_cases())
@pytest.mark.parametrize("k", [1, 3])
def test_lookahead_matches_reference_python(vname: str, pi: int, k: int) -> None:
    dfa = small_dfa(SMALL, vname, pi)
    v = vocab_of(vname)
    tn = SMALL[f"{vname}/{pi}/tok_next"]
    got = ORC.build_lookahead(tn, dfa["accept"], dfa["live"], v.eos_id, k)
    want = SMALL[f"{vname}/{pi}/lookahead{k}"].astype(np.float64)
    assert np.array_equal(np.isneginf(got), np.isneginf(want))
    fin = np.isfinite(want)
    np.testing.assert_allclose(got[fin], want[fin], rtol=1e-5, atol=1e-6)


@pytest.mark.skipif(not RefLib.available(), reason="reference C++ not compiled")
@pytest.mark.parametrize("vname,pi", small_cases())
def test_dense_matches_reference_cpp(vname: str, pi: int) -> None:
    ref = RefLib()
    dfa = small_dfa(SMALL, vname, pi)
    v = vocab_of(vname)
    offsets, symbols = dfa_with_vocab(dfa, v.token_bytes)
    tn = ORC.build_tok_next(dfa, offsets, symbols, v.eos_id)
    S = tn.shape[0]
    states = np.asarray(list(range(S)) + [-1, -2], np.int32)
    assert np.array_equal(ref.compute_mask_batch(dfa, offsets, symbols, v.eos_id, states),
                          ORC.dense_mask_bits(tn, states))
    ss, tt = np.meshgrid(np.arange(S, dtype=np.int32), np.arange(v.size, dtype=np.int32))
    ss, tt = ss.ravel(), tt.ravel()
    assert np.array_equal(ref.advance_state_batch(dfa, offsets, symbols, v.eos_id, ss, tt),
                          ORC.dense_advance(tn, ss, tt))
    a = np.random.default_rng(pi).standard_normal((S, v.size)).astype(np.float32)
    b = a.copy()
    ref.apply_mask_batch(dfa, offsets, symbols, v.eos_id, np.arange(S, dtype=np.int32), a, NINF)
    ORC.dense_apply_mask(b, tn, np.arange(S), NINF)
    assert np.array_equal(a, b)


def test_config1_decode_loop_matches_reference() -> None:
    """The whole config-1 loop (IPv4, V = 32,000, B = 64, 32 steps) through the
    oracle reproduces the reference ConstraintBatch's tokens and states."""
    import hashlib

    from bpdecode_b200 import tables
    from bpdecode_b200.workloads import CONFIG1, vocab_config1

    g = golden_npz("config1.npz")
    v = vocab_config1(0, CONFIG1.vocab_size)
    dfa = tables.load_dfa("ipv4")
    offsets, symbols = dfa_with_vocab(dfa, v.token_bytes)
    tn = ORC.build_tok_next(dfa, offsets, symbols, v.eos_id)
    assert hashlib.sha256(tn.tobytes()).hexdigest() == golden_checksums()["config1/ipv4/tok_next"]
    B = CONFIG1.batch
    states = np.full(B, dfa["start"], np.int32)
    for step in range(CONFIG1.steps):
        gen = torch.Generator().manual_seed(step)
        logits = (torch.randn(B, v.size, generator=gen) * CONFIG1.sigma).numpy().copy()
        ORC.dense_apply_mask(logits, tn, states, NINF)
        tok = np.argmax(logits, axis=1)
        states = ORC.dense_advance(tn, states, tok)
        assert np.array_equal(tok, g["config1/tokens"][step]), step
        assert np.array_equal(states, g["config1/states"][step]), step


# --- PDA -----------------------------------------------------------------------

def pda_host(name: str, token_bytes: list[bytes], eos: int) -> HostPda:
    from bpdecode_b200 import tables

    offs = np.zeros(len(token_bytes) + 1, np.int32)
    np.cumsum([len(t) for t in token_bytes], out=offs[1:])
    flat = np.frombuffer(b"".join(token_bytes), np.uint8)
    return HostPda(tables.load_pda(name), offs, flat, eos)


def paren_table() -> HostPda:
    """csrc/tests/test_pda.cpp:20-44 (make_paren_table / make_paren_tokens)."""
    a = {
        "accept": np.asarray([0, 0, 0, 0, 1, 0], np.uint8),
        "live": np.ones(6, np.uint8),
        "edge_offsets": np.asarray([0, 2, 3, 4, 5, 5, 6], np.int32),
        "edge_kind": np.asarray([0, 0, 1, 2, 1, 1], np.int32),
        "edge_lo": np.asarray([0, 0, ord("("), 0, ord(")"), ord("x")], np.int32),
        "edge_hi": np.asarray([0, 0, ord("("), 0, ord(")"), ord("x")], np.int32),
        "edge_dst": np.asarray([1, 5, 2, 3, 4, 4], np.int32),
        "edge_callee": np.asarray([-1, -1, -1, 0, -1, -1], np.int32),
        "root_start": 0, "root_accept": 4,
    }
    return HostPda(a, np.asarray([0, 1, 2, 3, 3], np.int32),
                   np.frombuffer(b"()x", np.uint8), 3)


def feed(g: HostPda, cfg: np.ndarray, s: bytes) -> bool:
    return all(ORC.pda_advance_byte(g, cfg, b) for b in s)


def test_pda_known_answers() -> None:
    g = paren_table()
    cfg = ORC.pda_init(g)
    assert not ORC.pda_is_complete(g, cfg)  # test_pda.cpp:56-61
    c = cfg.copy()
    assert feed(g, c, b"x") and ORC.pda_is_complete(g, c)  # 63-69
    c = cfg.copy()
    assert not feed(g, c, b"y")  # 71-76
    c = cfg.copy()
    assert feed(g, c, b"((x))") and ORC.pda_is_complete(g, c)  # 90-96
    c = cfg.copy()
    assert feed(g, c, b"((x)") and not ORC.pda_is_complete(g, c)  # 98-107
    bits = ORC.pda_mask_bits(g, cfg)[0, 0]  # 119-137
    assert (bits & 1) and not (bits & 2) and (bits & 4) and not (bits & 8)
    cfgs = cfg.reshape(1, NCFG).copy()
    assert ORC.pda_advance(g, cfgs, np.asarray([0]))[0] == 1  # 154-183
    before = cfgs.copy()
    assert ORC.pda_advance(g, cfgs, np.asarray([1]))[0] == 0
    assert np.array_equal(before, cfgs)  # rejected token leaves the row unchanged
    assert ORC.pda_advance(g, cfgs, np.asarray([2]))[0] == 1
    assert ORC.pda_advance(g, cfgs, np.asarray([1]))[0] == 1
    assert ORC.pda_is_complete(g, cfgs[0])
    assert ORC.pda_advance(g, cfgs, np.asarray([3]))[0] == 1


PDA_GOLDEN = golden_npz("pda.npz")


def _pda_case(name: str) -> HostPda:
    from bpdecode_b200.workloads import vocab_large

    if name.endswith("_v4096"):
        v = vocab_large(4096)
        return pda_host(name.split("_v")[0], list(v.token_bytes), v.eos_id)
    toks, eos = PDA_VOCAB
    return pda_host(name, [t.encode() for t in toks], eos)


PDA_CASES = ["paren", "pairs", "xy", "jsonvalue", "schema", "jsonvalue_v4096", "schema_v4096"]


@pytest.mark.parametrize("name", PDA_CASES)
def test_pda_walks_match_reference_rows(name: str) -> None:
    """Replay the reference's recorded walks: identical masks, ok flags and
    full raw config rows after every commit."""
    g = _pda_case(name)
    rows = PDA_GOLDEN[f"{name}/rows"]
    masks = PDA_GOLDEN[f"{name}/masks"]
    toks = PDA_GOLDEN[f"{name}/tokens"]
    oks = PDA_GOLDEN[f"{name}/ok"]
    init = ORC.pda_init(g)
    for i in range(rows.shape[0]):
        if i == 0 or np.array_equal(rows[i], init) and not np.array_equal(rows[i - 1], init):
            pass
        cfg = rows[i].reshape(1, NCFG).copy()
        assert np.array_equal(ORC.pda_mask_bits(g, cfg)[0], masks[i]), (name, i)
        ok = ORC.pda_advance(g, cfg, toks[i:i + 1])
        assert ok[0] == oks[i], (name, i)
        if i + 1 < rows.shape[0] and not np.array_equal(rows[i + 1], init):
            assert np.array_equal(cfg[0], rows[i + 1]), (name, i)
    assert np.array_equal(init, rows[0])


@pytest.mark.skipif(not RefLib.available(), reason="reference C++ not compiled")
@pytest.mark.parametrize("name", ["paren", "pairs", "jsonvalue", "schema"])
def test_pda_exhaustive_short_sequences_match_reference_cpp(name: str) -> None:
    """Every token sequence of length <= 2 over the test vocabulary: identical
    ok flags, masks and raw rows against the reference's compiled PDA."""
    import itertools

    ref = RefLib()
    g = _pda_case(name)
    alphabet = [t for t in range(g.vocab_size) if t != g.eos_id]
    for length in range(3):
        for combo in itertools.product(alphabet, repeat=length):
            a = ORC.pda_init(g).reshape(1, NCFG)
            b = ref.pda_init(g).reshape(1, NCFG)
            assert np.array_equal(a, b)
            for t in combo:
                oka = ORC.pda_advance(g, a, np.asarray([t]))
                okb = ref.pda_advance(g, b, np.asarray([t], np.int32))
                assert oka[0] == okb[0] and np.array_equal(a, b), (name, combo)
                if not oka[0]:
                    break
            assert np.array_equal(ORC.pda_mask_bits(g, a), ref.pda_mask_bits(g, b)), combo
