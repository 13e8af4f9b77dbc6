"""Dense regular path on the GPU against the oracle and the reference's goldens.

Every comparison is bit-exact: tables, packed bits, masked logits (fp32, bf16,
fp16), next states, argmax tokens. Full-size configurations are checked
through size-independent properties (sha256 of the reference's tables, fused
step == unfused step, oracle spot checks of sampled rows).
"""

from __future__ import annotations

import hashlib

import numpy as np
import pytest
import torch

from conftest import (
    golden_checksums,
    golden_npz,
    small_cases,
    small_dfa,
    vocab_of,
)
from oracle.oracle import Oracle, RefLib, dfa_with_vocab

pytestmark = pytest.mark.gpu

NINF = float("-inf")
SMALL = golden_npz("small.npz")


@pytest.fixture(scope="module")
def orc() -> Oracle:
    return Oracle()


def _fsa(vname: str, pi: int):
    from bpdecode_b200.ops import FsaTensors

    return FsaTensors.from_arrays(small_dfa(SMALL, vname, pi), vocab_of(vname)).to("cuda")


def _u16(t: torch.Tensor) -> np.ndarray:
    return t.cpu().view(torch.int16).numpy().view(np.uint16).copy()


def _fill_bits(neg_inf: float, dtype: torch.dtype) -> int:
    return int(torch.tensor(neg_inf, dtype=dtype).view(torch.int16).item()) & 0xFFFF


@pytest.mark.parametrize("vname,pi", small_cases())
def test_tok_next_allow_bits_mask_advance(vname: str, pi: int, orc: Oracle) -> None:
    from bpdecode_b200 import ops

    fsa = _fsa(vname, pi)
    want_tn = SMALL[f"{vname}/{pi}/tok_next"]
    tn, bits = fsa.dense_tables()
    assert np.array_equal(tn.cpu().numpy(), want_tn)
    S, V = want_tn.shape
    ob = orc.allow_bits(want_tn, bits.shape[1])
    assert np.array_equal(bits.cpu().numpy().view(np.uint32), ob)

    # fp32 apply against the reference's own masked output
    logits = torch.from_numpy(SMALL[f"{vname}/{pi}/logits"]).cuda()
    states = torch.arange(S, dtype=torch.int32, device="cuda")
    ops.apply_mask_(logits, fsa, states)
    assert np.array_equal(logits.cpu().numpy(), SMALL[f"{vname}/{pi}/masked"])

    # compute_mask against the oracle (and broken / free rows)
    st = torch.tensor(list(range(S)) + [-1, -2], dtype=torch.int32, device="cuda")
    got = ops.compute_mask(fsa, st).cpu().numpy().view(np.uint32)
    assert np.array_equal(got, orc.dense_mask_bits(want_tn, st.cpu().numpy()))

    # advance over every (state, token) pair, plus broken rows
    ss, tt = np.meshgrid(np.arange(-2, S, dtype=np.int32), np.arange(V, dtype=np.int64))
    ss, tt = ss.ravel(), tt.ravel()
    nxt = ops.advance_state(fsa, torch.from_numpy(ss).cuda(), torch.from_numpy(tt).cuda())
    assert np.array_equal(nxt.cpu().numpy(), orc.dense_advance(want_tn, ss, tt))


@pytest.mark.skipif(not RefLib.available(), reason="reference C++ not compiled")
@pytest.mark.parametrize("vname,pi", small_cases()[::3])
def test_compute_mask_matches_reference_cpp(vname: str, pi: int) -> None:
    from bpdecode_b200 import ops

    ref = RefLib()
    dfa = small_dfa(SMALL, vname, pi)
    v = vocab_of(vname)
    offsets, symbols = dfa_with_vocab(dfa, v.token_bytes)
    fsa = _fsa(vname, pi)
    S = fsa.num_states
    st = np.asarray(list(range(S)) + [-1], np.int32)
    got = ops.compute_mask(fsa, torch.from_numpy(st).cuda()).cpu().numpy().view(np.uint32)
    assert np.array_equal(got, ref.compute_mask_batch(dfa, offsets, symbols, v.eos_id, st))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("neg_inf", [NINF, -1e4, -3.3])
def test_apply_mask_16bit(dtype: torch.dtype, neg_inf: float, orc: Oracle) -> None:
    from bpdecode_b200 import ops

    for vname, pi in small_cases()[::5]:
        fsa = _fsa(vname, pi)
        tn = SMALL[f"{vname}/{pi}/tok_next"]
        S, V = tn.shape
        st = np.asarray([s % (S + 2) - 2 for s in range(3 * S)], np.int32)
        x = torch.randn(st.size, V, generator=torch.Generator().manual_seed(pi)).to(dtype)
        want = _u16(x)
        orc.dense_apply_mask(want, tn, st, _fill_bits(neg_inf, dtype))
        y = x.cuda()
        ops.apply_mask_(y, fsa, torch.from_numpy(st).cuda(), neg_inf)
        assert np.array_equal(_u16(y), want)


def _ipv4_large(V: int):
    from bpdecode_b200 import tables
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import vocab_large

    return FsaTensors.from_arrays(tables.load_dfa("ipv4"), vocab_large(V)).to("cuda")


@pytest.mark.parametrize("V,pad", [(1001, 0), (1001, 7), (4096, 3), (4099, 0), (32768, 64)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_strided_and_ragged_rows(V: int, pad: int, dtype: torch.dtype, orc: Oracle) -> None:
    """Row strides that break 16-byte alignment, vocab sizes that are not a
    multiple of the vector or tile width, and a logits view inside a wider
    buffer (the padded lm_head case): only the view's columns change."""
    from bpdecode_b200 import ops

    fsa = _ipv4_large(V)
    tn = fsa.dense_tables()[0].cpu().numpy()
    S = fsa.num_states
    B = 2 * S + 2
    st = np.asarray([(b % (S + 2)) - 2 for b in range(B)], np.int32)
    buf = torch.randn(B, V + pad, generator=torch.Generator().manual_seed(V + pad)).to(dtype)
    view_cpu = buf[:, :V].contiguous()
    if dtype == torch.float32:
        want = view_cpu.numpy().copy()
        orc.dense_apply_mask(want, tn, st, NINF)
    else:
        want = _u16(view_cpu)
        orc.dense_apply_mask(want, tn, st, _fill_bits(NINF, dtype))
    dev = buf.cuda()
    ops.apply_mask_(dev[:, :V], fsa, torch.from_numpy(st).cuda())
    got = dev[:, :V].contiguous()
    got = got.cpu().numpy() if dtype == torch.float32 else _u16(got)
    assert np.array_equal(got, want)
    assert torch.equal(dev[:, V:].cpu(), buf[:, V:])


def test_config1_loop_matches_reference() -> None:
    """The config-1 decode loop through ConstraintBatch (apply_mask + argmax +
    commit) and through the fused step both reproduce the reference's recorded
    tokens and states at every step."""
    from bpdecode_b200 import tables
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import CONFIG1, vocab_config1

    g = golden_npz("config1.npz")
    v = vocab_config1(0, CONFIG1.vocab_size)
    fsa = FsaTensors.from_arrays(tables.load_dfa("ipv4"), v).to("cuda")
    tn = fsa.dense_tables()[0].cpu().numpy()
    assert hashlib.sha256(tn.tobytes()).hexdigest() == golden_checksums()["config1/ipv4/tok_next"]
    B = CONFIG1.batch
    a = ConstraintBatch(fsa, capacity=B)
    b = ConstraintBatch(fsa, capacity=B)
    ids = list(range(B))
    for i in ids:
        a.add(i)
        b.add(i)
    for step in range(CONFIG1.steps):
        gen = torch.Generator().manual_seed(step)
        logits = (torch.randn(B, v.size, generator=gen) * CONFIG1.sigma).cuda()
        la = logits.clone()
        a.apply_mask(ids, la)
        tok = la.argmax(-1)
        nxt = a.commit(ids, tok)
        lb = logits.clone()
        tb = b.step_greedy(ids, lb)
        assert np.array_equal(tok.cpu().numpy(), g["config1/tokens"][step])
        assert np.array_equal(nxt.cpu().numpy(), g["config1/states"][step])
        assert torch.equal(tb, tok) and torch.equal(lb, la)
        assert torch.equal(b._state, a._state)


def test_full_size_tables_match_reference_checksums() -> None:
    from bpdecode_b200 import tables
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import DENSE_PATTERNS, vocab_large

    sums = golden_checksums()
    v = vocab_large(128_256)
    for name, _ in DENSE_PATTERNS:
        fsa = FsaTensors.from_arrays(tables.load_dfa(name), v).to("cuda")
        tn = fsa.dense_tables()[0].cpu().numpy()
        assert hashlib.sha256(tn.tobytes()).hexdigest() == sums[f"config2/{name}/tok_next"], name
    v3 = vocab_large(151_936)
    fsa = FsaTensors.from_arrays(tables.load_dfa("schema"), v3).to("cuda")
    tn = fsa.dense_tables()[0].cpu().numpy()
    assert hashlib.sha256(tn.tobytes()).hexdigest() == sums["config3/schema/tok_next"]


def _config2_batch(B: int):
    from bpdecode_b200 import tables
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import DENSE_PATTERNS, row_patterns, vocab_large

    v = vocab_large(128_256)
    fsas = [FsaTensors.from_arrays(tables.load_dfa(n), v).to("cuda") for n, _ in DENSE_PATTERNS]
    pats = row_patterns(B)
    mk = lambda: ConstraintBatch(fsas, capacity=B)  # noqa: E731
    batches = (mk(), mk())
    for bt in batches:
        for i in range(B):
            bt.add(i, grammar=pats[i])
    return batches, v


def test_config2_fused_step_equals_unfused_and_oracle(orc: Oracle) -> None:
    """Serving scale (8 regexes mixed in one batch, B = 1024, V = 128,256, bf16
    N(0, 2)): the fused step and apply_mask + argmax + commit agree exactly on
    masked logits, tokens and states; sampled rows agree with the oracle."""
    B = 1024
    (a, b), v = _config2_batch(B)
    ids = list(range(B))
    tn_all = a._t.tok_next.cpu().numpy()
    rows = np.arange(0, B, 37)
    fill = _fill_bits(NINF, torch.bfloat16)
    for step in range(6):
        gen = torch.Generator(device="cuda").manual_seed(1000 + step)
        logits = (torch.randn(B, v.size, generator=gen, device="cuda") * 2.0).to(torch.bfloat16)
        states_before = a._state.cpu().numpy()[rows]
        sample = _u16(logits[rows])
        la = logits.clone()
        a.apply_mask(ids, la)
        tok = la.argmax(-1)
        nxt = a.commit(ids, tok)
        lb = logits.clone()
        tb = b.step_greedy(ids, lb)
        assert torch.equal(lb, la)
        assert torch.equal(tb, tok)
        assert torch.equal(a._state, b._state)
        orc.dense_apply_mask(sample, tn_all, states_before, fill)
        assert np.array_equal(_u16(la[rows]), sample)
        sample_f = torch.from_numpy(sample.view(np.int16)).view(torch.bfloat16).float().numpy()
        assert np.array_equal(np.argmax(sample_f, axis=1), tok.cpu().numpy()[rows])
        assert np.array_equal(orc.dense_advance(tn_all, states_before, tok.cpu().numpy()[rows]),
                              nxt.cpu().numpy()[rows])


def test_config3_schema_steps_match_oracle(orc: Oracle) -> None:
    """Config 3 (the JSON-Schema object as a dense DFA, V = 151,936, B = 512,
    fp32 N(0, 1), greedy commit): every row of the first steps against the
    oracle -- masked logits, tokens and states -- and the fused step against
    the unfused one over 32 steps."""
    from bpdecode_b200 import tables
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import vocab_large

    B, V = 512, 151_936
    fsa = FsaTensors.from_arrays(tables.load_dfa("schema"), vocab_large(V)).to("cuda")
    a, b = ConstraintBatch(fsa, capacity=B), ConstraintBatch(fsa, capacity=B)
    ids = list(range(B))
    for i in ids:
        a.add(i)
        b.add(i)
    tn = fsa.dense_tables()[0].cpu().numpy()
    for step in range(32):
        gen = torch.Generator(device="cuda").manual_seed(3000 + step)
        logits = torch.randn(B, V, generator=gen, device="cuda")
        before = a._state.cpu().numpy().copy()
        la = logits.clone()
        a.apply_mask(ids, la)
        tok = la.argmax(-1)
        nxt = a.commit(ids, tok)
        lb = logits.clone()
        assert torch.equal(b.step_greedy(ids, lb), tok)
        assert torch.equal(lb, la) and torch.equal(a._state, b._state)
        if step < 3:
            want = logits.cpu().numpy()
            orc.dense_apply_mask(want, tn, before, NINF)
            assert np.array_equal(la.cpu().numpy(), want)
            assert np.array_equal(np.argmax(want, axis=1), tok.cpu().numpy())
            assert np.array_equal(orc.dense_advance(tn, before, tok.cpu().numpy()),
                                  nxt.cpu().numpy())


@pytest.mark.parametrize("k", [1, 2, 3, 7, 32])
def test_step_chunkings_agree(k: int) -> None:
    """Any cut of the rows into work items gives the unfused result, and the
    step scratch is zero again after the launch."""
    from bpdecode_b200 import ops

    fsa = _ipv4_large(32_000)
    S = fsa.num_states
    B = 96
    pool0 = torch.tensor([(i % (S + 2)) - 2 for i in range(B)], dtype=torch.int32, device="cuda")
    logits = torch.randn(B, fsa.vocab_size, device="cuda").to(torch.bfloat16)
    la = logits.clone()
    ops.apply_mask_(la, fsa, pool0)
    want_tok = la.argmax(-1)
    want_next = ops.advance_state(fsa, pool0, want_tok)
    lb = logits.clone()
    pool = pool0.clone()
    tok, nxt = ops.step_greedy_(lb, fsa, pool, chunks_per_row=k)
    assert torch.equal(lb, la) and torch.equal(tok, want_tok)
    assert torch.equal(nxt, want_next) and torch.equal(pool, want_next)
    assert int(ops.step_scratch(B, lb.device).count_nonzero()) == 0


def test_argmax_ties_nan_and_finite_fill() -> None:
    """First maximal index on ties, NaN counts as maximal, fully masked rows
    pick index 0, and a finite neg_inf above the allowed logits is what
    torch.argmax would pick."""
    from bpdecode_b200 import ops

    fsa = _ipv4_large(4096)
    tn, _ = fsa.dense_tables()
    S, V = fsa.num_states, fsa.vocab_size
    allowed = (tn[fsa.start] != -1).nonzero().flatten()
    B = 6
    logits = torch.zeros(B, V, device="cuda")
    logits[1, allowed[3]] = float("nan")
    logits[1, allowed[5]] = float("nan")
    logits[2] = -50.0  # below the finite fill of row 2's call below
    logits[3, allowed] = 1.0
    logits[4, allowed[-1]] = float("inf")
    states = torch.full((B,), fsa.start, dtype=torch.int32, device="cuda")
    states[5] = -1
    for fill in (NINF, -7.0):
        la = logits.clone()
        ops.apply_mask_(la, fsa, states, fill)
        want = la.argmax(-1)
        lb = logits.clone()
        pool = states.clone()
        tok, _ = ops.step_greedy_(lb, fsa, pool, neg_inf=fill)
        assert torch.equal(lb.isnan(), la.isnan())
        assert torch.equal(torch.nan_to_num(lb), torch.nan_to_num(la))
        assert torch.equal(tok, want), (fill, tok, want)
    assert int(tok[5]) == 0


def test_batch_lifecycle_like_reference() -> None:
    """tests/test_batch.py semantics: slot reuse, FREE / BROKEN, independent
    rows, MaskCache == uncached."""
    from bpdecode_b200.batch import BROKEN, FREE, ConstraintBatch, MaskCache
    from bpdecode_b200.ops import FsaTensors, apply_mask_

    patterns = list(SMALL["meta/patterns"])
    v = vocab_of("batch")
    fsa = FsaTensors.from_arrays(small_dfa(SMALL, "batch", patterns.index("[01]+")), v).to("cuda")
    batch = ConstraintBatch(fsa, capacity=2)
    s0, s1 = batch.add("r0"), batch.add("r1")
    assert {s0, s1} == {0, 1}
    with pytest.raises(RuntimeError):
        batch.add("r2")
    batch.evict("r0")
    assert int(batch._state[s0]) == FREE
    assert batch.add("r2") == s0
    assert "r0" not in batch and "r2" in batch

    tok = {t: i for i, t in enumerate(["a", "b", "c", "ab", "0", "1", "12", "-", ".", "<eos>"])}
    b3 = ConstraintBatch(fsa, capacity=3)
    for r in ("a", "b", "c"):
        b3.add(r)
    b3.commit(["a", "b", "c"], torch.tensor([4, 5, 4], dtype=torch.int32, device="cuda"))
    b3.commit(["b"], torch.tensor([5], dtype=torch.int32, device="cuda"))
    logits = torch.zeros(3, v.size, device="cuda")
    b3.apply_mask(["a", "b", "c"], logits)
    for row in range(3):
        assert logits[row, tok["0"]].item() == 0.0
        assert logits[row, tok["a"]].item() == NINF
        assert logits[row, v.eos_id].item() == 0.0
    assert b3.is_complete("a")
    b3.commit(["c"], torch.tensor([tok["a"]], dtype=torch.int32, device="cuda"))
    assert b3.state_of("c") == BROKEN and b3.is_broken("c")
    b3.reset("c")
    assert b3.state_of("c") == fsa.start

    for pat in ("[01]+", "-?[0-9]+(\\.[0-9]+)?", "(ab)+", "a|b|12"):
        f = FsaTensors.from_arrays(small_dfa(SMALL, "batch", patterns.index(pat)), v).to("cuda")
        st = torch.tensor(list(range(f.num_states)) * 2, dtype=torch.int32, device="cuda")
        base = torch.randn(len(st), v.size, device="cuda")
        want = base.clone()
        apply_mask_(want, f, st)
        mc = MaskCache(f)
        got = base.clone()
        mc.apply(st, got)
        assert torch.equal(want, got)


def test_mixed_grammar_batch_equals_separate_batches() -> None:
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.ops import FsaTensors

    patterns = list(SMALL["meta/patterns"])
    v = vocab_of("dense")
    fsas = [FsaTensors.from_arrays(small_dfa(SMALL, "dense", i), v).to("cuda")
            for i in range(len(patterns))]
    mixed = ConstraintBatch(fsas, capacity=len(fsas) * 2)
    singles = [ConstraintBatch(f, capacity=2) for f in fsas]
    for g in range(len(fsas)):
        for r in range(2):
            mixed.add((g, r), grammar=g)
            singles[g].add((g, r))
    gen = torch.Generator().manual_seed(5)
    for _ in range(6):
        logits = torch.randn(len(fsas) * 2, v.size, generator=gen).cuda()
        ids = [(g, r) for g in range(len(fsas)) for r in range(2)]
        lm = logits.clone()
        mixed.apply_mask(ids, lm)
        tok = lm.argmax(-1)
        mixed.commit(ids, tok)
        for g in range(len(fsas)):
            ls = logits[2 * g:2 * g + 2].clone()
            singles[g].apply_mask([(g, 0), (g, 1)], ls)
            assert torch.equal(ls, lm[2 * g:2 * g + 2])
            singles[g].commit([(g, 0), (g, 1)], tok[2 * g:2 * g + 2])
            for r in range(2):
                sm = mixed.state_of((g, r))
                ss = singles[g].state_of((g, r))
                assert (sm == ss == -1) or sm == ss + mixed._t.offsets[g]
                assert mixed.is_complete((g, r)) == singles[g].is_complete((g, r))


def test_reset_many_equals_per_row_reset() -> None:
    """reset_many(ids) puts exactly the named rows back at their own
    grammar's start state, like reset() per id, and leaves the rest alone."""
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.ops import FsaTensors

    patterns = list(SMALL["meta/patterns"])
    v = vocab_of("dense")
    fsas = [FsaTensors.from_arrays(small_dfa(SMALL, "dense", i), v).to("cuda")
            for i in range(len(patterns))]
    a = ConstraintBatch(fsas, capacity=3 * len(fsas))
    b = ConstraintBatch(fsas, capacity=3 * len(fsas))
    ids = [(g, r) for g in range(len(fsas)) for r in range(3)]
    for i in ids:
        a.add(i, grammar=i[0])
        b.add(i, grammar=i[0])
    gen = torch.Generator().manual_seed(9)
    for step in range(8):
        logits = torch.randn(len(ids), v.size, generator=gen).cuda()
        ta = a.step_greedy(ids, logits.clone())
        tb = b.step_greedy(ids, logits.clone())
        assert torch.equal(ta, tb)
        if step % 3 == 2:
            some = [i for i in ids if (i[1] + step) % 2]
            a.reset_many(some)
            for i in some:
                b.reset(i)
            assert [a.state_of(i) for i in ids] == [b.state_of(i) for i in ids]


def test_empty_batch_and_cpu_tensors_fail_loudly() -> None:
    from bpdecode_b200 import ops

    fsa = _ipv4_large(1024)
    empty = torch.empty(0, fsa.vocab_size, device="cuda")
    ops.apply_mask_(empty, fsa, torch.empty(0, dtype=torch.int32, device="cuda"))
    with pytest.raises(RuntimeError):
        ops.apply_mask_(torch.zeros(1, fsa.vocab_size), fsa,
                        torch.zeros(1, dtype=torch.int32, device="cuda"))


def test_invalid_tokens_and_states_are_rejected_not_read() -> None:
    """Fault injection from the host: token ids outside [0, V) and states
    outside [0, S) (the reference would read out of bounds) turn the row
    BROKEN / fully masked instead; valid rows are unaffected."""
    from bpdecode_b200.batch import BROKEN, ConstraintBatch

    fsa = _ipv4_large(4096)
    V, S = fsa.vocab_size, fsa.num_states
    b = ConstraintBatch(fsa, capacity=8)
    ids = list(range(8))
    for i in ids:
        b.add(i)
    start = b.state_of(0)
    digit = next(t for t in range(V) if int(fsa.dense_tables()[0][start, t]) >= 0)
    toks = torch.tensor([-3, V, V + 100, digit, -1, digit, 2**40, digit], device="cuda")
    nxt = b.commit(ids, toks)
    bad = [0, 1, 2, 4, 6]
    assert all(int(nxt[i]) == BROKEN for i in bad)
    assert all(int(nxt[i]) >= 0 for i in (3, 5, 7))
    # a state outside the table (corrupted pool entry) masks the whole row
    b._state[b._slot_of[3]] = S + 7
    logits = torch.randn(8, V, device="cuda")
    b.apply_mask(ids, logits)
    for i in bad + [3]:
        assert torch.isneginf(logits[i]).all()
    assert not torch.isneginf(logits[5]).all()
    tok = b.step_greedy(ids, torch.randn(8, V, device="cuda"))
    assert int(b.state_of(3)) == BROKEN and all(b.state_of(i) == BROKEN for i in bad)
    assert torch.equal(tok[bad], torch.zeros(len(bad), dtype=torch.int64, device="cuda"))
