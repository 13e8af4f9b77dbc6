"""PDA kernels on the GPU against the reference's compiled PDA and the oracle.

Bit-exact on masks, ok flags and full 266-int config rows (including words
outside the live region), with and without the HBM mask memo.
"""

from __future__ import annotations

import itertools

import numpy as np
import pytest
import torch

from conftest import PDA_VOCAB, golden_npz
from oracle.oracle import HostPda, Oracle, RefLib

pytestmark = pytest.mark.gpu

PDA_GOLDEN = golden_npz("pda.npz")
GRAMMARS = ["paren", "pairs", "xy", "jsonvalue", "schema"]


def _vocab(name: str):
    from bpdecode_b200.tokenizer import Vocabulary
    from bpdecode_b200.workloads import vocab_large

    if name.endswith("_v4096"):
        return vocab_large(4096)
    toks, eos = PDA_VOCAB
    return Vocabulary.from_tokens(toks, eos_id=eos)


def _grammar(name: str):
    return name.split("_v")[0]


def _dev(name: str):
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import PdaTensors

    return PdaTensors.from_arrays(tables.load_pda(_grammar(name)), _vocab(name), "cuda")


def _host(name: str) -> HostPda:
    from bpdecode_b200 import tables

    v = _vocab(name)
    offs = np.zeros(v.size + 1, np.int32)
    np.cumsum([len(t) for t in v.token_bytes], out=offs[1:])
    return HostPda(tables.load_pda(_grammar(name)), offs,
                   np.frombuffer(b"".join(v.token_bytes), np.uint8), v.eos_id)


@pytest.fixture(scope="module")
def orc() -> Oracle:
    return Oracle()


@pytest.mark.parametrize("name", GRAMMARS + ["jsonvalue_v4096", "schema_v4096"])
def test_init_config_matches_oracle(name: str, orc: Oracle) -> None:
    g = _dev(name)
    assert np.array_equal(g.init_config().cpu().numpy(), orc.pda_init(_host(name)))


@pytest.mark.parametrize("name", GRAMMARS + ["jsonvalue_v4096", "schema_v4096"])
@pytest.mark.parametrize("memo", [True, False])
def test_golden_walks(name: str, memo: bool) -> None:
    """Replay the reference's recorded walks: masks of every recorded
    config-set, ok flags and the raw row after every commit."""
    from bpdecode_b200.grammar.device import pda_advance_state, pda_compute_mask

    g = _dev(name)
    rows = PDA_GOLDEN[f"{name}/rows"]
    masks = PDA_GOLDEN[f"{name}/masks"]
    toks = PDA_GOLDEN[f"{name}/tokens"]
    oks = PDA_GOLDEN[f"{name}/ok"]
    cfg = torch.from_numpy(rows).cuda()
    got = pda_compute_mask(g, cfg, memo=memo).cpu().numpy().view(np.uint32)
    assert np.array_equal(got, masks)
    after = cfg.clone()
    ok = pda_advance_state(after, g, torch.from_numpy(toks).cuda()).cpu().numpy()
    assert np.array_equal(ok, oks)
    after = after.cpu().numpy()
    init = rows[0]
    for i in range(rows.shape[0] - 1):
        if np.array_equal(rows[i + 1], init) and not np.array_equal(after[i], init):
            continue  # a new walk starts at rows[i + 1]
        assert np.array_equal(after[i], rows[i + 1]), (name, i)


@pytest.mark.parametrize("name", GRAMMARS)
def test_exhaustive_sequences_match_oracle(name: str, orc: Oracle) -> None:
    """Every token sequence of length <= 3 (<= 2 for the JSON grammars),
    advanced as one batch per length: ok, raw rows and masks equal the
    oracle's."""
    from bpdecode_b200.grammar.device import pda_advance_state, pda_compute_mask

    g = _dev(name)
    h = _host(name)
    alphabet = [t for t in range(h.vocab_size) if t != h.eos_id]
    max_len = 2 if name in ("jsonvalue", "schema") else 3
    init = orc.pda_init(h)
    for length in range(1, max_len + 1):
        combos = list(itertools.product(alphabet, repeat=length))
        ref = np.tile(init, (len(combos), 1))
        alive = np.ones(len(combos), bool)
        dev = torch.from_numpy(ref.copy()).cuda()
        for pos in range(length):
            toks = np.asarray([c[pos] for c in combos], np.int64)
            ok_ref = orc.pda_advance(h, ref, toks)
            ok_dev = pda_advance_state(dev, g, torch.from_numpy(toks).cuda()).cpu().numpy()
            assert np.array_equal(ok_dev[alive], ok_ref[alive])
            alive &= ok_ref.astype(bool)
        got_rows = dev.cpu().numpy()
        assert np.array_equal(got_rows, ref)
        m_dev = pda_compute_mask(g, dev).cpu().numpy().view(np.uint32)
        assert np.array_equal(m_dev, orc.pda_mask_bits(h, ref))


@pytest.mark.skipif(not RefLib.available(), reason="reference C++ not compiled")
@pytest.mark.parametrize("name", ["jsonvalue_v4096", "schema_v4096"])
def test_apply_mask_matches_reference_cpp(name: str) -> None:
    from bpdecode_b200.grammar.device import pda_apply_mask_

    ref = RefLib()
    h = _host(name)
    g = _dev(name)
    rows = PDA_GOLDEN[f"{name}/rows"][:12]
    logits = np.random.default_rng(3).standard_normal((rows.shape[0], h.vocab_size)).astype(
        np.float32)
    want = logits.copy()
    ref.pda_apply_mask(h, rows, want, float("-inf"))
    got = torch.from_numpy(logits).cuda()
    pda_apply_mask_(got, g, torch.from_numpy(rows).cuda())
    assert np.array_equal(got.cpu().numpy(), want)
    for dtype in (torch.bfloat16, torch.float16):
        x = torch.from_numpy(logits).to(dtype)
        ref16 = x.clone()
        ref16[torch.from_numpy(np.isneginf(want))] = float("-inf")
        y = x.cuda()
        pda_apply_mask_(y, g, torch.from_numpy(rows).cuda())
        assert torch.equal(y.cpu(), ref16)


def test_memo_hits_and_clear(orc: Oracle) -> None:
    from bpdecode_b200.grammar.device import pda_compute_mask

    name = "jsonvalue_v4096"
    g = _dev(name)
    rows = torch.from_numpy(PDA_GOLDEN[f"{name}/rows"]).cuda()
    first = pda_compute_mask(g, rows)
    second = pda_compute_mask(g, rows)  # every row now hits the memo
    assert torch.equal(first, second)
    g.clear_memo()
    third = pda_compute_mask(g, rows)
    assert torch.equal(first, third)
    # duplicated rows inside one call (in-batch dedup) and a strided slot list
    dup = torch.cat([rows, rows.flip(0)])
    assert torch.equal(pda_compute_mask(g, dup), torch.cat([first, first.flip(0)]))


def test_batch_lifecycle(orc: Oracle) -> None:
    """grammar/device.py:189-300 semantics: slot reuse, sticky broken rows
    that mask everything until reset, int32 status, is_complete."""
    from bpdecode_b200.grammar.device import CFGConstraintBatch

    g = _dev("xy")
    h = _host("xy")
    toks, _ = PDA_VOCAB
    x, y = toks.index("x"), toks.index("y")
    batch = CFGConstraintBatch(g, capacity=2)
    batch.add("a")
    batch.add("b")
    with pytest.raises(RuntimeError):
        batch.add("c")
    batch.evict("a")
    assert batch.add("c") in (0, 1)
    assert "a" not in batch and "b" in batch and "c" in batch

    st = batch.commit(["b", "c"], torch.tensor([x, toks.index("(")], device="cuda"))
    assert st.tolist() == [1, -1]
    assert batch.is_complete("b") and not batch.is_complete("c")
    assert batch.is_broken("c") and not batch.is_broken("b")
    logits = torch.zeros(2, h.vocab_size, device="cuda")
    batch.apply_mask(["b", "c"], logits)
    assert torch.isneginf(logits[1]).all()
    assert logits[0, h.eos_id].item() == 0.0
    st = batch.commit(["c"], torch.tensor([x], device="cuda"))
    assert st.tolist() == [-1]  # broken is sticky
    batch.reset("c")
    assert not batch.is_broken("c")
    logits = torch.zeros(1, h.vocab_size, device="cuda")
    batch.apply_mask(["c"], logits)
    assert logits[0, y].item() == 0.0 and logits[0, x].item() == 0.0


def test_config4_workload_matches_oracle(orc: Oracle) -> None:
    """Recursive JSON-value grammar, V = 128,256, 256 rows, fp32 N(0,1) logits
    with +3 on { [ \" , : mask (memo cleared at start), argmax, commit for a
    few steps; sampled rows checked against the oracle each step."""
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import CFGConstraintBatch, PdaTensors
    from bpdecode_b200.workloads import BIASED, vocab_large

    v = vocab_large(128_256)
    g = PdaTensors.from_arrays(tables.load_pda("jsonvalue"), v, "cuda")
    g.clear_memo()
    offs = np.zeros(v.size + 1, np.int32)
    np.cumsum([len(t) for t in v.token_bytes], out=offs[1:])
    h = HostPda(tables.load_pda("jsonvalue"), offs,
                np.frombuffer(b"".join(v.token_bytes), np.uint8), v.eos_id)
    B = 256
    batch = CFGConstraintBatch(g, capacity=B)
    for i in range(B):
        batch.add(i)
    bias_ids = [v.token_bytes.index(t) for t in BIASED]
    sample = [0, 97, 255]
    for step in range(4):
        gen = torch.Generator(device="cuda").manual_seed(400 + step)
        logits = torch.randn(B, v.size, generator=gen, device="cuda")
        logits[:, bias_ids] += 3.0
        before = batch._configs.cpu().numpy()
        raw = logits[sample].cpu().numpy()
        batch.apply_mask(list(range(B)), logits)
        tok = logits.argmax(-1)
        batch.commit(list(range(B)), tok)
        for j, r in enumerate(sample):
            want = raw[j:j + 1].copy()
            orc.pda_apply_mask(h, before[r:r + 1], want, float("-inf"))
            assert np.array_equal(logits[r].cpu().numpy(), want[0]), (step, r)
            c = before[r:r + 1].copy()
            orc.pda_advance(h, c, tok[r:r + 1].cpu().numpy())
            assert np.array_equal(batch._configs[r].cpu().numpy(), c[0]), (step, r)


@pytest.mark.parametrize("name", ["paren", "pairs", "jsonvalue_v4096", "schema_v4096"])
def test_fused_step_equals_unfused(name: str) -> None:
    """step_greedy == apply_mask + argmax + commit: masked logits, tokens,
    config rows, broken flags and status, over a few steps with a broken row
    and bf16 logits."""
    from bpdecode_b200.grammar.device import CFGConstraintBatch

    g = _dev(name)
    B = 24
    a = CFGConstraintBatch(g, capacity=B)
    b = CFGConstraintBatch(g, capacity=B)
    ids = list(range(B))
    for i in ids:
        a.add(i)
        b.add(i)
    gen = torch.Generator(device="cuda").manual_seed(7)
    for step in range(8):
        logits = torch.randn(B, g.vocab_size, generator=gen, device="cuda")
        if step == 3:
            logits[5] = float("-inf")  # an all -inf row picks token 0
        if step % 2:
            logits = logits.to(torch.bfloat16)
        la, lb = logits.clone(), logits.clone()
        a.apply_mask(ids, la)
        tok = la.argmax(-1)
        st = a.commit(ids, tok)
        tb = b.step_greedy(ids, lb, chunks_per_row=(1, 2, 5, 16)[step % 4])
        assert torch.equal(la, lb)
        assert torch.equal(tb, tok)
        assert torch.equal(b.last_status, st)
        assert torch.equal(a._configs, b._configs)
        assert torch.equal(a._broken, b._broken)


def test_invalid_tokens_leave_config_unchanged_and_break_the_row() -> None:
    """Fault injection from the host: a token id outside [0, V) is rejected
    (ok = 0), the config-set is unchanged, the row is BROKEN (status -1) and
    masked entirely afterwards; valid rows are unaffected."""
    from bpdecode_b200.grammar.device import CFGConstraintBatch

    g = _dev("jsonvalue_v4096")
    b = CFGConstraintBatch(g, capacity=4)
    for i in range(4):
        b.add(i)
    before = b._configs.clone()
    V = g.vocab_size
    logits = torch.randn(4, V, device="cuda")
    b.apply_mask(list(range(4)), logits)
    good = int(logits[3].argmax())
    status = b.commit([0, 1, 2, 3], torch.tensor([-1, V, V + 9, good], device="cuda"))
    assert status.tolist() == [-1, -1, -1, 1]
    assert torch.equal(b._configs[:3], before[:3])
    assert b._broken[:3].all() and not bool(b._broken[3])
    masked = torch.randn(4, V, device="cuda")
    b.apply_mask(list(range(4)), masked)
    assert torch.isneginf(masked[:3]).all() and not torch.isneginf(masked[3]).all()
