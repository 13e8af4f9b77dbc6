"""Checkpoint / resume of the batch state: a batch restored from
``state_dict()`` (through ``torch.save`` / ``torch.load``) continues exactly
like the batch that never stopped -- same tokens, same automaton states and
config-set rows -- and keeps its slot bookkeeping (evict / add afterwards)."""

from __future__ import annotations

import io

import pytest
import torch

from conftest import PDA_VOCAB, golden_npz, small_dfa, vocab_of

pytestmark = pytest.mark.gpu

SMALL = golden_npz("small.npz")


def _roundtrip(sd: dict) -> dict:
    buf = io.BytesIO()
    torch.save(sd, buf)
    buf.seek(0)
    return torch.load(buf, weights_only=False)


def _dense_batch():
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.ops import FsaTensors

    v = vocab_of("dense")
    fsas = [FsaTensors.from_arrays(small_dfa(SMALL, "dense", i), v).to("cuda")
            for i in range(len(SMALL["meta/patterns"]))]
    return ConstraintBatch(fsas, capacity=3 * len(fsas)), fsas, v


def test_dense_batch_resumes_identically() -> None:
    a, fsas, v = _dense_batch()
    ids = [(g, r) for g in range(len(fsas)) for r in range(3)]
    for i in ids:
        a.add(i, grammar=i[0])
    gen = torch.Generator().manual_seed(3)
    for _ in range(3):
        a.step_greedy(ids, torch.randn(len(ids), v.size, generator=gen).cuda())
    sd = _roundtrip(a.state_dict())
    b, _, _ = _dense_batch()
    b.load_state_dict(sd)
    assert [b.state_of(i) for i in ids] == [a.state_of(i) for i in ids]
    for _ in range(4):
        logits = torch.randn(len(ids), v.size, generator=gen).cuda()
        ta = a.step_greedy(ids, logits.clone())
        tb = b.step_greedy(ids, logits.clone())
        assert torch.equal(ta, tb)
        assert [b.state_of(i) for i in ids] == [a.state_of(i) for i in ids]
    # bookkeeping survives: a restored batch evicts and re-adds like the original
    for x in (a, b):
        x.evict(ids[0])
        x.add(("new", 0), grammar=1)
    assert a._slot_of == b._slot_of
    assert torch.equal(a._state, b._state)


def test_dense_state_dict_rejects_other_batches() -> None:
    from bpdecode_b200.batch import ConstraintBatch

    a, fsas, _ = _dense_batch()
    with pytest.raises(ValueError):
        ConstraintBatch(fsas, capacity=a.capacity + 1).load_state_dict(a.state_dict())
    other = sorted(fsas, key=lambda f: f.num_states)
    if [f.num_states for f in other] != [f.num_states for f in fsas]:
        with pytest.raises(ValueError):
            ConstraintBatch(other, capacity=a.capacity).load_state_dict(a.state_dict())


def _pda_batch(cap: int = 6):
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import CFGConstraintBatch, PdaTensors
    from bpdecode_b200.tokenizer import Vocabulary

    toks, eos = PDA_VOCAB
    v = Vocabulary.from_tokens(toks, eos_id=eos)
    g = PdaTensors.from_arrays(tables.load_pda("pairs"), v, "cuda")
    return CFGConstraintBatch(g, capacity=cap), v


def test_pda_batch_resumes_identically() -> None:
    a, v = _pda_batch()
    ids = list(range(6))
    for i in ids:
        a.add(i)
    gen = torch.Generator().manual_seed(8)
    for _ in range(3):
        a.step_greedy(ids, torch.randn(len(ids), v.size, generator=gen).cuda())
    sd = _roundtrip(a.state_dict())
    b, _ = _pda_batch()
    b.load_state_dict(sd)
    assert torch.equal(a._configs, b._configs) and torch.equal(a._broken, b._broken)
    for _ in range(4):
        logits = torch.randn(len(ids), v.size, generator=gen).cuda()
        ta = a.step_greedy(ids, logits.clone())
        tb = b.step_greedy(ids, logits.clone())
        assert torch.equal(ta, tb)
        assert torch.equal(a._configs, b._configs) and torch.equal(a._broken, b._broken)
    with pytest.raises(ValueError):
        _pda_batch(cap=7)[0].load_state_dict(sd)
