"""The compile-time glue of the drop-in against bpdecode's own Python code.

Runs where bpdecode's source tree is on the machine (its front-end compiles
the grammars); skipped elsewhere. Checks, array for array:

* ``build_pda_tensors`` (grammar/device.py:79-158) on every benchmark and
  test grammar, at a small and a synthetic large vocabulary;
* the precompiled tables the GPU tests and the benchmark load
  (``bpdecode_b200/data/grammars.npz``) against a fresh build by the
  reference;
* ``FsaTensors.build`` (ops.py:127-140, with its dense ``tok_next``) and
  ``GrammarCache.get`` (batch.py:103-112) on the eight serving-scale
  regexes and the reference's test patterns.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import import_reference

PDA_FIELDS = ("accept", "live", "edge_offsets", "edge_kind", "edge_lo", "edge_hi", "edge_dst",
              "edge_callee", "tok_offsets", "tok_bytes")
FSA_FIELDS = ("trans", "accept", "live", "offsets", "symbols")


def _grammars():
    """(name, CompiledGrammar) of every PDA grammar the package precompiles."""
    import_reference()
    from bpdecode.grammar.gbnf import parse_gbnf
    from bpdecode.grammar.json_schema import _PRIMITIVES, json_schema_to_grammar
    from bpdecode.grammar.pda import CompiledGrammar

    from bpdecode_b200.data.make_tables import HF_SCHEMA, MISS_GRAMMARS, PDA_TEST_GRAMMARS
    from bpdecode_b200.workloads import SCHEMA_OBJECT

    out = [("jsonvalue", CompiledGrammar.build(parse_gbnf(_PRIMITIVES + "\nroot ::= json-value\n"))),
           ("schema", CompiledGrammar.build(json_schema_to_grammar(SCHEMA_OBJECT))),
           ("hf_object", CompiledGrammar.build(json_schema_to_grammar(HF_SCHEMA)))]
    out += [(n, CompiledGrammar.build(parse_gbnf(src)))
            for n, src in {**PDA_TEST_GRAMMARS, **MISS_GRAMMARS}.items()]
    return out


def _vocabs():
    from bpdecode.tokenizer import Vocabulary as RefVocab

    from bpdecode_b200.workloads import vocab_large

    small = ["(", ")", "x", "y", "{", "}", "a", "b", ":", "0", "1", ",", '"', "tr", "ue",
             "null", "<eos>"]
    big = vocab_large(4096)
    return [RefVocab.from_tokens(small, eos_id=len(small) - 1),
            RefVocab(token_bytes=big.token_bytes, eos_id=big.eos_id)]


def test_build_pda_tensors_equals_reference() -> None:
    import_reference()
    from bpdecode.grammar.device import build_pda_tensors as ref_build

    from bpdecode_b200.grammar.device import build_pda_tensors

    for name, cg in _grammars():
        for vocab in _vocabs():
            want = ref_build(cg, vocab)
            got = build_pda_tensors(cg, vocab)
            for f in ("num_states", "root_start", "root_accept", "vocab_size", "eos_id"):
                assert getattr(got, f) == getattr(want, f), (name, f)
            for f in PDA_FIELDS:
                a, b = getattr(got, f), getattr(want, f)
                assert a.dtype == b.dtype and torch.equal(a, b), (name, f)


def test_precompiled_pda_tables_equal_a_fresh_reference_build() -> None:
    import_reference()
    from bpdecode.grammar.device import build_pda_tensors as ref_build
    from bpdecode.tokenizer import Vocabulary as RefVocab

    from bpdecode_b200 import tables

    for name, cg in _grammars():
        want = ref_build(cg, RefVocab.from_tokens(["x"], eos_id=None))
        got = tables.load_pda(name)
        for f in ("num_states", "root_start", "root_accept"):
            assert got[f] == getattr(want, f), (name, f)
        for f in PDA_FIELDS[:8]:
            assert np.array_equal(np.asarray(got[f]), getattr(want, f).numpy()), (name, f)


PATTERNS = ["[01]+", "a+b*", "(ab)+", "-?[0-9]+(\\.[0-9]+)?", "a|bc|12", "caf(e|é)"]


def _fsa_equal(got, want, what: str) -> None:
    for f in FSA_FIELDS:
        a, b = getattr(got, f), getattr(want, f)
        assert torch.equal(a.to(b.dtype), b), (what, f)
    for f in ("num_symbols", "dead", "eos_id", "start", "accepting", "num_states",
              "vocab_size"):
        assert getattr(got, f) == getattr(want, f), (what, f)
    assert (got.tok_next is None) == (want.tok_next is None), what
    if want.tok_next is not None:
        assert torch.equal(got.tok_next, want.tok_next), what


def test_fsa_build_equals_reference() -> None:
    import_reference()
    from bpdecode.ops import FsaTensors as RefFsa
    from bpdecode.tokenizer import Vocabulary as RefVocab

    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import DENSE_PATTERNS, vocab_large

    v = vocab_large(2048)
    big = RefVocab(token_bytes=v.token_bytes, eos_id=v.eos_id)
    small = RefVocab.from_tokens(["a", "b", "c", "ab", "ba", "0", "1", "12", "-", ".", "aa",
                                  "café", "é", "<eos>"], eos_id=13)
    for pattern in [p for _, p in DENSE_PATTERNS] + PATTERNS:
        for vocab in (small, big):
            for dense in (True, False):
                want = RefFsa.build(pattern, vocab, dense=dense)
                got = FsaTensors.build(pattern, vocab, dense=dense)
                _fsa_equal(got, want, f"{pattern} dense={dense}")


def test_grammar_cache_get_equals_reference_and_is_shared() -> None:
    import_reference()
    from bpdecode.batch import GrammarCache as RefCache
    from bpdecode.tokenizer import Vocabulary as RefVocab

    from bpdecode_b200.batch import GrammarCache

    vocab = RefVocab.from_tokens(["a", "b", "c", "ab", "0", "1", "12", "-", ".", "<eos>"],
                                 eos_id=9)
    ours, ref = GrammarCache(vocab, max_size=2), RefCache(vocab, max_size=2)
    for p in ("[01]+", "-?[0-9]+(\\.[0-9]+)?", "(ab)+"):
        _fsa_equal(ours.get(p), ref.get(p), p)
    # the reference's tests/test_batch.py:26-35 semantics: shared, LRU of max_size
    a1 = ours.get("[01]+")
    assert ours.get("[01]+") is a1
    ours.get("(ab)+")
    ours.get("a|b|12")  # evicts the least recently used
    assert len(ours) == 2
    assert ours.get("(ab)+") is not None and len(ours) == 2
