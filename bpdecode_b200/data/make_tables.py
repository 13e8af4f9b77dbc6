"""Compile the benchmark grammars once, with bpdecode's own front-end, into
``grammars.npz`` (committed beside this script).

Grammar compilation (regex -> byte-class DFA, GBNF / JSON Schema -> rule NFAs)
is a compile-time front-end that this package does not rebuild; the GPU boxes
that run the benchmark have no copy of bpdecode. This script runs where
bpdecode's source tree is importable and stores, per grammar, exactly the
vocabulary-independent tables the device path consumes:

* dense DFAs -- ``fsa_from_dfa`` output (``trans``, ``accept``, ``live``,
  ``num_symbols``, ``dead``, ``start``) plus the 256-entry byte -> symbol-class
  table ``lut`` (``DFA.symbol_of``), so the token symbol sequences of any
  vocabulary are ``lut[token_bytes]``;
* PDAs -- the flattened global-state CSR grammar of ``build_pda_tensors``
  (``grammar/device.py:79-158``) without its vocabulary part.

Usage: ``python -m bpdecode_b200.data.make_tables --ref-src <bpdecode>/src``
"""

from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "grammars.npz")

# The JSON Schema of the reference's HF processor test (tests/test_grammar_hf.py:49-55).
HF_SCHEMA = {
    "type": "object",
    "properties": {"name": {"enum": ["a", "b"]}, "age": {"enum": [0, 1, 2]}},
    "required": ["name", "age"],
    "additionalProperties": False,
}

# Small grammars the reference's own PDA tests use (tests/test_pda_device.py:30-34).
PDA_TEST_GRAMMARS = {
    "paren": 'root ::= "(" root ")" | "x" | "y"',
    "pairs": 'root ::= "{" p ("," p)* "}"\np ::= [a-b] ":" [0-1]',
    "xy": 'root ::= "x" | "y"',
}

# A grammar whose stack records the sequence of open brackets, so greedy rows
# keep reaching config-sets no row held before (the PDA memo-miss workload).
MISS_GRAMMARS = {
    "brackets": 'root ::= item+\nitem ::= "(" item* ")" | "[" item* "]" | "x"',
}


def _dfa_arrays(prefix: str, dfa, out: dict) -> None:
    from bpdecode.fsa import fsa_from_dfa

    f = fsa_from_dfa(dfa)
    out[f"{prefix}/trans"] = np.asarray(f.trans, dtype=np.int32)
    out[f"{prefix}/accept"] = np.asarray(f.accept, dtype=np.uint8)
    out[f"{prefix}/live"] = np.asarray(f.live, dtype=np.uint8)
    out[f"{prefix}/meta"] = np.asarray([f.num_symbols, f.dead, f.start], dtype=np.int32)
    out[f"{prefix}/lut"] = np.asarray([dfa.symbol_of(b) for b in range(256)], dtype=np.int32)


def _pda_arrays(prefix: str, compiled, out: dict) -> None:
    from bpdecode.grammar.device import build_pda_tensors
    from bpdecode.tokenizer import Vocabulary

    g = build_pda_tensors(compiled, Vocabulary.from_tokens(["x"], eos_id=None))
    for name in ("accept", "live", "edge_offsets", "edge_kind", "edge_lo", "edge_hi",
                 "edge_dst", "edge_callee"):
        arr = getattr(g, name).numpy()
        out[f"{prefix}/{name}"] = arr.astype(np.uint8 if arr.dtype == np.uint8 else np.int32)
    out[f"{prefix}/meta"] = np.asarray([g.num_states, g.root_start, g.root_accept],
                                       dtype=np.int32)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", required=True, help="bpdecode's src/ directory")
    args = ap.parse_args()
    sys.path.insert(0, args.ref_src)
    sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

    from bpdecode.grammar.gbnf import parse_gbnf
    from bpdecode.grammar.json_schema import _PRIMITIVES, json_schema_to_grammar
    from bpdecode.grammar.pda import CompiledGrammar
    from bpdecode.grammar.regular import residual_dfa
    from bpdecode.regex import compile_regex

    from bpdecode_b200.workloads import DENSE_PATTERNS, SCHEMA_OBJECT

    out: dict[str, np.ndarray] = {}
    for name, pattern in DENSE_PATTERNS:
        _dfa_arrays(f"dfa/{name}", compile_regex(pattern), out)

    schema_cg = CompiledGrammar.build(json_schema_to_grammar(SCHEMA_OBJECT))
    root = schema_cg.root
    _dfa_arrays("dfa/schema", residual_dfa(schema_cg, root, schema_cg.rules[root].start), out)

    _pda_arrays("pda/jsonvalue",
                CompiledGrammar.build(parse_gbnf(_PRIMITIVES + "\nroot ::= json-value\n")), out)
    _pda_arrays("pda/schema", schema_cg, out)
    _pda_arrays("pda/hf_object", CompiledGrammar.build(json_schema_to_grammar(HF_SCHEMA)), out)
    for name, src in {**PDA_TEST_GRAMMARS, **MISS_GRAMMARS}.items():
        _pda_arrays(f"pda/{name}", CompiledGrammar.build(parse_gbnf(src)), out)

    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT}: {len(out)} arrays")


if __name__ == "__main__":
    main()
