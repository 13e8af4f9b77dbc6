"""Generate the golden fixtures of tests/golden/ from the reference itself.

Runs where bpdecode's source tree is importable (``--ref-src <bpdecode>/src``)
and its C++ CPU sources are compiled into oracle/_ref/ (``make -C oracle``).
Everything it writes is an output of the reference, never of this package:

* ``small.npz`` -- for every (pattern, vocabulary) pair of the reference's own
  dense tests (tests/test_dense.py, test_ops.py, test_cuda.py, test_soft.py):
  the DFA arrays, the reference's ``build_token_transitions`` table, its dense
  ``apply_mask_`` output on seeded logits, and its ``build_lookahead`` tables
  (k = 1 and 3);
* ``config1.npz`` -- the config-1 decode loop (IPv4, V = 32,000, B = 64, fp32,
  32 steps, logits from a seeded CPU generator) run through the reference's
  ``ConstraintBatch``: argmax token and state of every row at every step, plus
  the sha256 of its ``tok_next``;
* ``checksums.json`` -- sha256 of the reference's ``tok_next`` for the eight
  config-2 regexes at V = 128,256 and the config-3 schema DFA at V = 151,936;
* ``pda.npz`` -- raw 266-int config rows and packed masks of the reference's
  compiled PDA (oracle/_ref) along seeded random walks over the reference's
  test grammars and the JSON-value grammar.

Usage: ``python tests/golden/make_golden.py --ref-src <bpdecode>/src``
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import random
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

# (name, tokens, eos_id) -- the vocabularies of the reference's dense tests
VOCABS = {
    "dense": (["a", "b", "c", "ab", "ba", "0", "1", "12", "-", ".", "aa", "cafe", "\xc3",
               "<eos>"], 13),
    "cuda": (["a", "b", "c", "ab", "ba", "0", "1", "12", "-", ".", "aa", "café", "é",
              "<eos>"], 13),
    "ops": (["a", "b", "c", "ab", "ba", "0", "1", "12", "-", ".", "aa", "", "<eos>"], 12),
    "soft": (["a", "b", "c", "ab", "ba", "0", "1", "12", "-", ".", "ge", "<eos>"], 11),
    "batch": (["a", "b", "c", "ab", "0", "1", "12", "-", ".", "<eos>"], 9),
}
PATTERNS = ["[01]+", "a+b*", "(ab)+", "-?[0-9]+(\\.[0-9]+)?", "a|bc|12", "[a-c]*", "caf(e|)",
            "caf(e|é)", "a[012]+|b0", "age", "[012]+", "a|b|12"]

PDA_VOCAB = (["(", ")", "x", "y", "{", "}", "a", "b", ":", "0", "1", ",", "<eos>"], 12)


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def small(out: dict) -> None:
    import torch
    from bpdecode.ops import FsaTensors, apply_mask_, build_lookahead
    from bpdecode.regex import compile_regex
    from bpdecode.tokenizer import Vocabulary

    sys.path.insert(0, ROOT)
    from bpdecode_b200.ops import dfa_arrays

    for vname, (toks, eos) in VOCABS.items():
        vocab = Vocabulary.from_tokens(toks, eos_id=eos)
        for pi, pat in enumerate(PATTERNS):
            dfa = compile_regex(pat)
            arr = dfa_arrays(dfa)
            key = f"{vname}/{pi}"
            for k in ("trans", "accept", "live", "lut"):
                out[f"{key}/{k}"] = arr[k]
            out[f"{key}/meta"] = np.asarray([arr["num_symbols"], arr["dead"], arr["start"]],
                                            np.int32)
            fsa = FsaTensors.build(pat, vocab, dense=True)
            tn = fsa.tok_next.numpy()
            out[f"{key}/tok_next"] = tn
            g = torch.Generator().manual_seed(1000 + pi)
            logits = torch.randn(tn.shape[0], vocab.size, generator=g)
            states = torch.arange(tn.shape[0], dtype=torch.int32)
            out[f"{key}/logits"] = logits.numpy().copy()
            masked = logits.clone()
            apply_mask_(masked, fsa, states)
            out[f"{key}/masked"] = masked.numpy()
            for k in (1, 3):
                out[f"{key}/lookahead{k}"] = build_lookahead(fsa, k).numpy()
    out["meta/patterns"] = np.asarray(PATTERNS, dtype=object).astype(str)


def config1(out: dict, sums: dict) -> None:
    import torch
    from bpdecode.batch import ConstraintBatch
    from bpdecode.ops import FsaTensors
    from bpdecode.regex import compile_regex
    from bpdecode.tokenizer import Vocabulary

    from bpdecode_b200.workloads import CONFIG1, IPV4_PATTERN, vocab_config1

    v = vocab_config1(0, CONFIG1.vocab_size)
    vocab = Vocabulary(v.token_bytes, v.eos_id)
    fsa = FsaTensors.build(compile_regex(IPV4_PATTERN), vocab, dense=True)
    sums["config1/ipv4/tok_next"] = sha(fsa.tok_next.numpy())
    B, steps = CONFIG1.batch, CONFIG1.steps
    batch = ConstraintBatch(fsa, capacity=B)
    ids = list(range(B))
    for i in ids:
        batch.add(i)
    toks = np.zeros((steps, B), np.int64)
    states = np.zeros((steps, B), np.int32)
    for step in range(steps):
        g = torch.Generator().manual_seed(step)
        logits = torch.randn(B, vocab.size, generator=g) * CONFIG1.sigma
        batch.apply_mask(ids, logits)
        t = logits.argmax(-1)
        nxt = batch.commit(ids, t)
        toks[step] = t.numpy()
        states[step] = nxt.numpy()
    out["config1/tokens"] = toks
    out["config1/states"] = states


def checksums(sums: dict) -> None:
    from bpdecode.grammar.json_schema import json_schema_to_grammar
    from bpdecode.grammar.pda import CompiledGrammar
    from bpdecode.grammar.regular import residual_dfa
    from bpdecode.ops import FsaTensors
    from bpdecode.regex import compile_regex
    from bpdecode.tokenizer import Vocabulary

    from bpdecode_b200.workloads import DENSE_PATTERNS, SCHEMA_OBJECT, vocab_large

    v = vocab_large(128_256)
    vocab = Vocabulary(v.token_bytes, v.eos_id)
    for name, pat in DENSE_PATTERNS:
        fsa = FsaTensors.build(compile_regex(pat), vocab, dense=True)
        sums[f"config2/{name}/tok_next"] = sha(fsa.tok_next.numpy())
    v3 = vocab_large(151_936)
    vocab3 = Vocabulary(v3.token_bytes, v3.eos_id)
    cg = CompiledGrammar.build(json_schema_to_grammar(SCHEMA_OBJECT))
    dfa = residual_dfa(cg, cg.root, cg.rules[cg.root].start)
    fsa = FsaTensors.build(dfa, vocab3, dense=True)
    sums["config3/schema/tok_next"] = sha(fsa.tok_next.numpy())


def pda(out: dict) -> None:
    from bpdecode_b200 import tables
    from bpdecode_b200.workloads import vocab_large
    from oracle.oracle import NCFG, HostPda, RefLib

    ref = RefLib()
    toks, eos = PDA_VOCAB
    tb = [t.encode() for t in toks]

    def host(name: str, token_bytes: list[bytes], eos_id: int) -> HostPda:
        a = tables.load_pda(name)
        offs = np.zeros(len(token_bytes) + 1, np.int32)
        np.cumsum([len(t) for t in token_bytes], out=offs[1:])
        flat = np.frombuffer(b"".join(token_bytes), np.uint8)
        return HostPda(a, offs, flat, eos_id)

    def walks(name: str, g: HostPda, n_walks: int, length: int, seed: int) -> None:
        rng = random.Random(seed)
        rows, masks, tokseq, oks = [], [], [], []
        for _ in range(n_walks):
            cfg = ref.pda_init(g)
            for _ in range(length):
                m = ref.pda_mask_bits(g, cfg)[0]
                rows.append(cfg.copy())
                masks.append(m)
                allowed = [t for t in range(g.vocab_size) if (m[t >> 5] >> (t & 31)) & 1]
                # mostly valid tokens, sometimes an arbitrary one (rejections)
                t = rng.choice(allowed) if allowed and rng.random() < 0.85 else rng.randrange(
                    g.vocab_size)
                c = cfg.reshape(1, NCFG).copy()
                ok = ref.pda_advance(g, c, np.asarray([t], np.int32))[0]
                tokseq.append(t)
                oks.append(ok)
                cfg = c[0]
        out[f"{name}/rows"] = np.asarray(rows, np.int32)
        out[f"{name}/masks"] = np.asarray(masks, np.uint32)
        out[f"{name}/tokens"] = np.asarray(tokseq, np.int64)
        out[f"{name}/ok"] = np.asarray(oks, np.uint8)

    for name in ("paren", "pairs", "xy", "jsonvalue", "schema"):
        walks(name, host(name, tb, eos), 6, 12, 7)
    v = vocab_large(4096)
    walks("jsonvalue_v4096", host("jsonvalue", list(v.token_bytes), v.eos_id), 3, 10, 11)
    walks("schema_v4096", host("schema", list(v.token_bytes), v.eos_id), 3, 24, 13)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-src", required=True)
    ap.add_argument("--only", default="small,config1,checksums,pda")
    args = ap.parse_args()
    sys.path.insert(0, args.ref_src)
    sys.path.insert(0, ROOT)
    only = set(args.only.split(","))
    sums_path = os.path.join(HERE, "checksums.json")
    sums = json.load(open(sums_path)) if os.path.exists(sums_path) else {}
    if "small" in only:
        out: dict = {}
        small(out)
        np.savez_compressed(os.path.join(HERE, "small.npz"), **out)
    if "config1" in only:
        out = {}
        config1(out, sums)
        np.savez_compressed(os.path.join(HERE, "config1.npz"), **out)
    if "checksums" in only:
        checksums(sums)
    if "pda" in only:
        out = {}
        pda(out)
        np.savez_compressed(os.path.join(HERE, "pda.npz"), **out)
    with open(sums_path, "w") as f:
        json.dump(sums, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main()
