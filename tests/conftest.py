"""Shared test setup: the `gpu` marker, import paths and fixture loaders.

Tests marked `gpu` need a CUDA device (they run on a B200); everything else
runs on the CPU and never launches a kernel.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (runs on the B200 box)")


def pytest_collection_modifyitems(config: pytest.Config, items: list) -> None:
    try:
        import torch

        has_cuda = torch.cuda.is_available()
    except Exception:  # pragma: no cover
        has_cuda = False
    if has_cuda:
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


def golden_npz(name: str) -> dict[str, np.ndarray]:
    with np.load(os.path.join(GOLDEN, name), allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def golden_checksums() -> dict[str, str]:
    with open(os.path.join(GOLDEN, "checksums.json")) as f:
        return json.load(f)


# Vocabularies of the reference's dense tests (tests/golden/make_golden.py).
VOCABS = {
    "dense": (["a", "b", "c", "ab", "ba", "0", "1", "12", "-", ".", "aa", "cafe", "\xc3",
               "<eos>"], 13),
    "cuda": (["a", "b", "c", "ab", "ba", "0", "1", "12", "-", ".", "aa", "café", "é",
              "<eos>"], 13),
    "ops": (["a", "b", "c", "ab", "ba", "0", "1", "12", "-", ".", "aa", "", "<eos>"], 12),
    "soft": (["a", "b", "c", "ab", "ba", "0", "1", "12", "-", ".", "ge", "<eos>"], 11),
    "batch": (["a", "b", "c", "ab", "0", "1", "12", "-", ".", "<eos>"], 9),
}
PDA_VOCAB = (["(", ")", "x", "y", "{", "}", "a", "b", ":", "0", "1", ",", "<eos>"], 12)


def small_cases() -> list[tuple[str, int]]:
    z = golden_npz("small.npz")
    n = len(z["meta/patterns"])
    return [(v, i) for v in VOCABS for i in range(n)]


def small_dfa(z: dict, vname: str, pi: int) -> dict:
    p = f"{vname}/{pi}/"
    num_symbols, dead, start = (int(x) for x in z[p + "meta"])
    return {"trans": z[p + "trans"], "accept": z[p + "accept"], "live": z[p + "live"],
            "lut": z[p + "lut"], "num_symbols": num_symbols, "dead": dead, "start": start}


def vocab_of(vname: str):
    from bpdecode_b200.tokenizer import Vocabulary

    toks, eos = VOCABS[vname]
    return Vocabulary.from_tokens(toks, eos_id=eos)


def reference_src() -> str | None:
    """bpdecode's ``src/`` directory when its source tree is on this machine
    (BPDECODE_REFERENCE, else a checkout named ``reference`` beside this
    repository), for the tests that compare against its Python front-end;
    None elsewhere (those tests skip)."""
    for root in (os.environ.get("BPDECODE_REFERENCE"),
                 os.path.join(os.path.dirname(ROOT), "reference")):
        if root and os.path.isfile(os.path.join(root, "src", "bpdecode", "__init__.py")):
            return os.path.join(root, "src")
    return None


def import_reference():
    """Import bpdecode from its source tree (skips the test when absent)."""
    src = reference_src()
    if src is None:
        pytest.skip("bpdecode's source tree is not on this machine")
    if src not in sys.path:
        sys.path.append(src)
    import bpdecode  # noqa: F401

    return bpdecode
