"""Load the precompiled benchmark grammars of ``data/grammars.npz``.

The file is produced by ``data/make_tables.py`` with bpdecode's own compiler
front-end; see that script for the exact content. Dense DFAs come back as the
dict :meth:`bpdecode_b200.ops.FsaTensors.from_arrays` takes; PDA grammars as the
dict :func:`bpdecode_b200.grammar.device.PdaTensors.from_arrays` takes.
"""

from __future__ import annotations

import functools
import os

import numpy as np

PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "data", "grammars.npz")


@functools.lru_cache(maxsize=1)
def _npz() -> dict[str, np.ndarray]:
    with np.load(PATH) as z:
        return {k: z[k] for k in z.files}


def names(kind: str) -> list[str]:
    """Grammar names of one kind: ``"dfa"`` or ``"pda"``."""
    return sorted({k.split("/")[1] for k in _npz() if k.startswith(kind + "/")})


def load_dfa(name: str) -> dict:
    z = _npz()
    p = f"dfa/{name}/"
    num_symbols, dead, start = (int(x) for x in z[p + "meta"])
    return {
        "trans": z[p + "trans"], "accept": z[p + "accept"], "live": z[p + "live"],
        "lut": z[p + "lut"], "num_symbols": num_symbols, "dead": dead, "start": start,
    }


def load_pda(name: str) -> dict:
    z = _npz()
    p = f"pda/{name}/"
    num_states, root_start, root_accept = (int(x) for x in z[p + "meta"])
    out = {k: z[p + k] for k in ("accept", "live", "edge_offsets", "edge_kind", "edge_lo",
                                 "edge_hi", "edge_dst", "edge_callee")}
    out.update(num_states=num_states, root_start=root_start, root_accept=root_accept)
    return out
