"""The continuous-batching loop over both grammar paths (config 5 at a small
scale): the fused steps and the unfused drop-in sequence make the same
decisions -- tokens, dense states, PDA config rows and broken flags -- while
requests are retired and admitted every step; admitted rows start from their
grammar's start state / initial config-set."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _grammars(V: int):
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import PdaTensors
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import DENSE_PATTERNS, vocab_large

    vocab = vocab_large(V)
    dense = [FsaTensors.from_arrays(tables.load_dfa(n), vocab).to("cuda")
             for n, _ in DENSE_PATTERNS]
    dense.append(FsaTensors.from_arrays(tables.load_dfa("schema"), vocab).to("cuda"))
    dense = [f.with_lookahead(4) for f in dense]
    pda = PdaTensors.from_arrays(tables.load_pda("jsonvalue"), vocab, "cuda")
    return dense, pda, vocab


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_fused_loop_equals_unfused_loop(dtype: torch.dtype) -> None:
    from bpdecode_b200.serving import MixedServingLoop
    from bpdecode_b200.workloads import DENSE_PATTERNS

    dense, pda, vocab = _grammars(4096)
    rows = 96
    loops = [MixedServingLoop(rows, dense, pda, n_regex=len(DENSE_PATTERNS), seed=5, fused=f)
             for f in (True, False)]
    assert (loops[0].kind == loops[1].kind).all() and 0 < int(loops[0].kind.sum()) < rows
    gen = torch.Generator(device="cuda").manual_seed(11)
    for step in range(12):
        logits = (torch.randn(rows, vocab.size, generator=gen, device="cuda") * 2).to(dtype)
        keep = logits.clone()
        ta = loops[0].step(logits)
        tb = loops[1].step(logits)
        assert torch.equal(logits, keep)  # the model's logits are not modified
        assert torch.equal(ta, tb), step
        for x, y in zip(loops[0].states(), loops[1].states()):
            assert torch.equal(x, y), step
        ra = loops[0].turnover()
        rb = loops[1].turnover()
        assert ra == rb and len(ra) == round(rows * 0.1)


def test_admitted_rows_start_fresh() -> None:
    from bpdecode_b200.serving import MixedServingLoop
    from bpdecode_b200.workloads import DENSE_PATTERNS

    dense, pda, vocab = _grammars(4096)
    loop = MixedServingLoop(64, dense, pda, n_regex=len(DENSE_PATTERNS), seed=9)
    for _ in range(3):
        loop.step(torch.randn(64, vocab.size, device="cuda"))
    changed = loop.turnover()
    init = pda.init_config()
    for r in changed:
        q = int(loop.req[r])
        if loop.kind[r] == 0:
            g = loop.dense._grammar_of[q]
            assert loop.dense.state_of(q) == loop.dense._t.starts[g]
        else:
            slot = loop.pda._slot_of[q]
            assert torch.equal(loop.pda._configs[slot], init)
            assert not bool(loop.pda._broken[slot])
