"""The ``*_from`` fused steps (fp32 working values read straight from a
gathered 16-bit or fp32 source, optional fp32 output) against the in-place
steps on an explicit fp32 copy of the same rows: identical tokens, states
(dense) / config rows and broken flags (PDA) and output rows; the source is
never written."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

DTYPES = [torch.bfloat16, torch.float16, torch.float32]


def _dense(V: int, soft: bool):
    from bpdecode_b200 import tables
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import vocab_large

    vocab = vocab_large(V)
    fsas = [FsaTensors.from_arrays(tables.load_dfa(n), vocab).to("cuda")
            for n in ("ipv4", "name", "email")]
    if soft:
        fsas = [f.with_lookahead(3) for f in fsas]
    pair = []
    for _ in range(2):
        b = ConstraintBatch(fsas, capacity=64)
        for i in range(48):
            b.add(i, grammar=i % 3)
        pair.append(b)
    return pair, vocab


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("V,soft", [(32_000, False), (32_000, True), (4099, False)])
@pytest.mark.parametrize("with_out,pad", [(True, 8), (False, 8), (True, 5)])
def test_dense_and_soft_from_equal_fp32_copy(dtype, V, soft, with_out, pad) -> None:
    (a, b), vocab = _dense(V, soft)
    ids = list(range(47, -1, -1))
    gen = torch.Generator(device="cuda").manual_seed(V + soft)
    for step in range(5):
        src = (torch.randn(80, vocab.size + pad, generator=gen, device="cuda") * 2).to(dtype)
        keep = src.clone()
        rows = torch.randperm(80, generator=gen, device="cuda")[:48]
        work = src.index_select(0, rows)[:, : vocab.size].float()
        if soft:
            want = a.soft_step_greedy(ids, work, 1.0)
        else:
            want = a.step_greedy(ids, work)
        out = torch.full((48, vocab.size), 7.0, device="cuda") if with_out else None
        if soft:
            got = b.soft_step_greedy_from(ids, src, rows, out, 1.0)
        else:
            got = b.step_greedy_from(ids, src, rows, out)
        assert torch.equal(src, keep)
        assert torch.equal(got, want), step
        assert torch.equal(a._state, b._state)
        if with_out:
            assert torch.equal(out, work)


@pytest.mark.parametrize("dtype", DTYPES)
@pytest.mark.parametrize("with_out", [True, False])
def test_pda_from_equals_fp32_copy(dtype, with_out) -> None:
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import CFGConstraintBatch, PdaTensors
    from bpdecode_b200.workloads import BIASED, vocab_large

    vocab = vocab_large(8192)
    g = PdaTensors.from_arrays(tables.load_pda("jsonvalue"), vocab, "cuda")
    a, b = CFGConstraintBatch(g, capacity=40), CFGConstraintBatch(g, capacity=40)
    ids = list(range(32))
    for x in (a, b):
        for i in ids:
            x.add(i)
    bias = torch.tensor([vocab.token_bytes.index(t) for t in BIASED], device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(4)
    for step in range(8):
        src = torch.randn(50, vocab.size, generator=gen, device="cuda")
        src[:, bias] += 3.0
        src = src.to(dtype)
        keep = src.clone()
        rows = torch.randperm(50, generator=gen, device="cuda")[:32]
        work = src.index_select(0, rows).float()
        want = a.step_greedy(ids, work)
        out = torch.zeros(32, vocab.size, device="cuda") if with_out else None
        got = b.step_greedy_from(ids, src, rows, out)
        assert torch.equal(src, keep)
        assert torch.equal(got, want), step
        assert torch.equal(a._configs, b._configs) and torch.equal(a._broken, b._broken)
        assert torch.equal(a.last_status, b.last_status)
        if with_out:
            assert torch.equal(out, work)
