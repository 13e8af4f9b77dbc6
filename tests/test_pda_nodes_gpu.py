"""The PDA miss path with its transition cache, on workloads that keep
missing the mask memo, against the reference's own CUDA build.

Every config-set a token walk reaches is interned as a node with 256 byte
transitions filled in on demand, so repeated walks through the same stretch
of a grammar become table walks. Each transition is the bounded closure on
the node's exact content, so masks, tokens and full 266-int config rows must
stay bit-identical to the reference's apply_mask_pda / advance_state_pda
kernels (pda_cuda.cu:72-117). The node table lives in the grammar's memo
buffer; a memo of capacity c holds 4c nodes, so tiny capacities force the
fallbacks (a next set that cannot be interned, a first transition that is not
cached) on every step.
"""

from __future__ import annotations

import pytest
import torch

from oracle.oracle import RefCudaLib

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not RefCudaLib.available(),
                       reason="the reference's CUDA sources were not compiled (oracle/_ref)"),
]


def _grammar(name: str, V: int, memo_capacity: int):
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar import device
    from bpdecode_b200.workloads import vocab_large

    g = device.PdaTensors.from_arrays(tables.load_pda(name), vocab_large(V), "cuda")
    old = device.DEFAULT_MEMO_CAPACITY
    device.DEFAULT_MEMO_CAPACITY = memo_capacity
    try:
        g.mask_memo()  # allocated (and cleared) at this capacity
    finally:
        device.DEFAULT_MEMO_CAPACITY = old
    return g


def _run_against_reference(name: str, V: int, B: int, steps: int, memo_capacity: int,
                           seed: int, bias: float = 0.0, boost_tokens=None) -> int:
    """Greedy generation of B rows on fresh logits every step; returns how
    many distinct config-sets the rows went through."""
    from bpdecode_b200.grammar.device import CFGConstraintBatch
    from bpdecode_b200.workloads import BIASED, vocab_large

    ref = RefCudaLib()
    g = _grammar(name, V, memo_capacity)
    batch = CFGConstraintBatch(g, capacity=B)
    ids = list(range(B))
    for i in ids:
        batch.add(i)
    ref_cfg = batch._configs.clone()
    vocab = vocab_large(V)
    from bpdecode_b200.workloads import token_ids

    boost = torch.tensor(token_ids(vocab, boost_tokens or BIASED), device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(seed)
    seen: set[bytes] = set()
    ref_broken = torch.zeros(B, dtype=torch.bool, device="cuda")
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    ms_mine, ms_ref = [], []
    for step in range(steps):
        for row in batch._configs.cpu().numpy():
            seen.add(row.tobytes())
        logits = torch.randn(B, V, generator=gen, device="cuda")
        if bias:
            logits[:, boost] += bias
        mine, want = logits.clone(), logits.clone()
        ev[0].record()
        tok = batch.step_greedy(ids, mine)
        ev[1].record()
        # the reference's CFGConstraintBatch step (grammar/device.py:252-283)
        ev[2].record()
        ref.pda_apply_mask(g, ref_cfg, want)
        want[ref_broken] = float("-inf")
        ref_tok = want.argmax(-1)
        ok = ref.pda_advance(g, ref_cfg, ref_tok.to(torch.int32))
        ev[3].record()
        torch.cuda.synchronize()
        ms_mine.append(ev[0].elapsed_time(ev[1]))
        ms_ref.append(ev[2].elapsed_time(ev[3]))
        ref_broken |= ok == 0
        assert torch.equal(mine, want), (name, step)
        assert torch.equal(tok, ref_tok), (name, step)
        assert torch.equal(batch._configs, ref_cfg), (name, step)
        assert torch.equal(batch._broken.bool(), ref_broken), (name, step)
    # printed with -s: this library's fused step against the reference's mask +
    # argmax + advance on the same rows, ms per step (mean of the second half)
    h = steps // 2
    print(f"\n{name} V={V} B={B}: step {sum(ms_mine[h:]) / (steps - h):.3f} ms here, "
          f"{sum(ms_ref[h:]) / (steps - h):.3f} ms reference CUDA")
    return len(seen)


@pytest.mark.parametrize("memo_capacity", [4096, 16, 1])
@pytest.mark.parametrize("name", ["schema", "jsonvalue", "pairs", "paren", "hf_object",
                                  "brackets"])
def test_generation_equals_reference_cuda(name: str, memo_capacity: int) -> None:
    from bpdecode_b200.workloads import OPENERS

    bias = {"paren": 2.0, "jsonvalue": 2.0, "brackets": 1.0}.get(name, 0.0)
    distinct = _run_against_reference(name, 4096, 96, 24, memo_capacity, seed=5, bias=bias,
                                      boost_tokens=OPENERS if name == "brackets" else None)
    assert distinct > 1


def test_schema_misses_at_full_vocabulary_equal_reference_cuda() -> None:
    """The miss workload of the benchmark's PDA leg: the JSON-Schema object
    as a PDA, 256 rows, V = 128,256, fp32 N(0, 1), greedy, memo cleared at the
    start; most steps bring config-sets the memo has not seen."""
    distinct = _run_against_reference("schema", 128_256, 256, 24, 4096, seed=9)
    assert distinct > 24


def test_brackets_misses_at_full_vocabulary_equal_reference_cuda() -> None:
    """The benchmark's nesting leg: root ::= item+, item ::= "(" item* ")" |
    "[" item* "]" | "x"; the stack records the open brackets, so nearly every
    row holds a config-set no row held before at every step. 256 rows,
    V = 128,256, fp32 N(0, 1) + 1 on the "(" and "[" tokens."""
    from bpdecode_b200.workloads import OPENERS

    distinct = _run_against_reference("brackets", 128_256, 256, 16, 4096, seed=13, bias=1.0,
                                      boost_tokens=OPENERS)
    assert distinct > 256


def test_paren_nesting_walks_equal_reference_cuda() -> None:
    """paren = "(" paren ")" | "x" | "y" with "(" favoured: the stack deepens
    every step (a new config-set each step) up to the 32-frame cap, where the
    bounded PDA saturates."""
    from bpdecode_b200.grammar.device import CFGConstraintBatch

    ref = RefCudaLib()
    V = 8192
    g = _grammar("paren", V, 4096)
    from bpdecode_b200.workloads import vocab_large

    vocab = vocab_large(V)
    opens = torch.tensor([i for i, t in enumerate(vocab.token_bytes)
                          if t and set(t) <= {ord("(")}], device="cuda")
    assert len(opens) > 0
    B = 32
    batch = CFGConstraintBatch(g, capacity=B)
    ids = list(range(B))
    for i in ids:
        batch.add(i)
    ref_cfg = batch._configs.clone()
    gen = torch.Generator(device="cuda").manual_seed(3)
    for step in range(40):
        logits = torch.randn(B, V, generator=gen, device="cuda")
        logits[:, opens] += 6.0
        mine, want = logits.clone(), logits.clone()
        tok = batch.step_greedy(ids, mine)
        ref.pda_apply_mask(g, ref_cfg, want)
        ref_tok = want.argmax(-1)
        ref.pda_advance(g, ref_cfg, ref_tok.to(torch.int32))
        assert torch.equal(mine, want), step
        assert torch.equal(tok, ref_tok), step
        assert torch.equal(batch._configs, ref_cfg), step
