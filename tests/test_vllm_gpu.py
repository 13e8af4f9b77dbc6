"""vLLM adapters on the device path, exercised with synthetic inputs (vLLM is
not imported), after the reference's tests/test_vllm.py. The allowed sets
are checked against the oracle's token-transition table of the same DFA."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_npz, small_dfa
from oracle.oracle import Oracle, dfa_with_vocab

pytestmark = pytest.mark.gpu

SMALL = golden_npz("small.npz")
PATTERNS = [str(p) for p in SMALL["meta/patterns"]]
DECIMAL = small_dfa(SMALL, "dense", PATTERNS.index("-?[0-9]+(\\.[0-9]+)?"))
DIGITS012 = small_dfa(SMALL, "dense", PATTERNS.index("[012]+"))
TOKENS = ["0", "1", "2", "3", "4", "5", "6", "7", "8", "9", ".", "-", "x", "</s>"]


def _vocab():
    from bpdecode_b200.tokenizer import Vocabulary

    return Vocabulary.from_tokens(TOKENS, eos_id=len(TOKENS) - 1)


class _Ref:
    """Per-request oracle: state walk over the oracle's tok_next table."""

    def __init__(self, dfa: dict) -> None:
        v = _vocab()
        offs, syms = dfa_with_vocab(dfa, v.token_bytes)
        self.tn = Oracle().build_tok_next(dfa, offs, syms, v.eos_id)
        self.s = int(dfa["start"])

    def accepts(self, tok: int) -> bool:
        return self.s >= 0 and self.tn[self.s, tok] >= 0

    def advance(self, tok: int) -> None:
        self.s = int(self.tn[self.s, tok]) if self.s >= 0 else -1


def _allowed(row: torch.Tensor) -> set[int]:
    return set(np.flatnonzero(~torch.isneginf(row.float()).cpu().numpy()).tolist())


def _greedy(proc, bias: torch.Tensor, max_new: int = 12) -> list[int]:
    past: list[int] = []
    eos = len(TOKENS) - 1
    for _ in range(max_new):
        logits = proc(past, bias.clone())
        nxt = int(logits.argmax())
        if nxt == eos:
            break
        past.append(nxt)
    return past


def test_request_processor_output_is_a_valid_prefix() -> None:
    from bpdecode_b200.vllm import RegexLogitsProcessor

    bias = torch.zeros(len(TOKENS), device="cuda")
    bias[TOKENS.index("x")] = 9.0  # push toward an always-illegal token
    past = _greedy(RegexLogitsProcessor(DECIMAL, _vocab()), bias)
    ref = _Ref(DECIMAL)
    for tok in past:
        assert ref.accepts(tok)
        ref.advance(tok)
    assert TOKENS.index("x") not in past and past


def test_request_processor_tracks_reference_and_padding() -> None:
    from bpdecode_b200.vllm import RegexLogitsProcessor

    proc = RegexLogitsProcessor(DECIMAL, _vocab())
    ref = _Ref(DECIMAL)
    past: list[int] = []
    for tok in [TOKENS.index(c) for c in ("-", "4", ".", "2")]:
        logits = torch.zeros(len(TOKENS) + 3, device="cuda")  # padded lm_head
        proc(past, logits)
        assert torch.isneginf(logits[len(TOKENS):]).all()
        assert _allowed(logits[: len(TOKENS)]) == {i for i in range(len(TOKENS))
                                                   if ref.accepts(i)}
        ref.advance(tok)
        past.append(tok)
    proc(past, torch.zeros(len(TOKENS), device="cuda"))  # consume the final token
    assert proc.is_complete


def test_factory_shares_compiled_grammar() -> None:
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.vllm import RegexLogitsProcessorFactory

    fsa = FsaTensors.from_arrays(DECIMAL, _vocab()).to("cuda")
    factory = RegexLogitsProcessorFactory(_vocab())
    p1, p2 = factory.make(fsa), factory.make(fsa)
    assert p1._batch.fsa is p2._batch.fsa and p1 is not p2


def test_batch_state_masks_only_its_rows() -> None:
    from bpdecode_b200.vllm import BatchConstraintState

    st = BatchConstraintState(_vocab())
    st.add(0, DIGITS012)
    st.add(2, DIGITS012)
    logits = torch.zeros(3, len(TOKENS), device="cuda")
    logits[1, TOKENS.index("x")] = 3.0  # row 1 is some other request
    st.mask(logits)
    for r in (0, 2):
        assert torch.isneginf(logits[r, TOKENS.index("x")])
        assert logits[r, TOKENS.index("0")].item() == 0.0
    assert logits[1, TOKENS.index("x")].item() == 3.0  # untouched


def test_batch_state_lifecycle_matches_per_request_mixed_grammars() -> None:
    """Two patterns in one batch (the reference raises on a second pattern);
    per-row advance and one-launch advance_batch agree; remove + move keep
    the surviving row's state."""
    from bpdecode_b200.vllm import BatchConstraintState

    st = BatchConstraintState(_vocab())
    dfas = {0: DECIMAL, 1: DIGITS012}
    refs = {r: _Ref(d) for r, d in dfas.items()}
    for r, d in dfas.items():
        st.add(r, d)
    plans = {0: [TOKENS.index(c) for c in ("1", "2", "3")],
             1: [TOKENS.index(c) for c in ("2", "0")]}
    gen: dict[int, list[int]] = {0: [], 1: []}
    for step in range(3):
        logits = torch.zeros(2, len(TOKENS), device="cuda")
        st.mask(logits)
        for r in (0, 1):
            assert _allowed(logits[r]) == {i for i in range(len(TOKENS)) if refs[r].accepts(i)}
        rows = [r for r in (0, 1) if step < len(plans[r])]
        for r in rows:
            refs[r].advance(plans[r][step])
            gen[r].append(plans[r][step])
        if step % 2:
            st.advance_batch(rows, torch.tensor([plans[r][step] for r in rows]))
        else:
            for r in rows:
                st.advance(r, gen[r])
    st.remove(0)
    st.move(1, 0)  # vLLM compaction
    logits = torch.zeros(1, len(TOKENS), device="cuda")
    st.mask(logits)
    assert _allowed(logits[0]) == {i for i in range(len(TOKENS)) if refs[1].accepts(i)}
    assert st.is_complete(0)


def test_greedy_toward_eos_completes_a_full_match() -> None:
    from bpdecode_b200.vllm import RegexLogitsProcessor

    proc = RegexLogitsProcessor(DIGITS012, _vocab())
    bias = torch.zeros(len(TOKENS), device="cuda")
    bias[len(TOKENS) - 1] = 9.0
    bias[TOKENS.index("1")] = 10.0
    past = _greedy(proc, bias, max_new=3)
    assert past == [TOKENS.index("1")] * 3
