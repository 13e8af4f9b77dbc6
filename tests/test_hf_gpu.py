"""HF processors on the GPU (the reference's tests/test_grammar_hf.py and
test_hf.py conventions, with precompiled tables)."""

from __future__ import annotations

import json

import pytest
import torch

from conftest import golden_npz, small_dfa, vocab_of

pytestmark = pytest.mark.gpu

TOKENS = ["{", "}", "[", "]", '"', ":", ",", " ", "a", "b", "c", "0", "1", "2", "true", "false",
          "null", "name", "age", "</s>"]


def _greedy(lp, vocab, bias: torch.Tensor, max_new: int = 40, dtype=torch.float32) -> str:
    """Argmax decode; ties broken toward the longer token (test_grammar_hf.py:27-46)."""
    input_ids = torch.zeros(1, 1, dtype=torch.long, device="cuda")
    out: list[int] = []
    for _ in range(max_new):
        scores = lp(input_ids, bias.clone().unsqueeze(0).to(dtype))[0].float()
        best = max((i for i in range(vocab.size) if scores[i].item() > -1e30),
                   key=lambda i: (scores[i].item(), len(TOKENS[i])))
        if best == vocab.eos_id:
            break
        out.append(best)
        input_ids = torch.cat([input_ids, torch.tensor([[best]], device="cuda")], dim=1)
    return "".join(TOKENS[i] for i in out)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_grammar_processor_generates_valid_json(dtype: torch.dtype) -> None:
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import PdaTensors
    from bpdecode_b200.hf import GrammarLogitsProcessor
    from bpdecode_b200.tokenizer import Vocabulary

    vocab = Vocabulary.from_tokens(TOKENS, eos_id=len(TOKENS) - 1)
    g = PdaTensors.from_arrays(tables.load_pda("hf_object"), vocab)
    lp = GrammarLogitsProcessor(g, vocab, device="cuda")
    assert lp.backend == "device"
    bias = torch.zeros(vocab.size, device="cuda")
    bias[TOKENS.index(" ")] = -5.0
    obj = json.loads(_greedy(lp, vocab, bias, dtype=dtype))
    assert set(obj) == {"name", "age"}
    assert lp.is_complete(0)


def test_grammar_processor_masks_padded_columns() -> None:
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import PdaTensors
    from bpdecode_b200.hf import GrammarLogitsProcessor
    from bpdecode_b200.tokenizer import Vocabulary

    vocab = Vocabulary.from_tokens(TOKENS, eos_id=len(TOKENS) - 1)
    lp = GrammarLogitsProcessor(PdaTensors.from_arrays(tables.load_pda("hf_object"), vocab),
                                vocab, device="cuda")
    scores = torch.zeros(2, vocab.size + 12, device="cuda")
    lp(torch.zeros(2, 1, dtype=torch.long, device="cuda"), scores)
    assert torch.isneginf(scores[:, vocab.size:]).all()
    allowed = (~torch.isneginf(scores[0, :vocab.size])).nonzero().flatten().tolist()
    assert allowed == [TOKENS.index("{")]
    with pytest.raises(ValueError):
        GrammarLogitsProcessor(PdaTensors.from_arrays(tables.load_pda("xy"), vocab), vocab,
                               device="cpu")


@pytest.mark.parametrize("soft_k", [None, 3])
def test_regex_processor_matches_batch(soft_k) -> None:
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.hf import RegexLogitsProcessor
    from bpdecode_b200.ops import FsaTensors

    SMALL = golden_npz("small.npz")
    patterns = list(SMALL["meta/patterns"])
    dfa = small_dfa(SMALL, "dense", patterns.index("-?[0-9]+(\\.[0-9]+)?"))
    v = vocab_of("dense")
    lp = RegexLogitsProcessor(dfa, v, device="cuda", soft_k=soft_k, alpha=0.5)
    fsa = FsaTensors.from_arrays(dfa, v).to("cuda")
    if soft_k:
        fsa = fsa.with_lookahead(soft_k)
    ref = ConstraintBatch(fsa, capacity=2)
    ref.add(0)
    ref.add(1)
    gen = torch.Generator(device="cuda").manual_seed(3)
    input_ids = torch.zeros(2, 1, dtype=torch.long, device="cuda")
    for step in range(6):
        scores = torch.randn(2, v.size, generator=gen, device="cuda")
        want = scores.clone()
        if step:
            ref.commit([0, 1], input_ids[:, -1])
        if soft_k:
            ref.apply_soft([0, 1], want, 0.5)
        else:
            ref.apply_mask([0, 1], want)
        got = lp(input_ids, scores)
        assert torch.equal(got, want)
        tok = got.argmax(-1)
        input_ids = torch.cat([input_ids, tok.unsqueeze(1)], dim=1)
