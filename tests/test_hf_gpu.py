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


def _reference_processor_step(ref, hg, cfgs, broken, scores, input_ids, first: bool,
                              neg_inf: float = float("-inf")) -> None:
    """bpdecode's GrammarLogitsProcessor device backend (hf.py:226-259) on the
    host, with the reference's own compiled PDA (pda_cpu.cpp): commit the last
    token (CFGConstraintBatch.commit, grammar/device.py:268-283), then mask
    padded columns, mask the rows (broken rows entirely) on an fp32 working
    copy and copy it back."""
    import numpy as np

    if not first:
        ok = ref.pda_advance(hg, cfgs, input_ids[:, -1].cpu().numpy().astype(np.int32))
        broken |= ok == 0
    v = hg.vocab_size
    work = scores.float().cpu().numpy()
    work[:, v:] = neg_inf
    part = np.ascontiguousarray(work[:, :v])
    ref.pda_apply_mask(hg, cfgs, part, neg_inf)
    part[broken] = neg_inf
    work[:, :v] = part
    scores.copy_(torch.from_numpy(work).to(scores.device))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("name", ["hf_object", "jsonvalue", "schema"])
def test_grammar_processor_equals_reference_processor(name: str, dtype: torch.dtype) -> None:
    """Our processor and the reference processor's sequence on the same
    scores every step (padded columns, fp32 and bf16), greedy tokens fed back:
    the masked scores are identical."""
    import numpy as np

    from oracle.oracle import HostPda, RefLib

    if not RefLib.available():
        pytest.skip("the reference's CPU sources were not compiled (oracle/_ref)")
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import PdaTensors
    from bpdecode_b200.hf import GrammarLogitsProcessor
    from bpdecode_b200.workloads import vocab_large

    ref = RefLib()
    vocab = vocab_large(4096)
    arrays = tables.load_pda(name)
    lp = GrammarLogitsProcessor(PdaTensors.from_arrays(arrays, vocab), vocab, device="cuda")
    offs = np.zeros(vocab.size + 1, np.int32)
    np.cumsum([len(t) for t in vocab.token_bytes], out=offs[1:])
    hg = HostPda(arrays, offs, np.frombuffer(b"".join(vocab.token_bytes), np.uint8),
                 vocab.eos_id)
    rows, pad = 6, 11
    cfgs = np.stack([ref.pda_init(hg)] * rows)
    broken = np.zeros(rows, bool)
    gen = torch.Generator(device="cuda").manual_seed(17)
    input_ids = torch.zeros(rows, 1, dtype=torch.long, device="cuda")
    for step in range(16):
        scores = (torch.randn(rows, vocab.size + pad, generator=gen, device="cuda") * 2
                  ).to(dtype)
        want = scores.clone()
        _reference_processor_step(ref, hg, cfgs, broken, want, input_ids, step == 0)
        got = lp(input_ids, scores)
        assert got is scores
        assert torch.equal(got.view(torch.int16 if dtype != torch.float32 else torch.int32),
                           want.view(torch.int16 if dtype != torch.float32 else torch.int32)), step
        tok = got.float().argmax(-1)
        input_ids = torch.cat([input_ids, tok.unsqueeze(1)], dim=1)
