"""Byte-walk path (no tok_next table) and the torch.ops.bpdecode.* schemas on
the GPU, against the reference's goldens and the dense path."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import PDA_VOCAB, golden_npz, small_cases, small_dfa, vocab_of
from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu

SMALL = golden_npz("small.npz")
PDA_GOLDEN = golden_npz("pda.npz")


@pytest.mark.parametrize("vname,pi", small_cases())
def test_walk_ops_match_reference(vname: str, pi: int) -> None:
    from bpdecode_b200 import ops

    fsa = ops.FsaTensors.from_arrays(small_dfa(SMALL, vname, pi), vocab_of(vname)).to("cuda")
    assert fsa.tok_next is None  # stays non-dense: the byte-walk kernels run
    tn = SMALL[f"{vname}/{pi}/tok_next"]
    S, V = tn.shape
    logits = torch.from_numpy(SMALL[f"{vname}/{pi}/logits"]).cuda()
    ops.apply_mask_(logits, fsa, torch.arange(S, dtype=torch.int32, device="cuda"))
    assert np.array_equal(logits.cpu().numpy(), SMALL[f"{vname}/{pi}/masked"])
    st = np.asarray(list(range(S)) + [-1, -2], np.int32)
    bits = ops.compute_mask(fsa, torch.from_numpy(st).cuda()).cpu().numpy().view(np.uint32)
    assert np.array_equal(bits, Oracle().dense_mask_bits(tn, st))
    ss, tt = np.meshgrid(np.arange(-1, S, dtype=np.int32), np.arange(V, dtype=np.int32))
    nxt = ops.advance_state(fsa, torch.from_numpy(ss.ravel()).cuda(),
                            torch.from_numpy(tt.ravel()).cuda())
    assert np.array_equal(nxt.cpu().numpy(), Oracle().dense_advance(tn, ss.ravel(), tt.ravel()))
    assert fsa.tok_next is None


@pytest.mark.parametrize("vname,pi", small_cases()[::3])
def test_torch_ops_schemas_match_reference(vname: str, pi: int) -> None:
    import bpdecode_b200.torch_ops  # noqa: F401
    from bpdecode_b200 import ops

    f = ops.FsaTensors.from_arrays(small_dfa(SMALL, vname, pi), vocab_of(vname)).to("cuda")
    tn = SMALL[f"{vname}/{pi}/tok_next"]
    S = tn.shape[0]
    st = torch.arange(S, dtype=torch.int32, device="cuda")
    logits = torch.from_numpy(SMALL[f"{vname}/{pi}/logits"]).cuda()
    out = torch.ops.bpdecode.apply_mask_(logits, f.trans, f.accept, f.live, f.num_symbols,
                                         f.dead, f.offsets, f.symbols, f.eos_id, st,
                                         float("-inf"))
    assert out.data_ptr() == logits.data_ptr()
    assert np.array_equal(logits.cpu().numpy(), SMALL[f"{vname}/{pi}/masked"])
    bits = torch.ops.bpdecode.compute_mask(f.trans, f.accept, f.live, f.num_symbols, f.dead,
                                           f.offsets, f.symbols, f.eos_id, st)
    assert np.array_equal(bits.cpu().numpy().view(np.uint32), Oracle().dense_mask_bits(tn, st.cpu().numpy()))
    tok = torch.full((S,), 1, dtype=torch.int32, device="cuda")
    nxt = torch.ops.bpdecode.advance_state(f.trans, f.accept, f.live, f.num_symbols, f.dead,
                                           f.offsets, f.symbols, f.eos_id, st, tok)
    assert np.array_equal(nxt.cpu().numpy(), tn[np.arange(S), 1])


@pytest.mark.parametrize("name", ["paren", "pairs", "jsonvalue", "schema"])
def test_torch_ops_pda_schemas(name: str) -> None:
    import bpdecode_b200.torch_ops  # noqa: F401
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import PdaTensors

    toks, eos = PDA_VOCAB
    from bpdecode_b200.tokenizer import Vocabulary

    g = PdaTensors.from_arrays(tables.load_pda(name), Vocabulary.from_tokens(toks, eos), "cuda")
    gargs = (g.accept, g.live, g.edge_offsets, g.edge_kind, g.edge_lo, g.edge_hi, g.edge_dst,
             g.edge_callee, g.root_start, g.root_accept)
    init = torch.ops.bpdecode.pda_init(*gargs)
    rows = PDA_GOLDEN[f"{name}/rows"]
    assert np.array_equal(init.cpu().numpy(), rows[0])
    cfg = torch.from_numpy(rows).cuda()
    logits = torch.zeros(rows.shape[0], g.vocab_size, device="cuda")
    torch.ops.bpdecode.pda_apply_mask_(logits, *gargs, g.tok_offsets, g.tok_bytes, g.eos_id, cfg,
                                       float("-inf"))
    masks = PDA_GOLDEN[f"{name}/masks"][:, 0]
    allowed = ~torch.isneginf(logits).cpu().numpy()
    want = np.asarray([[(m >> t) & 1 for t in range(g.vocab_size)] for m in masks], bool)
    assert np.array_equal(allowed, want)
    ok = torch.ops.bpdecode.pda_advance_state(
        cfg, *gargs, g.tok_offsets, g.tok_bytes, g.eos_id,
        torch.from_numpy(PDA_GOLDEN[f"{name}/tokens"].astype(np.int32)).cuda())
    assert np.array_equal(ok.cpu().numpy(), PDA_GOLDEN[f"{name}/ok"])
