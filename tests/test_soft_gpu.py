"""Soft lookahead on the GPU: the sum-product table within 1e-5 relative of the
reference (fp32 torch) and of the double-precision oracle; the per-step
application against the oracle; alpha = 0 is exactly hard masking
(tests/test_soft.py semantics)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_npz, small_cases, small_dfa, vocab_of
from oracle.oracle import Oracle

pytestmark = pytest.mark.gpu

SMALL = golden_npz("small.npz")
RTOL = 1e-5  # the tolerance the soft-lookahead scores must meet, relative, fp32


def _fsa(vname: str, pi: int):
    from bpdecode_b200.ops import FsaTensors

    return FsaTensors.from_arrays(small_dfa(SMALL, vname, pi), vocab_of(vname)).to("cuda")


def _close(got: np.ndarray, want: np.ndarray) -> None:
    assert np.array_equal(np.isneginf(got), np.isneginf(want))
    fin = np.isfinite(want)
    assert np.isfinite(got[fin]).all()
    np.testing.assert_allclose(got[fin], want[fin], rtol=RTOL, atol=1e-6)


@pytest.mark.parametrize("vname,pi", small_cases())
@pytest.mark.parametrize("k", [1, 3])
def test_lookahead_matches_reference(vname: str, pi: int, k: int) -> None:
    from bpdecode_b200.ops import build_lookahead

    fsa = _fsa(vname, pi)
    fsa.dense_tables()
    got = build_lookahead(fsa, k).cpu().numpy()
    _close(got, SMALL[f"{vname}/{pi}/lookahead{k}"])


@pytest.mark.parametrize("name", ["ipv4", "name", "uuid"])
def test_lookahead_full_vocab_matches_oracle(name: str) -> None:
    from bpdecode_b200 import tables
    from bpdecode_b200.ops import FsaTensors, build_lookahead
    from bpdecode_b200.workloads import vocab_large

    dfa = tables.load_dfa(name)
    v = vocab_large(128_256)
    fsa = FsaTensors.from_arrays(dfa, v).to("cuda")
    tn = fsa.dense_tables()[0]
    got = build_lookahead(fsa, 4).cpu().numpy()
    want = Oracle().build_lookahead(tn.cpu().numpy(), dfa["accept"], dfa["live"], v.eos_id, 4)
    _close(got, want)


@pytest.mark.parametrize("alpha", [0.0, 1.0, -0.5, 2.5])
def test_apply_soft_matches_oracle(alpha: float) -> None:
    from bpdecode_b200.ops import apply_mask_, apply_soft_

    orc = Oracle()
    for vname, pi in small_cases()[::4]:
        fsa = _fsa(vname, pi).with_lookahead(3)
        S, V = fsa.num_states, fsa.vocab_size
        st = np.asarray([s % (S + 1) - 1 for s in range(2 * S + 1)], np.int32)
        base = torch.randn(st.size, V, generator=torch.Generator().manual_seed(pi))
        want = base.numpy().copy()
        orc.apply_soft(want, fsa.lookahead.cpu().numpy(), st, alpha)
        got = base.cuda()
        apply_soft_(got, fsa, torch.from_numpy(st).cuda(), alpha)
        got = got.cpu().numpy()
        _close(got, want)
        if alpha == 0.0:
            # exactly hard masking where the lookahead is finite; a token the
            # hard mask allows but whose continuations all die within k steps
            # is -inf in the lookahead table too (the reference's semantics)
            hard = base.cuda()
            apply_mask_(hard, fsa, torch.from_numpy(st).cuda())
            hard = hard.cpu().numpy()
            fin = np.isfinite(got)
            assert np.array_equal(got[fin], hard[fin])
            assert np.isneginf(got[np.isneginf(hard)]).all()


def test_batch_apply_soft_mixed_grammars() -> None:
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.ops import apply_soft_

    patterns = list(SMALL["meta/patterns"])
    fsas = [_fsa("soft", i).with_lookahead(3) for i in range(len(patterns))]
    batch = ConstraintBatch(fsas, capacity=len(fsas))
    for g in range(len(fsas)):
        batch.add(g, grammar=g)
    base = torch.randn(len(fsas), fsas[0].vocab_size, device="cuda")
    got = base.clone()
    batch.apply_soft(list(range(len(fsas))), got, alpha=1.5)
    for g, f in enumerate(fsas):
        want = base[g:g + 1].clone()
        apply_soft_(want, f, torch.tensor([f.start], dtype=torch.int32, device="cuda"), 1.5)
        assert torch.equal(got[g:g + 1], want)


def _soft_big(name: str = "ipv4", V: int = 128_256, k: int = 3):
    from bpdecode_b200 import tables
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import vocab_large

    fsa = FsaTensors.from_arrays(tables.load_dfa(name), vocab_large(V)).to("cuda")
    return fsa.with_lookahead(k)


def _soft_states(fsa, rows: int, seed: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(seed)
    st = torch.randint(0, fsa.num_states, (rows,), generator=g, dtype=torch.int32)
    st[::7] = -1  # BROKEN rows: every entry -inf
    return st.cuda()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("V", [128_256, 50_001])
def test_apply_soft_vector_path_matches_fp32_formula(dtype: torch.dtype, V: int) -> None:
    """Vector (V % 4 == 0) and scalar (odd V) paths: -inf where the bias is
    -inf, else x + alpha * bias in fp32 rounded once to the logits dtype."""
    from bpdecode_b200.ops import apply_soft_

    fsa = _soft_big(V=V)
    st = _soft_states(fsa, 40, V)
    base = (torch.randn(40, V, device="cuda") * 3).to(dtype)
    for alpha in (0.0, 0.75):
        got = base.clone()
        apply_soft_(got, fsa, st, alpha)
        bias = torch.full((40, V), float("-inf"), device="cuda")
        ok = st >= 0
        bias[ok] = fsa.lookahead[st[ok].long()]
        x = base.double()
        want = torch.where(bias == float("-inf"), torch.full_like(x, float("-inf")),
                           x if alpha == 0.0 else x + alpha * bias.double()).to(dtype)
        if alpha == 0.0:
            assert torch.equal(got, want)
        else:
            torch.testing.assert_close(got.float(), want.float(), rtol=RTOL if dtype ==
                                       torch.float32 else 1e-2, atol=1e-6)
            assert torch.equal(torch.isneginf(got), torch.isneginf(want))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16])
@pytest.mark.parametrize("ctas", [0, 1, 3, 16])
@pytest.mark.parametrize("V,pad", [(128_256, 0), (128_256, 64), (50_001, 3)])
def test_soft_step_greedy_equals_unfused(dtype: torch.dtype, ctas: int, V: int,
                                         pad: int) -> None:
    """The fused soft step gives exactly apply_soft_ + argmax + advance_state:
    same biased logits, same tokens (first maximal index), same next states."""
    from bpdecode_b200.ops import advance_state, apply_soft_, soft_step_greedy_

    fsa = _soft_big(V=V)
    rows = 96
    st = _soft_states(fsa, rows, 3 * V + pad)
    store = torch.randn(rows, V + pad, device="cuda").to(dtype)
    store[5, 100:2000] = store[5, 100:2000].abs().max()  # ties: the first wins
    base = store[:, :V]
    for alpha in (0.0, 1.0, -0.5):
        want = base.clone()
        apply_soft_(want, fsa, st, alpha)
        want_tok = want.argmax(-1)
        want_next = advance_state(fsa, st, want_tok)
        got_store = store.clone()
        got = got_store[:, :V]
        pool = st.clone()
        tok, nxt = soft_step_greedy_(got, fsa, pool, None, alpha, ctas)
        assert torch.equal(got, want)
        assert torch.equal(got_store[:, V:], store[:, V:])
        live = torch.isfinite(want.float()).any(-1) | torch.isnan(want.float()).any(-1)
        assert torch.equal(tok[live], want_tok[live])
        assert torch.equal(nxt[live], want_next[live].to(torch.int32))
        assert torch.equal(pool, nxt)


def test_batch_soft_step_greedy_slots() -> None:
    """ConstraintBatch.soft_step_greedy on a permuted subset of sequences
    equals apply_soft + argmax + commit through the same batch API."""
    from bpdecode_b200.batch import ConstraintBatch

    fsa = _soft_big("name")
    a = ConstraintBatch(fsa, capacity=64)
    b = ConstraintBatch(fsa, capacity=64)
    for i in range(64):
        a.add(i)
        b.add(i)
    g = torch.Generator(device="cuda").manual_seed(11)
    for step in range(6):
        ids = [i for i in range(63, -1, -1) if (i + step) % 3]
        logits = torch.randn(len(ids), fsa.vocab_size, device="cuda", generator=g,
                             dtype=torch.bfloat16)
        ref = logits.clone()
        b.apply_soft(ids, ref, alpha=1.0)
        want = ref.argmax(-1)
        b.commit(ids, want)
        got = a.soft_step_greedy(ids, logits, alpha=1.0)
        assert torch.equal(logits, ref)
        live = torch.isfinite(ref.float()).any(-1)
        assert torch.equal(got[live], want[live])
        for i in ids:
            if a.state_of(i) >= 0 or b.state_of(i) >= 0:
                assert a.state_of(i) == b.state_of(i)
