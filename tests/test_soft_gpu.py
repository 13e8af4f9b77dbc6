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
