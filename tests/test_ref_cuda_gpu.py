"""The kernels against the reference's own CUDA build (mask_cuda.cu and
pda_cuda.cu compiled unchanged for sm_100a into oracle/_ref/libbpdref_cuda.so)
on the same device inputs: packed masks, masked fp32 logits, ok flags and full
266-int config rows must be bit-identical. The last test does it at config 4's
full size (256 rows, V = 128,256) and prints both sides' device times."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden_npz, small_cases, small_dfa, vocab_of
from oracle.oracle import RefCudaLib

pytestmark = [
    pytest.mark.gpu,
    pytest.mark.skipif(not RefCudaLib.available(),
                       reason="the reference's CUDA sources were not compiled (oracle/_ref)"),
]

SMALL = golden_npz("small.npz")
PDA_GOLDEN = golden_npz("pda.npz")


def _pda(name: str, V: int):
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import PdaTensors
    from bpdecode_b200.workloads import vocab_large

    return PdaTensors.from_arrays(tables.load_pda(name), vocab_large(V), "cuda")


def _walked_rows(g, n: int, steps: int, seed: int) -> torch.Tensor:
    """n config-sets after up to `steps` greedy steps on random logits (a mix
    of fresh, deep, saturated and broken sets)."""
    from bpdecode_b200.grammar.device import CFGConstraintBatch

    b = CFGConstraintBatch(g, capacity=n)
    ids = list(range(n))
    for i in ids:
        b.add(i)
    gen = torch.Generator(device="cuda").manual_seed(seed)
    rows = [b._configs.clone()]
    for _ in range(steps):
        b.step_greedy(ids, torch.randn(n, g.vocab_size, generator=gen, device="cuda") * 3)
        rows.append(b._configs.clone())
    return torch.cat(rows)


@pytest.mark.parametrize("name", ["jsonvalue", "schema"])
def test_pda_mask_apply_advance_equal_reference_cuda(name: str) -> None:
    from bpdecode_b200.grammar.device import (pda_advance_state, pda_apply_mask_,
                                              pda_compute_mask)

    ref = RefCudaLib()
    g = _pda(name, 4096)
    cfg = torch.cat([torch.from_numpy(PDA_GOLDEN[f"{name}_v4096/rows"]).cuda(),
                     _walked_rows(g, 24, 6, seed=7)])
    want = ref.pda_mask(g, cfg)
    for memo in (True, False):
        assert torch.equal(pda_compute_mask(g, cfg, memo=memo), want), memo
    gen = torch.Generator(device="cuda").manual_seed(3)
    logits = torch.randn(cfg.shape[0], g.vocab_size, generator=gen, device="cuda")
    mine = logits.clone()
    ref.pda_apply_mask(g, cfg, logits)
    pda_apply_mask_(mine, g, cfg)
    assert torch.equal(mine, logits)
    # tokens: mostly allowed ones (the argmax of the masked logits), some random
    tok = mine.argmax(-1).to(torch.int32)
    tok[::3] = torch.randint(0, g.vocab_size, (len(tok[::3]),), generator=gen, device="cuda",
                             dtype=torch.int32)
    a, b = cfg.clone(), cfg.clone()
    ok_ref = ref.pda_advance(g, a, tok)
    ok = pda_advance_state(b, g, tok)
    assert torch.equal(ok, ok_ref)
    assert torch.equal(a, b)


@pytest.mark.parametrize("vname,pi", small_cases()[::2])
def test_walk_mask_and_advance_equal_reference_cuda(vname: str, pi: int) -> None:
    from bpdecode_b200 import ops

    ref = RefCudaLib()
    fsa = ops.FsaTensors.from_arrays(small_dfa(SMALL, vname, pi), vocab_of(vname)).to("cuda")
    S = int(fsa.accept.numel())
    V = int(fsa.offsets.numel()) - 1
    st = torch.tensor(list(range(S)) + [-1, -2], dtype=torch.int32, device="cuda")
    assert torch.equal(ops.compute_mask(fsa, st), ref.compute_mask(fsa, st))
    ss, tt = np.meshgrid(np.arange(-1, S, dtype=np.int32), np.arange(V, dtype=np.int32))
    s = torch.from_numpy(ss.ravel()).cuda()
    t = torch.from_numpy(tt.ravel()).cuda()
    assert torch.equal(ops.advance_state(fsa, s, t), ref.advance_state(fsa, s, t))


def test_config4_apply_mask_equals_reference_cuda_at_full_size() -> None:
    """Config 4's shape: 256 rows of the JSON-value grammar at V = 128,256 --
    initial and walked config-sets -- masked in place by the reference's
    apply_mask_pda kernel and by this library's memo pipeline + apply."""
    from bpdecode_b200.grammar.device import pda_apply_mask_
    from bpdecode_b200.workloads import BIASED, vocab_large

    ref = RefCudaLib()
    V = 128256
    g = _pda("jsonvalue", V)
    cfg = _walked_rows(g, 64, 3, seed=11)  # 256 rows
    assert cfg.shape[0] == 256
    vocab = vocab_large(V)
    bias = torch.tensor([vocab.token_bytes.index(x) for x in BIASED], device="cuda")
    gen = torch.Generator(device="cuda").manual_seed(40_000)
    src = torch.randn(256, V, generator=gen, device="cuda")
    src[:, bias] += 3.0
    a, b = src.clone(), src.clone()
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    ev[0].record()
    ref.pda_apply_mask(g, cfg, a)
    ev[1].record()
    g.clear_memo()
    pda_apply_mask_(b, g, cfg)  # cold memo
    ev[2].record()
    c = src.clone()
    pda_apply_mask_(c, g, cfg)  # every row hits the memo
    ev[3].record()
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(a, c)
    ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(3)]
    print(f"\nconfig-4 apply_mask, 256 x {V} fp32: reference CUDA {ms[0]:.3f} ms, "
          f"this library {ms[1]:.3f} ms (cold memo) / {ms[2]:.3f} ms (memo hits)")
