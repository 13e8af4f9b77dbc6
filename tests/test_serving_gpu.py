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


def _host_pda(vocab):
    import numpy as np

    from bpdecode_b200 import tables
    from oracle.oracle import HostPda

    arrays = tables.load_pda("jsonvalue")
    offs = np.zeros(vocab.size + 1, np.int32)
    np.cumsum([len(t) for t in vocab.token_bytes], out=offs[1:])
    return HostPda(arrays, offs, np.frombuffer(b"".join(vocab.token_bytes), np.uint8),
                   vocab.eos_id)


@pytest.mark.parametrize("dtype,steps", [(torch.bfloat16, 64), (torch.float32, 16),
                                         (torch.float16, 16)])
def test_device_loop_matches_oracle(dtype: torch.dtype, steps: int) -> None:
    """The device-turnover loop: before every step the row lists and counts
    match the kinds; every row's token and next state equal the C oracle's
    from that row's state (soft bias on fp32 working values for dense rows,
    bounded PDA for grammar rows, broken rows fully masked); after every
    turnover the retired rows start fresh and the others are untouched."""
    import numpy as np

    from bpdecode_b200.serving import DeviceServingLoop
    from bpdecode_b200.workloads import DENSE_PATTERNS
    from oracle.oracle import Oracle

    orc = Oracle()
    dense, pda, vocab = _grammars(4096)
    rows = 160
    loop = DeviceServingLoop(rows, dense, pda, n_regex=len(DENSE_PATTERNS), seed=21)
    tn = loop.dense._t.tok_next.cpu().numpy()
    la = loop.dense._t.lookahead.cpu().numpy()
    starts = set(loop.dense._t.starts)
    init = pda.init_config().cpu().numpy()
    hg = _host_pda(vocab)
    gen = torch.Generator(device="cuda").manual_seed(77)
    turned = 0
    for step in range(steps):
        logits = (torch.randn(rows, vocab.size, generator=gen, device="cuda") * 2).to(dtype)
        kind = loop.kind.cpu().numpy()
        pool, cfgs, broken = (x.cpu().numpy().copy() for x in loop.states())
        d, p = np.flatnonzero(kind == 0), np.flatnonzero(kind == 1)
        assert loop.counts.cpu().tolist() == [len(d), len(p)], step
        assert np.array_equal(loop.dense_rows.cpu().numpy()[:len(d)], d), step
        assert np.array_equal(loop.pda_rows.cpu().numpy()[:len(p)], p), step
        tok = loop.step(logits).cpu().numpy()
        work = logits.float().cpu().numpy()
        wd = np.ascontiguousarray(work[d])
        orc.apply_soft(wd, la, pool[d], 1.0)
        want_d = np.argmax(wd, axis=1)
        next_d = orc.dense_advance(tn, pool[d], want_d)
        wp = np.ascontiguousarray(work[p])
        c = np.ascontiguousarray(cfgs[p])
        orc.pda_apply_mask(hg, c, wp, float("-inf"))
        br = broken[p].astype(bool)
        wp[br] = float("-inf")
        want_p = np.argmax(wp, axis=1)
        ok = orc.pda_advance(hg, c, want_p)
        assert np.array_equal(tok[d], want_d), step
        assert np.array_equal(tok[p], want_p), step
        pool2, cfgs2, broken2 = (x.cpu().numpy().copy() for x in loop.states())
        assert np.array_equal(pool2[d], next_d), step
        assert np.array_equal(cfgs2[p], c), step
        assert np.array_equal(broken2[p].astype(bool), br | (ok == 0)), step
        loop.turnover()
        out = loop.retired.cpu().numpy().astype(bool)
        turned += int(out.sum())
        kind3 = loop.kind.cpu().numpy()
        pool3, cfgs3, broken3 = (x.cpu().numpy() for x in loop.states())
        keep = ~out
        assert np.array_equal(kind3[keep], kind[keep]), step
        assert np.array_equal(pool3[keep], pool2[keep]), step
        assert np.array_equal(cfgs3[keep], cfgs2[keep]), step
        for r in np.flatnonzero(out):
            if kind3[r] == 0:
                assert int(pool3[r]) in starts, (step, r)
            else:
                assert pool3[r] == -2 and not broken3[r], (step, r)
                assert np.array_equal(cfgs3[r], init), (step, r)
    # about 10 % of the rows turn over per step
    assert 0.05 * rows * steps < turned < 0.15 * rows * steps, turned


def test_device_loop_graph_replay_equals_eager() -> None:
    """The same loop replayed from CUDA graphs (one per input buffer, step +
    turnover captured together) makes the eager loop's decisions."""
    from bpdecode_b200.serving import DeviceServingLoop
    from bpdecode_b200.workloads import DENSE_PATTERNS

    dense, pda, vocab = _grammars(4096)
    rows = 128
    eager, replay = (DeviceServingLoop(rows, dense, pda, n_regex=len(DENSE_PATTERNS), seed=3)
                     for _ in range(2))
    gen = torch.Generator(device="cuda").manual_seed(5)
    src = [(torch.randn(rows, vocab.size, generator=gen, device="cuda") * 2).to(torch.bfloat16)
           for _ in range(8)]
    bufs = [torch.empty_like(src[0]) for _ in range(2)]
    # one eager step each before capturing (loads the kernels)
    for lp in (eager, replay):
        bufs[0].copy_(src[0])
        lp.step(bufs[0])
        lp.turnover()
    graphs = [replay.graph(b) for b in bufs]
    for step in range(1, 24):
        b = bufs[step % 2]
        b.copy_(src[step % 8])
        ta = eager.step(b).clone()
        eager.turnover()
        b.copy_(src[step % 8])
        graphs[step % 2].replay()
        assert torch.equal(replay.tokens, ta), step
        for x, y in zip(eager.states(), replay.states()):
            assert torch.equal(x, y), step
        assert torch.equal(eager.kind, replay.kind), step
        assert torch.equal(eager.counts, replay.counts), step
    del graphs


def test_device_loop_second_stream_equals_one_stream() -> None:
    """The PDA rows' launches on a second stream (the default) make the same
    decisions as the whole step on one stream: tokens, states, config rows,
    broken flags and the mix, step after step with turnover."""
    from bpdecode_b200.serving import DeviceServingLoop
    from bpdecode_b200.workloads import DENSE_PATTERNS

    dense, pda, vocab = _grammars(4096)
    rows = 96
    one, two = (DeviceServingLoop(rows, dense, pda, n_regex=len(DENSE_PATTERNS), seed=9,
                                  overlap=ov) for ov in (False, True))
    assert one._side is None and two._side is not None
    gen = torch.Generator(device="cuda").manual_seed(11)
    for step in range(16):
        logits = (torch.randn(rows, vocab.size, generator=gen, device="cuda") * 2).to(
            torch.bfloat16)
        ta = one.step(logits).clone()
        one.turnover()
        tb = two.step(logits).clone()
        two.turnover()
        assert torch.equal(ta, tb), step
        for x, y in zip(one.states(), two.states()):
            assert torch.equal(x, y), step
        assert torch.equal(one.kind, two.kind), step


def test_device_turnover_lists_over_many_rows() -> None:
    """The device turnover over 2500 rows (three blocks of the kernel's
    1024-row compaction): after every call the ascending row lists and their
    counts match the kinds, retired rows hold fresh states, the others keep
    theirs, and the retirement rate is about the configured fraction."""
    import numpy as np

    from bpdecode_b200.serving import DeviceServingLoop
    from bpdecode_b200.workloads import DENSE_PATTERNS

    dense, pda, _ = _grammars(1024)
    rows = 2500
    loop = DeviceServingLoop(rows, dense, pda, n_regex=len(DENSE_PATTERNS), seed=17,
                             evict_fraction=0.25)
    starts = set(loop.dense._t.starts)
    init = pda.init_config().cpu().numpy()
    turned = 0
    for _ in range(6):
        kind0 = loop.kind.cpu().numpy()
        pool0 = loop.dense._state.cpu().numpy().copy()
        loop.turnover()
        kind = loop.kind.cpu().numpy()
        out = loop.retired.cpu().numpy().astype(bool)
        turned += int(out.sum())
        d, p = np.flatnonzero(kind == 0), np.flatnonzero(kind == 1)
        assert len(d) + len(p) == rows
        assert loop.counts.cpu().tolist() == [len(d), len(p)]
        assert np.array_equal(loop.dense_rows.cpu().numpy()[:len(d)], d)
        assert np.array_equal(loop.pda_rows.cpu().numpy()[:len(p)], p)
        pool = loop.dense._state.cpu().numpy()
        cfgs = loop.pda._configs.cpu().numpy()
        assert np.array_equal(kind[~out], kind0[~out])
        assert np.array_equal(pool[~out], pool0[~out])
        assert all(int(pool[r]) in starts for r in np.flatnonzero(out & (kind == 0)))
        for r in np.flatnonzero(out & (kind == 1))[:50]:
            assert pool[r] == -2 and np.array_equal(cfgs[r], init)
    assert 0.20 * rows * 6 < turned < 0.30 * rows * 6, turned
    # the mix of admitted requests follows (0.5, 0.3, 0.2): dense about 80 %
    assert 0.72 < float((loop.kind == 0).float().mean()) < 0.88
