"""Parity on the exact trajectories the benchmark times, every row, every step.

* config 2: one whole 128-step generation of the benchmark's block of 1024
  rows (8 regexes mixed, V = 128,256, bf16 N(0, 2), the benchmark's seeds),
  fused step against the reference's own dense torch step (ops.py:271-276,
  301-306, restated in oracle/torch_port.py) run on the same device tensors:
  masked logits, tokens and states of all rows at every step;
* config 4: 512 steps of 256 JSON-value rows at V = 128,256 (the
  benchmark's logits, memo cleared at the start) against the reference's own
  CUDA build (apply_mask_pda_kernel / advance_state_pda_kernel,
  pda_cuda.cu:72-117): masked logits, tokens and full config rows;
* config 5: the continuous-batching loop with turnover against the C oracle
  (soft bias on the dense rows, bounded PDA on the grammar rows);
* sharding: the rows a rank owns (global row blocks, bench.py) reproduce,
  bit for bit, what one process running the whole global batch computes --
  in one process and as two ranks.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch

from oracle import torch_port
from oracle.oracle import HostPda, Oracle, RefCudaLib

pytestmark = pytest.mark.gpu

NINF = float("-inf")


def _bench():
    import bench

    return bench


def test_config2_generation_equals_reference_dense_step_every_row() -> None:
    bench = _bench()
    dev = torch.device("cuda", 0)
    _, fsas, pats = bench.build_workload(0, dev)
    batch = bench.make_batch(fsas, pats)
    ids = list(range(bench.ROWS_PER_GPU))
    tok_next = batch._t.tok_next
    ref_state = batch._state.clone()
    slots = torch.arange(bench.ROWS_PER_GPU, device=dev)
    changed = 0
    for step in range(bench.EPISODE):
        logits = bench.gen_logits(0, step, dev)
        want = logits.clone()
        ref_tok = torch_port.step(want, tok_next, ref_state, slots)
        tok = batch.step_greedy(ids, logits)
        assert torch.equal(logits.view(torch.int16), want.view(torch.int16)), step
        assert torch.equal(tok, ref_tok), step
        assert torch.equal(batch._state, ref_state), step
        changed += int(torch.isneginf(logits).sum())
    assert changed > 0
    # rows keep going through the whole generation (not all broken or done)
    assert int((batch._state >= 0).sum()) > 0


@pytest.mark.skipif(not RefCudaLib.available(),
                    reason="the reference's CUDA sources were not compiled (oracle/_ref)")
def test_config4_512_steps_equal_reference_cuda_every_row() -> None:
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import CFGConstraintBatch, PdaTensors
    from bpdecode_b200.workloads import BIASED, vocab_large

    ref = RefCudaLib()
    B, V = 256, 128_256
    vocab = vocab_large(V)
    g = PdaTensors.from_arrays(tables.load_pda("jsonvalue"), vocab, "cuda")
    g.clear_memo()
    batch = CFGConstraintBatch(g, capacity=B)
    ids = list(range(B))
    for i in ids:
        batch.add(i)
    ref_cfg = batch._configs.clone()
    bias = torch.tensor([vocab.token_bytes.index(t) for t in BIASED], device="cuda")
    ring = 32
    src = []
    for i in range(ring):  # bench.py _pda_config4's buffers (rank 0)
        gen = torch.Generator(device="cuda").manual_seed(40_000 + i)
        x = torch.randn(B, V, generator=gen, device="cuda")
        x[:, bias] += 3.0
        src.append(x)
    for step in range(512):
        mine = src[step % ring].clone()
        want = src[step % ring].clone()
        tok = batch.step_greedy(ids, mine)
        ref.pda_apply_mask(g, ref_cfg, want)
        ref_tok = want.argmax(-1)
        ok = ref.pda_advance(g, ref_cfg, ref_tok.to(torch.int32))
        assert torch.equal(mine, want), step
        assert torch.equal(tok, ref_tok), step
        assert torch.equal(batch._configs, ref_cfg), step
        assert bool(ok.all()) and not bool(batch._broken.any()), step


def test_config5_loop_with_turnover_matches_oracle() -> None:
    """64 steps of the serving loop (regex + schema rows with the k = 4 soft
    bias on fp32 working values, JSON-value PDA rows, 10 % of the requests
    retired and admitted every step): at each step every row's token and
    next state equal the oracle's from that row's state before the step."""
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import PdaTensors
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.serving import MixedServingLoop
    from bpdecode_b200.workloads import DENSE_PATTERNS, vocab_large

    orc = Oracle()
    V, rows = 4096, 160
    vocab = vocab_large(V)
    dense = [FsaTensors.from_arrays(tables.load_dfa(n), vocab).to("cuda")
             for n, _ in DENSE_PATTERNS]
    dense.append(FsaTensors.from_arrays(tables.load_dfa("schema"), vocab).to("cuda"))
    dense = [f.with_lookahead(4) for f in dense]
    arrays = tables.load_pda("jsonvalue")
    pda = PdaTensors.from_arrays(arrays, vocab, "cuda")
    loop = MixedServingLoop(rows, dense, pda, n_regex=len(DENSE_PATTERNS), seed=21)
    tn = loop.dense._t.tok_next.cpu().numpy()
    la = loop.dense._t.lookahead.cpu().numpy()
    offs = np.zeros(V + 1, np.int32)
    np.cumsum([len(t) for t in vocab.token_bytes], out=offs[1:])
    hg = HostPda(arrays, offs, np.frombuffer(b"".join(vocab.token_bytes), np.uint8),
                 vocab.eos_id)
    gen = torch.Generator(device="cuda").manual_seed(77)
    turned = 0
    for step in range(64):
        logits = (torch.randn(rows, V, generator=gen, device="cuda") * 2).to(torch.bfloat16)
        pool, cfgs, broken = (x.cpu().numpy().copy() for x in loop.states())
        kind, slot = loop.kind.copy(), loop.slot.copy()
        tok = loop.step(logits).cpu().numpy()
        work = logits.float().cpu().numpy()
        d, p = np.flatnonzero(kind == 0), np.flatnonzero(kind == 1)
        # dense rows: fp32 working values + soft bias, argmax, commit
        wd = np.ascontiguousarray(work[d])
        st = pool[slot[d]]
        orc.apply_soft(wd, la, st, 1.0)
        want_d = np.argmax(wd, axis=1)
        next_d = orc.dense_advance(tn, st, want_d)
        # PDA rows: mask, broken rows fully masked, argmax, advance
        wp = np.ascontiguousarray(work[p])
        c = np.ascontiguousarray(cfgs[slot[p]])
        orc.pda_apply_mask(hg, c, wp, NINF)
        br = broken[slot[p]].astype(bool)
        wp[br] = NINF
        want_p = np.argmax(wp, axis=1)
        ok = orc.pda_advance(hg, c, want_p)
        assert np.array_equal(tok[d], want_d), step
        assert np.array_equal(tok[p], want_p), step
        pool2, cfgs2, broken2 = (x.cpu().numpy() for x in loop.states())
        assert np.array_equal(pool2[slot[d]], next_d), step
        assert np.array_equal(cfgs2[slot[p]], c), step
        assert np.array_equal(broken2[slot[p]].astype(bool), br | (ok == 0)), step
        turned += len(loop.turnover())
    assert turned == 64 * round(rows * 0.1)


def _block_run(block_ids: list[int], steps: int, dev: torch.device):
    """Tokens and states of one ConstraintBatch holding the given global row
    blocks (in order) over `steps` benchmark steps."""
    bench = _bench()
    _, fsas, _ = bench.build_workload(0, dev)
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.workloads import block_patterns

    pats = [p for b in block_ids for p in block_patterns(b, bench.ROWS_PER_GPU)]
    batch = ConstraintBatch(fsas, capacity=len(pats))
    for i, p in enumerate(pats):
        batch.add(i, grammar=p)
    ids = list(range(len(pats)))
    toks = []
    for step in range(steps):
        logits = torch.cat([bench.gen_logits(b, step, dev) for b in block_ids])
        toks.append(batch.step_greedy(ids, logits).cpu())
    return torch.stack(toks), batch._state.cpu()


def test_sharded_blocks_equal_one_process_over_the_global_batch() -> None:
    bench = _bench()
    dev = torch.device("cuda", 0)
    R = bench.ROWS_PER_GPU
    whole_tok, whole_state = _block_run([0, 1], 16, dev)
    for world in (2,):
        for rank in range(world):
            block = bench.my_block(rank, world)
            tok, state = _block_run([block], 16, dev)
            assert torch.equal(tok, whole_tok[:, block * R:(block + 1) * R]), rank
            assert torch.equal(state, whole_state[block * R:(block + 1) * R]), rank


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_worker(rank: int, world: int, port: int, steps: int, outdir: str) -> None:
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank),
                      MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import sys

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    from bpdecode_b200 import shard

    import bench

    dev = torch.device("cuda", rank % torch.cuda.device_count())
    torch.cuda.set_device(dev)
    assert shard.init("gloo", timeout_s=120)
    block = bench.my_block(rank, world)
    tok, state = _block_run([block], steps, dev)
    shard.barrier()
    # results go to a file, not a pipe: a pipe holds 64 KB, and a writer
    # blocked on it would never reach the exit the parent joins on
    np.savez(os.path.join(outdir, f"rank{rank}.npz"), block=block, tok=tok.numpy(),
             state=state.numpy())
    shard.finish()


def test_two_ranks_reproduce_the_one_process_run(tmp_path) -> None:
    """Two processes (one GPU each where there are two, else both on cuda:0;
    no kernel of one waits on the other), gloo for the group: rank r runs its
    global row block; the gathered tokens and states equal one process over
    both blocks."""
    import torch.multiprocessing as mp

    bench = _bench()
    world, steps, R = 2, 8, bench.ROWS_PER_GPU
    mp.start_processes(_rank_worker, args=(world, _free_port(), steps, str(tmp_path)),
                       nprocs=world, join=True, start_method="spawn")
    whole_tok, whole_state = _block_run([0, 1], steps, torch.device("cuda", 0))
    for rank in range(world):
        with np.load(tmp_path / f"rank{rank}.npz") as z:
            block, tok, state = int(z["block"]), z["tok"], z["state"]
        assert block == rank
        assert np.array_equal(tok, whole_tok[:, block * R:(block + 1) * R].numpy()), rank
        assert np.array_equal(state, whole_state[block * R:(block + 1) * R].numpy()), rank
