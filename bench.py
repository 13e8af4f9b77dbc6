"""Benchmark of the constrained-decoding step (row-steps/s + HBM roofline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (the serving-scale dense configuration): V = 128,256 synthetic
tokens, 1024 rows per GPU, each row constrained by one of 8 regexes (IPv4,
date, e-mail, signed float, hex colour, UUID, name, phone) chosen from the
seed, bf16 logits ~ N(0, 2), greedy (argmax) commit. A step is mask + apply +
argmax + commit of every row: one fused launch per step
(ConstraintBatch.step_greedy). Rows are sharded by request: the global rows
are cut into blocks of 1024 (bpdecode_b200.workloads.ROW_BLOCK), rank r owns
block r (shard.shard_rows), every row's pattern and logits depend only on its
block, so rank r computes what one process over the global batch computes for
those rows, and no collective runs on the hot path (weak scaling).

Prints one JSON line (rank 0). Under torchrun each rank runs on LOCAL_RANK;
timing is the max over ranks of CUDA-event time.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

V = 128_256
ROWS_PER_GPU = 1024
SIGMA = 2.0
# Config 2 generates 128 steps per request: the timed run is a sequence of
# such episodes, every row restarting from its pattern's start state each
# EPISODE steps (ConstraintBatch.reset_many, one device write).
EPISODE = 128
METRIC = "constrained row-steps/sec (mask+apply+commit)"
UNIT = "row-steps/s"
# Algorithmic bytes of one row-step (bf16 logits, V = 128,256): logits read +
# write 2*V*2, packed allow row 4*ceil(V/32), state/token/tok_next gather 16.
E = 2
ALGO_BYTES_PER_ROW_STEP = 2 * V * E + 4 * ((V + 31) // 32) + 16


def _dist() -> tuple[int, int, int]:
    from bpdecode_b200.shard import dist_info

    return dist_info()


def _peaks() -> tuple[float, str]:
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def _profile_traffic(steps: int) -> tuple[float | None, str]:
    """Mean DRAM bytes (read + write) per launch of the fused step kernel over
    the generation steps a timed region of `steps` launches covers (step i of
    the region is generation step i mod EPISODE), from the committed ncu
    summary: one line `step_dram_bytes: <step> <read> <write>` per generation
    step. (None, why) when the summary does not cover those steps."""
    path = os.path.join(ROOT, "profiles", "dense_step_config2.md")
    per: dict[int, float] = {}
    try:
        with open(path) as f:
            for line in f:
                if line.strip().startswith("step_dram_bytes:"):
                    k, rd, wr = line.split(":", 1)[1].split()[:3]
                    per[int(k)] = float(rd) + float(wr)
    except OSError:
        return None, "no ncu summary"
    want = [i % EPISODE for i in range(steps)]
    if not per or any(k not in per for k in want):
        return None, "ncu summary does not cover the timed steps"
    return statistics.fmean(per[k] for k in want), (
        f"ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, mean over generation "
        f"steps {min(want)}..{max(want)} (the steps this run timed), profiles/dense_step_config2.md")


def _profile_bytes(name: str) -> float | None:
    """`traffic_bytes_per_launch: <bytes>` of a committed ncu summary under
    profiles/ (DRAM read + write per launch of that leg's kernel), or None."""
    try:
        with open(os.path.join(ROOT, "profiles", name)) as f:
            for line in f:
                if line.strip().startswith("traffic_bytes_per_launch:"):
                    return float(line.split(":", 1)[1].split()[0])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    HW = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
          "sw_power_cap": 0x4, "hw_power_brake_slowdown": 0x80}

    def __init__(self, index: int, period_s: float = 0.002) -> None:
        self.index, self.period = index, period_s
        self.samples: list[tuple[int, int]] = []
        self.max_mhz: int | None = None
        self._stop = threading.Event()
        self._thread: threading.Thread | None = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = int(pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM))
        except Exception:
            self._nv = None

    def _run(self) -> None:
        nv = self._nv
        while not self._stop.is_set():
            try:
                clk = int(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
                rs = int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))
                self.samples.append((clk, rs))
            except Exception:
                pass
            time.sleep(self.period)

    def __enter__(self) -> ClockSampler:
        if self._nv is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc: object) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unsampled"],
                    "samples": 0}
        reasons = set()
        for _, r in self.samples:
            for name, bit in self.HW.items():
                if r & bit:
                    reasons.add(name)
        return {"sm_mhz": statistics.median(c for c, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples": len(self.samples)}


def build_workload(block: int, device: torch.device):
    """Tables of the 8 patterns and the pattern of every row of global row
    block `block`."""
    from bpdecode_b200 import tables
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import DENSE_PATTERNS, block_patterns, vocab_large

    vocab = vocab_large(V)
    fsas = [FsaTensors.from_arrays(tables.load_dfa(n), vocab).to(device)
            for n, _ in DENSE_PATTERNS]
    return vocab, fsas, block_patterns(block, ROWS_PER_GPU)


def my_block(rank: int, world: int) -> int:
    """The global row block this rank owns (blocks of ROWS_PER_GPU rows)."""
    from bpdecode_b200 import shard

    rows = shard.shard_rows(ROWS_PER_GPU * world, world, rank)
    assert len(rows) == ROWS_PER_GPU and rows.start % ROWS_PER_GPU == 0
    return rows.start // ROWS_PER_GPU


def make_batch(fsas, pats):
    from bpdecode_b200.batch import ConstraintBatch

    batch = ConstraintBatch(fsas, capacity=ROWS_PER_GPU)
    for i in range(ROWS_PER_GPU):
        batch.add(i, grammar=pats[i])
    return batch


def gen_logits(block: int, step: int, device: torch.device, out: torch.Tensor | None = None):
    """bf16 logits N(0, SIGMA^2) of global row block `block` at step `step`."""
    from bpdecode_b200.workloads import block_logits_seed

    g = torch.Generator(device=device).manual_seed(block_logits_seed(block, step))
    x = torch.randn(ROWS_PER_GPU, V, generator=g, device=device) * SIGMA
    if out is None:
        return x.to(torch.bfloat16)
    out.copy_(x)
    return out


def _cpu_tables(tns: list[torch.Tensor], starts_local: list[int]) -> tuple[torch.Tensor, list[int]]:
    """The batch's global tok_next (grammars concatenated, state ids offset)
    and start states, on the host."""
    out, starts, off = [], [], 0
    for tn, st in zip(tns, starts_local):
        tn = tn.cpu()
        out.append(torch.where(tn >= 0, tn + off, tn))
        starts.append(st + off)
        off += tn.shape[0]
    return torch.cat(out), starts


def _time_cpu_reference(tok_next: torch.Tensor, starts: list[int], pats: list[int],
                        steps: int, warmup: int) -> float:
    """Seconds for `steps` steps of the reference's dense step on host cores
    over every row of the block (128-step generations from the start states,
    as on the GPU), after `warmup` untimed steps. Four seeded bf16 logits
    buffers of the workload's shape are cycled (the CPU arm masks them in
    place, which leaves later steps' allowed tokens unchanged)."""
    from oracle import torch_port

    rows = len(pats)
    state = torch.tensor([starts[p] for p in pats], dtype=torch.int32)
    start = state.clone()
    slots = torch.arange(rows)
    g = torch.Generator().manual_seed(12345)
    pool = [(torch.randn(rows, V, generator=g) * SIGMA).to(torch.bfloat16) for _ in range(4)]
    for i in range(warmup):
        torch_port.step(pool[i % 4], tok_next, state, slots)
    state.copy_(start)
    t0 = time.perf_counter()
    for i in range(steps):
        if i and i % EPISODE == 0:
            state.copy_(start)
        torch_port.step(pool[i % 4], tok_next, state, slots)
    return time.perf_counter() - t0


_CPU_SAMPLE = ("every row of the {rows}-row block, bf16, V={V}: torch CPU restatement of "
               "bpdecode's dense step (ops.py:271-276 mask, argmax, ops.py:301-306 commit; the "
               "reference's dense path is torch, not compiled code), {steps} steps, {dt:.1f} s")


def cpu_baseline(tok_next_cpu: torch.Tensor, starts: list[int], pats: list[int],
                 steps: int) -> dict:
    """The reference's own dense torch step on host cores (all torch threads),
    a bounded sample of this workload: every row, `steps` steps."""
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    dt = _time_cpu_reference(tok_next_cpu, starts, pats, steps, 1)
    rows = len(pats)
    return {"value": rows * steps / dt, "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port", "sample": _CPU_SAMPLE.format(rows=rows, V=V, steps=steps, dt=dt)}


def run_reference(args: argparse.Namespace) -> None:
    """--impl reference: the reference's CPU implementation of the step, timed
    on host cores on this arm's workload (the same 1024-row block, patterns,
    vocabulary, dtype and generation length); rank 0 only."""
    rank, world, _ = _dist()
    if rank != 0:
        return
    # torchrun sets OMP_NUM_THREADS=1 per rank; rank 0 runs alone here, so it
    # takes every host core it may use
    torch.set_num_threads(len(os.sched_getaffinity(0)))
    from bpdecode_b200 import tables
    from bpdecode_b200.workloads import DENSE_PATTERNS, block_patterns, vocab_large
    from oracle.oracle import Oracle, dfa_with_vocab

    vocab = vocab_large(V)
    orc = Oracle()
    tns, starts_local = [], []
    for n, _ in DENSE_PATTERNS:
        d = tables.load_dfa(n)
        o, sy = dfa_with_vocab(d, vocab.token_bytes)
        tns.append(torch.from_numpy(orc.build_tok_next(d, o, sy, vocab.eos_id)))
        starts_local.append(d["start"])
    tok_next, starts = _cpu_tables(tns, starts_local)
    pats = block_patterns(0, ROWS_PER_GPU)
    dt = _time_cpu_reference(tok_next, starts, pats, args.steps, args.warmup)
    value = ROWS_PER_GPU * args.steps / dt
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT,
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000.0 * dt / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _config(world),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(),
                         "kind": "port",
                         "sample": _CPU_SAMPLE.format(rows=ROWS_PER_GPU, V=V, steps=args.steps,
                                                      dt=dt)},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def _config(world: int) -> dict:
    """The workload, identical in both arms' lines."""
    return {
        "workload": "dense regex step at serving scale (config 2): 8 regexes mixed per batch, "
                    f"V={V}, {ROWS_PER_GPU} rows per GPU, bf16 logits N(0,{SIGMA:g}), argmax "
                    f"commit, {EPISODE}-step generations from the start states",
        "vocab": V, "rows_per_gpu": ROWS_PER_GPU, "global_batch": ROWS_PER_GPU * world,
        "parallelism": f"dp{world} (rows sharded by request in global blocks of "
                       f"{ROWS_PER_GPU}, no collective)",
        "l2": "inputs larger than L2: every step reads a 262 MB logits buffer (126 MB L2)",
    }


def run_config5(args: argparse.Namespace) -> None:
    """Config 5, per GPU: 1024 rows of continuous batching at V = 128,256 --
    50 % regex requests (the 8 patterns), 30 % the JSON-Schema object (dense
    DFA), 20 % the recursive JSON-value grammar (PDA); the dense rows are
    scored with the horizon-4 soft lookahead on fp32 working values read from
    their bf16 logits, all rows greedy; every step each request retires with
    probability 0.1 and a new one is admitted in its row
    (bpdecode_b200.serving.DeviceServingLoop: the turnover runs on the device,
    so a whole step -- both fused steps, the tokens in row order, the
    turnover -- is replayed from a CUDA graph, one per logits buffer).
    Timed: --steps steps, CUDA events around the replays, max over ranks.
    Side measurement: the same workload through MixedServingLoop (turnover
    bookkeeping on the host, eager launches)."""
    from bpdecode_b200 import shard, tables
    from bpdecode_b200.grammar.device import PdaTensors
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.serving import DeviceServingLoop, MixedServingLoop
    from bpdecode_b200.workloads import DENSE_PATTERNS, vocab_large

    rank, world, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    shard.init("nccl", device)
    vocab = vocab_large(V)
    t0 = time.perf_counter()
    dense = [FsaTensors.from_arrays(tables.load_dfa(n), vocab).to(device)
             for n, _ in DENSE_PATTERNS]
    dense.append(FsaTensors.from_arrays(tables.load_dfa("schema"), vocab).to(device))
    dense = [f.with_lookahead(4) for f in dense]
    pda = PdaTensors.from_arrays(tables.load_pda("jsonvalue"), vocab, device)
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    block = my_block(rank, world)
    loop = DeviceServingLoop(ROWS_PER_GPU, dense, pda, n_regex=len(DENSE_PATTERNS),
                             seed=block * 7 + 1)
    ring = 16
    bufs = [gen_logits(block, 20_000 + i, device) for i in range(ring)]
    for i in range(args.warmup):
        loop.step(bufs[i % ring])
        loop.turnover()
    graphs = [loop.graph(b) for b in bufs]
    torch.cuda.synchronize()
    shard.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    steps = args.steps
    with ClockSampler(local) as clocks:
        a.record()
        for i in range(steps):
            graphs[i % ring].replay()
        b.record()
        torch.cuda.synchronize()
    shard.barrier()
    ms = shard.max_over_ranks([a.elapsed_time(b)], device)[0]
    pda_rows = int(loop.counts[1])
    del graphs
    # the host-bookkeeping loop on the same workload, eager
    host = MixedServingLoop(ROWS_PER_GPU, dense, pda, n_regex=len(DENSE_PATTERNS),
                            seed=block * 7 + 1)
    hsteps = min(steps, 200)
    for i in range(3):
        host.step(bufs[i % ring])
        host.turnover()
    torch.cuda.synchronize()
    a.record()
    for i in range(hsteps):
        host.step(bufs[i % ring])
        host.turnover()
    b.record()
    torch.cuda.synchronize()
    host_ms = shard.max_over_ranks([a.elapsed_time(b)], device)[0] / hsteps
    line = {
        "metric": "constrained row-steps/sec (config 5 continuous batching)",
        "value": ROWS_PER_GPU * world * steps / (ms / 1e3), "unit": UNIT, "n_gpus": world,
        "steps": steps, "warmup": args.warmup, "ms_per_step": ms / steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic",
        "config": {"workload": "config 5: 1024 rows per GPU, V=128256, 50% regex (8 patterns) / "
                               "30% JSON-Schema object (dense DFA) / 20% recursive JSON-value "
                               "GBNF (PDA), soft lookahead k=4 fp32 on the dense rows, greedy, "
                               "every request retires with probability 0.1 per step and a new "
                               "one is admitted in its row",
                   "rows_per_gpu": ROWS_PER_GPU, "global_batch": ROWS_PER_GPU * world,
                   "parallelism": f"dp{world} (rows sharded by request, no collective)",
                   "pda_rows_at_end": pda_rows, "dense_rows_at_end": ROWS_PER_GPU - pda_rows,
                   "l2": f"{ring} logits buffers of 262 MB cycled (larger than L2)",
                   "table_build_s": build_s},
        "clocks": clocks.summary(),
        # per step: the dense soft step; prologue, lookup, compute and the
        # PDA step (second stream); the token gather; the turnover
        "gpu_launches": steps * 7,
        "timing": "CUDA events around the graph replays (a step = dense soft step, PDA "
                  "mask pipeline + step, token gather, device turnover); max over ranks",
        "host_turnover_loop": {"ms_per_step": host_ms,
                               "value": ROWS_PER_GPU * world / (host_ms / 1e3),
                               "path": "MixedServingLoop: exact 10 % turnover with host "
                                       "bookkeeping, eager launches, " + f"{hsteps} steps"},
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    shard.finish()


def run_profile_case(args: argparse.Namespace) -> None:
    """Small fixed cases for ncu captures (no timing, no side measurements).
    `dense` = the bench's fused dense step and `soft` = the fused soft step
    (k = 4, fp32 copy of the same logits): 1024 rows, and before step j of an
    episode the bench's logits buffer j is regenerated into one working
    buffer (262 MB bf16 / 525 MB fp32, larger than L2), so the rows follow the
    bench's trajectory with a device footprint of about 1 GB. `pda` = the
    config-4 PDA step (256 rows, fp32, one of 4 seeded buffers copied into the
    step's input each step). Each runs --warmup steps,
    restarts the rows (dense, soft), then --steps steps on cuda:0."""
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    n = args.warmup + args.steps
    if args.profile_case in ("dense", "soft"):
        _, fsas, pats = build_workload(0, device)
        soft = args.profile_case == "soft"
        if soft:
            from dataclasses import replace

            from bpdecode_b200.ops import build_lookahead

            fsas = [replace(f, lookahead=build_lookahead(f, 4)) for f in fsas]
        batch = make_batch(fsas, pats)
        ids = list(range(ROWS_PER_GPU))
        work = torch.empty(ROWS_PER_GPU, V, dtype=torch.float32 if soft else torch.bfloat16,
                           device=device)

        def step(j: int) -> None:
            if soft:
                work.copy_(gen_logits(0, j % EPISODE, device))
                batch.soft_step_greedy(ids, work, 1.0)
            else:
                gen_logits(0, j % EPISODE, device, out=work)
                batch.step_greedy(ids, work)

        for i in range(args.warmup):
            step(i)
        batch.reset_many(ids)  # the captured steps start an episode, as in the bench
        for i in range(args.steps):
            step(i)
    elif args.profile_case == "dense3":
        # config 3: the schema DFA at V = 151,936, 512 fp32 rows, the
        # _dense_config3 leg's first buffer copied into the step's input
        from bpdecode_b200 import tables
        from bpdecode_b200.batch import ConstraintBatch
        from bpdecode_b200.ops import FsaTensors
        from bpdecode_b200.workloads import vocab_large

        B3, V3 = 512, 151_936
        fsa = FsaTensors.from_arrays(tables.load_dfa("schema"), vocab_large(V3)).to(device)
        batch = ConstraintBatch(fsa, capacity=B3)
        ids = list(range(B3))
        for i in ids:
            batch.add(i)
        src = [torch.randn(B3, V3, device=device,
                           generator=torch.Generator(device=device).manual_seed(7 + i))
               for i in range(4)]
        work = torch.empty_like(src[0])
        for i in range(n):
            work.copy_(src[i % 4])
            batch.step_greedy(ids, work)
    elif args.profile_case in ("pda_misses", "pda_nesting"):
        from bpdecode_b200 import tables
        from bpdecode_b200.grammar.device import CFGConstraintBatch, PdaTensors
        from bpdecode_b200.workloads import BIASED, vocab_large

        nest = args.profile_case == "pda_nesting"
        vocab = vocab_large(V)
        g = PdaTensors.from_arrays(tables.load_pda("brackets" if nest else "schema"), vocab,
                                   device)
        batch = CFGConstraintBatch(g, capacity=256)
        ids = list(range(256))
        for i in ids:
            batch.add(i)
        src = [torch.randn(256, V, device=device,
                           generator=torch.Generator(device=device).manual_seed(500 + i))
               for i in range(4)]
        if nest:
            from bpdecode_b200.workloads import OPENERS, token_ids

            boost = torch.tensor(token_ids(vocab, OPENERS), device=device)
            for x in src:
                x[:, boost] += 1.0
        work = torch.empty_like(src[0])
        g.clear_memo()
        for i in range(n):
            work.copy_(src[i % 4])
            batch.step_greedy(ids, work)
    else:
        from bpdecode_b200 import tables
        from bpdecode_b200.grammar.device import CFGConstraintBatch, PdaTensors
        from bpdecode_b200.workloads import BIASED, vocab_large

        vocab = vocab_large(V)
        g = PdaTensors.from_arrays(tables.load_pda("jsonvalue"), vocab, device)
        batch = CFGConstraintBatch(g, capacity=256)
        ids = list(range(256))
        for i in ids:
            batch.add(i)
        bias = torch.tensor([vocab.token_bytes.index(t) for t in BIASED], device=device)
        src = []
        for i in range(4):
            gen = torch.Generator(device=device).manual_seed(40_000 + i)
            x = torch.randn(256, V, generator=gen, device=device)
            x[:, bias] += 3.0
            src.append(x)
        work = torch.empty_like(src[0])
        for i in range(n):
            work.copy_(src[i % 4])  # unmasked logits every step
            batch.step_greedy(ids, work)
    torch.cuda.synchronize()
    print(json.dumps({"profile_case": args.profile_case, "steps": n}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1024)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--ring", type=int, default=128, help="distinct logits buffers")
    ap.add_argument("--e2e-steps", type=int, default=24)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the PDA and soft-lookahead side measurements")
    ap.add_argument("--workload", default="config2", choices=["config2", "config5"],
                    help="config2 (default, the headline line) or config5 (whole-box continuous "
                         "batching: regex + schema + GBNF rows, soft lookahead, 10%% turnover)")
    ap.add_argument("--leg", choices=["pda_misses", "pda_nesting", "pda_config4"],
                    help="run one side measurement alone on cuda:0 and print it")
    ap.add_argument("--profile-case",
                    choices=["dense", "dense3", "pda", "soft", "pda_misses", "pda_nesting"],
                    help="run a few untimed steps of one hot kernel for an ncu capture "
                         "(1 GPU, --warmup steps then --steps steps) and exit")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    if args.profile_case:
        run_profile_case(args)
        return
    if args.leg:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        fn = {"pda_misses": _pda_misses, "pda_nesting": _pda_nesting,
              "pda_config4": _pda_config4}[args.leg]
        print(json.dumps({args.leg: fn(dev, 0)}), flush=True)
        return
    if args.workload == "config5" and args.impl == "ours":
        run_config5(args)
        return
    if args.impl == "reference":
        run_reference(args)
        return

    from bpdecode_b200 import shard

    rank, world, local = _dist()
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    shard.init("nccl", device)

    block = my_block(rank, world)
    vocab, fsas, pats = build_workload(block, device)
    batch = make_batch(fsas, pats)
    ids = list(range(ROWS_PER_GPU))

    ring = max(1, min(args.ring, args.steps + args.warmup))
    bufs = [gen_logits(block, i, device) for i in range(ring)]
    torch.cuda.synchronize()

    barrier = shard.barrier

    # warm-up, then every row back to its start state
    for i in range(args.warmup):
        batch.step_greedy(ids, bufs[i % ring])
    batch.reset_many(ids)
    torch.cuda.synchronize()
    barrier()

    stream = torch.cuda.current_stream(device)

    def run_steps(pairs: list | None) -> None:
        for i in range(args.steps):
            if i and i % EPISODE == 0:
                batch.reset_many(ids)
            if pairs is not None:
                pairs[i][0].record(stream)
            batch.step_greedy(ids, bufs[(i % EPISODE) % ring])
            if pairs is not None:
                pairs[i][1].record(stream)

    # the timed region: the launches back to back, nothing else on the stream
    t_all0 = torch.cuda.Event(enable_timing=True)
    t_all1 = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        torch.cuda.synchronize()
        t_all0.record(stream)
        run_steps(None)
        t_all1.record(stream)
        torch.cuda.synchronize()
    barrier()
    elapsed_ms = t_all0.elapsed_time(t_all1)

    # the step kernel's duration per launch: the same trajectory again (rows
    # back at their start states, the same logits buffers) with CUDA events
    # around every launch. A 1 GiB fill enqueued first keeps the GPU busy
    # while the first launches are issued, so every start event fires when
    # the previous launch ends, not when the host records it: the pairs time
    # the kernels, not the host's launch latency.
    batch.reset_many(ids)
    pairs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
             for _ in range(args.steps)]
    busy = torch.empty(1 << 30, dtype=torch.uint8, device=device)
    torch.cuda.synchronize()
    busy.fill_(1)
    run_steps(pairs)
    torch.cuda.synchronize()
    del busy
    per_launch_ms = [a.elapsed_time(b) for a, b in pairs]
    events_ms = statistics.fmean(per_launch_ms)
    rank_ms = shard.gather_over_ranks(elapsed_ms, device)
    elapsed_ms, events_ms = shard.max_over_ranks([elapsed_ms, events_ms], device)
    ms_per_step = elapsed_ms / args.steps
    # the timed region holds the step kernel's launches back to back and one
    # index_copy per generation, so its time per step bounds the kernel's own
    # duration from above (launch gaps included); the roofline uses it
    kern_ms = ms_per_step

    total_rows = ROWS_PER_GPU * world * args.steps
    value = total_rows / (elapsed_ms / 1000.0)
    peak, peak_kind = _peaks()
    achieved = ROWS_PER_GPU * ALGO_BYTES_PER_ROW_STEP / (kern_ms / 1000.0) / 1e9
    traffic, traffic_src = _profile_traffic(args.steps)

    # unfused drop-in path: apply_mask + torch.argmax + commit (3 launches),
    # the first 64 steps of an episode
    un_steps = min(args.steps, 64)
    for i in range(3):
        lg = bufs[i % ring]
        batch.apply_mask(ids, lg)
        batch.commit(ids, lg.argmax(-1))
    batch.reset_many(ids)
    torch.cuda.synchronize()
    u0 = torch.cuda.Event(enable_timing=True)
    u1 = torch.cuda.Event(enable_timing=True)
    u0.record(stream)
    for i in range(un_steps):
        lg = bufs[i % ring]
        batch.apply_mask(ids, lg)
        batch.commit(ids, lg.argmax(-1))
    u1.record(stream)
    torch.cuda.synchronize()
    un_ms = u0.elapsed_time(u1) / un_steps

    # greedy without the masked logits: step_greedy_from with no output reads
    # the allowed vectors, commits the argmax and writes nothing back
    tokens_only = _tokens_only(batch, ids, bufs, ring, stream)

    # reference GPU bar: bpdecode's dense torch composite on this B200
    batch.reset_many(ids)
    ref_gpu = _reference_torch_gpu(batch, bufs, ring, device)

    # end to end through the public API with host buffers
    batch.reset_many(ids)
    e2e = _e2e(batch, ids, block, device, args.e2e_steps, world)

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
        "config": _config(world),
        "timed_window": {"block": block, "logits_ring": ring, "episode_steps": EPISODE,
                         "episodes": (args.steps + EPISODE - 1) // EPISODE,
                         "note": (f"every row restarts from its start state each {EPISODE} "
                                  f"steps (one device write inside the timed region); step j "
                                  f"of an episode reads buffer j mod {ring}, so every episode "
                                  "replays the same trajectory (masking in place is "
                                  "idempotent)")},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "traffic": traffic,
                     "traffic_source": traffic_src,
                     "achieved_traffic_gbs": (traffic / (kern_ms / 1000.0) / 1e9
                                              if traffic else None),
                     "frac_traffic": (traffic / (kern_ms / 1000.0) / 1e9 / peak
                                      if traffic else None),
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                     if peak_kind == "measured" else "fallback 6.65 TB/s",
                     "kernel": "stream_step_kernel<bf16, DenseRows, DenseCommit> (fused "
                               "mask + argmax + commit)",
                     "kernel_ms": kern_ms,
                     "kernel_timing": "the timed region's device time per step (back-to-back "
                                      "launches of the step kernel, the only kernel there but "
                                      "one index_copy per generation), max over ranks: an upper "
                                      "bound of the kernel's duration",
                     "kernel_ms_events": events_ms,
                     "kernel_ms_events_first_last": [per_launch_ms[0], per_launch_ms[-1]],
                     "kernel_events_timing": f"diagnostic: CUDA events around each of the "
                                             f"{args.steps} launches of a replay of the timed "
                                             "steps, the GPU kept busy by a 1 GiB fill while the "
                                             "first launches were issued (each pair adds the "
                                             "event records' own cost)",
                     "algo_bytes_per_row_step": ALGO_BYTES_PER_ROW_STEP,
                     "algo_bytes_per_launch": ROWS_PER_GPU * ALGO_BYTES_PER_ROW_STEP},
        "clocks": clocks.summary(),
        "rank_ms": rank_ms,
        "gpu_launches": args.steps,
        "e2e": e2e,
        "unfused_dropin": {"ms_per_step": un_ms, "value": ROWS_PER_GPU * world / (un_ms / 1e3),
                           "path": "ConstraintBatch.apply_mask + torch.argmax + commit"},
        "reference_torch_gpu": ref_gpu,
        "tokens_only": tokens_only,
    }
    if not args.no_extra:
        # free the dense ring before the other workloads
        del bufs
        torch.cuda.empty_cache()
        line["pda_config4"] = _pda_config4(device, rank)
        line["pda_misses"] = _pda_misses(device, rank)
        line["pda_nesting"] = _pda_nesting(device, rank)
        line["dense_config3"] = _dense_config3(device, rank)
        line["soft_lookahead"] = _soft_lookahead(fsas, pats, device, rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        tok_next, starts = _cpu_tables([f.dense_tables()[0] for f in fsas],
                                       [f.start for f in fsas])
        line["cpu_baseline"] = cpu_baseline(tok_next, starts, pats, 80)
    if rank == 0:
        print(json.dumps(line), flush=True)
    shard.finish()


def _step_events(n: int, before, step) -> list[float]:
    """Per-step device time (µs) of `step(i)`, CUDA events right around it;
    `before(i)` (untimed, same stream) prepares step i's input."""
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(n)]
    for i in range(n):
        before(i)
        ev[i][0].record()
        step(i)
        ev[i][1].record()
    torch.cuda.synchronize()
    return [x.elapsed_time(y) * 1000 for x, y in ev]


def _pda_config4(device: torch.device, rank: int, steps: int = 512) -> dict:
    """Recursive JSON-value grammar on the PDA path (config 4): 256 rows,
    V = 128,256, fp32 logits N(0,1) + 3 on the { [ " , tokens, memo cleared at
    the start, 512 steps; one step = CFGConstraintBatch.step_greedy (mask +
    argmax + commit). Every step gets unmasked logits: one of 32 seeded
    buffers is copied into the step's input before it (untimed). Step latency
    from CUDA events around the step, run eagerly from Python and replayed
    from CUDA graphs (one graph per input buffer, captured after warm-up)."""
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import CFGConstraintBatch, PdaTensors
    from bpdecode_b200.workloads import BIASED, vocab_large

    B = 256
    vocab = vocab_large(V)
    g = PdaTensors.from_arrays(tables.load_pda("jsonvalue"), vocab, device)
    batch = CFGConstraintBatch(g, capacity=B)
    ids = list(range(B))
    for i in ids:
        batch.add(i)
    bias = torch.tensor([vocab.token_bytes.index(t) for t in BIASED], device=device)
    ring = 32
    src = []
    for i in range(ring):
        gen = torch.Generator(device=device).manual_seed(rank * 7919 + 40_000 + i)
        x = torch.randn(B, V, generator=gen, device=device)
        x[:, bias] += 3.0
        src.append(x)
    bufs = [x.clone() for x in src]

    def fresh(i: int) -> None:
        bufs[i % ring].copy_(src[i % ring])

    def restart() -> None:
        g.clear_memo()
        for r in ids:
            batch.reset(r)

    # one untimed step loads the kernels and allocates the memo / workspace
    fresh(0)
    batch.step_greedy(ids, bufs[0])
    restart()
    first = _step_events(1, fresh, lambda i: batch.step_greedy(ids, bufs[0]))[0]
    restart()
    eager = _step_events(steps, fresh, lambda i: batch.step_greedy(ids, bufs[i % ring]))
    # graphs: one captured step per buffer, replayed in sequence
    restart()
    s = torch.cuda.Stream(device)
    s.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(s):
        for i in range(3):
            fresh(i)
            batch.step_greedy(ids, bufs[i % ring])
    torch.cuda.current_stream(device).wait_stream(s)
    graphs = []
    for i in range(ring):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            batch.step_greedy(ids, bufs[i])
        graphs.append(gr)
    restart()
    torch.cuda.synchronize()
    us = sorted(_step_events(steps, fresh, lambda i: graphs[i % ring].replay()))
    del graphs
    # where an eager step's time goes: the unfused sequence on the same rows
    # (mask pipeline + apply, torch argmax, commit = advance_kernel), each
    # timed alone after warm steps (every row hits the memo by then)
    n = 32
    part = {"apply_mask": [], "argmax": [], "commit": []}
    for i in range(n):
        fresh(i)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        ev[0].record()
        batch.apply_mask(ids, bufs[i % ring])
        ev[1].record()
        tok = bufs[i % ring].argmax(-1)
        ev[2].record()
        batch.commit(ids, tok)
        ev[3].record()
        torch.cuda.synchronize()
        for k, name in enumerate(part):
            part[name].append(ev[k].elapsed_time(ev[k + 1]) * 1000)
    broken = int(batch._broken.sum())
    return {"workload": "recursive JSON-value GBNF, PDA, 256 rows, V=128256, fp32 N(0,1) "
                        f"+3 bias, memo cleared at start, {steps} steps, unmasked logits "
                        "every step",
            "step": "CFGConstraintBatch.step_greedy (mask + argmax + commit)",
            "graph_step_us_median": us[len(us) // 2], "graph_step_us_p90": us[int(len(us) * 0.9)],
            "eager_step_us_median": sorted(eager)[len(eager) // 2],
            "first_step_us_cold_memo": first,
            "unfused_us_median": {k: sorted(v)[len(v) // 2] for k, v in part.items()},
            "row_steps_per_s": B / (us[len(us) // 2] * 1e-6), "broken_rows_at_end": broken,
            "step_kernel_traffic_bytes": _profile_bytes("pda_step_config4.md"),
            "traffic_source": "ncu DRAM bytes per launch of the PDA step kernel, "
                              "profiles/pda_step_config4.md",
            "note": "the bounded PDA saturates at init on this grammar (8 configs), as the "
                    "reference does; after the first steps every row's config-set hits the memo"}


def _canon_rows(cfg) -> list[bytes]:
    """The live content of each 266-int config row (num_configs, depths and
    frames of the live configs), as bytes: equal content, equal mask."""
    import numpy as np

    out = []
    for r in cfg:
        n = int(r[0])
        d = r[2:2 + n]
        parts = [np.int32(n).tobytes(), d.tobytes()]
        parts += [r[10 + 32 * i:10 + 32 * i + int(d[i])].tobytes() for i in range(n)]
        out.append(b"".join(parts))
    return out


def _pda_nesting(device: torch.device, rank: int) -> dict:
    """The PDA path where nearly every row meets a config-set no row held
    before at every step: root ::= item+, item ::= "(" item* ")" | "[" item*
    "]" | "x" (the stack records the open brackets), 256 rows, V = 128,256,
    fp32 N(0, 1) + 1 on the "(" and "[" tokens; otherwise as _pda_misses."""
    from bpdecode_b200.workloads import OPENERS

    return _pda_misses(device, rank, name="brackets", bias=1.0, boost_tokens=OPENERS)


def _pda_misses(device: torch.device, rank: int, steps: int = 32, gens: int = 2,
                name: str = "schema", bias: float = 0.0, boost_tokens=None) -> dict:
    """The PDA path on a grammar that keeps producing config-sets the memo
    has not seen: the JSON-Schema object of config 3 as a PDA (its 1354-state
    rule NFAs, not the dense DFA), 256 rows, V = 128,256, fp32 N(0, 1), greedy;
    the memo and the transition cache are cleared at the start of each
    32-step generation. Per step: device time (CUDA events around
    CFGConstraintBatch.step_greedy, issued eagerly behind the step's input
    copy, as in _pda_config4) and the number of distinct
    config-sets the rows hold that the generation had not seen before (read
    between steps, untimed)."""
    from bpdecode_b200 import tables
    from bpdecode_b200.grammar.device import CFGConstraintBatch, PdaTensors
    from bpdecode_b200.workloads import vocab_large

    from bpdecode_b200.workloads import BIASED, token_ids

    B = 256
    vocab = vocab_large(V)
    g = PdaTensors.from_arrays(tables.load_pda(name), vocab, device)
    batch = CFGConstraintBatch(g, capacity=B)
    ids = list(range(B))
    for i in ids:
        batch.add(i)
    ring = 16
    src = [torch.randn(B, V, device=device,
                       generator=torch.Generator(device=device).manual_seed(rank * 97 + 500 + i))
           for i in range(ring)]
    if bias:
        boost = torch.tensor(token_ids(vocab, boost_tokens or BIASED), device=device)
        for x in src:
            x[:, boost] += bias
    work = torch.empty_like(src[0])
    for i in range(2):  # load the kernels, allocate the memo and workspace
        work.copy_(src[i])
        batch.step_greedy(ids, work)
    us: list[list[float]] = []
    new: list[list[int]] = []
    for gen in range(gens):
        g.clear_memo()
        for r in ids:
            batch.reset(r)
        seen: set[bytes] = set()
        us.append([])
        new.append([])
        for step in range(steps):
            rows = set(_canon_rows(batch._configs.cpu().numpy()))  # synchronises
            new[-1].append(len(rows - seen))
            seen |= rows
            # the input copy (131 MB) keeps the GPU busy while the step's
            # launches are issued, so the events time the step's kernels
            work.copy_(src[(gen * steps + step) % ring])
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            batch.step_greedy(ids, work)
            b.record()
            b.synchronize()
            us[-1].append(a.elapsed_time(b) * 1000)
    flat = [x for u in us for x in u]
    miss = [x for u, n in zip(us, new) for x, k in zip(u, n) if k > 0]
    what = {"schema": "JSON-Schema object as a PDA (1354 states)",
            "brackets": 'root ::= item+, item ::= "(" item* ")" | "[" item* "]" | "x" as a PDA'}
    return {"workload": f"{what.get(name, name)}, 256 rows, V=128256, fp32 N(0,1)"
                        + (f" + {bias:g} on the "
                           + " ".join(t.decode() for t in (boost_tokens or BIASED))
                           + " tokens" if bias else "")
                        + f", greedy, {gens} generations of {steps} steps, memo and "
                        "transition cache cleared at the start of each",
            "rows_per_step": B,
            "new_sets_share_late_mean": statistics.fmean(
                k / B for n in new for k in n[steps // 2:]),
            "step": "CFGConstraintBatch.step_greedy, eager",
            "us_per_step_mean": statistics.fmean(flat),
            "us_per_step_with_new_sets_mean": statistics.fmean(miss) if miss else None,
            "steps_with_new_sets": len(miss), "steps": len(flat),
            "us_first_step": [u[0] for u in us],
            "new_sets_per_step": new[0],
            "us_per_step": [round(x, 1) for x in us[0]]}


def _dense_config3(device: torch.device, rank: int, steps: int = 256) -> dict:
    """Config 3: the JSON-Schema object compiled to a dense DFA (1017 states),
    V = 151,936, 512 rows, fp32 logits N(0, 1), greedy commit, 256 steps from
    the start state; one step = ConstraintBatch.step_greedy. Every step gets
    unmasked logits (one of 16 seeded buffers copied into its input, untimed);
    CUDA events around each step."""
    from bpdecode_b200 import tables
    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.ops import FsaTensors
    from bpdecode_b200.workloads import vocab_large

    B3, V3 = 512, 151_936
    fsa = FsaTensors.from_arrays(tables.load_dfa("schema"), vocab_large(V3)).to(device)
    batch = ConstraintBatch(fsa, capacity=B3)
    ids = list(range(B3))
    for i in ids:
        batch.add(i)
    ring = 16
    src = [torch.randn(B3, V3, device=device,
                       generator=torch.Generator(device=device).manual_seed(rank * 131 + 7 + i))
           for i in range(ring)]
    work = torch.empty_like(src[0])

    def fresh(i: int) -> None:
        work.copy_(src[i % ring])

    for i in range(3):
        fresh(i)
        batch.step_greedy(ids, work)
    batch.reset_many(ids)
    us = _step_events(steps, fresh, lambda i: batch.step_greedy(ids, work))
    mean = statistics.fmean(us)
    algo = 2 * V3 * 4 + 4 * ((V3 + 31) // 32) + 16
    peak, _ = _peaks()
    achieved = B3 * algo / (mean * 1e-6) / 1e9
    traffic = _profile_bytes("dense_step_config3.md")
    return {"workload": "JSON-Schema object as a dense DFA (1017 states), V=151936, 512 rows, "
                        "fp32 N(0,1), greedy, 256 steps from the start state",
            "us_per_step": mean, "row_steps_per_s": B3 / (mean * 1e-6),
            "algo_bytes_per_row_step": algo, "achieved_gbs": achieved,
            "roofline_frac": achieved / peak,
            "traffic_bytes_per_launch": traffic,
            "traffic_gbs": traffic / (mean * 1e-6) / 1e9 if traffic else None,
            "roofline_frac_traffic": traffic / (mean * 1e-6) / 1e9 / peak if traffic else None,
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum per launch, "
                              "profiles/dense_step_config3.md (rejected vectors are written "
                              "without being read, so the algorithmic fraction exceeds 1)"}


def _soft_lookahead(fsas, pats, device: torch.device, rank: int, steps: int = 128) -> dict:
    """Soft lookahead (horizon 4) over the 8-regex dense rows in fp32: table
    build time, then one 128-step generation from the start states timed per
    step two ways -- apply_soft + argmax + commit (the reference's sequence)
    and the fused soft step (one launch). apply_soft adds the bias in place,
    so every step gets unbiased logits: one of 16 seeded buffers is copied
    into the step's input before it (untimed)."""
    from dataclasses import replace

    from bpdecode_b200.batch import ConstraintBatch
    from bpdecode_b200.ops import build_lookahead

    t0 = time.perf_counter()
    soft = [replace(f, lookahead=build_lookahead(f, 4)) for f in fsas]
    torch.cuda.synchronize()
    build_s = time.perf_counter() - t0
    ids = list(range(ROWS_PER_GPU))
    ring = 16
    src = [torch.randn(ROWS_PER_GPU, V, device=device,
                       generator=torch.Generator(device=device).manual_seed(rank * 31 + i))
           for i in range(ring)]
    work = torch.empty_like(src[0])

    def fresh(i: int) -> None:
        work.copy_(src[i % ring])

    def timed(step) -> float:
        batch = ConstraintBatch(soft, capacity=ROWS_PER_GPU)
        for i in ids:
            batch.add(i, grammar=pats[i])
        for i in range(3):
            fresh(i)
            step(batch)
        batch.reset_many(ids)
        return statistics.fmean(_step_events(steps, fresh, lambda i: step(batch)))

    def unfused(batch) -> None:
        batch.apply_soft(ids, work, 1.0)
        batch.commit(ids, work.argmax(-1))

    us = timed(unfused)
    us_fused = timed(lambda batch: batch.soft_step_greedy(ids, work, 1.0))
    logit_bytes = 2 * 4 * V * ROWS_PER_GPU
    return {"workload": f"soft lookahead k=4, 8 regexes, {ROWS_PER_GPU} rows, V={V}, fp32, "
                        f"{steps}-step generation from the start states",
            "table_build_s": build_s,
            "unfused_ms_per_step": us / 1e3, "unfused_row_steps_per_s": ROWS_PER_GPU / (us / 1e6),
            "fused_ms_per_step": us_fused / 1e3,
            "fused_row_steps_per_s": ROWS_PER_GPU / (us_fused / 1e6),
            "fused_logits_gbs": logit_bytes / (us_fused / 1e6) / 1e9,
            "note": "fused_logits_gbs counts the logits read + written once per step "
                    "(2 x 4 B x V per row); rejected tiles are written without a read"}


def _tokens_only(batch, ids, bufs, ring, stream) -> dict:
    """ConstraintBatch.step_greedy_from(ids, logits) with no output: the same
    mask + argmax + commit of every row on the config-2 trajectory, but the
    masked logits are not materialised (a sampler that needs only the greedy
    token). Logits are read where a token is allowed and never written. One
    generation of 128 steps, CUDA events around the whole run."""
    for i in range(3):
        batch.step_greedy_from(ids, bufs[i % ring])
    batch.reset_many(ids)
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for i in range(EPISODE):
        batch.step_greedy_from(ids, bufs[i % ring])
    b.record(stream)
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / EPISODE
    batch.reset_many(ids)
    return {"ms_per_step": ms, "value": ROWS_PER_GPU / (ms / 1e3),
            "algo_bytes_per_row_step": V * E + 4 * ((V + 31) // 32) + 16,
            "path": "ConstraintBatch.step_greedy_from(ids, bf16 logits) -- tokens and commits, "
                    "no masked logits written"}


def _reference_torch_gpu(batch, bufs, ring, device) -> dict:
    """bpdecode's dense path is torch (ops.py:271-276, 301-306): time that
    composite on this GPU on the same rows as the GPU bar the kernel beats."""
    tn = batch._t.tok_next
    state = batch._state.clone()
    slots = torch.arange(ROWS_PER_GPU, device=device)

    def step(lg: torch.Tensor) -> None:
        s = state[slots].long()
        broken = s < 0
        rejected = tn.index_select(0, s.clamp(min=0)) == -1
        rejected |= broken.unsqueeze(1)
        lg.masked_fill_(rejected, float("-inf"))
        tok = lg.argmax(-1)
        nxt = tn[s.clamp(min=0), tok]
        state[slots] = torch.where(broken, torch.full_like(nxt, -1), nxt)

    n = 16
    for i in range(3):
        step(bufs[i % ring])
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(n):
        step(bufs[i % ring])
    b.record()
    torch.cuda.synchronize()
    ms = a.elapsed_time(b) / n
    return {"ms_per_step": ms, "value": ROWS_PER_GPU / (ms / 1e3),
            "path": "ops.py dense composite (index_select + masked_fill_ + argmax + gather)"}


def _e2e(batch, ids, block, device, steps, world) -> dict:
    """Same step through the public API from pinned host logits: every step
    copies its logits host -> device, runs ConstraintBatch.step_greedy and
    reads the chosen tokens back."""
    from bpdecode_b200 import shard

    nhost = 2
    host = [gen_logits(block, 10_000 + i, device).cpu().pin_memory() for i in range(nhost)]
    dev = torch.empty(ROWS_PER_GPU, V, dtype=torch.bfloat16, device=device)
    out = torch.empty(ROWS_PER_GPU, dtype=torch.int64).pin_memory()
    for i in range(2):
        dev.copy_(host[i % nhost], non_blocking=True)
        out.copy_(batch.step_greedy(ids, dev), non_blocking=True)
    torch.cuda.synchronize()
    shard.barrier()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for i in range(steps):
        dev.copy_(host[i % nhost], non_blocking=True)
        out.copy_(batch.step_greedy(ids, dev), non_blocking=True)
    b.record()
    torch.cuda.synchronize()
    ms = shard.max_over_ranks([a.elapsed_time(b)], device)[0]
    return {"value": ROWS_PER_GPU * world * steps / (ms / 1e3), "unit": UNIT,
            "h2d_bytes_per_step": ROWS_PER_GPU * V * 2, "d2h_bytes_per_step": ROWS_PER_GPU * 8,
            "steps": steps, "ms_per_step": ms / steps,
            "path": "pinned host logits -> H2D -> ConstraintBatch.step_greedy -> tokens D2H"}


if __name__ == "__main__":
    main()
