#!/usr/bin/env python
"""Benchmark of the B200 decode engine for imi's brain token loop.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload ride2|b1|prefill|multi64|sweep] [--no-extra]

Headline (the batch-2 "riding" step): the Seoul-shaped synthetic backbone (seed 0);
conversation A prefilled with 1024 random ids (seed 1), conversation B with 256 (seed 2); then every timed step is
one step2 (imi_seoul::step2, seoul.cpp:208): both conversations advance one greedy position on one read of every
table. Under torchrun each rank runs the same workload on its own GPU (whole conversations per GPU, no collective):
weak scaling.

The default line also carries, unless --no-extra: `b1` (configs[0]: batch-1 greedy decode after a 32-id prompt),
`multi64` (configs[3]: 64 conversations per GPU with contexts drawn from 256..2048, one greedy position of all 64 per
step; box tokens/s summed over the ranks) and, on one GPU, `sweep` (configs[4]: the isolated table read, N x K in
{2048x2048, 8192x2048, 2048x8192, 97,496x2048} x B in {1, 2, 8, 32, 128}, GB/s). `--workload X` makes X the headline.
`--workload prefill` runs configs[2] (one step = one fresh conversation reading 400 input vectors and 16 ids in
chunks of 128, the last position's word scores; positions/s).

One JSON line on rank 0: `value` = tokens/s of the whole job with everything resident on the device (CUDA events on
the engine's stream, max over ranks); `e2e` = the same through the public calls with host token input and a host read
of every pick every step; `roofline` = the table-read kernel's bandwidth against the measured HBM peak;
`step_roofline` = the whole step's algorithmic bytes (every weight once per step, each conversation's K/V and conv
memory) over its time; `cpu_baseline` = the reference's own CPU code (oracle/_ref) on this host at all cores and at 4
threads pinned to cores 0-3, with the CPU model.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

A_PROMPT, B_PROMPT, B1_PROMPT = 1024, 256, 32


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0, help="timed steps (0 = the workload's default)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", choices=["ride2", "b1", "prefill", "multi64", "sweep"], default="ride2")
    ap.add_argument("--no-extra", action="store_true", help="headline only (no b1 / multi64 / sweep sub-objects)")
    ap.add_argument("--extra-steps", type=int, default=64, help="timed steps of the multi64 sub-object")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    a = ap.parse_args()
    if not a.steps:
        a.steps = {"prefill": 5, "multi64": 256, "sweep": 1}.get(a.workload, 128)
    return a


class Ranks:
    """RANK / WORLD_SIZE / LOCAL_RANK from torchrun; host-side barrier and max over a gloo group."""

    def __init__(self):
        self.rank = int(os.environ.get("RANK", 0))
        self.world = int(os.environ.get("WORLD_SIZE", 1))
        self.local = int(os.environ.get("LOCAL_RANK", 0))
        self.pg = None
        if self.world > 1:
            import datetime
            import torch.distributed as dist
            os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
            self.dist = dist

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, x: float) -> float:
        if self.world == 1:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


class Clocks:
    """nvidia-smi samples every 200 ms while the timed region runs (median SM clock under load, throttle reasons)."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,utilization.gpu,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index, self.proc, self.path = index, None, None

    def start(self):
        try:
            fd, self.path = tempfile.mkstemp(prefix="imi_clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.index), "-f", self.path],
                                         stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if not self.proc:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        self.proc.wait()
        rows = []
        with open(self.path) as f:
            for line in f:
                p = [x.strip() for x in line.split(",")]
                if len(p) >= 10:
                    rows.append(p)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        busy = [r for r in rows if (num(r[4]) or 0) > 0] or rows
        sm = [num(r[1]) for r in busy if num(r[1])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[k] for r in rows for k in range(4) if r[6 + k].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(rows[0][2]),
                "samples": len(rows), "reasons": reasons}


def table_traffic(ncol: int):
    """DRAM bytes (read + write) of one bench_tables pass at `ncol` inputs, from the committed ncu summary
    profiles/k_table_dram.txt (lines `ncol=<n> dram_bytes_per_pass=<bytes>`), or None when it has no such line."""
    p = os.path.join(ROOT, "profiles", "k_table_dram.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            kv = dict(x.split("=", 1) for x in line.split() if "=" in x)
            if kv.get("ncol") == str(ncol) and "dram_bytes_per_pass" in kv:
                return int(kv["dram_bytes_per_pass"])
    return None


def peaks() -> dict:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d.get("bf16_tflops"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


PREFILL_VECS, PREFILL_IDS, PREFILL_CHUNK = 400, 16, 128
MULTI_N, MULTI_CTX = 64, (256, 2048)


def multi_contexts(rank: int) -> list:
    """each session's context length, uniform in 256..2048 (seed 4 + the GPU's rank)."""
    rng = np.random.default_rng(4 + rank)
    return [int(x) for x in rng.integers(MULTI_CTX[0], MULTI_CTX[1] + 1, MULTI_N)]


def workload_desc(workload: str) -> dict:
    if workload == "prefill":
        return {"workload": f"configs[2] prefill: Seoul-shaped Q4_0 backbone (seed 0), a fresh conversation reads "
                            f"{PREFILL_VECS} input vectors N(0,1)*0.5 (seed 3) then {PREFILL_IDS} random ids (seed 3) "
                            f"in chunks of {PREFILL_CHUNK} (step_batch calls of 128, 128, 128, 16 vectors and 16 ids), "
                            "word scores of the last position; host inputs copied inside the timed region (the API "
                            "takes host vectors)", "tokens_per_step": PREFILL_VECS + PREFILL_IDS, "prompts": []}
    if workload == "multi64":
        return {"workload": f"configs[3] {MULTI_N} sessions per GPU: contexts uniform in {MULTI_CTX[0]}..{MULTI_CTX[1]} "
                            "(seed 4 + rank) read beforehand (not timed), then greedy steps of all sessions",
                "tokens_per_step": MULTI_N, "prompts": []}
    if workload == "sweep":
        return {"workload": "configs[4] isolated Q4_0 x Q8 table read: N x K in " +
                            ", ".join(f"{r}x{c}" for r, c in SWEEP_SHAPES) + f"; B in {list(SWEEP_B)}; random codes "
                            "and fp16 scales, table copies rotated through more than 256 MB so every read comes from "
                            "HBM", "tokens_per_step": 0, "prompts": []}
    if workload == "ride2":
        return {"workload": "configs[1] riding step2: Seoul-shaped Q4_0 backbone (seed 0), conversation A after a "
                            f"{A_PROMPT}-id prompt, B after {B_PROMPT} ids, greedy, one table read per step for both",
                "tokens_per_step": 2, "prompts": [A_PROMPT, B_PROMPT]}
    return {"workload": f"configs[0] batch-1 greedy decode: Seoul-shaped Q4_0 backbone (seed 0), {B1_PROMPT}-id prompt",
            "tokens_per_step": 1, "prompts": [B1_PROMPT]}


def step_bytes(info, positions) -> int:
    """Algorithmic HBM bytes of one decode step of conversations at `positions`: every weight byte once (layer tables,
    word table, small parameters), plus each conversation's K/V read over its positions and written at the new one,
    plus its conv memory read and written. Activations are negligible."""
    kvd = info.n_head_kv * info.head_dim
    kv = sum((p + 1) * info.n_attn * kvd * 2 * 2 + info.n_attn * kvd * 2 * 2 for p in positions)
    conv = len(positions) * (info.n_layer - info.n_attn) * 2 * info.d_conv * info.n_embd * 4
    return int(info.weight_bytes + kv + conv)


def step_roofline(bytes_per_step: int, ms_per_step: float, pk: dict) -> dict:
    gbs = bytes_per_step / (ms_per_step / 1e3) / 1e9
    return {"bytes_per_step": int(bytes_per_step), "achieved_gbs": gbs, "frac": gbs / pk["hbm_gbs"],
            "peak_gbs": pk["hbm_gbs"], "peak_source": pk["source"],
            "bytes": "algorithmic: every weight once per step + each conversation's K/V and conv memory"}


def run_ours(args, ranks: Ranks, workload: str, steps: int, e2e: bool = True) -> dict:
    """configs[1] (ride2) or configs[0] (b1): the conversations' prompts read, then `steps` greedy steps replayed on
    the device (CUDA events), then as many through the public step calls (e2e)."""
    import torch
    import nunchi_b200 as nb
    from nunchi_b200 import synth
    torch.cuda.set_device(ranks.local)
    wl = workload_desc(workload)
    prompts = wl["prompts"]
    n_ctx = max(prompts) + args.warmup + 2 * steps + 16
    path = synth.cached_gguf("seoul", 0)
    eng = nb.Engine(path, device=ranks.local, n_ctx=n_ctx, max_batch=8)
    info = eng.info
    states = [eng.new_state() for _ in prompts]
    for i, (s, n) in enumerate(zip(states, prompts)):
        s.step_batch(synth.random_ids(n, info.n_vocab, 1 + i), want_logits=True)
    st = torch.cuda.ExternalStream(eng.stream)
    ev = lambda: torch.cuda.Event(enable_timing=True)   # noqa: E731
    nb.greedy(states, args.warmup)
    torch.cuda.synchronize()
    ranks.barrier()
    pos0 = [s.pos for s in states]
    clocks = Clocks(ranks.local)
    clocks.start()
    e0, e1 = ev(), ev()
    torch.cuda.nvtx.range_push("timed")   # ncu --nvtx --nvtx-include "timed/" selects these launches
    e0.record(st)
    nb.greedy(states, steps)
    e1.record(st)
    torch.cuda.nvtx.range_pop()
    e1.synchronize()
    torch.cuda.synchronize()
    clk = clocks.stop()
    ranks.barrier()
    ms = ranks.max(e0.elapsed_time(e1))
    tps = wl["tokens_per_step"]
    value = ranks.world * tps * steps / (ms / 1e3)
    mid = [p + steps // 2 for p in pos0]
    out = {"ms": ms, "value": value, "clocks": clk, "info": info, "mid_positions": mid, "ncol": len(states)}
    out["step_bytes"] = step_bytes(info, mid)
    out["launches"] = eng.launches_per_step(len(states)) * steps
    # end to end through the public API: host token in, step, host read of the pick, every step
    if e2e and not args.no_e2e:
        picks = [s.argmax()[0] for s in states]
        ranks.barrier()
        e2, e3 = ev(), ev()
        torch.cuda.synchronize()
        e2.record(st)
        for _ in range(steps):
            if len(states) == 2:
                nb.step2(states[0], picks[0], None, True, states[1], picks[1], None, True)
            else:
                states[0].step(picks[0])
            picks = [s.argmax()[0] for s in states]
        e3.record(st)
        e3.synchronize()
        ms_e2e = ranks.max(e2.elapsed_time(e3))
        col_bytes, sess_bytes = 80, 24
        out["e2e"] = {"value": ranks.world * tps * steps / (ms_e2e / 1e3), "unit": "tok/s",
                      "h2d_bytes_per_step": col_bytes * len(states), "d2h_bytes_per_step": (sess_bytes + 4) * len(states),
                      "ms_per_step": ms_e2e / steps}
    # the table-read kernel alone: every layer table back to back (imi_seoul::bench_tables); the NVTX range lets a
    # profiler select exactly these launches (ncu --nvtx --nvtx-include "bench_tables/")
    torch.cuda.nvtx.range_push("bench_tables")
    t_ms, t_bytes = eng.bench_tables(ncol=len(states), reps=20)
    torch.cuda.nvtx.range_pop()
    out["tables"] = {"ms": t_ms, "bytes": t_bytes}
    for s in states:
        s.close()
    eng.close()
    return out


def prefill_inputs(n_embd: int, n_vocab: int):
    from nunchi_b200 import synth
    rng = np.random.default_rng(3)
    vecs = (rng.standard_normal((PREFILL_VECS, n_embd)) * 0.5).astype(np.float32)
    return vecs, synth.random_ids(PREFILL_IDS, n_vocab, 3)


def prefill_calls(s, vecs, ids):
    """configs[2]'s reads of one conversation: the vectors in chunks of 128, then the ids with the word scores."""
    for a in range(0, len(vecs), PREFILL_CHUNK):
        s.step_batch(embd=vecs[a:a + PREFILL_CHUNK], want_logits=False)
    s.step_batch(ids, want_logits=True)


def prefill_reads() -> int:
    """step_batch calls of one configs[2] prefill: the vector chunks, then the ids"""
    return -(-PREFILL_VECS // PREFILL_CHUNK) + 1


def run_prefill(args, ranks: Ranks, steps: int) -> dict:
    import torch
    import nunchi_b200 as nb
    from nunchi_b200 import synth
    torch.cuda.set_device(ranks.local)
    eng = nb.Engine(synth.cached_gguf("seoul", 0), device=ranks.local, n_ctx=512, max_batch=8)
    info = eng.info
    s = eng.new_state()
    vecs, ids = prefill_inputs(info.n_embd, info.n_vocab)
    st = torch.cuda.ExternalStream(eng.stream)
    ev = lambda: torch.cuda.Event(enable_timing=True)   # noqa: E731
    for _ in range(args.warmup):
        s.reset()
        prefill_calls(s, vecs, ids)
    torch.cuda.synchronize()
    ranks.barrier()
    clocks = Clocks(ranks.local)
    clocks.start()
    e0, e1 = ev(), ev()
    t0 = time.perf_counter()
    torch.cuda.nvtx.range_push("timed")
    e0.record(st)
    picks = []
    for _ in range(steps):
        s.reset()
        prefill_calls(s, vecs, ids)
        picks.append(s.argmax()[0])   # the host read of the prefill's result (the first greedy word)
    e1.record(st)
    torch.cuda.nvtx.range_pop()
    e1.synchronize()
    wall = time.perf_counter() - t0
    clk = clocks.stop()
    ranks.barrier()
    ms, ms_wall = ranks.max(e0.elapsed_time(e1)), ranks.max(wall * 1e3)
    assert len(set(picks)) == 1, "prefills of the same inputs gave different picks"
    n_pos = PREFILL_VECS + PREFILL_IDS
    out = {"ms": ms, "value": ranks.world * n_pos * steps / (ms / 1e3), "clocks": clk, "info": info,
           "ncol": min(PREFILL_CHUNK, info.cols_per_read)}
    out["launches"] = eng.prefill_launches(PREFILL_VECS, PREFILL_CHUNK, PREFILL_IDS) * steps
    out["e2e"] = {"value": ranks.world * n_pos * steps / (ms_wall / 1e3), "unit": "positions/s",
                  "h2d_bytes_per_step": int(vecs.nbytes + ids.nbytes), "d2h_bytes_per_step": 8,
                  "ms_per_step": ms_wall / steps, "clock": "host wall clock around the same calls"}
    t_ms, t_bytes = eng.bench_tables(ncol=out["ncol"], reps=20)
    out["tables"] = {"ms": t_ms, "bytes": t_bytes}
    # algorithmic: every weight once per step_batch call (the configuration's chunks), K/V of the positions written
    # once and read by the later ones; the word table once (the last position's scores)
    kvd = info.n_head_kv * info.head_dim
    out["step_bytes"] = int(prefill_reads() * (info.weight_bytes - table_bytes_word(info)) + table_bytes_word(info)
                            + info.n_attn * kvd * 4 * n_pos * (n_pos + 1) // 2)
    # the contraction (2 flops per weight per position; Q4_0 holds 32 weights in 18 bytes) + the last word scores
    out["flops_per_step"] = 2 * (t_bytes * 16 // 9) * n_pos + 2 * info.n_vocab * info.n_embd
    s.close()
    eng.close()
    return out


def table_bytes_word(info) -> int:
    """Bytes of the Q4_0 word table (the word table is read once per step with word scores)."""
    return info.n_vocab * info.n_embd // 32 * 18


def run_multi(args, ranks: Ranks, steps: int, e2e: bool = True) -> dict:
    """64 sessions per GPU, contexts read beforehand (not timed), then `steps` greedy steps of all."""
    import torch
    import nunchi_b200 as nb
    from nunchi_b200 import synth
    torch.cuda.set_device(ranks.local)
    ctx = multi_contexts(ranks.rank)
    n_ctx = MULTI_CTX[1] + args.warmup + 2 * steps + 8   # warm-up, timed steps, end-to-end steps
    eng = nb.Engine(synth.cached_gguf("seoul", 0), device=ranks.local, n_ctx=n_ctx, max_batch=MULTI_N)
    info = eng.info
    states = [eng.new_state() for _ in range(MULTI_N)]
    t0 = time.perf_counter()
    for i, (s, n) in enumerate(zip(states, ctx)):
        s.step_batch(synth.random_ids(n, info.n_vocab, 100 * ranks.rank + i), want_logits=True)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    st = torch.cuda.ExternalStream(eng.stream)
    ev = lambda: torch.cuda.Event(enable_timing=True)   # noqa: E731
    nb.greedy(states, args.warmup)
    torch.cuda.synchronize()
    ranks.barrier()
    pos0 = [s.pos for s in states]
    clocks = Clocks(ranks.local)
    clocks.start()
    e0, e1 = ev(), ev()
    torch.cuda.nvtx.range_push("timed")   # ncu --nvtx --nvtx-include "timed/" selects these launches
    e0.record(st)
    nb.greedy(states, steps)
    e1.record(st)
    torch.cuda.nvtx.range_pop()
    e1.synchronize()
    clk = clocks.stop()
    ranks.barrier()
    ms = ranks.max(e0.elapsed_time(e1))
    per_read = min(MULTI_N, info.cols_per_read)
    out = {"ms": ms, "value": ranks.world * MULTI_N * steps / (ms / 1e3), "clocks": clk, "info": info,
           "ncol": per_read, "prefill_s": prefill_s, "reads_per_step": -(-MULTI_N // per_read)}
    mid = [p + steps // 2 for p in pos0]
    out["step_bytes"] = step_bytes(info, mid)   # every weight once per step of all 64, plus each one's K/V
    out["launches"] = eng.launches_per_step(MULTI_N, 1) * steps
    if e2e and not args.no_e2e:   # host ids in, one step of all, host read of every pick, each step
        picks = np.array([s.argmax()[0] for s in states], np.int32)
        e2, e3 = ev(), ev()
        torch.cuda.synchronize()
        e2.record(st)
        for _ in range(steps):
            nb.step_multi(states, picks)
            picks = np.array([s.argmax()[0] for s in states], np.int32)
        e3.record(st)
        e3.synchronize()
        ms_e2e = ranks.max(e2.elapsed_time(e3))
        out["e2e"] = {"value": ranks.world * MULTI_N * steps / (ms_e2e / 1e3), "unit": "tok/s",
                      "h2d_bytes_per_step": 80 * MULTI_N, "d2h_bytes_per_step": 28 * MULTI_N,
                      "ms_per_step": ms_e2e / steps}
    t_ms, t_bytes = eng.bench_tables(ncol=per_read, reps=20)
    out["tables"] = {"ms": t_ms, "bytes": t_bytes}
    for s in states:
        s.close()
    eng.close()
    return out


SWEEP_SHAPES = ((2048, 2048), (8192, 2048), (2048, 8192), (97496, 2048))
SWEEP_B = (1, 2, 8, 32, 128)


def run_sweep(args, ranks: Ranks, pk: dict) -> dict:
    """the isolated table read (imi_cuda_bench_matvec) for every shape and batch, GB/s of its algorithmic
    bytes (table once, inputs' codes and scales, outputs) and, for the batches read as a contraction, TFLOP/s."""
    import torch
    import nunchi_b200 as nb
    torch.cuda.set_device(ranks.local)
    rows = []
    for n, k in SWEEP_SHAPES:
        for b in SWEEP_B:
            ms, byts = nb.bench_matvec(n, k, b, reps=20, device=ranks.local)
            gbs = byts / (ms / 1e3) / 1e9
            tf = 2.0 * b * n * k / (ms / 1e3) / 1e12
            rows.append({"N": n, "K": k, "B": b, "ms": ms, "bytes": byts, "gbs": gbs, "hbm_frac": gbs / pk["hbm_gbs"],
                         "tflops": tf, "tensor_frac": tf / pk["bf16_tflops"] if pk.get("bf16_tflops") else None})
    return {"rows": rows, "peak_gbs": pk["hbm_gbs"], "peak_tflops": pk.get("bf16_tflops"), "peak_source": pk["source"],
            "note": "one read = every input once against the table; inputs above 8 per read are read as groups of 8 "
                    "per table read by the small-batch kernel unless the tensor-core path runs them"}


MULTI_CPU_SESSIONS = 4


def cpu_model() -> str:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


class Pinned:
    """Run the reference's CPU code on a fixed set of cores: the affinity is set before its thread team starts (the
    workers inherit it) and restored afterwards (taskset -c 0-3, as the reference's 4-thread figures, README.md)."""

    def __init__(self, cpus):
        self.cpus = set(cpus) if cpus else None

    def __enter__(self):
        self.old = os.sched_getaffinity(0)
        if self.cpus:
            os.sched_setaffinity(0, self.cpus)
        return self

    def __exit__(self, *exc):
        os.sched_setaffinity(0, self.old)


def reference_threads() -> int:
    return len(os.sched_getaffinity(0)) or os.cpu_count() or 1


def run_reference_decode(workload: str, steps: int, threads: int) -> dict:
    """configs[0] / configs[1] on the reference's own CPU path (imi/core/seoul.cpp + tables.cpp compiled from the
    reference tree into oracle/_ref): `steps` timed positions after the same prompts."""
    import oracle
    from nunchi_b200 import synth
    wl = workload_desc(workload)
    prompts = wl["prompts"]
    if not oracle.reference_available():
        raise RuntimeError("oracle/_ref/libimi_ref.so is not built")
    n_ctx = max(prompts) + steps + 8
    r = oracle.Reference(synth.cached_gguf("seoul", 0), n_ctx=n_ctx, threads=threads)
    t0 = time.perf_counter()
    other = r.new_state() if len(prompts) == 2 else None
    if other is not None:   # B's prompt through the brain's own conversation, then parked in `other`
        r.step_batch(synth.random_ids(prompts[1], r.n_vocab, 2), want_logits=True)
        r.swap_state(other)
    r.step_batch(synth.random_ids(prompts[0], r.n_vocab, 1), want_logits=True)
    prefill_s = time.perf_counter() - t0
    ta = int(np.argmax(r.logits))
    tb = int(np.argmax(other.logits)) if other is not None else None
    t0 = time.perf_counter()
    for _ in range(steps):
        if other is not None:
            r.step2(ta, None, True, other, tb, None, True)
            ta, tb = int(np.argmax(r.logits)), int(np.argmax(other.logits))
        else:
            r.step(ta)
            ta = int(np.argmax(r.logits))
    dt = time.perf_counter() - t0
    tps = wl["tokens_per_step"]
    return {"value": tps * steps / dt, "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"{steps} steps ({tps * steps} tokens) of the same workload after the same prompts "
                      f"(prefill {prefill_s:.1f} s, not timed); imi_seoul from the reference's seoul.cpp/tables.cpp, "
                      f"AVX2, {threads} threads", "ms_per_step": dt / steps * 1e3}


def run_reference_prefill(steps: int, threads: int) -> dict:
    """configs[2] on the reference's CPU path: `steps` fresh conversations each reading the same 416 positions
    (imi_seoul::reset + step_batch, seoul.cpp:188-191,490-517)."""
    import oracle
    from nunchi_b200 import synth
    if not oracle.reference_available():
        raise RuntimeError("oracle/_ref/libimi_ref.so is not built")
    r = oracle.Reference(synth.cached_gguf("seoul", 0), n_ctx=512, threads=threads)
    vecs, ids = prefill_inputs(r.n_embd, r.n_vocab)
    t0 = time.perf_counter()
    for _ in range(steps):
        r.reset()
        prefill_calls(r, vecs, ids)
        int(np.argmax(r.logits))
    dt = time.perf_counter() - t0
    n = (PREFILL_VECS + PREFILL_IDS) * steps
    return {"value": n / dt, "unit": "positions/s", "cores": threads, "kind": "reference",
            "sample": f"{steps} prefills of the same 416 positions; imi_seoul from the reference's seoul.cpp/tables.cpp, "
                      f"AVX2, {threads} threads", "ms_per_step": dt / steps * 1e3}


def run_reference_multi(steps: int, threads: int) -> dict:
    """configs[3] on the reference's CPU path, a bounded sample: the first sessions of rank 0's draw, their contexts
    read beforehand (not timed), then `steps` greedy positions of each, the sessions one after another through
    swap_state (the reference runs one conversation at a time; no CPU batching is invented)."""
    import oracle
    from nunchi_b200 import synth
    if not oracle.reference_available():
        raise RuntimeError("oracle/_ref/libimi_ref.so is not built")
    ctx = multi_contexts(0)[:MULTI_CPU_SESSIONS]
    r = oracle.Reference(synth.cached_gguf("seoul", 0), n_ctx=MULTI_CTX[1] + steps + 8, threads=threads)
    parked = []
    for i, n in enumerate(ctx):
        r.reset()
        r.step_batch(synth.random_ids(n, r.n_vocab, i), want_logits=True)
        s = r.new_state()
        r.swap_state(s)   # the session's memory parks in s; the brain's own becomes a fresh one
        parked.append(s)
    picks = [int(np.argmax(s.logits)) for s in parked]
    t0 = time.perf_counter()
    for _ in range(steps):
        for i, s in enumerate(parked):
            r.swap_state(s)
            r.step(picks[i])
            picks[i] = int(np.argmax(r.logits))
            r.swap_state(s)
    dt = time.perf_counter() - t0
    n = len(parked) * steps
    return {"value": n / dt, "unit": "tok/s", "cores": threads, "kind": "reference",
            "sample": f"{len(parked)} of the 64 sessions (contexts {ctx}, read beforehand, not timed), {steps} greedy "
                      f"steps each, one session at a time via swap_state; imi_seoul from the reference's "
                      f"seoul.cpp/tables.cpp, AVX2, {threads} threads", "ms_per_step": dt / steps * 1e3}


def run_reference_tables(ncol: int, threads: int) -> dict:
    """the reference's own table reads alone (imi_seoul::bench_tables, seoul.cpp:657-685: every layer table back to
    back, 1 or 2 inputs riding each read): CPU GB/s of the layer tables"""
    import oracle
    from nunchi_b200 import synth
    r = oracle.Reference(synth.cached_gguf("seoul", 0), n_ctx=16, threads=threads)
    ms = r.bench_tables(ncol=ncol, reps=5)
    return {"ms": ms, "gbs": TABLE_BYTES / (ms / 1e3) / 1e9, "B": ncol, "cores": threads}


TABLE_BYTES = 582967296   # the Seoul shape's layer tables, every row once: one pass


def run_reference(workload: str, steps: int, threads: int) -> dict:
    if workload == "prefill":
        return run_reference_prefill(steps, threads)
    if workload == "multi64":
        return run_reference_multi(steps, threads)
    if workload == "sweep":
        rows = [run_reference_tables(b, threads) for b in (1, 2)]
        return {"value": rows[0]["gbs"], "unit": "GB/s", "cores": threads, "kind": "reference", "rows": rows,
                "sample": "imi_seoul::bench_tables (every layer table back to back, 5 passes, best) at 1 and 2 inputs; "
                          f"the reference's batched read (imi_q4_group_batch) is not timed alone; {threads} threads",
                "ms_per_step": rows[0]["ms"]}
    return run_reference_decode(workload, steps, threads)


def cpu_steps(workload: str) -> int:
    return {"ride2": 64, "prefill": 3, "multi64": 16, "sweep": 1}.get(workload, 128)


def cpu_baseline(workload: str, steps: int) -> dict:
    """The reference's CPU path at all of this host's cores and at 4 threads pinned to cores 0-3."""
    allc = reference_threads()
    try:
        with Pinned(None):
            full = run_reference(workload, steps, allc)
        four = None
        if len(os.sched_getaffinity(0)) >= 4:
            with Pinned(sorted(os.sched_getaffinity(0))[:4]):
                four = run_reference(workload, steps, 4)
    except Exception as ex:   # the reference build is missing: say so, keep the GPU line
        return {"value": None, "unit": "tok/s", "cores": 0, "kind": "reference", "sample": f"unavailable: {ex}"}
    out = {k: full[k] for k in ("value", "unit", "cores", "kind", "sample")}
    out["cpu_model"] = cpu_model()
    if "rows" in full:
        out["rows"] = full["rows"]
    if four is not None:
        out["at_4_threads"] = {"value": four["value"], "unit": four["unit"], "cores": 4,
                               "pinned": "the first 4 cores of this process's affinity (taskset -c 0-3 equivalent)"}
    return out


METRIC = {"ride2": "decode tok/s, batch-2 riding step (step2), Seoul-shaped Q4_0 backbone",
          "b1": "decode tok/s, batch-1 greedy step, Seoul-shaped Q4_0 backbone",
          "prefill": "prefill positions/s, 400 input vectors + 16 ids, Seoul-shaped Q4_0 backbone",
          "multi64": "decode tok/s, 64 sessions per GPU, Seoul-shaped Q4_0 backbone",
          "sweep": "isolated Q4_0 x Q8 table read GB/s (97,496 x 2048, B=1)"}


def sub_line(r: dict, steps: int, workload: str, pk: dict, cpu: dict = None) -> dict:
    """a sub-object of the default line: one more configuration, measured the same way"""
    ms_step = r["ms"] / steps
    o = {"workload": workload_desc(workload)["workload"], "value": r["value"], "unit": "tok/s", "steps": steps,
         "ms_per_step": ms_step, "step_roofline": step_roofline(r["step_bytes"], ms_step, pk),
         "gpu_launches": r["launches"], "clocks": r["clocks"]}
    for k in ("e2e", "prefill_s", "reads_per_step"):
        if k in r:
            o[k] = r[k]
    if "tables" in r:
        t_gbs = r["tables"]["bytes"] / (r["tables"]["ms"] / 1e3) / 1e9
        o["tables_roofline"] = {"ncol": r["ncol"], "achieved": t_gbs, "peak": pk["hbm_gbs"], "frac": t_gbs / pk["hbm_gbs"],
                                "launch_ms": r["tables"]["ms"]}
    if cpu:
        o["cpu_baseline"] = cpu
    return o


def main():
    args = parse()
    ranks = Ranks()
    wl = workload_desc(args.workload)
    unit = {"prefill": "positions/s", "sweep": "GB/s"}.get(args.workload, "tok/s")
    base = {"metric": METRIC[args.workload], "unit": unit, "n_gpus": ranks.world, "steps": args.steps,
            "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4 x int8 -> int32 block dots, fp32 scale and accumulate", "data": "synthetic",
            "config": {"workload": wl["workload"], "parallelism": f"whole conversations per GPU x{ranks.world}, "
                       "no collective", "l2": "no flush: every step reads ~696 MB of weights (> 126 MB L2)"}}
    if args.impl == "reference":
        if ranks.rank != 0:
            ranks.close()
            return
        ref = run_reference(args.workload, args.steps if args.workload != "sweep" else 1, reference_threads())
        line = dict(base, impl="reference", value=ref["value"], ms_per_step=ref["ms_per_step"], n_gpus=ranks.world,
                    cpu_baseline=dict({k: ref[k] for k in ("value", "unit", "cores", "kind", "sample")},
                                      cpu_model=cpu_model()),
                    e2e={"value": ref["value"], "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0})
        print(json.dumps(line), flush=True)
        ranks.close()
        return
    pk = peaks()
    if args.workload == "sweep":
        sw = run_sweep(args, ranks, pk)
        top = [r for r in sw["rows"] if r["N"] == 97496 and r["B"] == 1][0]
        line = dict(base, value=top["gbs"], ms_per_step=top["ms"], gpu_launches=None, sweep=sw,
                    roofline={"kernel": "k_table (isolated read)", "bound": "hbm", "achieved": top["gbs"],
                              "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": top["hbm_frac"], "peak_source": pk["source"],
                              "traffic": None})
        if ranks.rank == 0 and ranks.world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_baseline("sweep", 1)
        if ranks.rank == 0:
            print(json.dumps(line), flush=True)
        ranks.close()
        return
    if args.workload == "prefill":
        r = run_prefill(args, ranks, args.steps)
    elif args.workload == "multi64":
        r = run_multi(args, ranks, args.steps)
    else:
        r = run_ours(args, ranks, args.workload, args.steps)
    t_gbs = r["tables"]["bytes"] / (r["tables"]["ms"] / 1e3) / 1e9
    step_ms = r["ms"] / args.steps
    line = dict(base, value=r["value"], ms_per_step=step_ms, gpu_launches=r["launches"], clocks=r["clocks"])
    line["roofline"] = {
        "kernel": "k_table (every layer table of a step, read back to back: imi_seoul::bench_tables)",
        "bound": "hbm", "achieved": t_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": t_gbs / pk["hbm_gbs"],
        "peak_source": pk["source"], "traffic": table_traffic(r["ncol"]), "ncol": r["ncol"],
        "algorithmic_bytes_per_launch": r["tables"]["bytes"], "launch_ms": r["tables"]["ms"]}
    line["step_roofline"] = step_roofline(r["step_bytes"], step_ms, pk)
    if "flops_per_step" in r:   # prefill is a contraction: its tensor-pipe roofline
        tf = r["flops_per_step"] / (step_ms / 1e3) / 1e12
        line["flops_roofline"] = {"flops_per_step": r["flops_per_step"], "achieved_tflops": tf,
                                  "peak_tflops": pk.get("bf16_tflops"), "unit": "TFLOP/s",
                                  "frac": tf / pk["bf16_tflops"] if pk.get("bf16_tflops") else None}
    if "prefill_s" in r:
        line["config"]["prefill_s"] = r["prefill_s"]
    if "e2e" in r:
        line["e2e"] = r["e2e"]
    cpu_here = ranks.rank == 0 and ranks.world == 1 and not args.no_cpu_baseline
    if cpu_here:
        line["cpu_baseline"] = cpu_baseline(args.workload, cpu_steps(args.workload))
    if args.workload == "ride2" and not args.no_extra:
        b1 = run_ours(args, ranks, "b1", args.steps)
        line["b1"] = sub_line(b1, args.steps, "b1", pk, cpu_baseline("b1", cpu_steps("b1")) if cpu_here else None)
        m = run_multi(args, ranks, args.extra_steps)
        line["multi64"] = sub_line(m, args.extra_steps, "multi64", pk,
                                   cpu_baseline("multi64", cpu_steps("multi64")) if cpu_here else None)
        line["multi64"]["box_tok_s"] = m["value"]
        if ranks.world == 1:
            line["sweep"] = run_sweep(args, ranks, pk)
            if cpu_here:
                line["sweep"]["cpu_baseline"] = cpu_baseline("sweep", 1)
    if ranks.rank == 0:
        print(json.dumps(line), flush=True)
    ranks.close()


if __name__ == "__main__":
    main()
