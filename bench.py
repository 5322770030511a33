"""Benchmark of the B200 Needle-3 token loop (one JSON line on rank 0).

Workload (the reference's batched-decoding configuration): the synthetic
depth-20 Needle-3 archive (seed 0), 256 independent sequences per GPU with
prompt lengths uniform in [128, 1024] (one stratified draw, the same lengths
on every rank in a per-rank seeded order, with per-rank seeded ids), greedy
decoding. A
step is one batched decode step of every sequence on the GPU: tied logits,
argmax, and the forward pass of the chosen tokens through all 20 layers with
the paged int8 KV cache. Sequences are sharded across ranks with no
collective on the data path (weak scaling).

  value  tokens/s of the whole job, from CUDA events on the library's stream
         around K device-resident steps (max over ranks)
  e2e    the same through nb_batch_step with host buffers: per step the
         host->device staging of the step's metadata and the device->host
         read of the chosen tokens are inside the timed region
  batch1 the batch-1 configuration: depth 20, a 512-token prompt (prefill ms)
         and masked greedy steps (a seeded ~5% allowed bitset each step),
         host-loop latency and device time per token, with its roofline
         against the L2 read peak measured here and the HBM peak
  roofline  the attention kernel (the HBM-bound dominant kernel) against the
         measured HBM copy bandwidth; step_roofline the whole step's KV bytes
  products  the product microbenchmark (config 3) against the int8 tensor peak
  cpu_baseline  the CPU restatement's float path (what the reference runs on
         an x86 host) on a bounded sample of the same workload, with the
         reference's default 6 threads and the integer mode beside it
  float_agreement  device tokens against the reference's x86 float kernels
         (teacher-forced on the device's tokens) on configs 0 and 1

`--impl reference` times that CPU path alone on the host cores.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

SEQS_PER_GPU = 256
PROMPT_RANGE = (128, 1024)
DEPTH = 20
METRIC = "decode tokens/s (depth-20 Needle-3, 256 sequences per GPU, greedy)"
UNIT = "tokens/s"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=32)
    p.add_argument("--warmup", type=int, default=4)
    p.add_argument("--impl", default="b200", choices=["b200", "reference"])
    p.add_argument("--seqs", type=int, default=SEQS_PER_GPU)
    p.add_argument("--shard", type=int, default=None,
                   help="one GPU decoding the sequences rank SHARD gets at N > 1 (its shard timed alone)")
    p.add_argument("--no-batch1", action="store_true")
    p.add_argument("--no-cpu", action="store_true")
    p.add_argument("--profile", action="store_true", help="64 sequences, no extras: the small case for ncu captures")
    p.add_argument("--batch1-only", action="store_true", help="only the batch-1 configuration (ncu launch lists)")
    p.add_argument("--no-whistle", action="store_true", help="skip the Whistle decoder section (config 4)")
    p.add_argument("--whistle-only", action="store_true", help="only the Whistle decoder section (config 4; ncu launch lists)")
    p.add_argument("--ncu-range", action="store_true",
                   help="bracket the timed steps with cudaProfilerStart/Stop (ncu --profile-from-start off)")
    p.add_argument("--products", action="store_true",
                   help="the product microbenchmark (config 3) instead of decoding: one JSON line of GOP/s per shape")
    return p.parse_args()


def prompts(rank: int, count: int):
    from rustyneedle_b200 import workloads

    return workloads.config2_prompts(rank, count)


def kv_bytes_per_step(lengths, steps: int, depth: int = DEPTH, per_position: int = 544) -> float:
    """KV-cache bytes the attention reads and writes per decode step, averaged
    over `steps` steps from the given context lengths: every layer reads every
    cached position (64 B key + 64 B value + two 4-byte scales per kv head) and
    writes the new one."""
    lengths = np.asarray(lengths, dtype=np.float64)
    mean_positions = lengths.sum() * 1.0 + len(lengths) * (steps + 1) / 2.0
    return depth * per_position * (mean_positions + len(lengths))


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f), "measured"
    except OSError:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "fallback"


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = tempfile.mktemp(suffix=".csv")

    def __enter__(self):
        query = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                 "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                 "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={query}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=self.out,
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            self.proc.wait()
            self.out.close()

    def summary(self):
        if not self.proc:
            return None
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].isdigit():
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [int(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": int(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


REFERENCE_THREADS = 6  # the reference's pool: min(cores - 2, 5) workers plus the caller (crates/kernels/src/pool.rs:48-52)


def _cpu_sessions(oracle, model, rank_prompts, count: int):
    sessions = []
    for ids in rank_prompts[:count]:
        s = oracle.Session(model)
        s.feed(ids)
        sessions.append(s)
    return sessions


def _sample_note(rank_prompts, count: int) -> str:
    lengths = [len(p) for p in rank_prompts[:count]]
    return f"{count} of the rank's sequences (prompts {min(lengths)}-{max(lengths)} tokens, prefill untimed)"


def cpu_sequence_parallel(oracle, archive: str, rank_prompts, mode: int, threads: int, sequences: int, steps: int):
    """Decode tokens/s of `sequences` sequences stepped side by side, one
    sequence per host thread (the sessions of a step spread over `threads`
    threads; every thread has at least one sequence)."""
    model = oracle.Model.open(archive, mode, threads)
    sessions = _cpu_sessions(oracle, model, rank_prompts, sequences)
    model.set_threads(1)  # one thread per sequence inside the step
    tokens = np.array([oracle.argmax(s.logits()) for s in sessions], dtype=np.uint32)
    tokens = np.array([oracle.argmax(r) for r in oracle.sessions_step(sessions, tokens, threads)], dtype=np.uint32)
    start = time.perf_counter()
    for _ in range(steps):
        tokens = np.array([oracle.argmax(r) for r in oracle.sessions_step(sessions, tokens, threads)], dtype=np.uint32)
    elapsed = time.perf_counter() - start
    return len(sessions) * steps / elapsed


def cpu_reference_threading(oracle, archive: str, rank_prompts, mode: int, threads: int, sequences: int, steps: int):
    """Decode tokens/s the way rustyneedle serves: one session at a time, each
    token's products forked over the pool's `threads` threads (64-row tasks,
    matrix.rs:8-11)."""
    model = oracle.Model.open(archive, mode, threads)
    sessions = _cpu_sessions(oracle, model, rank_prompts, sequences)
    for s in sessions:
        s.push(oracle.argmax(s.logits()))
    start = time.perf_counter()
    for _ in range(steps):
        for s in sessions:
            s.push(oracle.argmax(s.logits()))
    elapsed = time.perf_counter() - start
    return len(sessions) * steps / elapsed


def cpu_baseline(archive: str, rank_prompts):
    """The CPU restatement on this host's cores for a bounded sample of the
    config-2 workload. `value`: FLOAT mode (the reference's x86 float kernels,
    what rustyneedle executes on this host) with one sequence per thread on
    every core, sequences >= threads; beside it the reference's own threading
    (6 threads inside each token, sessions in turn) and INT mode (the
    reference's aarch64 integer kernels restated in scalar C++, the parity
    target)."""
    from oracle import oracle

    cores = os.cpu_count() or 1
    steps = 8
    value = cpu_sequence_parallel(oracle, archive, rank_prompts, oracle.MODE_FLOAT, cores, cores, steps)
    six = cpu_reference_threading(oracle, archive, rank_prompts, oracle.MODE_FLOAT, REFERENCE_THREADS, 4, steps)
    int_seqs = 2
    int_mode = cpu_reference_threading(oracle, archive, rank_prompts, oracle.MODE_INT, cores, int_seqs, 4)
    return {"value": value, "unit": UNIT, "cores": cores, "kind": "port",
            "sample": f"{_sample_note(rank_prompts, cores)}, {steps} timed decode steps each after one untimed, "
                      f"oracle FLOAT mode (the reference's x86 float kernels), one sequence per thread on {cores} threads",
            "reference_threads": {"value": six, "cores": REFERENCE_THREADS,
                                  "sample": f"{_sample_note(rank_prompts, 4)}, {steps} timed steps; FLOAT mode; sessions one "
                                            f"after another, each token's products on the reference's default "
                                            f"{REFERENCE_THREADS}-thread pool"},
            "int_mode": {"value": int_mode, "cores": cores,
                         "sample": f"{_sample_note(rank_prompts, int_seqs)}, 4 timed steps; INT mode (the reference's "
                                   f"aarch64 integer kernels as scalar C++), sessions in turn on {cores} threads"}}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from rustyneedle_b200 import synthetic

    archive = synthetic.cached_archive(seed=0)
    threads = os.cpu_count() or 1
    from oracle import oracle

    oracle.build()
    model = oracle.Model.open(archive, oracle.MODE_FLOAT, threads)
    sample = min(max(16, threads), args.seqs)  # at least one sequence per thread
    sessions = []
    for ids in prompts(0, args.seqs)[:sample]:
        s = oracle.Session(model)
        s.feed(ids)
        sessions.append(s)
    model.set_threads(1)  # one thread per sequence inside the step
    tokens = np.array([oracle.argmax(s.logits()) for s in sessions], dtype=np.uint32)
    for _ in range(args.warmup):
        tokens = np.argmax(oracle.sessions_step(sessions, tokens, threads), axis=1).astype(np.uint32)
    start = time.perf_counter()
    for _ in range(args.steps):
        tokens = np.argmax(oracle.sessions_step(sessions, tokens, threads), axis=1).astype(np.uint32)
    elapsed = time.perf_counter() - start
    value = sample * args.steps / elapsed
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * elapsed / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "config": {"workload": "config2: depth-20 synthetic Needle-3, greedy decode",
                                            "sequences_timed": sample, "prompt_tokens": list(PROMPT_RANGE)},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"{sample} sequences of the workload, one decode step of each per step, "
                                       f"prefill untimed; oracle FLOAT mode (the reference's x86 float kernels), one "
                                       f"sequence per thread on {threads} threads"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


PRODUCT_SHAPES = [(512, 2048, 2), (2048, 512, 2), (512, 8192, 4)]  # (K, N, code bits)
PRODUCT_TOKENS = [1, 8, 64, 256, 4096]


def product_sweep(steps: int = 8):
    """Config 3: int8 codebook products M x K -> N through nb_debug_product,
    the product kernel alone timed with CUDA events (activations quantised and
    resident, the matrix L2-resident as the model's weights are between
    tokens), against twice the measured bf16 tensor peak (the int8 dense
    rate)."""
    from rustyneedle_b200 import debug, synthetic

    peaks, peak_kind = measured_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    rows = []
    for cols, n, bits in PRODUCT_SHAPES:
        packed, levels, norms = synthetic.product_matrix(seed=cols + n, rows=n, columns=cols, bits=bits)
        for m in PRODUCT_TOKENS:
            x = np.random.default_rng(m).standard_normal((m, cols)).astype(np.float32)
            _, ms = debug.product(bits, packed, levels, norms, n, cols, x, reps=max(3, steps))
            tops = 2.0 * m * cols * n / (ms / 1000.0) / 1e12
            weight_gbs = n * cols / (ms / 1000.0) / 1e9  # int8 weight bytes per product
            rows.append({"M": m, "K": cols, "N": n, "bits": bits, "us": round(ms * 1000.0, 2), "TOP/s": round(tops, 2),
                         "frac_int8_tensor": round(tops / int8_peak, 4), "weight_GB/s": round(weight_gbs, 1)})
    return {"workload": "config3: codebook int8 products, M in {1, 8, 64, 256, 4096} x (K, N) in {(512, 2048), "
                        "(2048, 512), (512, 8192)}; 2-bit codes for the first two, 4-bit for the third",
            "peak": {"int8_tensor_TOPs": int8_peak, "source": f"2 x {peak_kind} bf16_tflops"}, "rows": rows}


def product_sweep_cpu():
    """Config 3 on the CPU restatement, one thread: the three shapes at M = 1
    in FLOAT mode (the reference's x86 float kernel, matrix.rs:427-440) and
    INT mode (its aarch64 integer kernels); a product of M tokens costs M times
    one token's on these per-row kernels."""
    from oracle import oracle
    from rustyneedle_b200 import synthetic

    out = []
    for cols, n, bits in PRODUCT_SHAPES:
        packed, levels, norms = synthetic.product_matrix(seed=cols + n, rows=n, columns=cols, bits=bits)
        x = np.random.default_rng(1).standard_normal(cols).astype(np.float32)
        row = {"K": cols, "N": n, "bits": bits}
        for mode, name in ((oracle.MODE_FLOAT, "float"), (oracle.MODE_INT, "int")):
            oracle.product_raw(mode, bits, packed, levels, norms, n, cols, x)
            reps = 8
            t = time.perf_counter()
            for _ in range(reps):
                oracle.product_raw(mode, bits, packed, levels, norms, n, cols, x)
            sec = (time.perf_counter() - t) / reps
            row[f"{name}_GOP/s"] = round(2.0 * cols * n / sec / 1e9, 3)
        out.append(row)
    return {"cores": 1, "kind": "port", "sample": "M = 1 per shape, 8 timed products after one untimed", "rows": out}


def products(args):
    """--products: the config-3 sweep alone as one JSON line."""
    sweep = product_sweep(args.steps)
    print(json.dumps({"metric": "codebook int8 product throughput (config 3)", "unit": "TOP/s", "impl": "b200",
                      "peak": sweep["peak"], "data": "synthetic", "products": sweep["rows"]}), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        return run_reference(args)
    if args.products:
        return products(args)
    import rustyneedle_b200 as nb
    from rustyneedle_b200 import debug, dp, synthetic

    ranks = dp.ranks_from_env()
    rank, world, local = ranks.rank, ranks.world, ranks.local
    dist = dp.init_group(ranks, "nccl")

    if args.whistle_only:  # before the config-2 model and its KV pool
        print(json.dumps({"config4": whistle(nb, local, args.ncu_range)}), flush=True)
        return
    archive = synthetic.cached_archive(seed=0)
    seqs = 64 if args.profile else args.seqs
    shard = rank if args.shard is None or world > 1 else args.shard
    rank_prompts = prompts(shard, seqs)
    # KV pool sized to the run: every sequence's prompt plus the decode steps, plus the batch-1 session
    pages = dp.kv_pages_for(rank_prompts, 2 * args.steps + 2 * args.warmup + 8, DEPTH)
    model = nb.Model.open(archive, device=local, max_sessions=seqs + 4, kv_pages=pages)
    if DEPTH != model.config.num_layers:
        model = model.with_depth(DEPTH)
    if args.batch1_only:
        print(json.dumps({"batch1": batch1(nb, model, local, args.ncu_range)}), flush=True)
        return
    t0 = time.perf_counter()
    sessions = [nb.Session(model) for _ in rank_prompts]
    nb.feed_many(sessions, rank_prompts)  # the prompts packed into shared prefill passes
    setup_s = time.perf_counter() - t0
    batch = nb.Batch(model, sessions)

    def barrier():
        dp.barrier(dist)

    def max_over_ranks(x: float) -> float:
        return dp.max_over_ranks(dist, x, f"cuda:{local}")

    batch.run(args.warmup)
    barrier()
    if args.ncu_range:
        import torch

        torch.cuda.cudart().cudaProfilerStart()
    with Clocks(local) as clocks:
        ms = batch.run(args.steps)
    if args.ncu_range:
        import torch

        torch.cuda.cudart().cudaProfilerStop()
    barrier()
    rank_ms = ms
    ms = max_over_ranks(ms)
    total_tokens = seqs * world * args.steps
    value = total_tokens / (ms / 1000.0)
    # each rank's step time and KV traffic: whether the slowest rank is the one with the most KV to read
    step_kv = kv_bytes_per_step([len(p) + args.warmup for p in rank_prompts], args.steps)
    per_rank = [{"rank": r, "ms_per_step": round(v[0], 4), "kv_bytes_per_step": round(v[1])}
                for r, v in enumerate(dp.gather_over_ranks(dist, [rank_ms / args.steps, step_kv], f"cuda:{local}"))]

    # end to end through the public C ABI with host buffers
    batch.step()
    barrier()
    start = time.perf_counter()
    for _ in range(args.steps):
        batch.step()
    e2e_s = max_over_ranks(time.perf_counter() - start)
    e2e = {"value": seqs * world * args.steps / e2e_s, "unit": UNIT, "h2d_bytes_per_step": seqs * (16 + 4 + 4),
           "d2h_bytes_per_step": seqs * 4}

    att_ms, att_bytes = debug.time_attention(batch, reps=3)
    peaks, peak_kind = measured_peaks()
    achieved = att_bytes / (att_ms / 1000.0) / 1e9
    traffic = None
    try:
        with open(os.path.join(ROOT, "profiles", "k_attend_traffic.json")) as f:
            t = json.load(f)
            # the captured launch's DRAM bytes per algorithmic byte, scaled to this launch
            traffic = round(t["dram_bytes"] / t["algorithmic_bytes"] * att_bytes)
    except (OSError, KeyError, ZeroDivisionError):
        traffic = None
    roofline = {"kernel": "k_attend (paged int8 attention; one layer of the batch: the step's launches, one per group of 128 sequences)",
                "bound": "hbm",
                "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                "peak_source": f"{peak_kind} hbm_gbs", "launch_ms": att_ms, "algorithmic_bytes": att_bytes}

    step_roofline = {"bound": "hbm", "unit": "GB/s", "kv_bytes_per_step": round(step_kv),
                     "achieved": round(step_kv / (rank_ms / args.steps / 1000.0) / 1e9, 1), "peak": peaks["hbm_gbs"],
                     "frac": round(step_kv / (rank_ms / args.steps / 1000.0) / 1e9 / peaks["hbm_gbs"], 4),
                     "peak_source": f"{peak_kind} hbm_gbs",
                     "note": "the whole decode step of this rank: KV bytes read and written by all layers' attention "
                             "(algorithmic, 544 B per cached position per layer) over the device time per step; weights "
                             "(12.1 MB, L2-resident) not counted"}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8+f32", "data": "synthetic",
            "config": {"workload": "config2: depth-20 synthetic Needle-3 (seed 0), 256 sequences per GPU, prompts "
                                   "uniform in [128, 1024] (stratified: the same lengths on every rank), greedy decode, "
                                   "paged int8 KV (64-token pages)",
                       "sequences_per_gpu": seqs, "depth": DEPTH, "parallelism": f"dp{world} (sequences sharded)",
                       "l2": "inputs larger than L2 (KV cache ~2 GB per GPU)", "setup_s": round(setup_s, 1),
                       **({"shard": shard} if shard != rank else {})},
            "e2e": e2e, "roofline": roofline, "step_roofline": step_roofline,
            "gpu_launches": debug.step_kernels(batch) * args.steps, "clocks": clocks.summary(), "per_rank": per_rank}

    if not args.no_batch1 and rank == 0 and not args.profile:
        batch.close()
        line["batch1"] = batch1(nb, model, local)
        if world == 1:  # single-GPU configurations: a scaling run only repeats them
            line["config0"] = config0(nb, model)
            line["products"] = product_sweep()
            line["grammar"] = grammar_masks(nb, model)
            if not args.no_whistle:
                line["config4"] = whistle(nb, local)
    if rank == 0 and world == 1 and not args.no_cpu and not args.profile:
        from oracle import oracle

        oracle.build()
        line["cpu_baseline"] = cpu_baseline(archive, rank_prompts)
        if "batch1" in line:
            line["batch1"]["cpu"] = config1_cpu(archive)
            line["float_agreement"] = float_agreement(nb, model, archive)
        if "products" in line:
            line["products"]["cpu"] = product_sweep_cpu()
        if "config0" in line:
            line["config0"]["cpu"] = config0_cpu(archive)
        if "config4" in line:
            line["config4"]["cpu"] = whistle_cpu()
        if "grammar" in line:
            line["grammar"]["cpu"] = grammar_masks_cpu()
    if rank == 0:
        print(json.dumps(line), flush=True)
    batch.close()
    dp.close_group(dist)


def config0(nb, model):
    """Config 0: depth 2, batch 1, 32 prompt ids, 64 unconstrained greedy tokens."""
    from rustyneedle_b200 import workloads

    shallow = model.with_depth(workloads.CONFIG0["depth"])
    s = nb.Session(shallow)
    s.feed(workloads.config0_prompt())
    b = nb.Batch(shallow, [s])
    times = []
    for _ in range(64):
        t = time.perf_counter()
        b.step()
        times.append(1000 * (time.perf_counter() - t))
    b.close()
    s.close()
    shallow.close()
    times = times[4:]
    p50 = float(np.percentile(times, 50))
    return {"p50_ms_per_token": round(p50, 4), "tokens_per_s": round(1000.0 / p50, 1), "steps": len(times),
            "note": "depth 2, 32-token prompt, greedy through nb_batch_step (token out), unconstrained"}


def config0_cpu(archive: str):
    """Config 0 on the CPU oracle (FLOAT mode, one thread): the same prompt and 64 greedy tokens."""
    from oracle import oracle

    from rustyneedle_b200 import workloads

    model = oracle.Model.open(archive, oracle.MODE_FLOAT, 1).with_depth(workloads.CONFIG0["depth"])
    s = oracle.Session(model)
    s.feed(workloads.config0_prompt())
    times = []
    for _ in range(64):
        t = time.perf_counter()
        s.push(oracle.argmax(s.logits()))
        times.append(1000 * (time.perf_counter() - t))
    p50 = float(np.percentile(times[4:], 50))
    return {"p50_ms_per_token": round(p50, 4), "tokens_per_s": round(1000.0 / p50, 1), "cores": 1,
            "kind": "port", "sample": "60 timed greedy tokens after 4 untimed"}


GRAMMAR = dict(sequences=256, seed=5, tools="home_assistant.json")


def grammar_workload(vocab: int):
    """Whole tool calls over the reference's home-assistant tools (object
    arguments, enums, bounded integers, a choice; tests/golden/tool_schemas.json)
    and a vocabulary of the 256 byte pieces plus pieces cut from the tools'
    JSON. Each of the 256 sequences stands part-way into a call: a seeded walk
    of 0-80 accepted bytes through the call machine. Returns (tools, pieces,
    the sequences' byte prefixes)."""
    from rustyneedle_b200.grammar import call_automaton

    with open(os.path.join(ROOT, "tests", "golden", "tool_schemas.json")) as f:
        tools = json.load(f)[GRAMMAR["tools"]]
    rng = np.random.default_rng(GRAMMAR["seed"])
    text = json.dumps(tools).encode() + b'[{"name":"' + b',"arguments":{' + b'0123456789}],'
    pieces = [None, None, None] + [bytes([b]) for b in range(256)]
    while len(pieces) < vocab:
        a = int(rng.integers(0, len(text)))
        pieces.append(text[a:a + int(rng.integers(1, 8))])
    trans, complete, start = call_automaton(tools)
    structural = list(b'"}]:,{[0123456789')
    prefixes = []
    for _ in range(GRAMMAR["sequences"]):
        s, prefix = start, b""
        for _ in range(int(rng.integers(0, 81))):
            ok = [b for b in range(256) if trans[s, b] and not trans[s, b] & 0x80000000]
            if not ok or complete[s]:
                break
            pick = int(rng.choice(structural))
            b = pick if pick in ok and rng.random() < 0.5 else int(rng.choice(ok))
            s, prefix = int(trans[s, b]), prefix + bytes([b])
        prefixes.append(prefix)
    return tools, pieces, prefixes


def grammar_masks(nb, model):
    """Device grammar masks for 256 sequences inside whole tool calls: µs per batch mask and per advance."""
    import torch

    V = model.config.output_vocab
    B = GRAMMAR["sequences"]
    tools, pieces, prefixes = grammar_workload(V)
    t = time.perf_counter()
    trans, complete, start = nb.call_automaton(tools)
    compile_ms = 1000 * (time.perf_counter() - t)
    aut = nb.TokenAutomaton(model, trans, complete, start, pieces, 1, 2)
    states = np.zeros(B, dtype=np.uint32)
    for b, prefix in enumerate(prefixes):
        s = start
        for byte in prefix:
            s = int(trans[s, byte])
        states[b] = s
    d_states = torch.from_numpy(states.view(np.int32).copy()).cuda()
    d_mask = torch.zeros(B * V // 32, dtype=torch.int32, device="cuda")
    d_next = torch.full((B,), 0xFFFF, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    reps = 200
    for _ in range(10):
        aut.mask(d_states, d_mask, sync=False)
    model.synchronize()
    t = time.perf_counter()
    for _ in range(reps):
        aut.mask(d_states, d_mask, sync=False)
    model.synchronize()
    mask_us = 1e6 * (time.perf_counter() - t) / reps
    t = time.perf_counter()
    for _ in range(reps):
        aut.advance(d_next, d_states, sync=False)  # id 0xFFFF is beyond the vocabulary: the walk is skipped, the states stay
    model.synchronize()
    advance_us = 1e6 * (time.perf_counter() - t) / reps
    aut.check()
    aut.close()
    return {"workload": f"{B} sequences part-way into whole tool calls over the reference's {len(tools)} home-assistant "
                        f"tools ({trans.shape[0]} automaton states, compiled in {compile_ms:.1f} ms), vocabulary {V} "
                        f"pieces (256 bytes and cuts of the tools JSON)",
            "mask_us": round(mask_us, 2), "advance_us": round(advance_us, 2),
            "masks_per_s": round(B * 1e6 / mask_us, 1),
            "note": "host wall time per call (launch included) over 200 back-to-back calls, then a synchronise"}


def grammar_masks_cpu():
    """TokenBytes::allowed over the restated CallMachine (oracle/grammar.py,
    pure Python) for 4 sequences of the same workload."""
    from oracle import grammar as og

    tools, pieces, prefixes = grammar_workload(8192)
    grammar = og.CallGrammar(tools)
    machines = []
    for prefix in prefixes[:4]:
        m = grammar.start()
        for byte in prefix:
            m.step(byte)
        machines.append(m)
    t = time.perf_counter()
    for m in machines:
        og.allowed(pieces, m)
    per = (time.perf_counter() - t) / len(machines)
    return {"masks_per_s": round(1.0 / per, 1), "cores": 1, "kind": "port",
            "sample": "4 masks, pure-Python restatement of TokenBytes::allowed over CallMachine (the reference's is Rust)"}


from rustyneedle_b200.workloads import WHISTLE, whistle_archive  # noqa: E402


def whistle(nb, device: int = 0, ncu_range: bool = False):
    """Config 4: a Whistle decoder (depth 8), 64 utterances each cross-attending
    to its own 1500 x 512 N(0, 1) encoder output, bos and a language token,
    then 224 greedy text tokens (ids below text_vocab) on the device (with
    ncu_range, two more steps bracketed by cudaProfilerStart/Stop)."""
    import torch

    model = nb.Model.open(whistle_archive(), device=device, max_sessions=WHISTLE["batch"])
    B, V, T = WHISTLE["batch"], model.config.output_vocab, WHISTLE["tokens"]
    rng = np.random.default_rng(11)
    sessions, memories, mem_ms = [], [], []
    for i in range(B):
        enc = rng.standard_normal((WHISTLE["frames"], model.config.d_model)).astype(np.float32)
        t = time.perf_counter()
        mem = nb.CrossMemory(model, enc)
        mem_ms.append(1000 * (time.perf_counter() - t))
        s = nb.Session(model)
        s.set_cross(mem)
        s.push(1)
        s.push(WHISTLE["text_vocab"] + i % (V - WHISTLE["text_vocab"]))
        sessions.append(s)
        memories.append(mem)
    allowed = np.zeros(V, dtype=bool)
    allowed[:WHISTLE["text_vocab"]] = True
    words = np.packbits(allowed, bitorder="little").view(np.uint32)
    masks = torch.from_numpy(np.tile(words, (T + 6) * B).astype(np.int32)).to(f"cuda:{device}")
    batch = nb.Batch(model, sessions)
    warm = 4
    batch.run(warm, masks.data_ptr())
    with Clocks(device) as clocks:
        ms = batch.run(T, masks.data_ptr() + warm * B * (V // 32) * 4)
    if ncu_range:
        torch.cuda.synchronize(device)
        torch.cuda.cudart().cudaProfilerStart()
        batch.run(2, masks.data_ptr() + (warm + T) * B * (V // 32) * 4)
        torch.cuda.cudart().cudaProfilerStop()
    out = {"workload": "config4: synthetic Whistle decoder (depth 8, d 512, 8 heads, seed 0), 64 utterances per GPU, each "
                       "cross-attending to its own 1500 x 512 N(0,1) encoder output; bos and a language token, then 224 greedy "
                       "text tokens (ids < 8000 of 8192) per utterance, device-resident steps",
           "tokens_per_s": round(B * T / (ms / 1000.0), 1), "ms_per_step": round(ms / T, 4),
           "memory_ms_per_utterance": round(float(np.median(mem_ms)), 3), "clocks": clocks.summary()}
    batch.close()
    for s in sessions:
        s.close()
    for m in memories:
        m.close()
    model.close()
    return out


def whistle_cpu(sample_tokens: int = 4):
    """Config 4 on the CPU oracle (FLOAT mode, all host cores): one utterance's
    memory, bos and a language token, then a few greedy text tokens."""
    from oracle import oracle

    model = oracle.Model.open(whistle_archive(), oracle.MODE_FLOAT, os.cpu_count() or 1)
    enc = np.random.default_rng(11).standard_normal((WHISTLE["frames"], 512)).astype(np.float32)
    t = time.perf_counter()
    mem = oracle.CrossMemory(model, enc)
    mem_ms = 1000 * (time.perf_counter() - t)
    s = oracle.Session(model)
    s.push_cross(1, mem)
    s.push_cross(WHISTLE["text_vocab"], mem)
    allowed = np.zeros(8192, dtype=np.uint8)
    allowed[:WHISTLE["text_vocab"]] = 1
    t = time.perf_counter()
    for _ in range(sample_tokens):
        s.push_cross(oracle.argmax_allowed(s.logits(), allowed), mem)
    ms = 1000 * (time.perf_counter() - t) / sample_tokens
    return {"tokens_per_s": round(1000.0 / ms, 2), "ms_per_token": round(ms, 2), "memory_ms": round(mem_ms, 1),
            "cores": os.cpu_count() or 1, "kind": "port", "sample": f"one utterance, {sample_tokens} greedy tokens after bos and a language token"}


def batch1(nb, model, device: int = 0, ncu_range: bool = False):
    """Config 1: depth 20, batch 1, 512-token prompt, 256 masked greedy steps
    (with ncu_range, one prefill and steps 64 and 65 are bracketed by
    cudaProfilerStart/Stop).

    The prompt is fed once; two copy-on-write clones of the fed session then
    run the 256 steps: one through nb_batch_step with a host bitset each step
    (the per-token latency a caller sees), one device-resident (nb_batch_run
    with the bitsets on the device: the device time per token, which the
    roofline divides). Both must choose the same tokens."""
    import torch

    from rustyneedle_b200 import debug, workloads

    V = model.config.output_vocab
    ids, words, _ = workloads.config1(V)
    # prefill: one untimed feed (first launches of the large-pass kernels),
    # then the median of five timed feeds, each into a fresh session that is
    # closed before the next (feed returns once the device is done); with
    # ncu_range the third timed feed is bracketed too
    feeds = []
    for k in range(6):
        warm = nb.Session(model)
        if ncu_range and k == 3:
            torch.cuda.cudart().cudaProfilerStart()
        start = time.perf_counter()
        warm.feed(ids)
        if k:
            feeds.append(1000 * (time.perf_counter() - start))
        if ncu_range and k == 3:
            torch.cuda.cudart().cudaProfilerStop()
        warm.close()
    prefill_ms = float(np.median(feeds))
    base = nb.Session(model)
    base.feed(ids)
    s = base.clone()
    b = nb.Batch(model, [s])
    times, host_tokens = [], []
    with Clocks(device) as clocks:
        for k, m in enumerate(words):
            if ncu_range and k in (64, 66):
                (torch.cuda.cudart().cudaProfilerStart if k == 64 else torch.cuda.cudart().cudaProfilerStop)()
            t = time.perf_counter()
            host_tokens.append(int(b.step(m)[0]))
            times.append(1000 * (time.perf_counter() - t))
    b.close()
    s.close()
    times = times[4:]
    p50 = float(np.percentile(times, 50))
    out = {"prefill_ms_512": round(prefill_ms, 2), "p50_ms_per_token": round(p50, 4),
           "p90_ms_per_token": round(float(np.percentile(times, 90)), 4),
           "tokens_per_s": round(1000.0 / p50, 1), "steps": len(times), "clocks": clocks.summary(),
           "note": "per-token latency through nb_batch_step (host mask in, token out), depth 20"}
    if ncu_range:
        base.close()
        return out

    d = base.clone()
    bd = nb.Batch(model, [d])
    masks = torch.from_numpy(np.concatenate(words).view(np.int32)).to(f"cuda:{device}")
    chosen = torch.zeros(len(words), dtype=torch.int32, device=f"cuda:{device}")
    torch.cuda.synchronize(device)
    dev_ms = bd.run(len(words), masks.data_ptr(), chosen.data_ptr()) / len(words)
    device_tokens = chosen.cpu().numpy().view(np.uint32).tolist()
    bd.close()
    d.close()
    base.close()

    # the roofline: algorithmic bytes of one token (weights touched + KV read and written) over the device time
    weights = workloads.token_weight_bytes(DEPTH)
    steps = len(words)
    kv = DEPTH * 544 * (len(ids) + (steps + 1) / 2.0 + 1)
    per_token = weights + kv
    achieved = per_token / (dev_ms / 1000.0) / 1e9
    peaks, peak_kind = measured_peaks()
    l2_gbs = max(debug.read_bandwidth(size << 20, passes=32, reps=10, device=device) for size in (8, 16, 32))
    prefill_ops = 2.0 * workloads.prefill_product_macs(len(ids), DEPTH)
    out.update({
        "device_ms_per_token": round(dev_ms, 4),
        "device_tokens_equal_host_loop": device_tokens == host_tokens,
        "roofline": {"bound": "l2 (weights L2-resident across tokens) / hbm (cold)", "unit": "GB/s",
                     "algorithmic_bytes_per_token": round(per_token), "weight_bytes": weights, "kv_bytes": round(kv),
                     "achieved": round(achieved, 1),
                     "l2_peak": round(l2_gbs, 1), "frac_l2": round(achieved / l2_gbs, 4),
                     "l2_peak_source": "measured here: the best of plain 16-byte streaming reads of 8, 16 and 32 MiB "
                                       "buffers, 32 reads of the buffer per launch (nb_debug_read_bandwidth), CUDA "
                                       "events over 10 launches",
                     "hbm_peak": peaks["hbm_gbs"], "frac_hbm": round(achieved / peaks["hbm_gbs"], 4),
                     "hbm_peak_source": f"{peak_kind} hbm_gbs"},
        "prefill_roofline": {"bound": "tensor", "unit": "TOP/s", "product_ops": prefill_ops,
                             "achieved": round(prefill_ops / (prefill_ms / 1000.0) / 1e12, 3),
                             "peak": 2.0 * peaks["bf16_tflops"],
                             "frac": round(prefill_ops / (prefill_ms / 1000.0) / 1e12 / (2.0 * peaks["bf16_tflops"]), 5),
                             "note": "int8 product ops of the 512-token prefill (every layer's projections and lane maps "
                                     "per token, logits of the last token) over the host-timed prefill (median of "
                                     "five feeds after an untimed one); peak 2 x "
                                     f"{peak_kind} bf16_tflops"}})
    return out


def float_agreement(nb, model, archive: str):
    """Device tokens against the reference's x86 float kernels (oracle FLOAT
    mode, which rustyneedle executes on this host) on configs 0 and 1,
    teacher-forced: the float session is pushed the device's choice each step,
    so every step compares the two choices from the same history. Reports the
    fraction of steps whose choices agree and the cosine of the two logit
    vectors (the reference's own float/int comparison, docs/parity.md)."""
    from oracle import oracle
    from rustyneedle_b200 import workloads

    V = model.config.output_vocab
    fmodel = oracle.Model.open(archive, oracle.MODE_FLOAT, os.cpu_count() or 1)
    ids1, words1, allowed1 = workloads.config1(V)
    cases = [("config0", workloads.CONFIG0["depth"], workloads.config0_prompt(), None, None, workloads.CONFIG0["tokens"]),
             ("config1", workloads.CONFIG1["depth"], ids1, words1, allowed1, workloads.CONFIG1["steps"])]
    out = {}
    for name, depth, ids, words, allowed, steps in cases:
        dm = model.with_depth(depth)
        fm = fmodel.with_depth(depth)
        s = nb.Session(dm)
        s.feed(ids)
        o = oracle.Session(fm)
        o.feed(ids)
        agree, cosines = 0, []
        for k in range(steps):
            dl, fl = s.logits().astype(np.float64), o.logits()
            cosines.append(float(dl @ fl / (np.linalg.norm(dl) * np.linalg.norm(fl))))
            if words is None:
                token, want = s.step(), oracle.argmax(fl)
            else:
                token, want = s.step(words[k]), oracle.argmax_allowed(fl, allowed[k].astype(np.uint8))
            agree += int(token == want)
            o.push(token)
        s.close()
        dm.close()
        out[name] = {"steps": steps, "token_agreement": round(agree / steps, 4),
                     "logit_cosine_mean": round(float(np.mean(cosines)), 6),
                     "logit_cosine_min": round(float(np.min(cosines)), 6)}
    out["note"] = ("device (the reference's integer kernels, bit-exact) vs oracle FLOAT mode (its x86 float kernels), "
                   "teacher-forced on the device's tokens; float and integer products differ by ~0.7 % rRMS, so near "
                   "ties may choose differently")
    return out


def config1_cpu(archive: str):
    """Config 1 on the CPU restatement: the 512-token prefill and the per-token
    latency of the first 32 masked steps, FLOAT mode on the reference's default
    6 threads and on every core, and INT mode on every core (8 steps)."""
    from oracle import oracle
    from rustyneedle_b200 import workloads

    cores = os.cpu_count() or 1
    ids, _, allowed = workloads.config1(8192)
    out = {}
    for name, mode, threads, steps in (("float_6_threads", oracle.MODE_FLOAT, REFERENCE_THREADS, 32),
                                       ("float_all_cores", oracle.MODE_FLOAT, cores, 32),
                                       ("int_all_cores", oracle.MODE_INT, cores, 8)):
        model = oracle.Model.open(archive, mode, threads)
        s = oracle.Session(model)
        t = time.perf_counter()
        s.feed(ids)
        prefill = 1000 * (time.perf_counter() - t)
        times = []
        for k in range(steps):
            t = time.perf_counter()
            s.push(oracle.argmax_allowed(s.logits(), allowed[k].astype(np.uint8)))
            times.append(1000 * (time.perf_counter() - t))
        out[name] = {"prefill_ms_512": round(prefill, 1), "p50_ms_per_token": round(float(np.percentile(times, 50)), 3),
                     "tokens_per_s": round(1000.0 / float(np.percentile(times, 50)), 1), "cores": threads,
                     "steps": steps}
    out["kind"] = "port"
    return out


if __name__ == "__main__":
    main()
