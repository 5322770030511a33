"""Benchmark of the B200 Needle-3 token loop (one JSON line on rank 0).

Workload (the reference's batched-decoding configuration): the synthetic
depth-20 Needle-3 archive (seed 0), 256 independent sequences per GPU with
prompt lengths uniform in [128, 1024] (seeded per rank), greedy decoding. A
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
         and masked greedy steps (a seeded ~5% allowed bitset each step)
  roofline  the attention kernel (the HBM-bound dominant kernel) against the
         measured HBM copy bandwidth
  cpu_baseline  the CPU restatement's float path (what the reference runs on
         an x86 host) on a bounded sample of the same workload

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
    from rustyneedle_b200 import dp

    return dp.shard_prompts(rank, count, PROMPT_RANGE[0], PROMPT_RANGE[1])


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


def cpu_baseline(archive: str, rank_prompts, threads: int, steps: int = 2, sample: int = 8):
    from oracle import oracle

    model = oracle.Model.open(archive, oracle.MODE_FLOAT, threads)
    sessions = []
    for ids in rank_prompts[:sample]:
        s = oracle.Session(model)
        s.feed(ids)
        sessions.append(s)
    tokens = np.array([oracle.argmax(s.logits()) for s in sessions], dtype=np.uint32)
    oracle.sessions_step(sessions, tokens, threads)  # warm-up step
    start = time.perf_counter()
    for _ in range(steps):
        logits = oracle.sessions_step(sessions, tokens, threads)
        tokens = np.argmax(logits, axis=1).astype(np.uint32)
    elapsed = time.perf_counter() - start
    return {"value": len(sessions) * steps / elapsed, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{len(sessions)} of the rank's sequences (prompts {min(len(p) for p in rank_prompts[:sample])}-"
                      f"{max(len(p) for p in rank_prompts[:sample])} tokens, prefill untimed), {steps} decode steps each, "
                      f"oracle FLOAT mode (the reference's x86 float kernels) with one sequence per thread"}


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
    sample = min(16, args.seqs)
    sessions = []
    for ids in prompts(0, args.seqs)[:sample]:
        s = oracle.Session(model)
        s.feed(ids)
        sessions.append(s)
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
                                       "prefill untimed; oracle FLOAT mode (the reference's x86 float kernels)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


PRODUCT_SHAPES = [(512, 2048, 2), (2048, 512, 2), (512, 8192, 4)]  # (K, N, code bits)
PRODUCT_TOKENS = [1, 8, 64, 256, 4096]


def products(args):
    """Config 3: int8 codebook products M x K -> N through nb_debug_product,
    the product kernel alone timed with CUDA events (activations quantised and
    resident), against twice the measured bf16 tensor peak (int8 dense rate)."""
    from rustyneedle_b200 import debug, synthetic

    peaks, peak_kind = measured_peaks()
    int8_peak = 2.0 * peaks["bf16_tflops"]
    rows = []
    for cols, n, bits in PRODUCT_SHAPES:
        packed, levels, norms = synthetic.product_matrix(seed=cols + n, rows=n, columns=cols, bits=bits)
        for m in PRODUCT_TOKENS:
            x = np.random.default_rng(m).standard_normal((m, cols)).astype(np.float32)
            _, ms = debug.product(bits, packed, levels, norms, n, cols, x, reps=max(3, args.steps))
            tops = 2.0 * m * cols * n / (ms / 1000.0) / 1e12
            weight_gbs = n * cols / (ms / 1000.0) / 1e9  # int8 weight bytes per product
            rows.append({"M": m, "K": cols, "N": n, "bits": bits, "us": round(ms * 1000.0, 2), "TOP/s": round(tops, 2),
                         "frac_int8_tensor": round(tops / int8_peak, 4), "weight_GB/s": round(weight_gbs, 1)})
    print(json.dumps({"metric": "codebook int8 product throughput (config 3)", "unit": "TOP/s", "impl": "b200",
                      "peak": {"int8_tensor_TOPs": int8_peak, "source": f"2 x {peak_kind} bf16_tflops"},
                      "data": "synthetic", "products": rows}), flush=True)


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
    rank_prompts = prompts(rank, seqs)
    # KV pool sized to the run: every sequence's prompt plus the decode steps, plus the batch-1 session
    pages = dp.kv_pages_for(rank_prompts, 2 * args.steps + 2 * args.warmup + 8, DEPTH)
    model = nb.Model.open(archive, device=local, max_sessions=seqs + 2, kv_pages=pages)
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
    ms = max_over_ranks(ms)
    total_tokens = seqs * world * args.steps
    value = total_tokens / (ms / 1000.0)

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

    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8+f32", "data": "synthetic",
            "config": {"workload": "config2: depth-20 synthetic Needle-3 (seed 0), 256 sequences per GPU, prompts "
                                   "uniform in [128, 1024], greedy decode, paged int8 KV (64-token pages)",
                       "sequences_per_gpu": seqs, "depth": DEPTH, "parallelism": f"dp{world} (sequences sharded)",
                       "l2": "inputs larger than L2 (KV cache ~2 GB per GPU)", "setup_s": round(setup_s, 1)},
            "e2e": e2e, "roofline": roofline, "gpu_launches": debug.step_kernels(batch) * args.steps,
            "clocks": clocks.summary()}

    if not args.no_batch1 and rank == 0 and not args.profile:
        batch.close()
        line["batch1"] = batch1(nb, model, local)
        if world == 1:  # single-GPU configurations: a scaling run only repeats them
            line["config0"] = config0(nb, model)
            line["grammar"] = grammar_masks(nb, model)
            if not args.no_whistle:
                line["config4"] = whistle(nb, local)
    if rank == 0 and world == 1 and not args.no_cpu and not args.profile:
        from oracle import oracle

        oracle.build()
        line["cpu_baseline"] = cpu_baseline(archive, rank_prompts, os.cpu_count() or 1)
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
    rng = np.random.default_rng(3)
    shallow = model.with_depth(2)
    s = nb.Session(shallow)
    s.feed(rng.integers(10, 8000, 32).astype(np.uint32))
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

    rng = np.random.default_rng(3)
    model = oracle.Model.open(archive, oracle.MODE_FLOAT, 1).with_depth(2)
    s = oracle.Session(model)
    s.feed(rng.integers(10, 8000, 32).astype(np.uint32))
    times = []
    for _ in range(64):
        t = time.perf_counter()
        s.push(oracle.argmax(s.logits()))
        times.append(1000 * (time.perf_counter() - t))
    p50 = float(np.percentile(times[4:], 50))
    return {"p50_ms_per_token": round(p50, 4), "tokens_per_s": round(1000.0 / p50, 1), "cores": 1,
            "kind": "port", "sample": "60 timed greedy tokens after 4 untimed"}


GRAMMAR = dict(sequences=256, tools=64, seed=5)


def grammar_workload(vocab: int):
    """A tool-name choice over 64 names and a vocabulary of short pieces (the shapes of a call's name literal)."""
    rng = np.random.default_rng(GRAMMAR["seed"])
    letters = np.frombuffer(b"abcdefghijklmnopqrstuvwxyz_", dtype=np.uint8)
    names = [bytes(rng.choice(letters, size=int(rng.integers(6, 20))).tolist()) for _ in range(GRAMMAR["tools"])]
    joined = b"|".join(names)
    pieces = [None, None, None]
    while len(pieces) < vocab:
        a = int(rng.integers(0, len(joined)))
        pieces.append(joined[a:a + int(rng.integers(1, 7))] if rng.random() < 0.8
                      else bytes(rng.integers(32, 127, size=int(rng.integers(1, 8))).tolist()))
    return names, pieces


def grammar_masks(nb, model):
    """Device grammar masks for 256 sequences inside a tool-name literal: µs per batch mask and per advance."""
    import torch

    V = model.config.output_vocab
    B = GRAMMAR["sequences"]
    names, pieces = grammar_workload(V)
    trans, complete, start = nb.literal_automaton(names)
    aut = nb.TokenAutomaton(model, trans, complete, start, pieces, 1, 2)
    rng = np.random.default_rng(6)
    # every sequence inside the literal, part-way along one of the names
    states = np.full(B, start, dtype=np.uint32)
    for b in range(B):
        for byte in names[int(rng.integers(0, len(names)))][: int(rng.integers(0, 4))]:
            states[b] = trans[states[b], byte]
    d_states = torch.from_numpy(states.view(np.int32).copy()).cuda()
    d_mask = torch.zeros(B * V // 32, dtype=torch.int32, device="cuda")
    d_next = torch.full((B,), 0xFFFF, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    reps = 200
    for _ in range(10):
        aut.mask(d_states, d_mask)
    model.synchronize()
    t = time.perf_counter()
    for _ in range(reps):
        aut.mask(d_states, d_mask)
    model.synchronize()
    mask_us = 1e6 * (time.perf_counter() - t) / reps
    t = time.perf_counter()
    for _ in range(reps):
        aut.advance(d_next, d_states)  # id 0xFFFF is beyond the vocabulary: the walk is skipped, the states stay
    model.synchronize()
    advance_us = 1e6 * (time.perf_counter() - t) / reps
    aut.check()
    aut.close()
    return {"workload": f"{B} sequences inside a {len(names)}-name tool literal ({trans.shape[0]} automaton states), "
            f"vocabulary {V} pieces of 1-7 bytes", "mask_us": round(mask_us, 2), "advance_us": round(advance_us, 2),
            "masks_per_s": round(B * 1e6 / mask_us, 1),
            "note": "host wall time per call (launch included) over 200 back-to-back calls, then a synchronise"}


def grammar_masks_cpu():
    """TokenBytes::allowed restated in Python (oracle/grammar.py) for 4 sequences of the same workload."""
    from oracle import grammar as og

    names, pieces = grammar_workload(8192)
    rng = np.random.default_rng(6)
    t = time.perf_counter()
    for _ in range(4):
        m = og.LiteralMachine(names)
        for byte in names[int(rng.integers(0, len(names)))][: int(rng.integers(0, 4))]:
            m.step(byte)
        og.allowed(pieces, m)
    per = (time.perf_counter() - t) / 4
    return {"masks_per_s": round(1.0 / per, 1), "cores": 1, "kind": "port",
            "sample": "4 masks, pure-Python restatement of TokenBytes::allowed (the reference's is Rust)"}


WHISTLE = dict(layers=8, text_vocab=8000, frames=1500, batch=64, tokens=224)


def whistle_archive():
    from rustyneedle_b200 import synthetic

    return synthetic.cached_archive(seed=0, geometry=synthetic.Geometry(num_layers=WHISTLE["layers"], text_vocab=WHISTLE["text_vocab"]))


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
    (with ncu_range, steps 64 and 65 are bracketed by cudaProfilerStart/Stop)."""
    rng = np.random.default_rng(7)
    ids = rng.integers(10, 8000, 512).astype(np.uint32)
    s = nb.Session(model)
    start = time.perf_counter()
    s.feed(ids)
    prefill_ms = 1000 * (time.perf_counter() - start)
    b = nb.Batch(model, [s])
    words = model.config.output_vocab // 32
    masks = []
    for _ in range(256):
        allowed = rng.random(model.config.output_vocab) < 0.05
        allowed[rng.integers(0, model.config.output_vocab)] = True
        masks.append(np.packbits(allowed.astype(np.uint8), bitorder="little").view(np.uint32)[:words].copy())
    times = []
    with Clocks(device) as clocks:
        for k, m in enumerate(masks):
            if ncu_range and k in (64, 66):
                import torch

                (torch.cuda.cudart().cudaProfilerStart if k == 64 else torch.cuda.cudart().cudaProfilerStop)()
            t = time.perf_counter()
            b.step(m)
            times.append(1000 * (time.perf_counter() - t))
    b.close()
    times = times[4:]
    return {"prefill_ms_512": round(prefill_ms, 2), "p50_ms_per_token": round(float(np.percentile(times, 50)), 4),
            "p90_ms_per_token": round(float(np.percentile(times, 90)), 4),
            "tokens_per_s": round(1000.0 / float(np.percentile(times, 50)), 1), "steps": len(times),
            "clocks": clocks.summary(),
            "note": "per-token latency through nb_batch_step (host mask in, token out), depth 20"}


if __name__ == "__main__":
    main()
