#!/usr/bin/env python3
"""Decode benchmark of TinyBrain's hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--config C]

Default run (one JSON line from rank 0), at every N:
  * headline = BASELINE config 4: the TinyLlama-1.1B-shaped INT8 model decoding
    64 independent sequences (prompt lengths U[512, 4096], numpy PCG64 seed 4)
    greedily; the sequences are spread data parallel over the N ranks
    (longest prompt first to the least-loaded rank, no collective on the data
    path).  A step is one decode token of every sequence; W warm-up steps,
    then K timed ones (W + K <= 128, the config's decode length).  value =
    64 * K / (max over ranks of the device time of K graph replays): strong
    scaling, the 64 sequences are fixed.
  * "tp": BASELINE config 5, the Llama-2-7B-shaped INT4-g32 model, batch 1,
    tensor parallel over the same N ranks (column q/k/v and gate/up, row
    o_proj/down with the residual all-reduce over NVLink peer memory).
  * at N = 1 also "b1" (TinyLlama INT8, batch 1, prompt 128,
    greedy decode) and "gemv_config1" (config 1: one INT8 GEMV 2048 x 4096 and
    its INT4-g32 twin, HBM GB/s).
Every object carries `e2e` (the same metric through the public API from host
prompts, per-token read-back), a roofline of its dominant kernel family on
the graph-replayed device timeline, clocks sampled during the timed region and
a check of its greedy tokens against the oracle's lists in
tests/golden/config_tokens.json where they exist.  `--impl reference` times
the reference's CPU algorithm (the oracle restatement in reference-faithful
mode, all host cores) on bounded samples of the headline workload.
`--config 1..6` runs one configuration alone (6 = the perplexity harness, the
only workload with published reference numbers).
"""
import argparse
import gc
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tok/s (INT8/INT4, b=1 & b=64); dequant-GEMV HBM GB/s as % of peak"
UNIT = "tok/s"
MODEL_SEED = 0
C4_SEQS, C4_NEW, C4_MAXLEN = 64, 128, 4224
GOLDEN = os.path.join(ROOT, "tests", "golden", "config_tokens.json")
TRAFFIC = os.path.join(ROOT, "profiles", "dram_traffic.md")


# ------------------------------------------------------------------ helpers --
class Env:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.dist = None

    def init(self):
        if self.world > 1 and self.dist is None:
            import torch
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", device_id=torch.device("cuda", self.local))
            self.dist = dist

    def barrier(self):
        if self.dist:
            self.dist.barrier()

    def max(self, v):
        if not self.dist:
            return v
        import torch
        t = torch.tensor([float(v)], device=f"cuda:{self.local}")
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def gather(self, obj):
        if not self.dist:
            return [obj]
        out = [None] * self.world
        self.dist.all_gather_object(out, obj)
        return out


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def golden(name):
    try:
        with open(GOLDEN) as f:
            return json.load(f).get(name)
    except Exception:
        return None


def traffic_per_launch(kernel_key):
    """DRAM bytes per launch (dram__bytes_read.sum + dram__bytes_write.sum) of
    an ncu capture summarised in profiles/dram_traffic.md: table rows
    `| key | ... | bytes per launch | ...` (third column)."""
    try:
        with open(TRAFFIC) as f:
            for line in f:
                cells = [c.strip() for c in line.strip().strip("|").split("|")]
                if len(cells) >= 3 and cells[0] == kernel_key:
                    return float(cells[2].replace(",", ""))
    except Exception:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region (read-only query)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
            return
        import select
        r, _, _ = select.select([self.proc.stdout], [], [], 5.0)
        if r:
            self.proc.stdout.readline()  # the sample before the timed region is dropped

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=5)
        except Exception:
            self.proc.kill()
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


class profile_range:
    """TB_PROFILE_RANGE=1: bracket the timed decode loop with
    cudaProfilerStart / Stop, so `ncu --profile-from-start off` records only
    the timed steps' launches (the launch list in profiles/)."""

    def __enter__(self):
        self.on = os.environ.get("TB_PROFILE_RANGE") == "1"
        if self.on:
            import torch
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
        return self

    def __exit__(self, *exc):
        if self.on:
            import torch
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
        return False


def timeline_roofline(runner, attn_bytes_per_launch, family_names, traffic_keys, peak, peak_kind):
    """Roofline of the dominant kernel family on the device timeline of one
    graph-replayed step (tb_runner_trace_launches: globaltimer stamps per
    launch).  With programmatic dependent launch the next kernel's CTAs start
    while the previous one runs, so each launch is charged the interval
    between the previous launch's last CTA exit and its own (the sum over the
    step is the step's device time, launches overlap nowhere twice).
    Algorithmic bytes per launch: tb_runner_profile_step (weights + scales as
    stored + activations) for GEMVs, K/V rows of the context for attention."""
    import numpy as np
    stamps, kinds = runner.trace_launches()
    _, _, nbytes = runner.profile_step()
    exits = stamps[:, 6].astype(np.float64)
    for i in range(1, len(exits)):  # a launch without stamps inherits its predecessor's exit
        if exits[i] <= 0:
            exits[i] = exits[i - 1]
    start = float(stamps[0, 0])
    prev = np.concatenate([[start], exits[:-1]])
    excl_us = np.maximum(exits - prev, 0.0) / 1000.0
    step_us = float(exits[-1] - start) / 1000.0
    fam = {}
    gm, am, dg = kinds == 0, kinds == 1, kinds == 6
    fam["gemv"] = (float(nbytes[gm].sum()), float(excl_us[gm].sum() + excl_us[dg].sum()), int(gm.sum()))
    fam["attention"] = (float(attn_bytes_per_launch) * int(am.sum()), float(excl_us[am].sum()), int(am.sum()))
    dom = max(fam, key=lambda k: fam[k][1])
    b, us, n = fam[dom]
    achieved = b / (us * 1e-6) / 1e9 if us > 0 else 0.0
    tr = traffic_per_launch(traffic_keys[dom])
    out = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
           "traffic": tr, "peak_source": f"{peak_kind} hbm_gbs (burst copy)", "kernel": family_names[dom],
           "bytes_per_launch": b / max(n, 1), "launches_per_step": n, "us_per_launch": us / max(n, 1),
           "timing": "device timeline of one graph-replayed step (globaltimer), exit-to-exit per launch",
           "traced_step_us": step_us,
           "families": {k: {"bytes": v[0], "us": v[1], "launches": v[2],
                            "gbs": v[0] / (v[1] * 1e-6) / 1e9 if v[1] > 0 else None} for k, v in fam.items()}}
    if tr is not None:
        out["traffic_key"] = traffic_keys[dom]
    return out


def tokens_vs_fixture(name, key_to_tokens):
    """Greedy tokens of the device run against the oracle lists (exact match,
    or a near-tie flip at a step whose oracle top-2 gap < 1e-4: reported)."""
    fx = golden(name)
    if not fx:
        return None
    checked, identical, flips = 0, True, []
    for seq in fx["sequences"]:
        got = key_to_tokens.get(seq["key"])
        if got is None:
            continue
        want = seq["tokens"][:len(got)]
        checked += 1
        for i, (a, b) in enumerate(zip(got, want)):
            if a != b:
                if seq["gaps"][i] < 1e-4:
                    flips.append([seq["key"], i, seq["gaps"][i]])
                else:
                    identical = False
                break
    return {"fixture": name, "sequences_checked": checked, "identical": identical and not flips,
            "near_tie_flips": flips}


def build_tinyllama(ctx, mode="perChannel", max_seq_len=None):
    from tinybrain_b200.runtime import ModelConfig
    from tinybrain_b200.synthetic import TINYLLAMA, make_llama_model
    cfg = ModelConfig(**{**TINYLLAMA, **({"max_seq_len": max_seq_len} if max_seq_len else {})})
    return make_llama_model(cfg, seed=MODEL_SEED, mode=mode, ctx=ctx)


def config4_workload(world):
    import numpy as np
    rng = np.random.default_rng(4)
    lens = rng.integers(512, 4097, size=C4_SEQS)
    prompts = [rng.integers(0, 32000, size=int(n)).tolist() for n in lens]
    load = [0] * world
    owner = [0] * C4_SEQS
    for i in sorted(range(C4_SEQS), key=lambda i: -lens[i]):
        r = min(range(world), key=lambda q: load[q])
        load[r] += int(lens[i])
        owner[i] = r
    return lens, prompts, owner


# ------------------------------------------------------------ CPU baselines --
def cpu_sample_config4(seconds, warmup=1, max_steps=None, threads=None):
    """The reference's CPU algorithm (oracle, mode 0: dequantize each weight
    per call then a sequential fp32 GEMV; scalar attention over the gathered
    context) on a bounded sample of the headline workload: sequence-steps of
    8 of the 64 sequences spread over the length distribution, each at its own
    context (prompt length + a few steps; the KV rows are synthetic, filled
    through the cache's paging rules, so no CPU prefill is needed), cycled
    round robin.  Uses only oracle/ (never the product library)."""
    import numpy as np
    import oracle
    from oracle.synthetic import TINYLLAMA, llama_model
    n = threads or host_cores()
    oracle.set_threads(n)
    lens, _, _ = config4_workload(1)
    order = np.argsort(lens, kind="stable")
    pick = [int(order[j]) for j in range(4, C4_SEQS, 8)]  # 8 sequences across the distribution
    w = llama_model({**TINYLLAMA, "max_seq_len": C4_MAXLEN}, seed=MODEL_SEED, mode="perChannel")
    runners = []
    for i in pick:
        om = oracle.OracleModel(w, mode=0)
        om.fill_context(int(lens[i]), seed=i + 1)
        runners.append(om)
    for j in range(warmup):
        runners[j % len(runners)].step(1)
    steps, t0 = 0, time.perf_counter()
    while (time.perf_counter() - t0) < seconds and (max_steps is None or steps < max_steps):
        runners[steps % len(runners)].step(7)
        steps += 1
    dt = time.perf_counter() - t0
    ctxs = [int(lens[i]) for i in pick]
    return steps, dt, n, (f"{steps} single-sequence decode steps cycled over 8 of config 4's 64 sequences "
                          f"(contexts {min(ctxs)}..{max(ctxs)}, synthetic KV rows), oracle mode 0 "
                          f"(reference-faithful fp32), OpenMP over {n} host threads")


# ------------------------------------------------------------------ config 4 --
def run_config4(args, env, cpu=True):
    import numpy as np
    from tinybrain_b200.runtime import Context, ModelRunner
    lens, prompts, owner = config4_workload(env.world)
    if args.prompt_len:  # profiling captures only: cap the prompt lengths
        lens = np.minimum(lens, args.prompt_len)
        prompts = [p[:args.prompt_len] for p in prompts]
    mine = [i for i in range(C4_SEQS) if owner[i] == env.rank]
    ctx = Context(env.local)
    t_build = time.perf_counter()
    # profiling captures (--prompt-len) size the KV pool for the capped prompts
    maxlen = C4_MAXLEN if not args.prompt_len else args.prompt_len + C4_NEW + 64
    weights = build_tinyllama(ctx, max_seq_len=maxlen)
    runner = ModelRunner(weights, ctx, max_batch=len(mine), max_positions=maxlen + 64)
    build_s = time.perf_counter() - t_build
    my_prompts = [prompts[i] for i in mine]
    W = args.warmup
    K = min(args.steps, C4_NEW - W)
    t0 = time.perf_counter()
    runner.prefill_device(my_prompts, W + K)
    prefill_s = time.perf_counter() - t0
    runner.decode_device(W)
    clocks = ClockSampler(env.local)
    env.barrier()
    clocks.start()
    with profile_range():
        ms = runner.decode_device(K)
    clk = clocks.stop()
    t_dev = env.max(ms / 1000.0)
    value = C4_SEQS * K / t_dev
    dev_tokens = runner.read_tokens(len(mine), W + K)
    peak, peak_kind = measured_peaks()
    # context of the traced step: prompt + W + K decode steps + this one
    kvd = 256
    att_bytes = sum((len(p) + W + K + 1) * kvd * 2 * 4 for p in my_prompts)
    roof = timeline_roofline(
        runner, att_bytes,
        {"gemv": "gemv_kernel<8,128,64> (+ wide_digits): all projections + LM head of one step, all rows"
                 if len(mine) > 16 else "gemv_kernel<8,128,*>: all projections + LM head of one step",
         "attention": ("attn_flat_gqa8_kernel (persistent chunked paged attention, all layers)" if len(mine) * 4 >= 64
                       else "attn_gqa8_d64_kernel (cluster-split paged attention, all layers)")},
        {"gemv": f"gemv int8 M={len(mine)} tinyllama", "attention": f"attention tinyllama config4 M={len(mine)}"},
        peak, peak_kind)
    launches = int(len(runner.profile_step()[1]))

    # ---- end to end through the public API (host prompts in, per-token read-back) ----
    runner.io_bytes(reset=True)
    stamps = {}

    def on_token(seq, idx, tok):
        stamps[idx] = time.perf_counter()
        return False

    env.barrier()
    e2e_tokens = runner.generate_batch(my_prompts, W + K, stop_tokens=(), callback=on_token)
    h2d, d2h = runner.io_bytes()
    n_steps_e2e = W + K
    e2e_t = env.max(stamps[W + K - 1] - stamps[W - 1])
    e2e_value = C4_SEQS * K / e2e_t
    same = e2e_tokens == [t[:W + K] for t in dev_tokens]
    parity = env.gather(tokens_vs_fixture("config4", {i: dev_tokens[j] for j, i in enumerate(mine)}))
    runner.close()
    del runner, weights
    gc.collect()
    cpu_line = None
    if cpu and env.world == 1 and env.rank == 0 and not args.no_cpu:
        steps, dt, n, sample = cpu_sample_config4(20.0)
        cpu_line = {"value": steps / dt, "unit": UNIT, "cores": n, "kind": "port", "sample": sample}
    checked = [p for p in parity if p]
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": env.world, "steps": K, "warmup": W,
        "ms_per_step": 1000.0 * t_dev / K, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "int8 weights x fp32 activations (exact integer tensor-core products, fp32 epilogue)",
        "data": "synthetic (seeded LCG normal std 0.02 weights; numpy PCG64 seed 4 prompt lengths and ids)",
        "config": {"workload": "TinyLlama-1.1B-shaped INT8, 64 sequences, prompts U[512,4096], greedy decode "
                               "(BASELINE config 4)", "global_batch": C4_SEQS,
                   "parallelism": f"dp{env.world} (sequences longest-first to the least-loaded rank, no collective)",
                   "batch_rank0": len(mine), "prefill_s_rank0": round(prefill_s, 1),
                   "model_build_s": round(build_s, 1),
                   "l2": "weights (1.04 GB) and KV (GBs) streamed every step exceed L2; no flush needed"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": round(h2d / n_steps_e2e, 1),
                "d2h_bytes_per_step": round(d2h / n_steps_e2e, 1),
                "api": "ModelRunner.generate_batch (tb_runner_generate, per-token callback; prompt prefill "
                       "outside the timed window)", "tokens_match_device_run": same},
        "roofline": roof,
        "parity": {"sequences_checked": sum(p["sequences_checked"] for p in checked),
                   "identical": all(p["identical"] for p in checked) if checked else None,
                   "near_tie_flips": [f for p in checked for f in p["near_tie_flips"]]},
        "gpu_launches": launches * K,
        "clocks": clk,
    }
    if cpu_line:
        line["cpu_baseline"] = cpu_line
    return line


# ------------------------------------------------------------------ config 2 --
def run_config2(args, env, mode="perChannel", steps=None):
    """BASELINE config 2 (mode int4: config 3): one sequence, batch 1.
    steps: timed steps (default --steps when run alone, --b1-steps nested)."""
    from tinybrain_b200.runtime import Context, ModelRunner
    from tinybrain_b200.synthetic import random_prompt
    cfg3 = mode == "int4"
    ctx = Context(env.local)
    t_build = time.perf_counter()
    weights = build_tinyllama(ctx, mode=mode)
    runner = ModelRunner(weights, ctx, max_batch=1, max_positions=2048 + 64)
    runner.persistent = bool(args.persistent)
    build_s = time.perf_counter() - t_build
    if cfg3:
        prompt = random_prompt(args.prompt_len or 1920, 32000, 3)
        W, K = args.warmup, min(args.steps, 128 - args.warmup)
    else:
        prompt = random_prompt(args.prompt_len or 128, 32000, 2)
        W, K = args.warmup, min(steps or args.steps, 256 - args.warmup)
    runner.ctx.synchronize()
    t_pf = time.perf_counter()
    runner.prefill_device([prompt], W + K)
    runner.ctx.synchronize()
    prefill_s = time.perf_counter() - t_pf
    runner.decode_device(W)
    clocks = ClockSampler(env.local)
    clocks.start()
    with profile_range():
        ms = runner.decode_device(K)
    clk = clocks.stop()
    t_dev = ms / 1000.0
    dev_tokens = runner.read_tokens(1, W + K)[0]
    peak, peak_kind = measured_peaks()
    L = len(prompt) + W + K
    tag = "int4" if cfg3 else "int8"
    roof = None
    if not runner.persistent:
        roof = timeline_roofline(runner, L * 256 * 2 * 4,
                                 {"gemv": f"gemv_kernel<{4 if cfg3 else 8},128,1>: all projections + LM head of one step",
                                  "attention": "attn_decode_kernel (paged KV, all layers)"},
                                 {"gemv": f"gemv {tag} M=1 tinyllama", "attention": f"attention tinyllama {tag} M=1"},
                                 peak, peak_kind)
    launches = int(len(runner.profile_step()[1]))
    runner.io_bytes(reset=True)
    stamps = []

    def on_token(seq, idx, tok):
        stamps.append(time.perf_counter())
        return False

    e2e_tokens = runner.generate_batch([prompt], W + K, stop_tokens=(), callback=on_token)[0]
    h2d, d2h = runner.io_bytes()
    n_steps_e2e = (len(prompt) - 1) + W + K
    e2e_value = K / (stamps[-1] - stamps[W - 1])
    step_bytes = float(runner.model.weight_bytes)
    parity = tokens_vs_fixture("config3" if cfg3 else "config2", {"seq": dev_tokens})
    runner.close()
    del runner, weights
    gc.collect()
    return {
        "metric": "decode tok/s, batch 1", "value": K / t_dev, "unit": UNIT, "steps": K, "warmup": W,
        "ms_per_step": 1000.0 * t_dev / K,
        "dtype": ("int4-g32 weights x fp32 activations" if cfg3 else
                  "int8 weights x fp32 activations (exact integer tensor-core products, fp32 epilogue)"),
        "config": {"workload": ("TinyLlama-1.1B-shaped INT4-g32, batch 1, prompt 1920, greedy decode (BASELINE config 3)"
                                if cfg3 else "TinyLlama-1.1B-shaped INT8, batch 1, prompt 128, greedy decode "
                                             "(BASELINE config 2)"),
                   "prompt": len(prompt), "decode_tokens": W + K, "model_build_s": round(build_s, 1),
                   "l2": "weights streamed per step exceed L2; no flush needed"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": round(h2d / n_steps_e2e, 1),
                "d2h_bytes_per_step": round(d2h / n_steps_e2e, 1),
                "api": "ModelRunner.generate_stream path (tb_runner_generate with per-token callback)",
                "tokens_match_device_run": e2e_tokens == dev_tokens},
        "roofline": roof,
        "step_roofline": {"weight_bytes_per_step": step_bytes, "achieved_gbs": step_bytes / (t_dev / K) / 1e9,
                          "frac": step_bytes / (t_dev / K) / 1e9 / peak},
        "parity": parity,
        "prefill": {"tokens": len(prompt) - 1, "seconds": round(prefill_s, 4),
                    "tok_s": round((len(prompt) - 1) / max(prefill_s, 1e-9), 1)},
        "gpu_launches": launches * K, "clocks": clk,
    }


# ------------------------------------------------------------------ config 5 --
def run_config5(args, env, steps=None):
    """Llama-2-7B-shaped INT4-g32, batch 1, prompt 512 (seed 5),
    greedy decode, tensor parallel over the ranks."""
    from tinybrain_b200.runtime import Context, ModelConfig, ModelRunner, tp_unique_id
    from tinybrain_b200.synthetic import LLAMA2_7B, make_llama_model, random_prompt
    world, rank = env.world, env.rank
    n_prompt, n_new = (args.prompt_len or 512), 256
    cfg = ModelConfig(**{**LLAMA2_7B, "max_seq_len": 768})
    ctx = Context(env.local)
    if world > 1:
        uid = [tp_unique_id() if rank == 0 else None]
        env.dist.broadcast_object_list(uid, src=0)
        ctx.init_tensor_parallel(uid[0], rank, world)
    t_build = time.perf_counter()
    weights = make_llama_model(cfg, seed=MODEL_SEED, mode="int4", ctx=ctx, shard=(rank, world) if world > 1 else None)
    dm = weights.upload(ctx, tp=(rank, world))
    runner = ModelRunner(dm, ctx, max_batch=1, max_positions=cfg.max_seq_len + 64)
    peer = world > 1 and os.environ.get("TB_TP_ALLREDUCE", "peer") != "nccl"
    if peer:
        runner.tp_connect(env.gather(runner.tp_handle()))
        env.barrier()
    build_s = time.perf_counter() - t_build
    prompt = random_prompt(n_prompt, 32000, 5)
    W = args.warmup
    K = min(steps or args.steps, n_new - W)
    t0 = time.perf_counter()
    runner.prefill_device([prompt], W + K)
    prefill_s = time.perf_counter() - t0
    runner.decode_device(W)
    clocks = ClockSampler(env.local)
    env.barrier()
    clocks.start()
    ms = runner.decode_device(K)
    clk = clocks.stop()
    t_dev = env.max(ms / 1000.0)
    dev_tokens = runner.read_tokens(1, W + K)[0]
    peak, peak_kind = measured_peaks()
    roof = timeline_roofline(runner, (n_prompt + W + K + 1) * (4096 // world) * 2 * 4,
                             {"gemv": "gemv_kernel<4,128,1>: all projection shards + LM head of one step (rank 0)",
                              "attention": "attn_decode_kernel (paged KV, all layers)"},
                             {"gemv": f"gemv int4 M=1 7b tp{world}", "attention": f"attention 7b tp{world}"},
                             peak, peak_kind)
    kinds = runner.profile_step()[1]
    runner.io_bytes(reset=True)
    stamps = []

    def on_token(seq, idx, tok):
        stamps.append(time.perf_counter())
        return False

    env.barrier()
    e2e_tokens = runner.generate_batch([prompt], W + K, stop_tokens=(), callback=on_token)[0]
    h2d, d2h = runner.io_bytes()
    n_steps_e2e = (len(prompt) - 1) + W + K
    e2e_value = K / env.max(stamps[-1] - stamps[W - 1])
    all_tokens = env.gather(dev_tokens)
    parity = tokens_vs_fixture("config5", {"seq": dev_tokens})
    wbytes = float(dm.weight_bytes)
    runner.close()
    del runner, dm, weights
    gc.collect()
    return {
        "metric": "decode tok/s, batch 1, tensor parallel", "value": K / t_dev, "unit": UNIT, "n_gpus": world,
        "steps": K, "warmup": W, "ms_per_step": 1000.0 * t_dev / K, "scaling": "strong",
        "dtype": "int4-g32 weights x fp32 activations",
        "config": {"workload": "Llama-2-7B-shaped INT4-g32, batch 1, prompt 512, greedy decode (BASELINE config 5)",
                   "parallelism": f"tp{world} (column q/k/v, gate/up; row o_proj/down + residual all-reduce "
                                  + ("through NVLink peer memory fused into the GEMV launches" if peer else
                                     ("by NCCL" if world > 1 else "none")) + "; LM head replicated)",
                   "prefill_s": round(prefill_s, 1), "model_build_s": round(build_s, 1),
                   "l2": "weights streamed per step per GPU exceed L2; no flush needed"},
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": round(h2d / n_steps_e2e, 1),
                "d2h_bytes_per_step": round(d2h / n_steps_e2e, 1),
                "tokens_match_device_run": e2e_tokens == dev_tokens},
        "roofline": roof,
        "step_roofline": {"weight_bytes_per_step_per_gpu": wbytes, "achieved_gbs": wbytes / (t_dev / K) / 1e9,
                          "frac": wbytes / (t_dev / K) / 1e9 / peak},
        "tokens_identical_across_ranks": all(t == all_tokens[0] for t in all_tokens),
        "parity": parity,
        "gpu_launches": int((kinds != 3).sum()) * K, "clocks": clk,
    }


# ------------------------------------------------------------------ config 1 --
def run_config1(args):
    """one INT8 GEMV x[1,2048] . W[2048 in, 4096 out] (and the
    INT4-g32 twin).  W ~ N(0, 0.02) seed 0, x ~ N(0, 1) seed 1; quantized on the
    GPU; the timed pass cycles through enough weight copies to exceed L2 (126 MB)
    so every GEMV streams its weights from HBM."""
    import numpy as np
    import torch
    from tinybrain_b200.runtime import Context, QuantizedWeight, SeededGenerator, gemv_stream_time, quantize
    ctx = Context(0)
    K, N = 2048, 4096
    w = SeededGenerator(0).normal((K, N), 0.0, 0.02)
    x = SeededGenerator(1).normal((1, K), 0.0, 1.0)
    peak, peak_kind = measured_peaks()
    l2 = 126 * 2**20
    lines = {}
    for mode, algo in (("perChannel", K * N + N * 4 + K * 4 + N * 4),
                       ("int4", K * N // 2 + (K * N // 32) * 4 + K * 4 + N * 4)):
        q = quantize(w, mode, ctx=ctx)
        copies = max(8, -(-3 * l2 // algo))
        ws = [QuantizedWeight(q, ctx) for _ in range(copies)]
        xd = torch.tensor(x, device="cuda:0")
        yd = torch.empty((1, N), dtype=torch.float32, device="cuda:0")
        got = ws[0].matmul(x)
        reps = max(3, args.steps // 10)
        per = gemv_stream_time(ws, xd.data_ptr(), 1, yd.data_ptr(), reps=reps, pdl=2) / copies
        per_dep = gemv_stream_time(ws, xd.data_ptr(), 1, yd.data_ptr(), reps=reps, pdl=1) / copies
        gbs = algo / (per / 1000.0) / 1e9
        gbs_dep = algo / (per_dep / 1000.0) / 1e9
        lines[mode] = {"gemv_us": per * 1000.0, "gbs": gbs, "frac": gbs / peak, "bytes": algo, "copies": copies,
                       "dependent_chain": {"gemv_us": per_dep * 1000.0, "gbs": gbs_dep, "frac": gbs_dep / peak},
                       "y_norm": float(np.linalg.norm(got))}
        for wq in ws:
            wq.close()
    return {
        "metric": "dequant-GEMV HBM GB/s (BASELINE config 1)", "value": lines["perChannel"]["gbs"], "unit": "GB/s",
        "dtype": "int8 weights x fp32 activations", "peak": peak, "peak_source": peak_kind,
        "config": {"workload": "single INT8 GEMV 2048 in x 4096 out, batch 1 (BASELINE config 1)",
                   "l2": f"{lines['perChannel']['copies']} weight copies cycled (> 3 x L2) per pass",
                   "launch": "one CUDA graph of back-to-back GEMVs; gbs: independent launches (executions overlap), "
                             "dependent_chain: each waits for its predecessor, as inside a step"},
        "int8": lines["perChannel"], "int4_g32": lines["int4"],
    }


# ------------------------------------------------------------------ config 6 --
def run_config6(args):
    """The reference's only published figures for this path: the step rate of
    its perplexity harness (PerplexityHarness.computePerplexity: 64 teacher-
    forced steps at context <= 65 on TinyLlama), 1.66 tok/s INT8 and 1.52 tok/s
    INT4-g32 on an M4 Max.  The same work here through ModelRunner.perplexity
    (one chunk of 64 positions; host slice in, fp64 sum out)."""
    from tinybrain_b200.runtime import Context, ModelRunner, convert_to_int4
    from tinybrain_b200.synthetic import random_prompt
    ctx = Context(0)
    w8 = build_tinyllama(ctx)
    w4 = convert_to_int4(w8, 32, ctx)
    slice_ids = [1] + [int(t) for t in random_prompt(64, 32000, 6)]
    W, K = args.warmup, max(1, min(args.steps, 100))
    out = {}
    for name, w, published in (("int8", w8, 64 / 38.45), ("int4_g32", w4, 64 / 42.24)):
        r = ModelRunner(w, ctx, max_batch=1, max_positions=len(slice_ids) + 8)
        for _ in range(W):
            r.perplexity([slice_ids])
        clocks = ClockSampler(0)
        clocks.start()
        t0 = time.perf_counter()
        for _ in range(K):
            res = r.perplexity([slice_ids])[0]
        dt = time.perf_counter() - t0
        clk = clocks.stop()
        rate = K * res.num_predictions / dt
        out[name] = {"value": rate, "ms_per_call": 1000.0 * dt / K, "perplexity": res.perplexity,
                     "published_tok_s": round(published, 3), "vs_published": rate / published, "clocks": clk}
        r.close()
    v = out["int8"]["value"]
    return {
        "metric": "perplexity-harness step rate (teacher-forced TinyLlama steps/s)", "value": v, "unit": "tok/s",
        "n_gpus": 1, "steps": K, "warmup": W, "ms_per_step": 1000.0 / v, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": out["int8"]["vs_published"],
        "dtype": "int8 weights x fp32 activations; fp64 log-sum-exp",
        "data": "synthetic (seeded LCG normal std 0.02 weights; slice = BOS + 64 seeded uniform ids)",
        "config": {"workload": "PerplexityHarness.computePerplexity, TinyLlama-1.1B shape, 65-token slice "
                               "(64 predictions), INT8 and convertToINT4 g32",
                   "l2": "weights (1.04 GB INT8) exceed L2 every step"},
        "e2e": {"value": v, "unit": "tok/s", "h2d_bytes_per_step": round(4 * 65 / 64, 1),
                "d2h_bytes_per_step": round(8 / 64, 2),
                "api": "ModelRunner.perplexity (tb_runner_perplexity): host slice in, fp64 sum out"},
        "int8": out["int8"], "int4_g32": out["int4_g32"], "clocks": out["int8"]["clocks"],
        "gpu_launches": K * (5 * 22 + 2),
    }


# ------------------------------------------------- standalone attention --
def run_attention_kernel(args):
    """--kernel attention: the paged decode attention of one layer at the
    headline shape (64 sequences, contexts = config 4's prompt lengths + 128,
    32 query / 4 KV heads, d 64, scattered pages), through
    tb_paged_attention_dev, CUDA events over `--steps` launches on the
    context's stream.  K/V bytes per launch: every context position's K and V
    row of its KV head, once."""
    import ctypes as C
    import numpy as np
    import torch
    from tinybrain_b200 import _lib
    from tinybrain_b200.runtime import Context
    ctx = Context(0)
    lens = [int(n) + C4_NEW for n in config4_workload(1)[0]]
    H, Hkv, d = 32, 4, 64
    pages = [(n + 15) // 16 for n in lens]
    stride, total = max(pages), sum(pages)
    perm = np.random.default_rng(1).permutation(total)
    ptab = np.full((len(lens), stride), -1, dtype=np.int32)
    k = 0
    for s_, n in enumerate(pages):
        ptab[s_, :n] = perm[k:k + n]
        k += n
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    pool = torch.randn(total, 1, 2, Hkv, 16, d, device=dev, generator=g)
    q = torch.randn(len(lens), H * d, device=dev, generator=g)
    out = torch.zeros(len(lens), H * d, device=dev)
    pt = torch.tensor(ptab, device=dev)
    ln = torch.tensor(lens, dtype=torch.int32, device=dev)
    lib = _lib.load()
    P = lambda t: C.c_void_p(t.data_ptr())  # noqa: E731

    def launch():
        _lib.check(lib.tb_paged_attention_dev(ctx.handle, P(q), len(lens), P(pool), P(pt), stride, P(ln), max(lens),
                                              0, 1, H, Hkv, d, P(out)))

    for _ in range(args.warmup):
        launch()
    ctx.synchronize()
    st = torch.cuda.ExternalStream(lib.tb_context_stream(ctx.handle))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    K = max(1, args.steps)
    clocks = ClockSampler(0)
    clocks.start()
    e0.record(st)
    for _ in range(K):
        launch()
    e1.record(st)
    e1.synchronize()
    clk = clocks.stop()
    ctx.check_device()
    us = e0.elapsed_time(e1) * 1000.0 / K
    nbytes = sum(lens) * Hkv * d * 2 * 4
    peak, kind = measured_peaks()
    print(json.dumps({"metric": "paged decode attention HBM GB/s (one layer, config 4 shape)",
                      "value": nbytes / (us * 1e-6) / 1e9, "unit": "GB/s", "us_per_launch": us,
                      "bytes_per_launch": nbytes, "frac": nbytes / (us * 1e-6) / 1e9 / peak,
                      "peak": peak, "peak_source": kind, "launches": K, "warmup": args.warmup,
                      "config": {"sequences": len(lens), "tokens": sum(lens), "heads": "32q/4kv", "head_dim": d,
                                 "l2": "K/V of one launch (350 MB) exceed L2"},
                      "clocks": clk}), flush=True)
    return 0


# ------------------------------------------------------------------ arms --
def run_reference(args):
    """--impl reference: the reference's CPU algorithm on the host cores, on the
    headline workload (config 4), with every host thread; oracle only."""
    env = Env()
    if env.rank != 0:
        return 0
    W = args.warmup
    K = min(args.steps, C4_NEW - W)
    steps, dt, n, sample = cpu_sample_config4(float(os.environ.get("TB_REF_BUDGET_S", "90")), warmup=W,
                                              max_steps=K)
    v = steps / dt
    try:
        with open("/proc/self/maps") as f:
            product_loaded = "libtinybrain_cuda" in f.read()
    except OSError:
        product_loaded = None
    line = {
        "impl": "reference", "product_library_loaded": product_loaded, "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus, "steps": steps,
        "warmup": W, "ms_per_step": 1000.0 * dt / steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded LCG, std 0.02)",
        "config": {"workload": "TinyLlama-1.1B-shaped INT8, 64 sequences, prompts U[512,4096], greedy decode "
                               "(BASELINE config 4)", "global_batch": C4_SEQS,
                   "impl": "the reference's CPU path restated in C (oracle port, mode 0); the Swift/Accelerate "
                           "reference does not build on Linux",
                   "step": "one decode step of one sequence (bounded sample of the 64-sequence step)"},
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": n, "kind": "port", "sample": sample},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    env = Env()
    env.init()
    cfg = args.config
    if cfg == 1:
        line = run_config1(args)
    elif cfg in (2, 3):
        line = run_config2(args, env, mode="int4" if cfg == 3 else "perChannel")
    elif cfg == 5:
        line = run_config5(args, env)
    elif cfg == 6:
        line = run_config6(args)
    else:
        line = run_config4(args, env)
        if cfg is None:
            if env.world == 1:
                line["b1"] = run_config2(args, env, steps=args.b1_steps)
                line["gemv_config1"] = run_config1(args)
            line["tp"] = run_config5(args, env, steps=args.tp_steps)
    if env.rank == 0:
        line.setdefault("n_gpus", env.world)
        print(json.dumps(line), flush=True)
    if env.dist:
        env.dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=125, help="timed decode steps of the headline (W + K <= 128)")
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--b1-steps", type=int, default=253, help="timed steps of the batch-1 object (config 2)")
    ap.add_argument("--tp-steps", type=int, default=253, help="timed steps of the tensor-parallel object (config 5)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--persistent", action="store_true",
                    help="config 2/3: one persistent kernel per step instead of the per-projection launch chain")
    ap.add_argument("--prompt-len", type=int, default=0,
                    help="cap / set the prompt length (profiling captures only; 0 = the config's)")
    ap.add_argument("--config", type=int, default=None, choices=[1, 2, 3, 4, 5, 6],
                    help="run one BASELINE config alone: 1 single GEMV, 2 TinyLlama INT8 b=1, 3 INT4 at context 2k, "
                         "4 64 sequences data parallel, 5 7B INT4 tensor parallel, 6 perplexity harness")
    ap.add_argument("--kernel", default=None, choices=["attention"],
                    help="time one kernel alone at the headline shape (profiling)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    if args.kernel == "attention":
        return run_attention_kernel(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
