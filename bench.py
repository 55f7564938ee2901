"""Batch-1 decode throughput of the Llama-3-8B-shape decoder (bf16) on B200.

Workload (the default, --preset 3): Llama-3-8B shape (vocab 128256, d 4096, 32 layers, 32 q /
8 kv heads of 128, SwiGLU 14336, RoPE theta 5e5), weights N(0, 0.02) from seed 0, a 2048-token
prompt of uniform ids from seed 1, then greedy decode.  A step is one decoded token at batch 1;
the timed steps are decode positions 2048 .. 2048+K-1 (warm-up steps run at the same positions
first and are overwritten).  Every step streams ~15.3 GB of weights and KV, far above the
126 MB L2, so no L2 flush is needed between steps.  --preset 2 is the TinyLlama-1.1B shape
(prompt 512, 512 steps, 2.09 GB per step); --preset 1 the tiny d288 fp32 model (prompt 16,
240 steps), whose 61 MB of weights stay in L2, so it reports latency per step.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--preset 1|2|3]

Prints one JSON line (rank 0).  `value` is device-timed (CUDA events on the library's
stream, max over ranks); `e2e` times the per-token public call inf_forward() with the id
copied in from pinned host memory and the argmax read back every step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "inference-project_b200"))

METRIC = "batch-1 decode tokens/s and % of HBM roofline (Llama-3-8B shape, bf16), TP 1/2/4/8"
# DRAM bytes (read + write) that ncu counted for one gate/up + SwiGLU launch at TP 1
# (234.96 MB read + 3.38 MB write; the algorithmic figure is 234.9 MB)
GATEUP_NCU_TRAFFIC = 238.34e6
PROMPT = 2048
DECODE_STEPS = 1024

# The decode workloads as plain model dicts (the oracle's form), so that the reference arm runs
# without loading the library under test; tests/test_bench_cpu.py checks them against the
# library's presets.
_LLAMA3 = dict(vocab=128256, dim=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128, ffn=14336, max_seq=3072,
               eps=1e-5, rope_theta=500000.0, dtype="bf16", init_std=0.02)
DECODE = {
    1: dict(model=dict(vocab=32000, dim=288, n_layers=6, n_heads=6, n_kv_heads=6, head_dim=48, ffn=768, max_seq=256,
                       eps=1e-5, rope_theta=10000.0, dtype="fp32", init_std=0.02),
            prompt=16, steps=240, name="tiny-llama-d288-fp32",
            metric="batch-1 greedy decode latency per step (tiny Llama d288, 6 layers, fp32; weights L2-resident)"),
    2: dict(model=dict(vocab=32000, dim=2048, n_layers=22, n_heads=32, n_kv_heads=4, head_dim=64, ffn=5632,
                       max_seq=1024, eps=1e-5, rope_theta=10000.0, dtype="bf16", init_std=0.02),
            prompt=512, steps=512, name="tinyllama-1.1b-shape",
            metric="batch-1 decode tokens/s and % of HBM roofline (TinyLlama-1.1B shape, bf16), 1 GPU"),
    3: dict(model=_LLAMA3, prompt=2048, steps=1024, name="llama-3-8b-shape", metric=METRIC),
    # the Gemma-4-E2B shape of the reference's comments (src/model.cuh:9-14); not a BASELINE config
    6: dict(model=dict(vocab=262144, dim=1536, n_layers=35, n_heads=8, n_kv_heads=2, head_dim=512, ffn=6144,
                       max_seq=4096, eps=1e-6, rope_theta=1000000.0, dtype="bf16", init_std=0.02, arch=1, ple_dim=256,
                       final_softcap=30.0),
            prompt=1024, steps=512, name="gemma-4-e2b-shape",
            metric="batch-1 decode tokens/s and % of HBM roofline (Gemma-4-E2B shape, bf16), 1 GPU"),
}


def load_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        """Starts nvidia-smi and returns once its first sample is in, so that starting the sampler
        (a fork of this process and nvidia-smi's start-up) happens before the timed region's
        barrier: under tensor parallelism a rank that started late would make the others' first
        exchanges wait for it inside their timed regions."""
        self.first = []
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.device)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.first.append(self.proc.stdout.readline())
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in self.first + out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx.append(float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def oracle_decode_rate(cfg_dict: dict, ctx: int, budget_s: float, warmup: int = 1, max_tokens=None):
    """Tokens/s of the CPU oracle's decode at context `ctx` on all host cores."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import numpy as np

    import oracle as O
    threads = os.cpu_count() or 1
    t0 = time.time()
    m = O.OracleModel(cfg_dict, seed=0, n_threads=threads)
    m.fill_kv_synthetic(ctx)
    setup_s = time.time() - t0
    tid = int(O.gen_ids(1, 1, cfg_dict["vocab"])[0])
    pos = ctx
    for _ in range(warmup):
        _, tid = m.forward(np.array([tid], np.uint32), pos)
    n, t0 = 0, time.perf_counter()
    while True:
        _, tid = m.forward(np.array([tid], np.uint32), pos + n)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s or (max_tokens and n >= max_tokens) or pos + n + 1 >= cfg_dict["max_seq"]:
            break
    m.close()
    return n / el, n, el, threads, setup_s


def run_reference(args, rank: int, world: int):
    """The reference arm: the oracle's CPU restatement of the decoder (the reference itself has
    no forward pass), timed on the host cores on this workload's config.  It loads only the
    oracle (oracle/libllama_ref.so), never the library under test."""
    if rank != 0:
        return
    w = DECODE[args.preset]
    d = dict(w["model"])
    prompt = w["prompt"] if args.prompt is None else args.prompt
    # each step is one decoded token at ctx prompt+; bounded so the run ends in a few minutes
    budget = float(os.environ.get("INF_REF_BUDGET_S", "60"))
    rate, n, el, threads, setup_s = oracle_decode_rate(d, prompt, budget, warmup=min(args.warmup, 1))
    latency = args.preset == 1
    line = {
        "impl": "reference", "metric": w["metric"], "value": 1000.0 / rate if latency else rate,
        "unit": "ms" if latency else "tokens/s", "n_gpus": world,
        "steps": n, "warmup": min(args.warmup, 1), "ms_per_step": 1000.0 * el / n, "higher_is_better": not latency,
        "scaling": "strong", "vs_baseline": None, "dtype": d["dtype"], "data": "synthetic",
        "config": {"workload": f"{w['name']} batch-1 decode at ctx {prompt}+", "model": w["name"],
                   "global_batch": 1, "seq_len": prompt, "parallelism": "cpu"},
        "cpu_baseline": {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
                         "sample": f"{n} decode tokens at ctx {prompt}+ with a synthetic KV cache; "
                                   f"CPU restatement (oracle/llama_ref.c, OpenMP), the reference has no forward pass; "
                                   f"setup {setup_s:.0f}s untimed"},
    }
    line["e2e"] = {"value": line["value"], "unit": line["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}
    print(json.dumps(line), flush=True)


def run_ours(args, rank: int, world: int, dist):
    import numpy as np
    import torch

    import infb200 as I

    w = DECODE[args.preset]
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    layers = args.layers or w["model"]["n_layers"]
    cfg = I.preset(args.preset, n_layers=layers, tp_rank=rank if world > 1 else 0, tp_size=world)
    prompt_len = w["prompt"] if args.prompt is None else args.prompt
    steps, warmup = args.steps or w["steps"], args.warmup
    if prompt_len + max(steps, warmup) > cfg.max_seq:
        raise SystemExit(f"--steps/--warmup above {cfg.max_seq - prompt_len}")
    prompt = I.synth_ids(1, prompt_len, cfg.vocab_size)  # seed-1 uniform prompt ids

    eng = I.Engine(cfg, seed=0)
    if world > 1:
        # tensor parallelism: exchange the arenas' IPC handles (host plumbing), then every
        # rank's kernels reach the peers' exchange buffers directly over NVLink
        gloo = dist.new_group(backend="gloo")
        handles = [None] * world
        dist.all_gather_object(handles, eng.tp_export(), group=gloo)
        eng.tp_connect(handles)
    stream = torch.cuda.ExternalStream(eng.stream)
    t0 = time.time()
    _, first = eng.forward(prompt, 0)
    prefill_s = time.time() - t0
    sampling = None
    if args.sample:
        t_, p_, k_ = (float(x) for x in args.sample.split(","))
        sampling = {"temperature": t_, "top_p": p_, "top_k": int(k_), "seed": 7}
        eng.set_sampling(t_, p_, int(k_), seed=7)
    eng.decode(first, prompt_len, warmup)

    def barrier():
        if dist is not None:
            dist.barrier()

    def gather(x):
        """x from every rank, in rank order (one float each)."""
        if dist is None:
            return [x]
        t = torch.tensor([x], device="cuda", dtype=torch.float64)
        out = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [float(v.item()) for v in out]

    # ---- timed region: K decode steps chained on the device (one graph replay per step); the
    # clock sampler is running before the barrier, so no rank starts late
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.synchronize()
        barrier()
        l0 = eng.launches
        torch.cuda.nvtx.range_push("timed")  # lets ncu --nvtx-include "timed/" select these launches
        ev0.record(stream)
        ids, st = eng.decode(first, prompt_len, steps, want_ids=True)  # ids: one 4-byte read per step, at the end
        ev1.record(stream)
        torch.cuda.synchronize()
        torch.cuda.nvtx.range_pop()
        launches = eng.launches - l0
        barrier()
    rank_ms = gather(ev0.elapsed_time(ev1))
    ms = max(rank_ms)
    ms_per_step = ms / steps
    # every rank must have chosen the same ids (the cross-shard argmax is exchanged on the device)
    checksum = int(np.bitwise_xor.reduce((ids.astype(np.uint64) * np.arange(1, steps + 1, dtype=np.uint64))
                                         ^ np.arange(steps, dtype=np.uint64)))
    sums = gather(float(checksum % (1 << 52)))
    ranks_agree = all(v == sums[0] for v in sums)

    # ---- per-kernel durations of one eager step (events around each launch, same stream)
    prof = {}
    for _ in range(3):
        for k, v in eng.profile_step(prompt_len + steps - 1, first).items():
            prof[k] = prof.get(k, 0.0) + v / 3

    # ---- e2e: the per-token public call with host buffers
    tid = first
    e2e_ids = []
    torch.cuda.synchronize()
    barrier()
    e0 = time.perf_counter()
    for s_ in range(steps):
        _, tid = eng.forward([tid], prompt_len + s_, want_logits=False)
        e2e_ids.append(tid)
    e2e_s = max(gather(time.perf_counter() - e0))
    e2e_same = bool(np.array_equal(np.asarray(e2e_ids, np.uint32), ids)) if not sampling else None

    # ---- roofline of the dominant kernel (gate/up projection + SwiGLU)
    peak, peak_kind = load_peaks()
    L, d, F = cfg.n_layers, cfg.dim, cfg.ffn_dim
    Fl = F // world  # this rank's FFN shard
    esz = 2 if cfg.dtype == I.BF16 else 4
    gu_bytes = 2 * Fl * d * esz + d * 4 + Fl * esz
    gu_ms = prof.get("gate_up", 0.0) / L
    achieved = gu_bytes / (gu_ms * 1e-3) / 1e9 if gu_ms > 0 else None
    avg_ctx = prompt_len + (steps - 1) / 2
    step_bytes = I.decode_bytes(cfg, int(avg_ctx))
    step_gbs = step_bytes / (ms_per_step * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.skip_cpu:
        rate, n, el, threads, setup_s = oracle_decode_rate(dict(w["model"], n_layers=layers), prompt_len,
                                                           args.cpu_budget)
        cpu = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"{n} decode tokens ({el:.1f}s) at ctx {prompt_len}+ with a synthetic KV cache, CPU "
                         f"restatement (oracle/llama_ref.c, OpenMP); weight generation {setup_s:.0f}s untimed"}

    latency = args.preset == 1  # weights in L2: latency per step is the figure of merit
    value = ms_per_step if latency else steps / (ms * 1e-3)  # tensor parallel: every rank works on the same tokens
    if rank == 0:
        model = w["name"] if layers == DECODE[args.preset]["model"]["n_layers"] else f"{w['name']}-{layers}-layers"
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": (achieved / peak) if achieved else None,
                    "kernel": f"k_gemv gate/up+SwiGLU (per launch: 2*{Fl}*{d} weights)", "peak_kind": peak_kind}
        if args.preset == 3:
            # dram__bytes_read.sum + dram__bytes_write.sum of one full-width launch (ncu capture of the
            # same kernel and shape), scaled to this rank's shard
            roofline.update(traffic=GATEUP_NCU_TRAFFIC * Fl / F, traffic_unit="bytes per launch")
        else:
            roofline.update(traffic=None)
        if latency:
            roofline["note"] = "61 MB of weights stay in the 126 MB L2: the HBM figure is an upper bound, not the limit"
        line = {
            "metric": w["metric"], "value": value, "unit": "ms" if latency else "tokens/s", "n_gpus": world,
            "steps": steps, "warmup": warmup, "ms_per_step": ms_per_step, "higher_is_better": not latency,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16" if cfg.dtype == I.BF16 else "f32",
            "data": "synthetic (Philox seed-0 N(0,0.02) weights, seed-1 uniform prompt ids)",
            "config": {"workload": f"{w['name']} batch-1 " + ("sampled" if sampling else "greedy")
                                   + f" decode, prompt {prompt_len}, timed positions {prompt_len}..{prompt_len}+K-1",
                       "sampling": sampling, "model": model, "global_batch": 1, "seq_len": prompt_len,
                       "parallelism": f"tp{world}",
                       "l2": "no flush: each step streams the weights (%.2f GB)" % (step_bytes / 1e9)
                             + (", which fit in L2" if latency else " (> 126 MB L2)"),
                       "step_bytes": step_bytes, "step_gbs": step_gbs,
                       "step_roofline_frac": step_gbs / (peak * world), "prefill_s": prefill_s,
                       "kernel_ms_per_step": prof, "rank_ms": rank_ms, "ranks_agree": ranks_agree,
                       "ids_checksum": checksum, "e2e_ids_equal_timed_ids": e2e_same,
                       "tokens_per_s": steps / (ms * 1e-3)},
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": (e2e_s * 1e3 / steps) if latency else steps / e2e_s, "unit": "ms" if latency else "tokens/s",
                    "h2d_bytes_per_step": 12, "d2h_bytes_per_step": 20},
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    eng.close()


def linear_params(cfg, world: int) -> int:
    """Projection weights of one layer on one rank (QKV, O, gate/up, down)."""
    d, hd = cfg.dim, cfg.head_dim
    H, KV, F = cfg.n_heads // world, cfg.n_kv_heads // world, cfg.ffn_dim // world
    return (H + 2 * KV) * hd * d + H * hd * d + 2 * F * d + F * d


def run_workload(args, rank: int, world: int, dist):
    """The long-prefill (32768-token prompt), batched-decode (64 sequences) and continuous-batching
    (192 requests through inf_server into 64 slots) workloads."""
    import numpy as np
    import torch

    import infb200 as I

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    preset = 5 if args.workload == "prefill" else 4
    cfg = I.preset(preset, n_layers=args.layers or 32, tp_rank=rank if world > 1 else 0, tp_size=world)
    eng = I.Engine(cfg, seed=0)
    if world > 1:
        gloo = dist.new_group(backend="gloo")
        handles = [None] * world
        dist.all_gather_object(handles, eng.tp_export(), group=gloo)
        eng.tp_connect(handles)
    stream = torch.cuda.ExternalStream(eng.stream)

    def barrier():
        if dist is not None:
            dist.barrier()

    def max_over_ranks(x):
        if dist is None:
            return x
        t = torch.tensor([x], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    L = cfg.n_layers
    bf16_peak = None
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        bf16_peak, peak_kind = float(p["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:
        bf16_peak, peak_kind = 1400.0, "fallback (sustained)"
    hbm_peak, hbm_kind = load_peaks()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    if args.workload == "prefill":
        T = 32768 if args.prompt is None else args.prompt
        prompt = I.synth_ids(3, T, cfg.vocab_size)  # seed-3 uniform ids
        for _ in range(args.warmup):
            eng.reset(0)
            eng.forward(prompt, 0, want_logits=False)
        torch.cuda.synchronize()
        barrier()
        l0 = eng.launches
        with ClockSampler(local) as clk:
            ms = 0.0
            wall = 0.0
            torch.cuda.nvtx.range_push("timed")
            for _ in range(args.steps):
                eng.reset(0)
                torch.cuda.synchronize()
                w0 = time.perf_counter()
                ev0.record(stream)
                _, first = eng.forward(prompt, 0, want_logits=False)
                ev1.record(stream)
                torch.cuda.synchronize()
                wall += time.perf_counter() - w0
                ms += ev0.elapsed_time(ev1)
            torch.cuda.nvtx.range_pop()
        launches = eng.launches - l0
        barrier()
        ms, wall = max_over_ranks(ms), max_over_ranks(wall)
        # FLOPs of one rank: projections of every token + causal attention (QK and PV)
        H = cfg.n_heads // world
        flop = 2.0 * L * linear_params(cfg, world) * T + 4.0 * L * H * cfg.head_dim * T * (T + 1) / 2
        achieved = flop / (ms / args.steps * 1e-3) / 1e12
        tok_s = args.steps * T / (ms * 1e-3)
        # decode after the long prefill: 128 steps at context ~32k (reported, not the metric)
        dec_steps = 128 if T + 128 <= cfg.max_seq else 0
        dec = None
        if dec_steps:
            torch.cuda.synchronize()
            ev0.record(stream)
            eng.decode(first, T, dec_steps, want_ids=False)
            ev1.record(stream)
            torch.cuda.synchronize()
            dec = max_over_ranks(dec_steps / (ev0.elapsed_time(ev1) * 1e-3))
        if rank == 0:
            print(json.dumps({
                "metric": "prefill tokens/s (Llama-3-8B shape, bf16, 32768-token prompt), TP 1/2/4/8",
                "value": tok_s, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (Philox seed-0 N(0,0.02) weights, seed-3 uniform prompt ids)",
                "config": {"workload": f"llama3-8b-shape prefill of {T} tokens (one sequence), then {dec_steps} decode steps",
                           "model": "llama-3-8b-shape" if L == 32 else f"llama-3-8b-shape-{L}-layers",
                           "global_batch": 1, "seq_len": T, "parallelism": f"tp{world}",
                           "l2": "no flush: a step streams 16 GB of weights and writes 4 GB of K/V",
                           "flop_per_step": flop, "decode_tokens_per_s_at_32k": dec},
                "roofline": {"bound": "tensor", "achieved": achieved, "peak": bf16_peak, "unit": "TFLOP/s",
                             "frac": achieved / bf16_peak, "traffic": None,
                             "kernel": "whole prefill pass (tcgen05 GEMMs + tcgen05 causal attention)",
                             "peak_kind": peak_kind},
                "e2e": {"value": args.steps * T / wall, "unit": "tokens/s", "h2d_bytes_per_step": 4 * T,
                        "d2h_bytes_per_step": 4},
                "gpu_launches": launches, "clocks": clk.summary(),
            }), flush=True)
    elif args.workload == "serve":
        if world > 1:
            raise SystemExit("--workload serve runs on one GPU")
        B = cfg.max_batch
        n_req = 3 * B
        rng = np.random.default_rng(6)
        lens = rng.integers(128, 1025, n_req)
        news = rng.integers(32, 257, n_req)
        prompts = [I.synth_ids(200 + i, int(lens[i]), cfg.vocab_size) for i in range(n_req)]
        for _ in range(args.warmup):  # short requests through a server of their own
            with I.Server(eng) as s:
                for i in range(8):
                    s.submit(prompts[i][:64], 4)
                while s.stats()["waiting"] or s.stats()["active"]:
                    s.step()
        torch.cuda.synchronize()
        l0 = eng.launches
        with ClockSampler(local) as clk:
            with I.Server(eng) as s:
                torch.cuda.nvtx.range_push("timed")
                w0 = time.perf_counter()
                rids = [s.submit(p, int(m)) for p, m in zip(prompts, news)]
                steps = 0
                while True:
                    s.step()
                    steps += 1
                    st = s.stats()
                    if st["waiting"] == 0 and st["active"] == 0:
                        break
                wall = time.perf_counter() - w0
                torch.cuda.nvtx.range_pop()
                outs = [s.result(r) for r in rids]
        launches = eng.launches - l0
        out_tok = int(sum(o[0].size for o in outs))
        assert all(o[1] and o[2] == 0 for o in outs)
        print(json.dumps({
            "metric": "continuous-batching output tokens/s (Llama-3-8B shape, bf16, 192 requests into 64 slots)",
            "value": out_tok / wall, "unit": "tokens/s", "n_gpus": 1, "steps": steps, "warmup": args.warmup,
            "ms_per_step": wall * 1e3 / steps, "higher_is_better": True, "scaling": "none", "vs_baseline": None,
            "dtype": "bf16", "data": "synthetic (Philox seed-0 N(0,0.02) weights, per-request uniform ids, "
                                     "prompt lengths 128-1024 and 32-256 new tokens from numpy seed 6)",
            "config": {"workload": f"{n_req} requests submitted at once to inf_server over {B} slots; greedy; "
                                   "every step: admissions (prefill), one batched decode step, retirements",
                       "model": "llama-3-8b-shape" if L == 32 else f"llama-3-8b-shape-{L}-layers",
                       "global_batch": B, "prompt_tokens": int(lens.sum()), "output_tokens": out_tok,
                       "mean_decode_batch": st["batched_tokens"] / max(1, st["batched_steps"]),
                       "timing": "host wall clock: the server synchronizes with the device every step"},
            "roofline": None,
            "e2e": {"value": out_tok / wall, "unit": "tokens/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None},
            "gpu_launches": launches, "clocks": clk.summary(),
        }), flush=True)
    else:
        B = cfg.max_batch
        lens = I.synth_uniform(2, I.STREAM_CTX_LEN, B, 512, 4096)  # seed-2 context lengths
        cur = []
        t0 = time.time()
        for i in range(B):
            _, am = eng.forward(I.synth_ids(100 + i, int(lens[i]), cfg.vocab_size), 0, slot=i, want_logits=False)
            cur.append(am)
        fill_s = time.time() - t0
        slots = np.arange(B, dtype=np.uint32)
        pos = lens.astype(np.uint32).copy()
        cur = np.asarray(cur, np.uint32)
        if int(pos.max()) + args.warmup + args.steps > cfg.max_seq:
            raise SystemExit("--steps/--warmup beyond max_seq")
        for _ in range(args.warmup):
            _, cur = eng.forward_batch(slots, cur, pos)
            pos += 1
        torch.cuda.synchronize()
        barrier()
        l0, h0 = eng.launches, eng.batch_h2d_bytes
        with ClockSampler(local) as clk:
            torch.cuda.nvtx.range_push("timed")
            w0 = time.perf_counter()
            ev0.record(stream)
            for _ in range(args.steps):
                _, cur = eng.forward_batch(slots, cur, pos)
                pos += 1
            ev1.record(stream)
            torch.cuda.synchronize()
            wall = time.perf_counter() - w0
            torch.cuda.nvtx.range_pop()
        launches, h2d = eng.launches - l0, (eng.batch_h2d_bytes - h0) / args.steps
        barrier()
        ms, wall = max_over_ranks(ev0.elapsed_time(ev1)), max_over_ranks(wall)
        avg_ctx = float(lens.mean()) + args.warmup + (args.steps - 1) / 2
        # bytes of one step on one rank: every weight once + every sequence's K/V
        step_bytes = I.decode_bytes(cfg, 0) + B * (I.decode_bytes(cfg, int(avg_ctx)) - I.decode_bytes(cfg, 0))
        achieved = step_bytes / (ms / args.steps * 1e-3) / 1e9
        if rank == 0:
            print(json.dumps({
                "metric": "batched decode tokens/s (Llama-3-8B shape, bf16, 64 sequences, contexts 512-4096), TP 1/2/4/8",
                "value": B * args.steps / (ms * 1e-3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None, "dtype": "bf16",
                "data": "synthetic (Philox seed-0 N(0,0.02) weights, seed-2 context lengths, per-sequence uniform ids)",
                "config": {"workload": f"llama3-8b-shape batched greedy decode, {B} sequences, paged KV (16-token pages)",
                           "model": "llama-3-8b-shape" if L == 32 else f"llama-3-8b-shape-{L}-layers",
                           "global_batch": B, "seq_len": int(lens.max()), "parallelism": f"tp{world}",
                           "l2": "no flush: a step streams ~34 GB (> 126 MB L2)", "fill_s": fill_s,
                           "step_bytes": step_bytes},
                "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                             "frac": achieved / hbm_peak, "traffic": None,
                             "kernel": "whole batched step (tcgen05 projections, split-K attention)",
                             "peak_kind": hbm_kind},
                "e2e": {"value": B * args.steps / wall, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
                        "d2h_bytes_per_step": 4 * B},
                "gpu_launches": launches, "clocks": clk.summary(),
            }), flush=True)
    eng.close()


def run_tokenize(args):
    """Host tokenizer encode throughput (no GPU): inf_tokenizer_encode against the reference's
    own tokenizer_encode (oracle/_ref/libref_tokenizer.so, built from src/tokenizer.c) on the
    synthetic BPE tokenizer.json of the tests and a seeded corpus of space-separated words drawn
    from its vocabulary (64 documents of 64 KB).  One thread each."""
    import numpy as np

    import infb200 as I
    tok_path = os.path.join(ROOT, "tests", "golden", "tokenizer_synth.json")
    with open(tok_path, encoding="utf-8") as f:
        vocab = json.load(f)["model"]["vocab"]
    words = [p.replace("\u2581", "") for p in vocab if not p.startswith("<")]
    words = [w for w in words if w]
    rng = np.random.default_rng(5)
    zipf = np.array([1.0 / (i + 1) for i in range(len(words))])
    zipf /= zipf.sum()
    docs = []
    for _ in range(64):
        d = " ".join(words[i] for i in rng.choice(len(words), size=40000, p=zipf))
        docs.append(d.encode()[:65536].decode("utf-8", errors="ignore").rstrip(" "))
    n_bytes = sum(len(d.encode()) for d in docs)
    tok = I.Tokenizer(tok_path)
    for _ in range(args.warmup):
        n_tok = sum(tok.encode(d).size for d in docs)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for d in docs:
            tok.encode(d)
    dt = (time.perf_counter() - t0) / args.steps
    tok.close()
    line = {"metric": "tokenizer encode throughput (synthetic BPE tokenizer.json, 700 merges)", "value": round(n_tok / dt, 1),
            "unit": "tokens/s", "mb_per_s": round(n_bytes / dt / 1e6, 2), "n_gpus": 0, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(dt * 1e3, 3), "higher_is_better": True, "scaling": "none",
            "vs_baseline": None, "dtype": "utf-8", "data": "synthetic",
            "config": {"workload": f"encode {len(docs)} documents, {n_bytes} bytes, {n_tok} tokens per step"},
            "roofline": None, "gpu_launches": 0}
    ref_lib = os.path.join(ROOT, "oracle", "_ref", "libref_tokenizer.so")
    if os.path.exists(ref_lib):
        sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
        from gen_tokenizer import RefTokenizer
        ref = RefTokenizer(tok_path, ref_lib)
        t0 = time.perf_counter()
        done, n_ref = 0, 0
        while done < len(docs) and time.perf_counter() - t0 < args.cpu_budget:
            n_ref += len(ref.encode(docs[done]))
            done += 1
        rdt = time.perf_counter() - t0
        ref.close()
        line["cpu_baseline"] = {"value": round(n_ref / rdt, 1), "unit": "tokens/s", "cores": 1, "kind": "reference",
                                "sample": f"{done} of the {len(docs)} documents, reference tokenizer_encode"}
    print(json.dumps(line))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=0, help="timed steps (0: the workload's own count)")
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--skip-cpu", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--prompt", type=int, default=None, help="prompt length (profiling runs use a short one)")
    ap.add_argument("--preset", type=int, default=3, choices=[1, 2, 3, 6],
                    help="decode workload: 3 Llama-3-8B shape (the headline), 2 TinyLlama-1.1B shape, 1 tiny fp32 d288, "
                         "6 Gemma-4-E2B shape (Gemma-style decoder)")
    ap.add_argument("--layers", type=int, default=0,
                    help="decoder layers (0: the workload's own); fewer only for ncu captures of the same shapes")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "batch", "serve", "tokenize"],
                    help="decode: batch-1 decode (the headline); prefill: 32768-token prefill; batch: 64-sequence "
                         "decode; serve: continuous batching of 192 requests; tokenize: host tokenizer encode (no GPU)")
    ap.add_argument("--sample", default="", help="decode workload with sampling: temperature,top_p,top_k")
    args = ap.parse_args()
    if args.prompt is not None:
        globals()["PROMPT"] = args.prompt
    if args.steps == 0 and args.workload != "decode":  # the workload's own count
        args.steps = {"prefill": 3, "batch": 64, "serve": 1, "tokenize": 20}[args.workload]
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")

    if args.workload == "tokenize":
        return run_tokenize(args)
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        backend = "gloo" if args.impl == "reference" else "nccl"
        if backend == "nccl":
            import torch
            torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600))
    try:
        if args.impl == "reference":
            run_reference(args, rank, world)
        elif args.workload != "decode":
            run_workload(args, rank, world, dist)
        else:
            run_ours(args, rank, world, dist)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
