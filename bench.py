#!/usr/bin/env python
"""bench.py -- audio-seconds per second of the Ming-3.0-tts-0.5B per-step loop on B200.

Workload (the serving configuration, per GPU): R = 64 concurrent requests, each a 128-token prompt of
uniform random ids in [0, 151936) (per-request seeds), prefill, then generation steps with CFG 2.0
and N(0,1) noise; random-init weights (seed 1). One bench step = one engine step over all R
requests: LLM token (24 layers, R rows), stop head, 10 Euler steps of the CFG flow DiT (6R rows),
the aggregator DiT (2R rows), VAE fc1, and the VAE decode of latent n-2 (24-layer windowed Qwen,
4R rows, head, ISTFT, overlap-add). Each step yields 0.08 s of audio per request.

  value     device-timed throughput of K steps (CUDA events on the engine stream, inputs resident),
            whole job = all ranks' requests / max-over-ranks time (weak scaling: R per GPU).
  e2e       mt_engine_generate from host memory (ids + noise H2D, prefill, steps, flush, every PCM
            chunk and stop logit D2H), wall time of the call, max over ranks.
  roofline  the dominant kernel (tcgen05 GEMM at the flow-DiT ff1 shape) timed alone with events.
  gemv      the decode GEMV alone: M=2, W[4864x896] (and the down proj) over a >= 1 GiB pool.
  single_request  the reference's published shape (one request, 174-token prompt): prefill ms,
            ms per step, audio-s/s and p50 time to first audio.
  cpu_baseline / --impl reference: the CPU oracle (C restatement of the reference's kernels and
            loop, OpenMP) on a bounded sample: one request, full model, timed per step.

Multi-GPU: launched by torchrun, one rank per GPU, independent replicas (no collective on the data
path); torch.distributed is used only for barriers and the max-over-ranks of the timings.
"""
from __future__ import annotations

import argparse
import ctypes
import importlib.util
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
AUDIO_PER_STEP = 0.08  # 3528 samples at 44.1 kHz (Text/MingRequest.swift:104)


def load_package():
    name = "mingtts_b200"
    if name in sys.modules:
        return sys.modules[name]
    pkg = os.path.join(ROOT, "ming-tts_b200")
    spec = importlib.util.spec_from_file_location(name, os.path.join(pkg, "__init__.py"), submodule_search_locations=[pkg])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d.get("hbm_gbs", 6650.0), d.get("bf16_tflops", 1590.0), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.device)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            out, _ = self.proc.communicate(timeout=10)
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for name, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx or None,
                "reasons": sorted(reasons), "samples": len(sm)}


def dist_setup(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        import torch.distributed as dist
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))
    return rank, world, local


def dist_max(value: float, world: int, device: str = "cuda") -> float:
    """Maximum of `value` over the ranks (the timing rule: a multi-GPU time is the slowest rank's)."""
    if world == 1:
        return value
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world: int, device: str = "cuda"):
    import torch
    if device == "cuda":
        torch.cuda.synchronize()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def rank_requests(rank: int, per_rank: int):
    """Requests of one replica: rank r serves global requests [r * per_rank, (r + 1) * per_rank), so
    every rank draws different prompts and noise (seeds follow the global request index)."""
    return rank * per_rank, per_rank


def request_inputs(mt, cfg, requests, prompt, steps, first_request):
    """Per-request prompt ids (uniform over the vocabulary) and N(0,1) noise, seeded by request index."""
    import numpy as np
    ids = np.stack([np.random.default_rng(1000 + first_request + r).integers(0, cfg.vocab, prompt, dtype=np.int32)
                    for r in range(requests)])
    noise = np.empty((requests, steps, cfg.latent_dim), np.float32)
    for r in range(requests):
        mt.lib().mt_gaussian_noise_host(noise[r].ctypes.data, noise[r].size, 3 + first_request + r)
    return ids, noise


# ------------------------------------------------------------------------------------------------
# Kernel-level measurements
# ------------------------------------------------------------------------------------------------
def time_gemm(mt, ctx, m, n, k, flags, iters=100, rounds=3):
    """Average duration of the tcgen05 GEMM at one shape: `iters` launches replayed from a CUDA
    graph (so host launch cost is not measured), CUDA events, best of `rounds`."""
    import torch
    g = torch.Generator(device="cuda").manual_seed(0)
    xh = (torch.randn(m, k, device="cuda", generator=g)).to(torch.bfloat16)
    xl = (torch.randn(m, k, device="cuda", generator=g) * 2 ** -9).to(torch.bfloat16)
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, device="cuda", generator=g) * 0.02).to(torch.bfloat16)
    yh = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    yl = torch.empty_like(yh)
    args = (xh, xl, k, m, w, None, b, n, k, None, 0, yh, yl, n, flags | mt.BIAS)
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for _ in range(3):
            ctx.call("linear_split", *args)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for _ in range(iters):
                ctx.call("linear_split", *args)
        graph.replay()
        torch.cuda.synchronize()
        best = None
        for _ in range(rounds):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            graph.replay()
            e.record(stream)
            e.synchronize()
            t = s.elapsed_time(e) * 1e-3 / iters
            best = t if best is None else min(best, t)
    ctx.check()
    return best


def time_gemv_pool(mt, ctx, n, k, m=2, pool_bytes=1 << 30, rounds=3):
    """Decode GEMV over a rotating pool of distinct weight copies (no cache serves a weight twice),
    replayed from a CUDA graph. Returns seconds per launch."""
    import torch
    copies = max(1, pool_bytes // (n * k * 2))
    pool = (torch.randn(copies, n, k, device="cuda") * 0.02).to(torch.bfloat16)
    x = torch.randn(m, k, device="cuda")
    y = torch.empty(m, n, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        for i in range(3):
            ctx.call("linear", x, k, m, pool[i], None, None, n, k, y, n, 0)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(copies):
                ctx.call("linear", x, k, m, pool[i], None, None, n, k, y, n, 0)
        graph.replay()
        torch.cuda.synchronize()
        best = None
        for _ in range(rounds):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record(stream)
            graph.replay()
            e.record(stream)
            e.synchronize()
            t = s.elapsed_time(e) * 1e-3 / copies
            best = t if best is None else min(best, t)
    del graph, pool
    torch.cuda.empty_cache()
    return best, copies


# ------------------------------------------------------------------------------------------------
# CPU oracle runs (baseline)
# ------------------------------------------------------------------------------------------------
def time_to_first_audio(eng, requests, prompt, noise_host, ids_host, steps, world, reps=7):
    """p50 time to the first non-empty PCM chunk through mt_engine_generate_stream (host ids and noise,
    prefill, steps 0-2; the first chunk follows step 2). All requests of the batch receive their
    first chunk in the same callback, so the batch's time is every request's time; the p50 is over
    repeated calls and the max over ranks."""
    samples = []
    for _ in range(reps):
        t_first = []
        t0 = time.perf_counter()

        def on_chunk(index, pcm):
            if not t_first:
                t_first.append(time.perf_counter())
            return 0

        eng.generate_stream(requests, prompt, noise_host, steps, on_chunk, ids_host=ids_host)
        samples.append(t_first[0] - t0)
    return dist_max(statistics.median(samples), world), reps


def single_request(mt, ctx, model, cfg, first_request, world, prompt=174, steps=50, warmup=5, reps=5):
    """The reference's own benchmark shape (.claude/skills/verify/features/bench.md:25: one request, a
    174-token prompt):
    prefill time and step time with device-resident inputs (CUDA events on the launching stream,
    medians over `reps`), audio-s/s of the steps, and the p50 time to first audio through the
    streaming host API. One request runs its LLM and aggregator rows on the CUDA-core GEMV."""
    import numpy as np
    import torch
    ids, noise = request_inputs(mt, cfg, 1, prompt, warmup + steps, first_request)
    eng = mt.Engine(ctx, model, 1, prompt, warmup + steps)
    ids_d, noise_d = torch.from_numpy(ids).cuda(), torch.from_numpy(noise).cuda()
    stream = torch.cuda.current_stream()
    pre, per_step = [], []
    for _ in range(reps):
        a, b, c = (torch.cuda.Event(enable_timing=True) for _ in range(3))
        eng.begin(1, prompt, token_ids=ids_d, noise=noise_d, steps=warmup + steps)
        a.record(stream)
        eng.prefill()
        b.record(stream)
        for _ in range(warmup):
            eng.step()
        b2 = torch.cuda.Event(enable_timing=True)
        b2.record(stream)
        for _ in range(steps):
            eng.step()
        c.record(stream)
        c.synchronize()
        pre.append(a.elapsed_time(b))
        per_step.append(b2.elapsed_time(c) / steps)
    ctx.check()
    ids_h = torch.from_numpy(ids).pin_memory().numpy()
    noise_h = torch.from_numpy(np.ascontiguousarray(noise)).pin_memory().numpy()
    ttfa, calls = time_to_first_audio(eng, 1, prompt, noise_h, ids_h, 12, world)
    eng.close()
    prefill_ms = dist_max(statistics.median(pre), world)
    step_ms = dist_max(statistics.median(per_step), world)
    return {"prompt_tokens": prompt, "requests": 1, "prefill_ms": round(prefill_ms, 3),
            "ms_per_step": round(step_ms, 3), "audio_s_per_s": round(AUDIO_PER_STEP / (step_ms * 1e-3), 2),
            "ttfa_ms_p50": round(ttfa * 1e3, 2), "ttfa_calls": calls,
            "reference_published": {"prefill_ms": 26.0, "ms_per_step_gpu": 15.01, "ttfa_ms": 65,
                                    "hardware": "Apple M-series GPU (.claude/skills/verify/features/bench.md:25)"}}


def host_model(mt, oracle, cfg, seed):
    import numpy as np
    tensors = mt.tensor_table(cfg, seed)
    arena = np.zeros(mt.lib().mt_model_arena_bytes(ctypes.byref(cfg), 1), np.uint8)
    for t in tensors:
        if t.dtype == mt.MT_DTYPE_BF16:
            v = arena[t.offset:t.offset + 2 * t.numel].view(np.uint16)
            v[:] = 0x3F80 if t.init == 1 else oracle.randn_bf16(t.numel, t.seed, t.std)
        else:
            v = arena[t.offset:t.offset + 4 * t.numel].view(np.float32)
            if t.init == 0:
                v[:] = oracle.bf16_to_f32(oracle.randn_bf16(t.numel, t.seed, t.std))
            elif t.init == 2:
                v[:] = (1.0 / np.power(10000.0, 2 * np.arange(t.numel) / 64.0)).astype(np.float32)
            elif t.init == 3:
                v[:] = (0.5 - 0.5 * np.cos(2 * np.pi * np.arange(t.numel) / t.numel)).astype(np.float32)
    w, keep = mt.weights_struct(cfg, arena.ctypes.data, tensors)
    return arena, tensors, w, keep


def use_all_host_threads() -> int:
    """The CPU legs use every host core. torchrun sets OMP_NUM_THREADS=1 for its workers, and the
    OpenMP runtime may already be initialised by the time the oracle runs, so set both the
    environment and the running runtime's thread count."""
    n = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(n)
    except OSError:
        pass
    return n


def cpu_oracle_rate(mt, cfg, prompt, warm_steps, timed_steps):
    """Times the oracle's generation loop (one request) per step; returns (audio-s/s, seconds, threads)."""
    import numpy as np
    sys.path.insert(0, ROOT)
    import oracle
    arena, tensors, w, keep = host_model(mt, oracle, cfg, seed=1)
    steps = warm_steps + timed_steps
    ids, noise = request_inputs(mt, cfg, 1, prompt, steps, 0)
    off = {t.name.decode(): t.offset for t in tensors}["model.model.embed_tokens.weight"]
    table = arena[off:off + cfg.vocab * cfg.llm.hidden * 2].view(np.uint16).reshape(cfg.vocab, cfg.llm.hidden)
    embeds = np.ascontiguousarray(oracle.bf16_to_f32(table[ids[0]]))
    io = oracle.GenerateIO()
    stamps = np.zeros(steps, np.float64)
    io.prompt_rows, io.embeds, io.steps, io.cfg, io.obey_stop = prompt, embeds.ctypes.data, steps, 2.0, 0
    n0 = np.ascontiguousarray(noise[0])
    io.noise = n0.ctypes.data
    io.step_seconds = stamps.ctypes.data
    threads = use_all_host_threads()
    oracle.lib().or_generate(ctypes.addressof(cfg), ctypes.addressof(w), ctypes.byref(io))
    secs = stamps[steps - 1] - stamps[warm_steps - 1]
    return timed_steps * AUDIO_PER_STEP / secs, secs, threads


# ------------------------------------------------------------------------------------------------
def run_reference(args, rank, world):
    if rank != 0:
        return
    use_all_host_threads()
    mt = load_package()
    cfg = mt.default_config()
    # One step of this arm = one generation step of one request on the host cores (a bounded sample
    # of the per-GPU workload: ~0.3 s on 16 cores); W untimed and K timed steps, K capped so the
    # positions fit the 512-entry cache.
    warm = max(1, args.warmup)
    timed = max(1, min(args.steps, cfg.llm_capacity - args.cpu_prompt - warm - 1))
    rate, secs, threads = cpu_oracle_rate(mt, cfg, args.cpu_prompt, warm, timed)
    sample = (f"1 request, {args.cpu_prompt}-token prompt, {warm} untimed + {timed} timed steps of the full "
              f"model (CPU oracle: C restatement of the reference kernels, fp64 dot products, OpenMP)")
    line = {"impl": "reference", "metric": METRIC, "value": round(rate, 5), "unit": "audio-s/s", "n_gpus": args.gpus,
            "steps": timed, "warmup": warm, "ms_per_step": round(secs / timed * 1e3, 2),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: random-init weights seed 1, uniform prompt ids, N(0,1) noise",
            "config": config_block(args),
            "cpu_baseline": {"value": round(rate, 5), "unit": "audio-s/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(rate, 5), "unit": "audio-s/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


METRIC = "audio-sec/sec of the Ming-3.0-tts-0.5B step loop (config 5 serving, per-GPU replicas)"
# DRAM bytes (read + write) of one launch of the roofline GEMM, from the ncu capture summarised in
# profiles/gemm_tc_flow_ff1_m384_n4096_k1024.md (dram__bytes_read.sum + dram__bytes_write.sum).
ROOFLINE_TRAFFIC_BYTES = 10_003_456


def config_block(args):
    return {"workload": (f"config5 serving step: {args.requests} requests/GPU, {args.prompt}-token prompts, "
                         "1 step = LLM token + stop head + 10-step CFG flow DiT + aggregator + VAE decode of one "
                         "latent per request (0.08 s audio each)"),
            "model": "Ming-3.0-tts-0.5B dims (LLM 896x24, flow/agg DiT 1024x8, VAE decoder 896x24 window 65)",
            "requests_per_gpu": args.requests, "prompt_tokens": args.prompt, "global_batch": args.requests * args.gpus,
            "parallelism": f"replicas x{args.gpus} (no data-path collective)",
            "l2": "inputs larger than L2: ~3.6 GB of weights streamed per step"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--prompt", type=int, default=128)
    ap.add_argument("--e2e-steps", type=int, default=64)
    ap.add_argument("--cpu-steps", type=int, default=3)
    ap.add_argument("--cpu-prompt", type=int, default=16)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-graphs", action="store_true")
    ap.add_argument("--groups", type=int, default=0,
                    help="request groups stepped concurrently (0 = the engine's automatic choice)")
    ap.add_argument("--gemm", type=str, default="",
                    help="M,N,K[,flags]: time one tensor-core GEMM shape alone and exit (for focused profiling)")
    ap.add_argument("--gemv", type=str, default="",
                    help="N,K[,M]: time the CUDA-core GEMV over a >= 1 GiB weight pool alone and exit (for focused profiling)")
    ap.add_argument("--profile", action="store_true",
                    help="prefill, warm-up and timed steps only (for a profiler's launch list); prints ms/step")
    args = ap.parse_args()
    assert args.warmup >= 3, "at least 3 warm-up steps"
    if args.impl == "reference":
        # The CPU reference arm needs no process group: rank 0 times the oracle, the others exit.
        run_reference(args, int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")))
        return
    rank, world, local = dist_setup(args)
    if args.gemm:
        mt = load_package()
        ctx = mt.Context(local)
        f = [int(v) for v in args.gemm.split(",")]
        m, n, k, flags = f[0], f[1], f[2], (f[3] if len(f) > 3 else 0)
        t = time_gemm(mt, ctx, m, n, k, flags, iters=20, rounds=1)
        print(json.dumps({"gemm": [m, n, k, flags], "us": round(t * 1e6, 2),
                          "tflops": round(2.0 * m * n * k / t / 1e12, 1)}), flush=True)
        return
    if args.gemv:
        mt = load_package()
        ctx = mt.Context(local)
        f = [int(v) for v in args.gemv.split(",")]
        n, k, m = f[0], f[1], (f[2] if len(f) > 2 else 2)
        t, copies = time_gemv_pool(mt, ctx, n, k, m=m)
        nbytes = n * k * 2 + m * k * 4 + m * n * 4
        print(json.dumps({"gemv": [m, n, k], "us": round(t * 1e6, 3), "gbs": round(nbytes / t / 1e9, 1),
                          "pool_copies": copies}), flush=True)
        return

    import numpy as np
    import torch
    mt = load_package()
    ctx = mt.Context(local)
    cfg = mt.default_config()
    model = mt.Model(ctx, cfg, seed=1, with_embeddings=True)
    R, T = args.requests, args.prompt
    total_steps = args.warmup + args.steps
    assert T + total_steps <= cfg.llm_capacity, f"prompt + steps must fit the {cfg.llm_capacity}-position cache"
    eng = mt.Engine(ctx, model, R, T, max(total_steps, args.e2e_steps), use_graphs=not args.no_graphs,
                    groups=args.groups)
    first, _ = rank_requests(rank, R)
    ids, noise = request_inputs(mt, cfg, R, T, total_steps, first)
    ids_d, noise_d = torch.from_numpy(ids).cuda(), torch.from_numpy(noise).cuda()
    stream = torch.cuda.current_stream()

    # ---- device-timed steps (inputs resident) ----
    eng.begin(R, T, token_ids=ids_d, noise=noise_d, steps=total_steps)
    eng.prefill()
    for _ in range(args.warmup):
        eng.step()
    barrier(world)
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kernels = 0
    if args.profile:
        torch.cuda.cudart().cudaProfilerStart()  # a profiler started with --profile-from-start off sees only these steps
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(args.steps):
            eng.step()
            kernels += mt.lib().mt_engine_step_kernels(eng.handle)
        end.record(stream)
        end.synchronize()
    if args.profile:
        torch.cuda.cudart().cudaProfilerStop()
    ctx.check()
    t_local = start.elapsed_time(end) * 1e-3
    t_max = dist_max(t_local, world)
    value = world * R * args.steps * AUDIO_PER_STEP / t_max
    if args.profile:
        if rank == 0:
            print(json.dumps({"profile": True, "ms_per_step": round(t_max / args.steps * 1e3, 3),
                              "kernels_per_step": kernels // max(args.steps, 1)}), flush=True)
        return

    # ---- per-stage split of one eager step (reference StepRecorder semantics) ----
    eng.stage_timing(True)
    eng.begin(R, T, token_ids=ids_d, noise=noise_d, steps=min(total_steps, 8))
    eng.prefill()
    stage_samples = []
    for n in range(min(total_steps, 8)):
        eng.step()
        if n >= 3:
            torch.cuda.synchronize()
            stage_samples.append(eng.stage_ms())
    eng.stage_timing(False)
    stage_ms = [round(statistics.median(x[i] for x in stage_samples), 3) for i in range(4)]

    # ---- end to end through the host API ----
    E = args.e2e_steps
    ids_h = torch.from_numpy(ids).pin_memory().numpy()
    noise_e = torch.from_numpy(np.ascontiguousarray(noise[:, :E] if E <= total_steps else
                                                    np.resize(noise, (R, E, cfg.latent_dim)))).pin_memory().numpy()
    eng.generate(R, T, noise_e, min(E, 8), ids_host=ids_h)  # warm the host path
    barrier(world)
    t0 = time.perf_counter()
    pcm, stop = eng.generate(R, T, noise_e, E, ids_host=ids_h)
    t_e2e = dist_max(time.perf_counter() - t0, world)
    e2e_value = world * R * (pcm.shape[1] / (4 * cfg.hop)) * AUDIO_PER_STEP / t_e2e
    max_chunk = 4 * cfg.hop + (cfg.nfft - cfg.hop) // 2
    h2d = (ids_h.nbytes + noise_e.nbytes) / E
    d2h = (R * max_chunk * 4 * (E + 0.0) + R * 2 * 4 * E) / E
    ttfa = time_to_first_audio(eng, R, T, noise_e, ids_h, min(E, 12), world)
    single = single_request(mt, ctx, model, cfg, first + R, world)

    # ---- kernel roofline: the tcgen05 GEMM at the flow-DiT ff1 shape; decode GEMV (config 1) ----
    hbm_peak, bf16_peak, peak_kind = peaks()
    M, N, K = 6 * R, cfg.flow.ff, cfg.flow.hidden
    t_gemm = time_gemm(mt, ctx, M, N, K, mt.GELU)
    flops = 2.0 * M * N * K
    achieved = flops / t_gemm / 1e12
    t_gv, copies = time_gemv_pool(mt, ctx, 4864, 896)
    gv_bytes = 4864 * 896 * 2 + 2 * 896 * 4 + 2 * 4864 * 4
    t_gv_down, _ = time_gemv_pool(mt, ctx, 896, 4864)
    gv_down_bytes = 896 * 4864 * 2 + 2 * 4864 * 4 + 2 * 896 * 4

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        rate, secs, threads = cpu_oracle_rate(mt, cfg, args.cpu_prompt, 1, args.cpu_steps)
        cpu = {"value": round(rate, 5), "unit": "audio-s/s", "cores": threads, "kind": "port",
               "sample": f"1 request, {args.cpu_prompt}-token prompt, 1 untimed + {args.cpu_steps} timed steps of the "
                         "full model on the CPU oracle (C restatement, fp64 dot products, OpenMP)"}

    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "audio-s/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(t_max / args.steps * 1e3, 3), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None,
                "dtype": "f32 (bf16 weights; tensor-core GEMMs on bf16 hi+lo activation pairs, fp32 accumulate)",
                "data": "synthetic: random-init weights seed 1, uniform prompt ids per request seed, N(0,1) noise",
                "config": config_block(args),
                "e2e": {"value": round(e2e_value, 2), "unit": "audio-s/s", "steps": E,
                        "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                        "includes": "ids+noise H2D, prefill, steps, flush, PCM+stop D2H (mt_engine_generate)"},
                "ttfa_ms": {"p50": round(ttfa[0] * 1e3, 2), "calls": ttfa[1], "requests_per_call": R,
                            "includes": "ids+noise H2D, prefill of all requests, steps 0-2, first PCM chunk D2H "
                                        "(mt_engine_generate_stream callback)"},
                "roofline": {"kernel": "gemm_tc_kernel (flow DiT ff1, GELU, hi/lo out)",
                             "shape": f"M={M} N={N} K={K}", "bound": "tensor", "achieved": round(achieved, 1),
                             "peak": bf16_peak, "unit": "TFLOP/s", "frac": round(achieved / bf16_peak, 4),
                             "peak_kind": f"{peak_kind} bf16 dense (burst)",
                             "note": "algorithmic 2MNK; the fp32-faithful hi+lo split issues 2 bf16 MMAs per product",
                             "ms_per_launch": round(t_gemm * 1e3, 4), "traffic": ROOFLINE_TRAFFIC_BYTES,
                             "traffic_unit": "bytes per launch (ncu dram read+write)"},
                "gemv": {"shape": "config 1: M=2 W[4864x896] bf16, fp32 x/y", "gbs": round(gv_bytes / t_gv / 1e9, 1),
                         "frac": round(gv_bytes / t_gv / 1e9 / hbm_peak, 4), "us": round(t_gv * 1e6, 3),
                         "down_proj_gbs": round(gv_down_bytes / t_gv_down / 1e9, 1),
                         "pool": f"{copies} distinct weight copies (>= 1 GiB), graph replay",
                         "peak_gbs": hbm_peak, "peak_kind": peak_kind},
                "single_request": single,
                "stages_ms": {"llm": stage_ms[0], "flow": stage_ms[1], "agg": stage_ms[2], "vae_concurrent": stage_ms[3],
                              "note": "one eager step, events per stage; the VAE decode runs on a second stream"},
                "gpu_launches": kernels, "clocks": clocks.summary()}
        if cpu:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    eng.close()
    model.close()
    ctx.close()
    barrier(world)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
