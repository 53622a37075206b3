"""Decode benchmark for the B200 `.gaje.flat` engine.

Workload (N=1): the Qwen2-0.5B-shaped model of BASELINE.json configs[1] --
random-init weights N(0, 0.02) written as `.gaje.flat` v2 by the synthetic
writer (Q4_0 body, tied FP32 embedding / lm_head), batch 1, a 256-token
uniform-random prompt, then greedy decode.  One "step" is one decode step
(one token).  K-WTA is off, as benchmarks/performance/bench_decode.py:158-159
sets it.

  value      decode tok/s with the model resident in HBM: K steps of the
             device-resident greedy loop (gaje_cuda_decode_greedy), timed
             with CUDA events on the model's stream, max over ranks.
  e2e        the same K steps through gaje_cuda_forward (the reference-facing
             call: host token in, host argmax out, a host sync every step).
  roofline   the lm_head GEMV (70 % of the step's bytes), from per-kernel CUDA
             events around each launch (gaje_cuda_profile_steps).
  cpu_baseline  the CPU oracle (the reference's AVX2 decode path restated in
             C++, all host threads) on a bounded sample of the same workload.

Multi-GPU (torchrun): batch-1 decode does not shard ("replicas only"): every
rank decodes its own stream on its own GPU; value = all ranks' tokens / the
slowest rank's time.

--impl reference runs the reference's CPU decode path (the C++ restatement
under oracle/, as the Rust crate cannot be built here) on the host cores.
"""
from __future__ import annotations

import argparse
import importlib
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

CONFIG_KEY = "qwen2-0.5b"
PROMPT_LEN = 256
SEED = 1234


def _pkg():
    return importlib.import_module("gaje-semantic-compression_b200")


def _model_path(cfg_key: str, seed: int) -> str:
    base = "/dev/shm" if os.path.isdir("/dev/shm") and os.access("/dev/shm", os.W_OK) else "/tmp"
    return os.path.join(base, f"gaje_bench_{cfg_key}_{seed}.flat")


def _ensure_model(g, cfg_key: str, seed: int, rank: int, dist) -> str:
    path = _model_path(cfg_key, seed)
    if rank == 0 and not os.path.exists(path):
        tmp = path + f".tmp{os.getpid()}"
        g.write_synthetic(tmp, seed=seed, **g.configs.CONFIGS[cfg_key])
        os.replace(tmp, path)
    if dist is not None:
        dist.barrier()
    return path


def _prompt(vocab: int, n: int, seed: int):
    import numpy as np

    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.samples = []
        self._stop = threading.Event()
        self._t = None

    def _run(self):
        while not self._stop.is_set():
            try:
                out = subprocess.run(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                      "--format=csv,noheader,nounits"], capture_output=True, text=True,
                                     timeout=5).stdout.strip()
                if out:
                    self.samples.append([c.strip() for c in out.split(",")])
            except Exception:
                pass
            self._stop.wait(0.2)

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(s[1]) for s in self.samples if s[1].replace(".", "").isdigit()]
        mx = [float(s[2]) for s in self.samples if s[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for s in self.samples for i in range(4)
                          if len(s) > 5 + i and s[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.samples)}


def _peaks() -> dict:
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d.get("bf16_tflops", 1590.0)),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "source": "fallback"}


def _ncu_traffic(kernel: str, cfg_key: str):
    """Per-launch DRAM bytes of a kernel from the committed ncu summary, if any."""
    p = os.path.join(REPO, "profiles", "ncu_traffic.json")
    if not os.path.exists(p):
        return None
    try:
        return json.load(open(p)).get(f"{kernel}@{cfg_key}")
    except Exception:
        return None


def cpu_oracle_decode(path: str, prompt, budget_s: float, max_tokens: int, threads: int = 0):
    """The CPU oracle decoding greedily after the prompt: (tok/s, tokens, cores)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import numpy as np
    import oracle

    oracle.build()
    if threads:
        oracle.set_threads(threads)
    cores = oracle.max_threads()
    m = oracle.OracleModel(path)
    m.set_k_wta_ratio(0.0)
    logits = None
    for i, t in enumerate(prompt):
        logits = m.forward(t, i == 0)
    tok = int(np.argmax(logits))
    n, t0 = 0, time.perf_counter()
    while n < max_tokens and (time.perf_counter() - t0) < budget_s:
        logits = m.forward(tok)
        tok = int(np.argmax(logits))
        n += 1
    dt = time.perf_counter() - t0
    return n / dt, n, cores


def run_reference(args, rank: int) -> None:
    """The reference arm: the reference's CPU decode path on the host cores."""
    if rank != 0:
        return
    g = _pkg()
    path = _ensure_model(g, args.config, SEED, 0, None)
    cfg = g.configs.CONFIGS[args.config]
    prompt = _prompt(cfg["vocab_size"], PROMPT_LEN, SEED)
    budget = max(5.0, min(120.0, 0.05 * (args.steps + args.warmup) + 20.0))
    tps, n, cores = cpu_oracle_decode(path, prompt, budget_s=budget, max_tokens=args.steps)
    line = {
        "impl": "reference",
        "metric": "decode tok/s (batch 1)",
        "value": round(tps, 3),
        "unit": "tok/s",
        "n_gpus": args.gpus,
        "steps": n,
        "warmup": args.warmup,
        "ms_per_step": round(1000.0 / tps, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded random-init weights, uniform random prompt ids",
        "config": {"workload": f"{args.config} batch-1 greedy decode after a {PROMPT_LEN}-token prompt",
                   "global_batch": 1, "prompt_len": PROMPT_LEN},
        "cpu_baseline": {"value": round(tps, 3), "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": f"{n} greedy decode steps after a {PROMPT_LEN}-token prompt "
                                   f"(time-bounded to {budget:.0f} s)"},
        "e2e": {"value": round(tps, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args, rank: int, world: int, local_rank: int, dist) -> None:
    import numpy as np
    import torch

    g = _pkg()
    torch.cuda.set_device(local_rank)
    cfg_key = args.config
    cfg = g.configs.CONFIGS[cfg_key]
    path = _ensure_model(g, cfg_key, SEED, rank, dist)
    K, W = args.steps, args.warmup
    max_ctx = PROMPT_LEN + max(K, W) + 64
    model = g.load_genomic_auto(path, device=local_rank, max_ctx=max_ctx, use_megakernel=ENGINES[args.engine])
    model.set_k_wta_ratio(0.0)
    prompt = _prompt(model.vocab_size, PROMPT_LEN, SEED + rank)
    stream = torch.cuda.ExternalStream(model.stream, device=local_rank)

    def prefill():
        model.clear_cache_py()
        last = 0
        for i, t in enumerate(prompt):
            last = model.forward_argmax(t, i == 0)
        return last

    # warm-up: graph capture, caches, clocks
    first = prefill()
    model.decode_greedy(first, W)
    first = prefill()
    torch.cuda.synchronize()

    # ---- value: device-resident loop, CUDA events on the model stream
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize()
    with ClockSampler(local_rank) as clk:
        torch.cuda.nvtx.range_push("timed_decode")
        e0.record(stream)
        toks = model.decode_greedy(first, K)
        e1.record(stream)
        e1.synchronize()
        torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    ms_max = ms
    if dist is not None:
        t = torch.tensor([ms], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_max = float(t.item())
    value = world * K / (ms_max / 1000.0)

    # ---- e2e: the reference-facing call, one host round trip per step
    first2 = prefill()
    torch.cuda.synchronize()
    if dist is not None:
        dist.barrier()
    t0 = time.perf_counter()
    tok = first2
    e2e_toks = []
    for _ in range(K):
        tok = model.forward_argmax(tok)
        e2e_toks.append(tok)
    e2e_s = time.perf_counter() - t0
    if dist is not None:
        t = torch.tensor([e2e_s], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    e2e = world * K / e2e_s
    same_stream = e2e_toks == toks

    # ---- roofline and phase profile
    peaks = _peaks()
    d, V = cfg["n_embd"], cfg["vocab_size"]
    step_ms_dev = ms / K
    sb_mean = g.configs.step_bytes(cfg, PROMPT_LEN + K // 2)
    step_gbs = sb_mean["total"] / (step_ms_dev / 1000.0) / 1e9
    prof_steps = min(K, 64)
    first3 = prefill()
    engine = int(model.info().megakernel)
    mega = engine == 1
    if engine == 2:
        # the two-exchange persistent kernel is the whole step: one launch for all K steps
        kernel = "k_decode_fused (persistent, two exchanges per block: every phase of K decode steps)"
        k_gbs, k_bytes, k_ms = step_gbs, sb_mean["total"], step_ms_dev
        launches = 1
        lm_us = 0.0
        breakdown = {"note": "one launch per K steps; no per-phase stamps in this kernel"}
        breakdown_unit = "-"
    elif mega:
        phases = model.profile_phases(first3, prof_steps, detail=True)
        # the persistent kernel is the whole step: one launch for all K steps
        kernel = "k_decode_mega (persistent: every phase of K decode steps)"
        k_gbs, k_bytes, k_ms = step_gbs, sb_mean["total"], step_ms_dev
        launches = 1
        lm_us = phases["lmhead"]
        breakdown = {k: (round(v, 2) if not isinstance(v, dict) else v) for k, v in phases.items()}
        breakdown_unit = "us per step (grid-barrier stamps, CTA 0)"
    else:
        prof = model.profile_steps(first3, prof_steps)
        kernel = "k_lmhead (final RMSNorm + f32 lm_head GEMV + argmax)"
        k_ms = prof["lmhead"][0]
        k_bytes = V * d * 4 + V * 4 + 2 * d * 4
        k_gbs = k_bytes / (k_ms / 1000.0) / 1e9
        launches = sum(n for _, n in prof.values()) * K
        lm_us = k_ms * 1000.0
        breakdown = {k: round(v[0] * 1000.0, 2) for k, v in prof.items()}
        breakdown_unit = "us per step (events around each launch)"
    lm_bytes = V * d * 4
    lm_gbs = lm_bytes / (lm_us / 1e6) / 1e9 if lm_us > 0 else None

    if rank != 0:
        return
    # ---- CPU baseline (rank 0, N=1 only): bounded oracle sample of the same workload
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        tps, n, cores = cpu_oracle_decode(path, prompt, budget_s=12.0, max_tokens=K)
        cpu = {"value": round(tps, 3), "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": f"{n} greedy decode steps after the same {PROMPT_LEN}-token prompt, "
                         f"oracle/ AVX2 restatement, {cores} OpenMP threads, 12 s budget"}
    line = {
        "metric": "decode tok/s (batch 1)",
        "value": round(value, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": W,
        "ms_per_step": round(ms_max / K, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded random-init N(0,0.02) weights quantised by the Q4_0 exporter "
                "restatement, uniform random prompt ids",
        "config": {"workload": f"{cfg_key} batch-1 greedy decode after a {PROMPT_LEN}-token prompt",
                   "global_batch": world, "prompt_len": PROMPT_LEN, "decode_steps": K,
                   "parallelism": f"replicas{world}" if world > 1 else "single",
                   "l2": "inputs larger than L2 (778 MB of weights streamed per step vs 126 MB L2)"},
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 4, "d2h_bytes_per_step": 32,
                "path": "gaje_cuda_forward (host token in, host argmax out)",
                "same_tokens_as_device_loop": same_stream},
        "roofline": {"bound": "hbm", "kernel": kernel,
                     "achieved": round(k_gbs, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(k_gbs / peaks["hbm_gbs"], 4),
                     "traffic": _ncu_traffic("k_decode_fused" if engine == 2 else "k_decode_mega" if mega else "k_lmhead",
                                            cfg_key),
                     "algorithmic_bytes": k_bytes, "ms_per_step": round(k_ms, 4),
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs, of measured)"},
        "lm_head_phase": {"us_per_step": round(lm_us, 2), "bytes": lm_bytes,
                          "achieved_gbs": round(lm_gbs, 1) if lm_gbs else None,
                          "frac": round(lm_gbs / peaks["hbm_gbs"], 4) if lm_gbs else None},
        "step_breakdown": {"unit": breakdown_unit, **breakdown},
        "gpu_launches": int(launches),
        "clocks": clk.summary(),
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


SWEEP_NK = [(896, 896), (4864, 896), (896, 4864), (8960, 1536), (1536, 8960)]
SWEEP_M = [1, 8, 64, 512]


def run_sweep(args) -> None:
    """the isolated Q4_0 dequant-GEMV/GEMM sweep.  One
    JSON line per (M, N, K): weights N(0, 0.02) quantised by the Q4_0 quantiser,
    activations N(0, 1); each launch timed alone with CUDA events after an L2
    flush (a 256 MB write), median of the timed launches.  GB/s counts the
    weight bytes N*(K/32)*20 plus activations and outputs 4*M*(K+N); TFLOP/s
    counts 2*M*N*K."""
    import numpy as np
    import torch

    g = _pkg()
    torch.cuda.set_device(0)
    peaks = _peaks()
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    reps = max(3, args.steps if args.steps != 256 else 20)
    for (N, K) in SWEEP_NK:
        rng = np.random.default_rng(N * 7 + K)
        W = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
        mat = g.Q4Matrix(np.frombuffer(g.quantize_q4_0_native(W), dtype=np.uint8), N, K)
        for M in SWEEP_M:
            x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
            y = torch.empty((M, N), dtype=torch.float32, device="cuda")
            times = []
            for it in range(reps + 3):
                flush.fill_(float(it))
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                mat.gemv(x.data_ptr(), y.data_ptr(), M)
                e1.record()
                e1.synchronize()
                if it >= 3:
                    times.append(e0.elapsed_time(e1) / 1000.0)
            t = statistics.median(times)
            wbytes = N * (K // 32) * 20
            nbytes = wbytes + 4 * M * (K + N)
            flops = 2.0 * M * N * K
            gbs, tfl = nbytes / t / 1e9, flops / t / 1e12
            bound = "hbm" if M <= 8 else "tensor"
            tc = M >= 16 and K % 64 == 0
            # the tensor-core kernel issues three bf16 MMAs per product (hi*hi, hi*lo, lo*hi):
            # its ceiling in useful TFLOP/s is a third of the measured bf16 peak
            tpeak = peaks.get("bf16_tflops", 1.0) / (3.0 if tc else 1.0)
            line = {"metric": "q4_0 dequant-GEMV/GEMM", "config": {"workload": "configs[2] sweep", "M": M, "N": N,
                                                                 "K": K, "l2": "flushed (256 MB write) before each launch"},
                    "us": round(t * 1e6, 2), "gbs": round(gbs, 1), "tflops": round(tfl, 3),
                    "kernel": ("k_gemv<G_PLAIN>" if M == 1 else
                               "k_q4_gemm_tc (tcgen05, bf16 hi/lo x3)" if tc else "k_q4_gemm_skinny<8> (CUDA cores)"),
                    "roofline": {"bound": bound,
                                 "achieved": round(gbs if bound == "hbm" else tfl, 3),
                                 "peak": round(peaks["hbm_gbs"] if bound == "hbm" else tpeak, 1),
                                 "unit": "GB/s" if bound == "hbm" else "TFLOP/s",
                                 "frac": round(gbs / peaks["hbm_gbs"] if bound == "hbm" else tfl / tpeak, 4),
                                 "peak_source": "measured (MEASURED_PEAKS.json" +
                                                (" hbm_gbs)" if bound == "hbm" else
                                                 " bf16_tflops / 3: three MMAs per product)" if tc else
                                                 " bf16_tflops)")}}
            print(json.dumps(line), flush=True)
        del mat


def lpt_assign(lengths, world: int):
    """Streams to ranks, longest prompt first onto the least-loaded rank that
    still has room (every rank gets len/world streams: the sharded head is
    collective, so every rank runs the same number of prefills and the same
    batch size).  Returns one list of stream indices per rank."""
    per = len(lengths) // world
    order = sorted(range(len(lengths)), key=lambda i: (-lengths[i], i))
    load, out = [0] * world, [[] for _ in range(world)]
    for i in order:
        r = min((r for r in range(world) if len(out[r]) < per), key=lambda r: (load[r], r))
        out[r].append(i)
        load[r] += lengths[i]
    return out


def run_batched(args, rank: int = 0, world: int = 1, local_rank: int = 0, dist=None) -> None:
    """BASELINE.json configs[3] shape (--batch B --prompt P): B streams per GPU,
    a P-token random prompt each, then K greedy decode steps (each stream fed
    its own argmax) through gaje_cuda_forward_batch.  With --serve, configs[4]:
    512 streams in all, prompt lengths uniform in [64, 1024], LPT-balanced over
    the ranks.  value = all streams' decode tokens / the decode time (CUDA
    events on the model stream, max over ranks); prefill tok/s likewise.
    Under torchrun the ranks are request-parallel and the f32 lm_head is split
    by vocabulary (gaje_cuda_load_sharded): every step all-gathers the
    residual rows and the argmax keys over NCCL."""
    import numpy as np
    import torch

    g = _pkg()
    torch.cuda.set_device(local_rank)
    cfg_key = args.config
    cfg = g.configs.CONFIGS[cfg_key]
    path = _ensure_model(g, cfg_key, SEED, rank, dist)
    K = args.steps
    pass_prefill = args.prefill_mode == "pass"
    rng = np.random.default_rng(SEED)
    if args.serve:
        n_all = 512
        lengths = [int(v) for v in rng.integers(64, 1025, n_all)]
        mine = lpt_assign(lengths, world)[rank]
        all_prompts = [rng.integers(0, cfg["vocab_size"], n) for n in lengths]
        plist = [all_prompts[i] for i in mine]
    else:
        plist = [np.random.default_rng(SEED + rank * 1000 + b).integers(0, cfg["vocab_size"], args.prompt)
                 for b in range(args.batch)]
    B = len(plist)
    P = max(len(p) for p in plist)
    max_ctx = P + K + 8
    kw = dict(device=local_rank, max_ctx=max_ctx, max_streams=B,
              max_prefill=min(P, 4096) if pass_prefill else 0)
    if world > 1:
        obj = [g.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        model = g.load_genomic_sharded(path, world, rank, obj[0], **kw)
    else:
        model = g.load_genomic_auto(path, **kw)
    model.set_k_wta_ratio(0.0)
    stream = torch.cuda.ExternalStream(model.stream, device=local_rank)
    sids = list(range(B))
    # warm-up (also the prefill timing)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if dist is not None:
        dist.barrier()
    e0.record(stream)
    am = None
    if pass_prefill:  # each stream's prompt in one pass (tensor-core GEMMs + causal attention)
        am = [model.prefill(sid, [int(t) for t in plist[sid]]) for sid in sids]
    else:  # token by token as batched steps (equal prompt lengths only)
        for t in range(P):
            am = model.forward_batch(sids, [int(plist[b][t]) for b in sids])
    e1.record(stream)
    e1.synchronize()
    pre_ms = e0.elapsed_time(e1)
    with ClockSampler(local_rank) as clk:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        toks = [int(v) for v in am]
        for _ in range(K):
            toks = [int(v) for v in model.forward_batch(sids, toks)]
        e1.record(stream)
        e1.synchronize()
    dec_ms = e0.elapsed_time(e1)
    dec_max, pre_max = dec_ms, pre_ms
    if dist is not None:
        tt = torch.tensor([dec_ms, pre_ms], dtype=torch.float64, device=f"cuda:{local_rank}")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        dec_max, pre_max = float(tt[0].item()), float(tt[1].item())
    if rank != 0:
        return
    peaks = _peaks()
    mean_p = sum(len(p) for p in plist) / B
    sb = g.configs.step_bytes(cfg, int(mean_p + K // 2))
    # per rank and step: the body once, this rank's share of the lm_head, every local stream's KV
    lm_share = sb["lm_head"] * (1.0 - 1.0 / world) if world > 1 else 0.0
    step_bytes = sb["total"] - sb["kv"] - lm_share + B * sb["kv"]
    step_s = dec_max / 1000.0 / K
    n_prompt_tokens = sum(len(p) for p in plist)
    workload = (f"{cfg_key} batched serving: 512 streams, prompts uniform in [64, 1024] (LPT over {world} ranks, "
                f"{B} per rank), {K} greedy steps" if args.serve else
                f"{cfg_key} batched greedy decode, {B} streams per GPU after a {P}-token prompt each")
    line = {
        "metric": "decode tok/s (batched)",
        "value": round(world * B * K / (dec_max / 1000.0), 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": P,
        "ms_per_step": round(dec_max / K, 4),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded random-init N(0,0.02) weights quantised by the Q4_0 exporter restatement, "
                "uniform random prompt ids",
        "config": {"workload": workload, "global_batch": world * B, "prompt_len": P if not args.serve else "64-1024",
                   "decode_steps": K,
                   "parallelism": (f"request-parallel x{world}, lm_head vocab-sharded over NCCL" if world > 1
                                   else "single"),
                   "l2": "inputs larger than L2"},
        "prefill": {"value": round(world * n_prompt_tokens / (pre_max / 1000.0), 2), "unit": "tok/s",
                    "how": ("gaje_cuda_prefill: each stream's prompt in one pass (tcgen05 GEMMs over the prompt "
                            "rows, causal attention kernel); the reference prefills token by token"
                            if pass_prefill else "token by token as batched steps (as the reference)")},
        "e2e": {"value": round(world * B * K / (dec_max / 1000.0), 2), "unit": "tok/s",
                "h2d_bytes_per_step": 12 * B, "d2h_bytes_per_step": 4 * B + 32,
                "path": "gaje_cuda_forward_batch (host tokens in, host argmax out, a sync per step)"},
        "roofline": {"bound": "hbm", "kernel": "batched step (Q4 GEMMs + lm_head for B vectors), bytes per rank",
                     "achieved": round(step_bytes / step_s / 1e9, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(step_bytes / step_s / 1e9 / peaks["hbm_gbs"], 4), "traffic": None,
                     "algorithmic_bytes": step_bytes,
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs, of measured)"},
        "gpu_launches": (5 * cfg["n_blocks"] + 1 + (B + (8 if B <= 8 else 16) - 1) // (8 if B <= 8 else 16)) * K,
        "clocks": clk.summary(),
    }
    print(json.dumps(line), flush=True)


# batch-1 engines (the load option use_megakernel): the two-exchange fused
# kernel (default), the five-exchange persistent kernel, a kernel per phase
ENGINES = {"fused": 1, "mega": 2, "phase": 0}


def run_ncu_case(args) -> None:
    """Two launches of the persistent kernel on one GPU: PROMPT_LEN greedy steps
    (the context a bench step sees), then args.steps steps, the launch a
    profiler captures.  No timing: numbers taken under a profiler are not bench
    values."""
    import torch

    g = _pkg()
    torch.cuda.set_device(0)
    path = _ensure_model(g, args.config, SEED, 0, None)
    model = g.load_genomic_auto(path, device=0, max_ctx=PROMPT_LEN + args.steps + 64,
                                use_megakernel=ENGINES[args.engine])
    model.set_k_wta_ratio(0.0)
    model.clear_cache_py()
    t = model.decode_greedy(5, PROMPT_LEN)[-1]
    toks = model.decode_greedy(t, args.steps)
    print(json.dumps({"ncu_case": args.config, "context": PROMPT_LEN, "steps": args.steps,
                      "last_token": int(toks[-1])}), flush=True)


def run_ncu_batch(args) -> None:
    """Profiling case for the batched kernels (no timing): --ncu-case with
    --batch B runs args.steps batched greedy steps of B streams, from empty
    caches unless --context P prefills each stream with P tokens first; with
    --prompt-only P it prefills two streams with P-token prompts instead."""
    import numpy as np
    import torch

    g = _pkg()
    torch.cuda.set_device(0)
    path = _ensure_model(g, args.config, SEED, 0, None)
    rng = np.random.default_rng(SEED)
    if args.prompt_only > 0:
        P = args.prompt_only
        model = g.load_genomic_auto(path, device=0, max_ctx=P + 16, max_streams=2, max_prefill=P)
        model.set_k_wta_ratio(0.0)
        out = [int(model.prefill(s, [int(t) for t in rng.integers(0, model.vocab_size, P)])) for s in range(2)]
        print(json.dumps({"ncu_case": args.config, "prefill": P, "streams": 2, "argmax": out}), flush=True)
        return
    B, P = args.batch, args.context
    model = g.load_genomic_auto(path, device=0, max_ctx=P + args.steps + 16, max_streams=B,
                                max_prefill=max(P, 16))
    model.set_k_wta_ratio(0.0)
    toks = [int(t) for t in rng.integers(0, model.vocab_size, B)]
    if P > 0:  # each stream's cache filled by one prefill pass first
        toks = [int(model.prefill(s, [int(t) for t in rng.integers(0, model.vocab_size, P)])) for s in range(B)]
    for _ in range(args.steps):
        toks = [int(t) for t in model.forward_batch(list(range(B)), toks)]
    print(json.dumps({"ncu_case": args.config, "streams": B, "steps": args.steps, "tokens": toks[:4]}), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", default=CONFIG_KEY)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0,
                    help="batched decode of this many streams per GPU (configs[3]/[4] shape) instead of batch 1")
    ap.add_argument("--prompt", type=int, default=PROMPT_LEN, help="prompt tokens per stream (--batch)")
    ap.add_argument("--serve", action="store_true",
                    help="configs[4]: 512 streams over all ranks, prompts uniform in [64, 1024], LPT-balanced")
    ap.add_argument("--prefill-mode", choices=["pass", "steps"], default="pass",
                    help="--batch prompts: one gaje_cuda_prefill pass per stream, or token-by-token batched steps")
    ap.add_argument("--sweep", action="store_true",
                    help="the isolated Q4_0 GEMV/GEMM sweep of configs[2] instead of the decode benchmark")
    ap.add_argument("--engine", choices=sorted(ENGINES), default="fused",
                    help="batch-1 engine: fused (two exchanges per block, default), mega (five), phase")
    ap.add_argument("--context", type=int, default=0,
                    help="with --ncu-case --batch B: prefill each stream with this many tokens first")
    ap.add_argument("--prompt-only", type=int, default=0,
                    help="with --ncu-case: prefill two streams with prompts of this many tokens (profiling)")
    ap.add_argument("--ncu-case", action="store_true",
                    help="the small profiling case: one launch filling the prompt's positions, then one "
                         "launch of --steps decode steps (capture it with -k regex:k_decode_fused -s 1 -c 1); "
                         "with --batch B: --steps batched steps of B streams from empty caches; with "
                         "--prompt-only P: two P-token prefills")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if args.ncu_case:
        if args.batch > 0 or args.prompt_only > 0:
            run_ncu_batch(args)
        else:
            run_ncu_case(args)
        return
    if args.sweep:
        run_sweep(args)
        return
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist

        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                 device_id=torch.device(f"cuda:{local_rank}"))
        dist = tdist
    try:
        if args.batch > 0 or args.serve:
            run_batched(args, rank, world, local_rank, dist)
        else:
            run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
