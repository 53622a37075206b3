"""Decode benchmark for the B200 `.gaje.flat` engine.

Workload, plain `python bench.py` (N=1): the Qwen2-0.5B-shaped model --
random-init weights N(0, 0.02) written as `.gaje.flat` v2 by the
synthetic writer (Q4_0 body, tied FP32 embedding / lm_head), batch 1, a
256-token uniform-random prompt, then greedy decode.  One "step" is one
decode step (one token).  K-WTA is off, as
benchmarks/performance/bench_decode.py:158-159 sets it.

  value      decode tok/s with the model resident in HBM: K steps of the
             device-resident greedy loop (gaje_cuda_decode_greedy), timed
             with CUDA events on the model's stream.
  e2e        the same K steps through gaje_cuda_forward (the reference-facing
             call: host token in, host argmax out, a host sync every step).
  roofline   the persistent decode kernel (the whole step): algorithmic bytes
             per step / the CUDA-event step time.
  cpu_baseline  the CPU oracle (the reference's AVX2 decode path restated in
             C++, all host threads) on a bounded sample of the same workload.
  serving    the multi-GPU workload (below) at N=1, for the scaling curve.

Under torchrun (any N, 1 included) the workload is batched serving on the
Qwen2.5-1.5B shape: 512 streams in all, prompt lengths uniform in [64, 1024],
LPT-balanced over the ranks, each prompt prefilled in one pass, then K
batched greedy steps (K <= 256) through gaje_cuda_forward_batch.  Ranks are
request-parallel and the f32 lm_head is split by vocabulary over NCCL
(gaje_cuda_load_sharded); the total work is fixed, so the scaling is strong.
Batch-1 decode does not shard (one GPU per stream: replicas only).

--impl reference runs the reference's CPU decode path (the C++ restatement
under oracle/, as the Rust crate cannot be built here) on the host cores, on
the same workload, without loading this repository's library: its model file
comes from the oracle's quantiser and tests/golden/flat_numpy.py.
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


def _configs():
    """The model shapes (configs.py), loaded by path: importing the package
    would load the product library, which the reference arm must not."""
    import importlib.util

    spec = importlib.util.spec_from_file_location(
        "gaje_bench_configs", os.path.join(REPO, "gaje-semantic-compression_b200", "configs.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


SERVE_CONFIG = "qwen2.5-1.5b"
SERVE_STREAMS = 512


def _under_torchrun() -> bool:
    return "WORLD_SIZE" in os.environ and "LOCAL_RANK" in os.environ


def _batch1_config(cfg_key: str, K: int, world: int) -> dict:
    return {"workload": f"{cfg_key} batch-1 greedy decode after a {PROMPT_LEN}-token prompt",
            "global_batch": world, "prompt_len": PROMPT_LEN, "decode_steps": K,
            "parallelism": f"replicas{world}" if world > 1 else "single",
            "l2": "inputs larger than L2 (the weights streamed per step exceed the 126 MB L2)"}


def _serve_config(K: int, world: int) -> dict:
    return {"workload": f"{SERVE_CONFIG} batched serving: {SERVE_STREAMS} streams, prompts uniform in [64, 1024], "
                        f"LPT over the ranks, {K} greedy steps",
            "global_batch": SERVE_STREAMS, "prompt_len": "64-1024", "decode_steps": K,
            "parallelism": (f"request-parallel x{world}, lm_head vocab-sharded over NCCL" if world > 1
                            else "single"),
            "l2": "inputs larger than L2 (1.75 GB of weights + the KV caches per step)"}


def _serve_prompts(vocab: int):
    """The serving workload's prompts: lengths uniform in [64, 1024], ids uniform."""
    import numpy as np

    rng = np.random.default_rng(SEED)
    lengths = [int(v) for v in rng.integers(64, 1025, SERVE_STREAMS)]
    return lengths, [rng.integers(0, vocab, n) for n in lengths]


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


def cpu_oracle_decode(path: str, prompt, budget_s: float, max_tokens: int, threads: int = 0,
                      hidden_prompt: bool = False):
    """The CPU oracle decoding greedily after the prompt: (tok/s, tokens, cores).
    hidden_prompt feeds the prompt without its discarded lm_head products
    (the cache is the same; only the last prompt token's logits are used)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import numpy as np
    import oracle

    oracle.build()
    if threads:
        oracle.set_threads(threads)
    cores = oracle.max_threads()
    m = oracle.OracleModel(path)
    m.set_k_wta_ratio(0.0)
    for i, t in enumerate(prompt[:-1]):
        if hidden_prompt:
            m.forward_hidden(int(t), i == 0)
        else:
            m.forward(int(t), i == 0)
    logits = m.forward(int(prompt[-1]), len(prompt) == 1)
    tok = int(np.argmax(logits))
    n, t0 = 0, time.perf_counter()
    while n < max_tokens and (time.perf_counter() - t0) < budget_s:
        logits = m.forward(tok)
        tok = int(np.argmax(logits))
        n += 1
    dt = time.perf_counter() - t0
    return n / dt, n, cores


def _reference_model(cfg_key: str) -> str:
    """The benchmark model written without the product: the oracle's synthetic
    generator and quantiser, and the numpy restatement of the exporter (the
    file equals the product's write_synthetic byte for byte)."""
    path = _model_path(cfg_key, SEED)
    if not os.path.exists(path):
        for p in (os.path.join(REPO, "oracle"), os.path.join(REPO, "tests", "golden")):
            if p not in sys.path:
                sys.path.insert(0, p)
        import flat_numpy

        tmp = path + f".tmp{os.getpid()}"
        flat_numpy.write_synthetic(tmp, seed=SEED, **_configs().CONFIGS[cfg_key])
        os.replace(tmp, path)
    return path


def run_reference(args, rank: int, world: int) -> None:
    """The reference arm: the reference's CPU decode path on the host cores, on
    the workload the GPU arm runs at this N (rank 0 only)."""
    if rank != 0:
        return
    serving = _under_torchrun() or args.serve
    cfg_key = SERVE_CONFIG if serving else args.config
    cfg = _configs().CONFIGS[cfg_key]
    path = _reference_model(cfg_key)
    budget = max(5.0, min(60.0, 0.05 * (args.steps + args.warmup) + 20.0))
    if serving:
        lengths, prompts = _serve_prompts(cfg["vocab_size"])
        # one stream of the workload (the reference decodes one stream at a
        # time): the prompt whose length is nearest the mean, prefilled untimed
        mean = sum(lengths) / len(lengths)
        i = min(range(len(lengths)), key=lambda j: (abs(lengths[j] - mean), j))
        tps, n, cores = cpu_oracle_decode(path, [int(t) for t in prompts[i]], budget_s=budget,
                                          max_tokens=args.steps, hidden_prompt=True)
        metric = "decode tok/s (batched)"
        config = _serve_config(args.steps, world)
        sample = (f"{n} greedy decode steps of one serving stream after its {lengths[i]}-token prompt "
                  f"(time-bounded to {budget:.0f} s; the reference has no batched path)")
    else:
        prompt = _prompt(cfg["vocab_size"], PROMPT_LEN, SEED)
        tps, n, cores = cpu_oracle_decode(path, prompt, budget_s=budget, max_tokens=args.steps)
        metric = "decode tok/s (batch 1)"
        config = _batch1_config(cfg_key, args.steps, world)
        sample = f"{n} greedy decode steps after a {PROMPT_LEN}-token prompt (time-bounded to {budget:.0f} s)"
    line = {
        "impl": "reference",
        "metric": metric,
        "value": round(tps, 3),
        "unit": "tok/s",
        "n_gpus": args.gpus,
        "steps": n,
        "warmup": args.warmup,
        "ms_per_step": round(1000.0 / tps, 3),
        "higher_is_better": True,
        "scaling": "strong" if serving else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded random-init weights, uniform random prompt ids",
        "config": config,
        "cpu_baseline": {"value": round(tps, 3), "unit": "tok/s", "cores": cores, "kind": "port",
                         "sample": sample},
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
    model.close()

    # ---- the multi-GPU workload at N=1, for the scaling curve (its own line under torchrun)
    serving = None
    if world == 1 and not args.no_serving:
        try:
            r = measure_batched(args, 0, 1, local_rank, None, serve=True, steps=min(K, 256))
            serving = {"value": round(r["value"], 2), "unit": "tok/s", "ms_per_step": round(r["ms_per_step"], 4),
                       "e2e": round(r["e2e"], 2), "prefill_tok_s": round(r["prefill"], 2),
                       "config": _serve_config(r["K"], 1),
                       "roofline_frac": round(r["achieved_gbs"] / r["peak"]["hbm_gbs"], 4),
                       "note": "the workload bench.py times under torchrun at every N (the scaling curve); "
                               "the headline above is batch-1 decode, which does not shard"}
        except Exception as ex:  # reported, not fatal: the headline line still prints
            serving = {"error": f"{type(ex).__name__}: {ex}"}

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
        "config": _batch1_config(cfg_key, K, world),
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
    if serving is not None:
        line["serving"] = serving
    print(json.dumps(line), flush=True)


SWEEP_NK = [(896, 896), (4864, 896), (896, 4864), (8960, 1536), (1536, 8960)]
SWEEP_M = [1, 8, 64, 512]


def run_sweep(args) -> None:
    """The isolated Q4_0 dequant-GEMV/GEMM sweep.  One
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
            line = {"metric": "q4_0 dequant-GEMV/GEMM", "config": {"workload": "isolated Q4_0 GEMV/GEMM sweep", "M": M, "N": N,
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


def measure_batched(args, rank: int = 0, world: int = 1, local_rank: int = 0, dist=None, serve: bool = False,
                    steps: int = 0):
    """Batched decode through gaje_cuda_forward_batch.  serve: the serving
    workload (SERVE_STREAMS streams over all ranks, prompts uniform in
    [64, 1024], LPT-balanced); else --batch B streams per GPU with --prompt P
    tokens each.  Each prompt is prefilled in one gaje_cuda_prefill pass (or
    token by token with --prefill-mode steps), then `steps` greedy steps, each
    stream fed its own argmax.  Under torchrun the ranks are request-parallel
    and the f32 lm_head is split by vocabulary (gaje_cuda_load_sharded).

    Returns (rank 0; None elsewhere) the decode tok/s from the steps' device
    time (CUDA events around each step's device work, max over ranks), the
    end-to-end tok/s of the host loop (tokens in, argmax out, a sync per step,
    max over ranks), the prefill tok/s, each rank's time per segment and the
    roofline of the step."""
    import numpy as np
    import torch

    g = _pkg()
    torch.cuda.set_device(local_rank)
    cfg_key = SERVE_CONFIG if serve else args.config
    cfg = g.configs.CONFIGS[cfg_key]
    path = _ensure_model(g, cfg_key, SEED, rank, dist)
    K = steps or args.steps
    pass_prefill = args.prefill_mode == "pass"
    if serve:
        lengths, all_prompts = _serve_prompts(cfg["vocab_size"])
        mine = lpt_assign(lengths, world)[rank]
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
    toks = [int(v) for v in am]
    # warm-up steps: graph capture for this batch size, clocks
    for _ in range(max(3, args.warmup)):
        toks = [int(v) for v in model.forward_batch(sids, toks)]
    model.batch_timings(reset=True)
    with ClockSampler(local_rank) as clk:
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(K):
            toks = [int(v) for v in model.forward_batch(sids, toks)]
        e1.record(stream)
        e1.synchronize()
    host_ms = e0.elapsed_time(e1)
    seg = model.batch_timings(reset=True)
    dev_ms = sum(seg[k] for k in model.BATCH_SEGMENTS)
    mine_t = [dev_ms, host_ms, pre_ms, float(sum(len(p) for p in plist))] + [seg[k] for k in model.BATCH_SEGMENTS]
    per_rank = [mine_t]
    if dist is not None:
        t = torch.tensor(mine_t, dtype=torch.float64, device=f"cuda:{local_rank}")
        gath = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(gath, t)
        per_rank = [[float(v) for v in x.cpu().tolist()] for x in gath]
    model.close()
    if rank != 0:
        return None
    dev_max = max(r[0] for r in per_rank)
    host_max = max(r[1] for r in per_rank)
    pre_max = max(r[2] for r in per_rank)
    peaks = _peaks()
    mean_p = sum(len(p) for p in plist) / B
    sb = g.configs.step_bytes(cfg, int(mean_p + K // 2))
    # per rank and step: the body once, this rank's share of the lm_head, every local stream's KV
    lm_share = sb["lm_head"] * (1.0 - 1.0 / world) if world > 1 else 0.0
    step_bytes = sb["total"] - sb["kv"] - lm_share + B * sb["kv"]
    step_s = dev_max / 1000.0 / K
    n_prompt = sum(r[3] for r in per_rank)
    segs = {k: [round(r[4 + i] / K, 4) for r in per_rank] for i, k in enumerate(("body", "gather_rows", "lm_head",
                                                                                  "gather_keys"))}
    seg_max = {k: max(v) for k, v in segs.items()}
    limiter = max(seg_max, key=seg_max.get)
    return {
        "value": world * B * K / (dev_max / 1000.0),
        "ms_per_step": dev_max / K,
        "e2e": world * B * K / (host_max / 1000.0),
        "host_ms_per_step": host_max / K,
        "prefill": n_prompt / (pre_max / 1000.0),
        "B": B, "P": P, "K": K, "world": world, "cfg_key": cfg_key,
        "segments_ms_per_step": {"per_rank": segs, "limiter": limiter},
        "step_bytes": step_bytes,
        "achieved_gbs": step_bytes / step_s / 1e9,
        "peak": peaks,
        "clocks": clk.summary(),
        "launches": (5 * cfg["n_blocks"] + 1 + (B + (8 if B <= 8 else 16) - 1) // (8 if B <= 8 else 16)) * K,
    }


def run_batched(args, rank: int = 0, world: int = 1, local_rank: int = 0, dist=None) -> None:
    """The batched line: --serve / torchrun (serving) or --batch B (B streams per GPU)."""
    serve = args.serve or args.batch <= 0
    K = min(args.steps, 256) if serve else args.steps
    r = measure_batched(args, rank, world, local_rank, dist, serve=serve, steps=K)
    if r is None:
        return
    peaks = r["peak"]
    cpu = None
    if world == 1 and serve and not args.no_cpu_baseline:
        cpu = _serve_cpu_baseline(K)
    workload = (_serve_config(K, world) if serve else
                {"workload": f"{r['cfg_key']} batched greedy decode, {r['B']} streams per GPU after a "
                             f"{r['P']}-token prompt each", "global_batch": world * r["B"], "prompt_len": r["P"],
                 "decode_steps": K,
                 "parallelism": (f"request-parallel x{world}, lm_head vocab-sharded over NCCL" if world > 1
                                 else "single"),
                 "l2": "inputs larger than L2"})
    line = {
        "metric": "decode tok/s (batched)",
        "value": round(r["value"], 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": K,
        "warmup": max(3, args.warmup),
        "ms_per_step": round(r["ms_per_step"], 4),
        "higher_is_better": True,
        "scaling": "strong" if serve else "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic: seeded random-init N(0,0.02) weights quantised by the Q4_0 exporter restatement, "
                "uniform random prompt ids",
        "config": workload,
        "timing": "value: CUDA events around each step's device work on every rank (body graph, all-gathers, "
                  "sharded head), summed over the K steps, max over ranks; e2e: the host loop",
        "prefill": {"value": round(r["prefill"], 2), "unit": "tok/s",
                    "how": "gaje_cuda_prefill: each stream's prompt in one pass (tcgen05 GEMMs over the prompt "
                           "rows, causal attention kernel); the reference prefills token by token"},
        "e2e": {"value": round(r["e2e"], 2), "unit": "tok/s", "ms_per_step": round(r["host_ms_per_step"], 4),
                "h2d_bytes_per_step": 12 * r["B"] * world, "d2h_bytes_per_step": (4 * r["B"] + 32) * world,
                "path": "gaje_cuda_forward_batch (host tokens in, host argmax out, a sync per step)"},
        "segments_ms_per_step": r["segments_ms_per_step"],
        "roofline": {"bound": "hbm", "kernel": "batched step (Q4 GEMMs + lm_head for B vectors), bytes per rank",
                     "achieved": round(r["achieved_gbs"], 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(r["achieved_gbs"] / peaks["hbm_gbs"], 4), "traffic": None,
                     "algorithmic_bytes": r["step_bytes"],
                     "peak_source": peaks["source"] + " (MEASURED_PEAKS.json hbm_gbs, of measured)"},
        "gpu_launches": r["launches"],
        "clocks": r["clocks"],
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
    print(json.dumps(line), flush=True)


def _serve_cpu_baseline(K: int) -> dict:
    """The oracle on one stream of the serving workload (bounded sample)."""
    g = _pkg()
    cfg = g.configs.CONFIGS[SERVE_CONFIG]
    path = _model_path(SERVE_CONFIG, SEED)
    lengths, prompts = _serve_prompts(cfg["vocab_size"])
    i = min(range(len(lengths)), key=lambda j: (abs(lengths[j] - sum(lengths) / len(lengths)), j))
    tps, n, cores = cpu_oracle_decode(path, [int(t) for t in prompts[i]], budget_s=10.0, max_tokens=K,
                                      hidden_prompt=True)
    return {"value": round(tps, 3), "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} greedy steps of one serving stream after its {lengths[i]}-token prompt, oracle/ AVX2 "
                      f"restatement, {cores} OpenMP threads, 10 s budget"}


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


def run_trace_fused(args) -> None:
    """Per-segment times of the two-exchange decode kernel from its %globaltimer
    stamps (gaje_cuda_trace_fused): the workload's prompt is fed first, then
    one launch of --steps greedy steps is traced.  Per block, each CTA's stamps
    give its segments; an exchange is the time from the last writer's publish
    to a reader's gate.  Prints one JSON object: for every segment the median
    over blocks and steps of (median over CTAs, max over CTAs), microseconds.
    No timing claim: the stamps themselves cost a little."""
    import numpy as np
    import torch

    g = _pkg()
    torch.cuda.set_device(0)
    path = _ensure_model(g, args.config, SEED, 0, None)
    model = g.load_genomic_auto(path, device=0, max_ctx=PROMPT_LEN + args.steps + 64)
    model.set_k_wta_ratio(0.0)
    if int(model.info().megakernel) != 2:
        raise SystemExit("--trace-fused: the model does not run on the two-exchange kernel")
    prompt = _prompt(model.vocab_size, PROMPT_LEN, SEED)
    first = 0
    for i, t in enumerate(prompt):
        first = model.forward_argmax(t, i == 0)
    tr = model.trace_fused(first, args.steps) / 1000.0  # [grid, steps, L+1, 24] us
    G, K, L1, _ = tr.shape
    L = L1 - 1
    info = model.info()
    # attention CTAs stamp 0-8 and 15-20; every CTA with FFN outputs stamps 9-14
    segs_a = [("input gate + residual (A)", 0, 1), ("attn_norm staging", 1, 2), ("q/k/v GEMV + RoPE", 2, 3),
              ("K/V rows wait", 3, 4), ("split attention math", 4, 5),
              ("  attention entry -> K/V landed", 16, 4), ("  scores", 4, 17), ("  softmax + (m, l)", 17, 18),
              ("  P*V", 18, 19), ("  return -> CTA barrier", 19, 5),
              ("attn_output columns", 5, 6),
              ("split weight", 6, 15),
              ("red.add + publish (A)", 7, 8)]
    segs_b = [("residual x_a", 9, 10), ("ffn_norm staging", 10, 11), ("gate/up GEMV + SwiGLU", 11, 12),
              ("ffn_down columns", 12, 13), ("red.add + publish (B)", 13, 14)]
    out = {"config": args.config, "steps": K, "blocks": L, "grid": G, "unit": "us", "segments": {}}

    def stat(vals):  # vals [G] per (step, block); nan = CTA without that stamp
        v = vals[np.isfinite(vals)]
        return (float(np.median(v)), float(np.max(v))) if v.size else (float("nan"), float("nan"))

    t = np.where(tr > 0, tr, np.nan)
    for name, a, b in segs_a + segs_b:
        meds, maxs = [], []
        for k in range(K):
            for l in range(L):
                m, x = stat(t[:, k, l, b] - t[:, k, l, a])
                meds.append(m)
                maxs.append(x)
        out["segments"][name] = {"median_cta": round(float(np.nanmedian(meds)), 3),
                                 "max_cta": round(float(np.nanmedian(maxs)), 3)}
    # exchanges: last writer's publish -> readers' gate
    exA, exB, blk = [], [], []
    for k in range(K):
        for l in range(L):
            wA = np.nanmax(t[:, k, l, 8])
            exA.append(float(np.nanmedian(t[:, k, l, 9] - wA)))
            if l + 1 < L:
                wB = np.nanmax(t[:, k, l, 14])
                exB.append(float(np.nanmedian(t[:, k, l + 1, 1] - wB)))
                blk.append(float(np.nanmax(t[:, k, l + 1, 14]) - np.nanmax(t[:, k, l, 14])))
    out["exchange_A_us"] = round(float(np.median(exA)), 3)
    out["exchange_B_us"] = round(float(np.median(exB)), 3) if exB else None
    out["block_us"] = round(float(np.median(blk)), 3) if blk else None
    lm = [float(np.nanmax(t[:, k, L, 4]) - np.nanmax(t[:, k, L - 1, 14])) for k in range(K)]
    out["lm_head_us"] = round(float(np.median(lm)), 3)
    stepus = [float(np.nanmax(t[:, k, L, 4]) - (np.nanmax(t[:, k - 1, L, 4]) if k else np.nanmin(t[:, 0, 0, 0])))
              for k in range(K)]
    out["step_us"] = round(float(np.median(stepus[1:] if K > 1 else stepus)), 3)
    out["plan"] = {"grid": int(info.grid)}
    print(json.dumps(out), flush=True)


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
    ap.add_argument("--config", default=None,
                    help="model shape (configs.py); default qwen2-0.5b, or qwen2.5-1.5b with --batch")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-serving", action="store_true",
                    help="plain N=1 run: skip the serving workload's N=1 measurement (the 'serving' object)")
    ap.add_argument("--batch", type=int, default=0,
                    help="batched decode of this many streams per GPU (Qwen2.5-1.5B shape by default) instead of batch 1")
    ap.add_argument("--prompt", type=int, default=PROMPT_LEN, help="prompt tokens per stream (--batch)")
    ap.add_argument("--serve", action="store_true",
                    help="batched serving: 512 streams over all ranks, prompts uniform in [64, 1024], LPT-balanced")
    ap.add_argument("--prefill-mode", choices=["pass", "steps"], default="pass",
                    help="--batch prompts: one gaje_cuda_prefill pass per stream, or token-by-token batched steps")
    ap.add_argument("--sweep", action="store_true",
                    help="the isolated Q4_0 GEMV/GEMM sweep instead of the decode benchmark")
    ap.add_argument("--engine", choices=sorted(ENGINES), default="fused",
                    help="batch-1 engine: fused (two exchanges per block, default), mega (five), phase")
    ap.add_argument("--context", type=int, default=0,
                    help="with --ncu-case --batch B: prefill each stream with this many tokens first")
    ap.add_argument("--prompt-only", type=int, default=0,
                    help="with --ncu-case: prefill two streams with prompts of this many tokens (profiling)")
    ap.add_argument("--trace-fused", action="store_true",
                    help="per-segment table of the two-exchange kernel from its timer stamps (--steps steps)")
    ap.add_argument("--ncu-case", action="store_true",
                    help="the small profiling case: one launch filling the prompt's positions, then one "
                         "launch of --steps decode steps (capture it with -k regex:k_decode_fused -s 1 -c 1); "
                         "with --batch B: --steps batched steps of B streams from empty caches; with "
                         "--prompt-only P: two P-token prefills")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.config is None:  # configs[3] (--batch) is quoted on the Qwen2.5-1.5B shape
        args.config = SERVE_CONFIG if args.batch > 0 else CONFIG_KEY
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
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
    if args.trace_fused:
        run_trace_fused(args)
        return
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist

        torch.cuda.set_device(local_rank)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device(f"cuda:{local_rank}"))
        dist = tdist
    try:
        if args.batch > 0 or args.serve or _under_torchrun():
            run_batched(args, rank, world, local_rank, dist)
        else:
            run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
