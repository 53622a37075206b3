"""Parity on the workloads the benchmark measures, against the CPU oracle.

The reference's decode loop is generate_native_core
(src/nn/llm/forward.rs:215-271): the prompt fed token by token through
forward_core, then the first maximum of each step's logits fed back.  Each
test below drives the GPU path the benchmark times on the same model file,
prompt and step count:

  * the Qwen2-0.5B shape, a 256-token prompt, then greedy steps (the batch-1
    headline; the default two-exchange fused kernel), through the host loop
    (gaje_cuda_forward, logits every step) and through the device loop
    (gaje_cuda_decode_greedy, the benchmark's timed call);
  * the SmolLM2-135M shape, a 128-token prompt, 128 greedy steps;
  * the Qwen2.5-1.5B shape (head_dim 128, d 1536, ffn 8960): the batch-1
    engine, batched steps of 8 streams (CUDA-core GEMMs) and 16 streams
    (tcgen05 GEMMs), and a 2048-token prompt in one prefill pass followed by
    decode steps over that context;
  * two runs of the fused kernel on one prompt (it adds CTA partial sums in
    arrival order).

Bars (the north star's): per-step logits within 1e-3 max relative error
(max|gpu - oracle| / max|oracle| over the vocabulary); an identical greedy
stream for the first 64 generated tokens.  Past 64 tokens, streams may part
only where the oracle's top-2 margin is itself inside that tolerance (a near
tie that either order of float additions may break).  Each test prints its
worst error and the smallest top-1/top-2 margin it saw.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3
SEED = 1234  # bench.py's model seed


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _margin(lr):
    top2 = np.sort(lr)[-2:]
    return float(top2[1] - top2[0])


def _bench_prompt(vocab, n, seed=SEED):
    """bench.py's prompt: uniform random ids from a fixed seed."""
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def _oracle_run(O, path, prompt, steps):
    """The oracle's prompt loop and greedy steps: (stream, per-step logits of
    the greedy steps, last prompt logits)."""
    ref = O.OracleModel(path)
    ref.set_k_wta_ratio(0.0)
    lr = None
    for i, t in enumerate(prompt):
        lr = ref.forward(t, i == 0)
    last_prompt = lr
    stream, logits = [], []
    tok = int(np.argmax(lr))
    for _ in range(steps):
        stream.append(tok)
        lr = ref.forward(tok)
        logits.append(lr)
        tok = int(np.argmax(lr))
    return stream, logits, last_prompt


def _check_stream(sg, sr, ref_logits_before, label):
    """Identical for the first 64 tokens; later a divergence only at a near tie.
    ref_logits_before[i] are the oracle logits that chose sr[i]."""
    n = min(len(sg), len(sr))
    first = next((i for i in range(n) if sg[i] != sr[i]), n)
    assert first >= min(64, n), f"{label}: greedy streams differ at token {first}"
    if first < n:
        lr = ref_logits_before[first]
        tol = REL_TOL * float(np.max(np.abs(lr)))
        assert _margin(lr) <= tol, f"{label}: streams part at {first} without a near tie"
        print(f"{label}: streams identical for {first} tokens, then part at a near tie "
              f"(margin {_margin(lr):.2e})")
    return first


def _host_loop_parity(g, O, path, prompt, steps, label, **load):
    gpu = g.load_genomic_auto(path, device=0, max_ctx=len(prompt) + steps + 16, **load)
    gpu.set_k_wta_ratio(0.0)
    ref = O.OracleModel(path)
    ref.set_k_wta_ratio(0.0)
    worst, margins = 0.0, []
    for i, t in enumerate(prompt):
        lg, lr = gpu.forward(t, i == 0), ref.forward(t, i == 0)
        worst = max(worst, _rel(lg, lr))
    sg, sr, before = [], [], []
    tg, tr = int(np.argmax(lg)), int(np.argmax(lr))
    diverged = False
    for _ in range(steps):
        sg.append(tg)
        sr.append(tr)
        before.append(lr)
        if tg != tr:
            diverged = True
            break
        lg, lr = gpu.forward(tg), ref.forward(tr)
        worst = max(worst, _rel(lg, lr))
        margins.append(_margin(lr))
        tg, tr = int(np.argmax(lg)), int(np.argmax(lr))
    print(f"{label}: max rel logit err {worst:.2e}, min top1-top2 margin "
          f"{min(margins) if margins else float('nan'):.2e} over {len(margins)} steps")
    assert worst <= REL_TOL, f"{label}: {worst:.3e}"
    if diverged:
        # the logits compared so far are within the bar; where the streams part
        # the oracle's choice must be a near tie
        _check_stream(sg, sr, before, label)
    return gpu, ref


@pytest.mark.parametrize("name,prompt_len,steps", [("qwen2-0.5b", 256, 256), ("smollm2-135m", 128, 128)])
def test_batch1_workload_as_benchmarked(g, O, make_model, name, prompt_len, steps):
    """The batch-1 benchmark workload on the default engine (two-exchange fused
    kernel): host loop with logits every step, then the device loop the
    benchmark times, both against the oracle's stream."""
    path = make_model(name, seed=SEED)
    gpu, _ = _host_loop_parity(g, O, path, _bench_prompt(g.configs.CONFIGS[name]["vocab_size"], prompt_len),
                               steps, f"{name} host loop")
    print(f"{name}: engine {gpu.info().megakernel} (2: the two-exchange fused kernel)")
    if name == "qwen2-0.5b":
        assert gpu.info().megakernel == 2  # the benchmark's engine
    prompt = _bench_prompt(gpu.vocab_size, prompt_len)
    stream, logits, last_prompt = _oracle_run(O, path, prompt, steps)
    gpu.clear_cache_py()
    first = 0
    for i, t in enumerate(prompt):
        first = gpu.forward_argmax(t, i == 0)
    assert first == int(np.argmax(last_prompt))
    toks = gpu.decode_greedy(first, steps)  # toks[i] is the argmax after feeding the i-th token
    dev_stream = [first] + list(toks[:-1])
    _check_stream(dev_stream, stream, [last_prompt] + logits[:-1], f"{name} device loop")
    gpu.close()


def test_q8_lm_head_fused_kernel(g, O, make_model):
    """The exporter's --quant-embed variant of the Qwen2-0.5B shape (Q8_0
    token_embd / lm_head): the fused kernel streams the Q8_0 rows themselves
    (genomic.rs:381-448 values, q * scale) instead of dequantised f32 rows."""
    path = make_model("qwen2-0.5b-q8e", seed=SEED)
    gpu, _ = _host_loop_parity(g, O, path, _bench_prompt(151936, 32), 64, "qwen2-0.5b-q8e host loop")
    assert gpu.info().megakernel == 2
    gpu.close()


def test_fused_kernel_run_to_run(g, make_model):
    """Two runs of the fused kernel on one prompt and 64 greedy steps: the
    token streams are identical; the logit spread between the runs is printed
    and must stay far inside the parity bar."""
    path = make_model("qwen2-0.5b", seed=SEED)
    gpu = g.load_genomic_auto(path, device=0, max_ctx=256)
    gpu.set_k_wta_ratio(0.0)
    prompt = _bench_prompt(gpu.vocab_size, 64)
    runs = []
    for _ in range(2):
        lgs = []
        for i, t in enumerate(prompt):
            lgs.append(gpu.forward(t, i == 0))
        tok = int(np.argmax(lgs[-1]))
        for _ in range(64):
            lgs.append(gpu.forward(tok))
            tok = int(np.argmax(lgs[-1]))
        runs.append(lgs)
    spread = max(_rel(a, b) for a, b in zip(runs[0], runs[1]))
    toks = [[int(np.argmax(x)) for x in r] for r in runs]
    print(f"fused kernel run-to-run: max rel logit spread {spread:.2e}")
    assert toks[0] == toks[1]
    assert spread <= REL_TOL / 100
    gpu.close()


# ---------------------------------------------------------- Qwen2.5-1.5B shape
@pytest.fixture(scope="module")
def q15(make_model):
    return make_model("qwen2.5-1.5b", seed=SEED)


@pytest.mark.parametrize("engine", [1, 2, 0], ids=["default", "five-exchange", "phase"])
def test_q15_batch1_engine(g, O, q15, engine):
    """The batch-1 path on head_dim 128 / d 1536, whichever engine the load
    option leads to for the shape (n_head * head_dim = 1536 is past what the
    persistent kernels' plans accept, so every option must end on an engine
    that computes it)."""
    rng = np.random.default_rng(15)
    prompt = [int(t) for t in rng.integers(0, 151936, 24)]
    gpu, _ = _host_loop_parity(g, O, q15, prompt, 64, f"qwen2.5-1.5b batch-1 (option {engine})",
                               use_megakernel=engine)
    print(f"qwen2.5-1.5b batch-1 engine: {gpu.info().megakernel}")
    gpu.close()


@pytest.mark.parametrize("n_streams", [8, 16])
def test_q15_batched_streams(g, O, q15, n_streams):
    """forward_batch at 8 streams (CUDA-core GEMMs) and 16 (tcgen05 GEMMs): each
    stream's 12-token prompt as batched steps, then 24 greedy steps; every
    stream against its own oracle run (one oracle model, stream by stream)."""
    P, steps = 12, 24
    rng = np.random.default_rng(100 + n_streams)
    prompts = [[int(t) for t in rng.integers(0, 151936, P)] for _ in range(n_streams)]
    gpu = g.load_genomic_auto(q15, device=0, max_ctx=P + steps + 8, max_streams=n_streams)
    gpu.set_k_wta_ratio(0.0)
    sids = list(range(n_streams))
    gl, ga = [], []
    for t in range(P):
        am, lg = gpu.forward_batch(sids, [prompts[s][t] for s in sids], logits=True)
        gl.append(lg)
        ga.append(list(am))
    for _ in range(steps):
        am, lg = gpu.forward_batch(sids, [int(a) for a in ga[-1]], logits=True)
        gl.append(lg)
        ga.append(list(am))
    gpu.close()
    ref = O.OracleModel(q15)
    ref.set_k_wta_ratio(0.0)
    worst, margin = 0.0, np.inf
    for s in sids:
        toks = prompts[s] + [int(ga[P - 1 + i][s]) for i in range(steps)]
        for i, t in enumerate(toks):
            lr = ref.forward(t, i == 0)
            worst = max(worst, _rel(gl[i][s], lr))
            assert int(ga[i][s]) == int(np.argmax(lr)), (s, i)
            if i >= P - 1:
                margin = min(margin, _margin(lr))
    print(f"qwen2.5-1.5b {n_streams} streams: max rel logit err {worst:.2e}, min margin {margin:.2e}")
    assert worst <= REL_TOL


def test_q15_prefill_2048(g, O, q15):
    """One 2048-token prompt in one gaje_cuda_prefill pass (tcgen05 GEMMs +
    causal attention) against the oracle fed token by token, then 16 batched
    decode steps over that context."""
    P = 2048
    gpu = g.load_genomic_auto(q15, device=0, max_ctx=P + 32, max_streams=1, max_prefill=P)
    gpu.set_k_wta_ratio(0.0)
    prompt = [int(t) for t in np.random.default_rng(2048).integers(0, 151936, P)]
    am, lg = gpu.prefill(0, prompt, logits=True)
    ref = O.OracleModel(q15)
    ref.set_k_wta_ratio(0.0)
    for i, t in enumerate(prompt[:-1]):
        ref.forward_hidden(t, i == 0)  # the cache only: the discarded logits of the prompt
    lr = ref.forward(prompt[-1])
    worst = _rel(lg, lr)
    assert am == int(np.argmax(lr))
    tok = am
    for _ in range(16):
        a, lgb = gpu.forward_batch([0], [tok], logits=True)
        lr = ref.forward(tok)
        worst = max(worst, _rel(lgb[0], lr))
        assert int(a[0]) == int(np.argmax(lr))
        tok = int(a[0])
    print(f"qwen2.5-1.5b prefill 2048 + 16 steps: max rel logit err {worst:.2e}")
    assert worst <= REL_TOL
    gpu.close()
