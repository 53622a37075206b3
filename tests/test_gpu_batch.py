"""Batched decode (gaje_cuda_forward_batch) against the CPU oracle: every
stream of a batch must give the logits and greedy tokens the single-stream
reference path gives for that stream alone (its own oracle model and cache).

Bar: per-step logits within 1e-3 max relative error (max|Δ|/max|oracle|),
identical argmax.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REL_TOL = 1e-3


def _rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _run_schedule(g, O, path, schedule, n_streams, max_ctx=256, kwta=0.0):
    """schedule: list of steps, each a list of (stream, token or None=greedy)."""
    gpu = g.load_genomic_auto(path, max_ctx=max_ctx, max_streams=n_streams)
    refs = [O.OracleModel(path) for _ in range(n_streams)]
    if kwta == 0.0:  # else: the post-load state, K-WTA 0.5 on the logits only
        gpu.set_k_wta_ratio(0.0)
        for r in refs:
            r.set_k_wta_ratio(0.0)
    last = [None] * n_streams
    worst = 0.0
    for step in schedule:
        sids = [s for s, _ in step]
        toks = [t if t is not None else last[s] for s, t in step]
        am, lg = gpu.forward_batch(sids, toks, logits=True)
        for i, s in enumerate(sids):
            lr = refs[s].forward(toks[i], refs[s].cache_len == 0)
            if kwta > 0:
                keep = (lg[i] != np.float32(-1e9)) & (lr != np.float32(-1e9))
                worst = max(worst, _rel(lg[i][keep], lr[keep]))
            else:
                worst = max(worst, _rel(lg[i], lr))
                assert int(am[i]) == int(np.argmax(lr)), (s, int(am[i]), int(np.argmax(lr)))
            last[s] = int(am[i])
    for s in range(n_streams):
        assert gpu.stream_len(s) == refs[s].cache_len
    return worst


@pytest.mark.parametrize("name", ["tiny", "small"])
def test_batch_streams_join_at_different_positions(g, O, make_model, name):
    path = make_model(name, seed=31)
    rng = np.random.default_rng(3)
    V = g.load_genomic_auto(path, max_ctx=8).vocab_size
    schedule = []
    for t in range(14):
        step = [(0, int(rng.integers(0, V)) if t < 4 else None)]
        if t >= 3:
            step.append((1, int(rng.integers(0, V)) if t < 6 else None))
        if t >= 6:
            step.append((2, int(rng.integers(0, V)) if t < 8 else None))
        schedule.append(step)
    assert _run_schedule(g, O, path, schedule, 3) <= REL_TOL


def test_batch_of_17_streams_two_tiles(g, O, make_model):
    """17 streams: two 8-vector GEMM tiles and two 16-vector lm_head tiles."""
    path = make_model("tiny", seed=32)
    V = g.load_genomic_auto(path, max_ctx=8).vocab_size
    rng = np.random.default_rng(4)
    schedule = [[(s, int(rng.integers(0, V))) for s in range(17)] for _ in range(3)]
    schedule += [[(s, None) for s in range(17)] for _ in range(3)]
    assert _run_schedule(g, O, path, schedule, 17, max_ctx=64) <= REL_TOL


@pytest.mark.parametrize("name", ["smollm2-135m", "qwen2-0.5b"])
def test_batch_baseline_shapes(g, O, make_model, name):
    path = make_model(name, seed=1234)
    V = g.load_genomic_auto(path, max_ctx=8).vocab_size
    rng = np.random.default_rng(5)
    schedule = [[(s, int(rng.integers(0, V))) for s in range(4)] for _ in range(6)]
    schedule += [[(s, None) for s in range(4)] for _ in range(10)]
    assert _run_schedule(g, O, path, schedule, 4, max_ctx=64) <= REL_TOL


def test_batch_default_logit_kwta(g, O, make_model):
    """load_genomic leaves K-WTA 0.5 on the logits (flat_reader.rs:234)."""
    path = make_model("small", seed=33)
    V = g.load_genomic_auto(path, max_ctx=8).vocab_size
    rng = np.random.default_rng(6)
    schedule = [[(s, int(rng.integers(0, V))) for s in range(2)] for _ in range(3)]
    assert _run_schedule(g, O, path, schedule, 2, kwta=0.5) <= REL_TOL


def test_batch_argument_errors(g, make_model):
    path = make_model("tiny", seed=34)
    m = g.load_genomic_auto(path, max_ctx=8, max_streams=2)
    with pytest.raises(ValueError):
        m.forward_batch([0, 0], [1, 2])
    with pytest.raises(ValueError):
        m.forward_batch([2], [1])
    m0 = g.load_genomic_auto(path, max_ctx=8)
    with pytest.raises(ValueError):
        m0.forward_batch([0], [1])
    for _ in range(8):
        m.forward_batch([1], [3])
    with pytest.raises(ValueError) as e:
        m.forward_batch([1], [3])
    assert e.value.status == 8
    m.clear_stream(1)
    assert m.stream_len(1) == 0
    m.forward_batch([1], [3])
    assert m.stream_len(1) == 1


@pytest.mark.parametrize("name,n_streams", [("smollm2-135m", 20), ("qwen2-0.5b", 16)])
def test_batch_tensor_core_path(g, O, make_model, name, n_streams):
    """From 16 streams the step's projections and the lm_head run on the
    tcgen05 kernels (bf16 hi/lo x3); same bar as the CUDA-core path."""
    path = make_model(name, seed=1235)
    V = g.load_genomic_auto(path, max_ctx=8).vocab_size
    rng = np.random.default_rng(7)
    schedule = [[(s, int(rng.integers(0, V))) for s in range(n_streams)] for _ in range(3)]
    schedule += [[(s, None) for s in range(n_streams)] for _ in range(2)]
    assert _run_schedule(g, O, path, schedule, n_streams, max_ctx=32) <= REL_TOL
