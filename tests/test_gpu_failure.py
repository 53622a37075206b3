"""Failure detection without a GPU fault.

1. A bounded device wait that runs out.  The two-exchange decode kernel waits
   (bounded) for every attention CTA's flag before the FFN half of a block;
   gaje_cuda_debug_withhold_flag makes one CTA skip that flag in the next
   launch, so the flag is one that nothing sets.  With the wait limit cut to
   0.2 s the call must return GAJE_ERR_TIMEOUT within a few seconds, and the
   CUDA context must stay usable: a fresh handle then decodes and matches the
   oracle.  (The reference's only comparable error path is its NaN guards,
   src/nn/block/forward.rs:11-13,97-99; a CPU engine has no device waits.)

2. A sharded rank that stops calling between steps.  Two ranks serve batched
   streams with the lm_head split by vocabulary; after a few steps rank 1
   leaves (no kernel or collective of it in flight) and rank 0 makes one more
   call.  Its NCCL all-gather can never complete: after GAJE_NCCL_TIMEOUT_S the
   library aborts the communicator and the call returns GAJE_ERR_TIMEOUT; the
   model then refuses further sharded calls.  NVLS is off.  Two spawned
   processes, one per GPU; skipped with fewer than two GPUs.
"""
import multiprocessing as mp
import os
import sys
import time

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu

GAJE_ERR_TIMEOUT = 9


def test_device_wait_runs_out_and_context_stays_usable(g, O, make_model):
    path = make_model("small", seed=61)
    g.set_wait_limit(0, 200_000_000)  # 0.2 s
    try:
        m = g.load_genomic_auto(path, device=0, max_ctx=64)
        assert int(m.info().megakernel) == 2  # the two-exchange kernel
        m.set_k_wta_ratio(0.0)
        m.forward(3, clear_cache=True)  # a normal step first
        m.debug_withhold_flag(1)
        t0 = time.time()
        with pytest.raises(g.GajeError) as ei:
            m.forward(5)
        elapsed = time.time() - t0
        assert ei.value.status == GAJE_ERR_TIMEOUT, str(ei.value)
        assert "bounded device wait" in ei.value.message
        assert elapsed < 10.0, elapsed
        m.close()
    finally:
        g.set_wait_limit(0, 0)
    # the context is usable: a fresh handle decodes and matches the oracle
    m = g.load_genomic_auto(path, device=0, max_ctx=64)
    m.set_k_wta_ratio(0.0)
    ref = O.OracleModel(path)
    ref.set_k_wta_ratio(0.0)
    tok = 3
    for i in range(6):
        lg, lr = m.forward(tok, i == 0), ref.forward(tok, i == 0)
        assert float(np.max(np.abs(lg - lr)) / np.max(np.abs(lr))) <= 1e-3
        assert int(np.argmax(lg)) == int(np.argmax(lr))
        tok = int(np.argmax(lr))
    m.close()


def test_withhold_rejects_bad_arguments(g, make_model):
    path = make_model("tiny", seed=62)
    m = g.load_genomic_auto(path, device=0, max_ctx=32, use_megakernel=0)  # kernel per phase
    with pytest.raises(g.GajeError) as ei:
        m.debug_withhold_flag(0)
    assert ei.value.status == 5  # GAJE_ERR_UNSUPPORTED
    m.close()
    m = g.load_genomic_auto(path, device=0, max_ctx=32)
    with pytest.raises(g.GajeError):
        m.debug_withhold_flag(10_000)
    m.close()


def _post(q, item, exit_after=False):
    """Queue.put is asynchronous: flush the feeder before an os._exit."""
    q.put(item)
    if exit_after:
        q.close()
        q.join_thread()
        os._exit(0)


def _leaver(rank, world, nid, path, B, P, steps, q, ev):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        os.environ["GAJE_NCCL_TIMEOUT_S"] = "5"
        sys.path.insert(0, REPO)
        import importlib

        import torch

        torch.cuda.set_device(rank)
        g = importlib.import_module("gaje-semantic-compression_b200")
        m = g.load_genomic_sharded(path, world, rank, nid, device=rank, max_ctx=64, max_streams=B, max_prefill=32)
        m.set_k_wta_ratio(0.0)
        rng = np.random.default_rng(200 + rank)
        toks = [m.prefill(s, [int(t) for t in rng.integers(0, m.vocab_size, P)]) for s in range(B)]
        for _ in range(steps):
            toks = [int(t) for t in m.forward_batch(list(range(B)), toks)]
        torch.cuda.synchronize()
        if rank == 1:  # leaves between steps: nothing of it in flight
            q.put((rank, "left", None, 0.0))
            ev.wait(120)  # stays alive (and silent) until rank 0 has seen the timeout
            _post(q, (rank, "done", None, 0.0), exit_after=True)
        time.sleep(0.5)
        t0 = time.time()
        status = None
        try:
            m.forward_batch(list(range(B)), toks)
        except g.GajeError as e:
            status = e.status
        elapsed = time.time() - t0
        after = None
        try:
            m.forward_batch(list(range(B)), toks)
        except g.GajeError as e:
            after = e.status
        ev.set()
        _post(q, (rank, status, after, elapsed), exit_after=True)
    except Exception as e:  # noqa: BLE001
        ev.set()
        _post(q, (rank, repr(e), None, 0.0), exit_after=True)


def test_sharded_rank_leaving_makes_peer_time_out(g, make_model):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    path = make_model("tiny", seed=63)
    nid = g.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ev = ctx.Event()
    procs = [ctx.Process(target=_leaver, args=(r, 2, nid, path, 3, 7, 3, q, ev)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(3):
            rank, a, b, t = q.get(timeout=180)
            res.setdefault(rank, []).append((a, b, t))
    finally:
        ev.set()
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert [r[0] for r in res[1]] == ["left", "done"], res
    status, after, elapsed = res[0][0]
    assert status == GAJE_ERR_TIMEOUT, res
    assert after is not None and after != 0, res  # the aborted model refuses further sharded calls
    assert 4.0 <= elapsed < 60.0, elapsed
