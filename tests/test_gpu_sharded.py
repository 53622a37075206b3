"""Vocab-sharded batched serving on two GPUs (gaje_cuda_load_sharded): each
rank runs its own streams through the whole body, the f32 lm_head is split by
vocabulary over the ranks, and the argmax keys are merged over NCCL.  Every
stream's greedy tokens (the prompt pass, then decode steps) must be the ones
the CPU oracle gives for that stream alone.

Runs as two spawned processes, one per GPU; skipped with fewer than two.
"""
import multiprocessing as mp
import os
import sys

import numpy as np
import pytest

from conftest import REPO

pytestmark = pytest.mark.gpu


def _worker(rank, world, nid, path, B, P, steps, q):
    try:
        os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
        os.environ.setdefault("GAJE_NCCL_TIMEOUT_S", "60")
        sys.path.insert(0, REPO)
        import importlib

        import torch

        torch.cuda.set_device(rank)
        g = importlib.import_module("gaje-semantic-compression_b200")
        m = g.load_genomic_sharded(path, world, rank, nid, device=rank, max_ctx=64, max_streams=B, max_prefill=32)
        m.set_k_wta_ratio(0.0)
        inf = m.info()
        rng = np.random.default_rng(100 + rank)
        prompts = rng.integers(0, m.vocab_size, (B, P))
        toks = [m.prefill(s, [int(t) for t in prompts[s]]) for s in range(B)]  # collective: B calls on every rank
        out = [list(toks)]
        for _ in range(steps):
            toks = [int(t) for t in m.forward_batch(list(range(B)), toks)]
            out.append(toks)
        refused = []
        try:
            m.forward(1)
        except ValueError as e:
            refused.append(e.status)
        try:
            m.forward_batch(list(range(B)), toks, logits=True)
        except ValueError as e:
            refused.append(e.status)
        q.put((rank, prompts.tolist(), out, (int(inf.vocab_row0), int(inf.vocab_rows)), refused))
        m.close()
    except Exception as e:
        q.put((rank, repr(e), None, None, None))


def _run(g, O, path, B, P, steps):
    import torch

    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    nid = g.nccl_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, nid, path, B, P, steps, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, prompts, out, shard, refused = q.get(timeout=600)
            assert out is not None, prompts
            res[rank] = (prompts, out, shard, refused)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    V = g.inspect_flat(path)["vocab_size"]
    assert res[0][2][0] == 0 and res[1][2][0] == res[0][2][1] and sum(r[2][1] for r in res.values()) == V
    for rank, (prompts, out, _, refused) in res.items():
        assert refused == [5, 5]  # GAJE_ERR_UNSUPPORTED: single-stream call, full logits
        for s in range(B):
            ref = O.OracleModel(path)
            ref.set_k_wta_ratio(0.0)
            lr = None
            for i, t in enumerate(prompts[s]):
                lr = ref.forward(int(t), i == 0)
            for k in range(steps + 1):
                assert out[k][s] == int(np.argmax(lr)), (rank, s, k)
                if k < steps:
                    lr = ref.forward(out[k][s])


def test_sharded_two_gpus_cuda_core_head(g, O, make_model):
    """3 streams per rank: 6 gathered rows through the CUDA-core lm_head kernel."""
    _run(g, O, make_model("tiny", seed=51), B=3, P=9, steps=6)


def test_sharded_two_gpus_tensor_core_head(g, O, make_model):
    """8 streams per rank: 16 gathered rows through the tcgen05 lm_head."""
    _run(g, O, make_model("small", seed=52), B=8, P=5, steps=3)
