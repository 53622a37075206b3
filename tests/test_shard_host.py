"""Host logic of vocab-sharded serving (gaje_cuda_load_sharded), on the CPU
with two gloo ranks: the vocabulary split the ranks load and the argmax-key
merge they run after the key all-gather.

Each rank takes its lm_head rows (gaje_vocab_shard), reduces its slice of a
logit row to the best gaje_argmax_key, the keys are all-gathered over gloo,
and the largest key must name the first maximum of the whole row, as the
reference's greedy argmax picks it (src/nn/llm/forward.rs:262-271: strict
`>` against a -inf start, so NaN never wins and ties keep the lower index).
"""
import multiprocessing as mp
import os
import socket
import sys
from datetime import timedelta

import numpy as np
import pytest

from conftest import REPO


def _reference_argmax(row):
    best, idx = -np.inf, 0
    for i, v in enumerate(row.tolist()):
        if v > best:
            best, idx = v, i
    return idx


def _rows(V):
    rng = np.random.default_rng(17)
    R = rng.standard_normal((7, V)).astype(np.float32)
    h = V // 2
    R[0, 3] = R[0, h + 5] = 9.0          # the maximum on both shards: the first one wins
    R[1, h - 1] = R[1, h] = 8.0          # a tie across the shard boundary
    R[2, :] = np.nan
    R[2, h + 7] = -1.0                   # NaNs never win
    R[2, 1] = -np.inf
    R[3, :] = 0.0
    R[3, 0] = -0.0                       # -0.0 ties with +0.0: index 0
    R[4, :] = np.nan                     # no valid value: index 0
    R[5, V - 1] = 50.0                   # the last row of the last shard
    return R


def _worker(rank, world, port, V, q):
    try:
        sys.path.insert(0, REPO)
        import importlib

        import torch
        import torch.distributed as dist

        g = importlib.import_module("gaje-semantic-compression_b200")
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=timedelta(seconds=60))
        R = _rows(V)
        r0, n = g.vocab_shard(V, world, rank)
        keys = np.zeros(R.shape[0], dtype=np.uint64)
        for b in range(R.shape[0]):
            best = 0
            for i in range(r0, r0 + n):
                best = max(best, g.argmax_key(float(R[b, i]), i))
            keys[b] = best
        t = torch.from_numpy(keys.view(np.int64).copy())
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        allk = np.stack([o.numpy().view(np.uint64) for o in out])  # [world][rows]
        merged = allk.max(axis=0)
        q.put((rank, [g.argmax_key_index(int(k)) for k in merged], (r0, n)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e), None))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("V", [1000, 999])
def test_two_gloo_ranks_merge_to_the_first_maximum(g, V):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, V, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in range(2):
        rank, idx, shard = q.get(timeout=120)
        assert shard is not None, idx
        res[rank] = (idx, shard)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    R = _rows(V)
    expected = [_reference_argmax(R[b]) for b in range(R.shape[0])]
    assert res[0][0] == expected and res[1][0] == expected
    # the two shards tile the vocabulary
    (a0, n0), (a1, n1) = res[0][1], res[1][1]
    assert a0 == 0 and a1 == n0 and a1 + n1 == V


@pytest.mark.parametrize("V,n", [(151936, 8), (151936, 3), (49152, 4), (10, 4), (7, 8)])
def test_vocab_shards_tile_the_vocabulary(g, V, n):
    end = 0
    for r in range(n):
        r0, rows = g.vocab_shard(V, n, r)
        assert r0 == min(V, end) and rows >= 0
        end = r0 + rows
    assert end == V
    chunk = -(-V // n)
    assert g.vocab_shard(V, n, 0) == (0, min(chunk, V))


def test_argmax_key_orders_value_then_lower_index(g):
    k = g.argmax_key
    assert k(1.0, 5) > k(1.0, 6) > k(0.5, 0)
    assert k(-0.0, 3) == k(0.0, 3)
    assert k(float("nan"), 0) == 0 and k(float("-inf"), 0) == 0
    assert k(-1e30, 0) > 0
    assert g.argmax_key_index(k(2.5, 123456)) == 123456
