"""Data-parallel sharding and failure handling on the host (gloo, world 2, no GPU)."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch.distributed as dist
import torch.multiprocessing as mp

from laya_js_b200.dp import lpt_shards, prompt_cost, run_data_parallel


def test_lpt_balances_and_covers():
    rng = np.random.default_rng(0)
    lens = rng.integers(32, 513, size=256)
    costs = [prompt_cost(int(L)) for L in lens]
    for world in (1, 2, 4, 8):
        shards = lpt_shards(costs, world)
        assert sorted(i for s in shards for i in s) == list(range(256))
        loads = [sum(costs[i] for i in s) for s in shards]
        assert max(loads) / (sum(loads) / world) < 1.02


def test_prompt_cost_grows_superlinearly():
    assert prompt_cost(512) > 2 * prompt_cost(256) > 4 * prompt_cost(128) * 0.99


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, fail_rank, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        costs = [float(L) for L in range(10, 30)]
        calls = {"n": 0}

        def worker(idx):
            calls["n"] += 1
            if rank == fail_rank and calls["n"] == 1:
                raise RuntimeError("injected worker failure")
            return [i * i for i in idx]

        def gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        res = run_data_parallel(costs, worker, rank, world, gather)
        q.put((rank, res))
    finally:
        dist.destroy_process_group()


def _spawn(fail_rank):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank_main, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=120) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return got


def test_gloo_world2_all_results():
    got = _spawn(fail_rank=-1)
    want = [i * i for i in range(20)]
    assert got[0] == want and got[1] == want


def test_gloo_world2_failed_rank_is_resharded():
    """Rank 1's worker raises: its prompts move to rank 0, every prompt still gets a result."""
    got = _spawn(fail_rank=1)
    want = [i * i for i in range(20)]
    assert got[0] == want and got[1] == want


def _encoder_rank(rank, world, port, fail_rank, q):
    """One rank: an encoder worker (the C++ CPU encoder stands in for the GPU
    one on these CPU ranks) over its LPT shard of 24 prompts; probabilities of
    every prompt gathered on the host."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from laya_js_b200 import workloads as WL
        from oracle import cpu
        cfg = {**WL.BASE, "num_hidden_layers": 2, "vocab_size": 1024}
        W = WL.random_weights(cfg, seed=5)
        hw, hb = WL.classifier(cfg, 8, seed=6)
        lens = WL.lengths(24, 8, 96, seed=7)
        ids, cu = WL.token_batch(cfg, lens, seed=8)
        enc = cpu.Encoder(cfg, W)
        calls = {"n": 0}

        def worker(idx):
            calls["n"] += 1
            if rank == fail_rank and calls["n"] == 1:
                raise RuntimeError("injected worker failure")
            _, probs, _ = enc.forward([ids[cu[i]:cu[i + 1]] for i in idx], hw, hb, threads=1, want_hidden=False)
            return [p for p in probs]

        def gather(obj):
            out = [None] * world
            dist.all_gather_object(out, obj)
            return out

        res = run_data_parallel([prompt_cost(int(L), layers=2) for L in lens], worker, rank, world, gather)
        q.put((rank, np.stack(res)))
    finally:
        dist.destroy_process_group()


def _spawn_encoder(fail_rank):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_encoder_rank, args=(r, world, port, fail_rank, q)) for r in range(world)]
    for p in ps:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(world))
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    return got


def test_gloo_world2_encoder_worker_matches_one_process():
    """run_data_parallel driving an encoder on two gloo ranks gives every
    prompt's probabilities, equal to one process running the whole batch;
    with a rank failing its first shard, its prompts are re-run on the other."""
    from laya_js_b200 import workloads as WL
    from oracle import cpu
    cfg = {**WL.BASE, "num_hidden_layers": 2, "vocab_size": 1024}
    W = WL.random_weights(cfg, seed=5)
    hw, hb = WL.classifier(cfg, 8, seed=6)
    lens = WL.lengths(24, 8, 96, seed=7)
    ids, cu = WL.token_batch(cfg, lens, seed=8)
    _, want, _ = cpu.Encoder(cfg, W).forward([ids[cu[i]:cu[i + 1]] for i in range(len(lens))], hw, hb, threads=1, want_hidden=False)
    for fail in (-1, 1):
        got = _spawn_encoder(fail)
        assert np.array_equal(got[0], want) and np.array_equal(got[1], want), f"fail_rank={fail}"
