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


def _store_rank(rank, world, port, fault, q):
    """One rank of run_data_parallel_store over a TCPStore held by rank 0;
    `fault` = (rank, kind): that rank's first worker call exits the process,
    hangs, or raises."""
    import time
    from datetime import timedelta

    from torch.distributed import TCPStore

    from laya_js_b200.dp import run_data_parallel_store
    store = TCPStore("127.0.0.1", port, world, rank == 0, timedelta(seconds=60), wait_for_workers=False)
    calls = {"n": 0}

    def worker(idx):
        calls["n"] += 1
        if fault[0] == rank and calls["n"] == 1:
            if fault[1] == "exit":
                os._exit(3)  # the process dies mid-run
            if fault[1] == "hang":
                time.sleep(600)
            raise RuntimeError("injected worker failure")
        return [i * i for i in idx]

    res = run_data_parallel_store([float(L) for L in range(10, 40)], worker, rank, world, store, timeout_s=3.0)
    q.put((rank, res))


def _spawn_store(fault):
    world, port = 3, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_store_rank, args=(r, world, port, fault, q)) for r in range(world)]
    for p in ps:
        p.start()
    survivors = [r for r in range(world) if not (r == fault[0] and fault[1] in ("exit", "hang"))]
    got = dict(q.get(timeout=120) for _ in survivors)
    for r, p in enumerate(ps):
        if r in survivors:
            p.join(timeout=60)
            assert p.exitcode == 0, f"rank {r} exit code {p.exitcode}"
        elif fault[1] == "exit":
            p.join(timeout=60)
            assert p.exitcode == 3
        else:
            p.kill()  # the hung rank (a child of this test)
            p.join(timeout=60)
    return got


def test_store_runner_survives_a_dead_rank():
    """Rank 2's process exits inside its worker: rank 0 stops waiting for it
    after the timeout and re-runs its prompts on ranks 0 and 1."""
    got = _spawn_store((2, "exit"))
    want = [i * i for i in range(30)]
    assert set(got) == {0, 1} and got[0] == want and got[1] == want


def test_store_runner_survives_a_hung_rank():
    got = _spawn_store((1, "hang"))
    want = [i * i for i in range(30)]
    assert set(got) == {0, 2} and got[0] == want and got[2] == want


def test_store_runner_reshards_a_raising_rank():
    got = _spawn_store((1, "raise"))
    want = [i * i for i in range(30)]
    assert got == {0: want, 1: want, 2: want}
