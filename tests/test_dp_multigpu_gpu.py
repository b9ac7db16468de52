"""Data parallel over two GPUs with a rank that dies (needs 2 GPUs; skipped
otherwise). Each rank is a child process with its own GPU and a full weight
replica, running the fused encoder on its LPT shard through
run_data_parallel_store (rank 0 coordinates through a TCPStore). In the
fault case rank 1's process exits inside its first worker call, before that
call launches anything (a rank leaves between steps, never with a kernel in
flight; no collective and no NVLink multicast is involved). Rank 0 re-runs
rank 1's prompts after the timeout; every prompt's probabilities must match a
single-process forward of the whole batch."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus() -> int:
    import torch
    return torch.cuda.device_count()


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, fault, q):
    from datetime import timedelta

    from torch.distributed import TCPStore

    from laya_js_b200 import createCudaBackend, workloads as WL
    from laya_js_b200.dp import prompt_cost, run_data_parallel_store
    from laya_js_b200.encoder import FusedEncoder
    from laya_js_b200.host import HostTensor
    from laya_js_b200.modernbert import loadModernBert, parseModernBertConfig
    try:
        store = TCPStore("127.0.0.1", port, world, rank == 0, timedelta(seconds=120), wait_for_workers=False)
        b = createCudaBackend(rank)
        cfg = {**WL.BASE, "num_hidden_layers": 2}
        enc = loadModernBert(b, parseModernBertConfig(cfg), WL.host_getter(WL.random_weights(cfg, seed=3)), "f16")
        fused = FusedEncoder(enc)
        hw, hb = WL.classifier(cfg, 8, seed=4)
        thw, thb = b.fromHost(HostTensor("f16", hw.shape, hw)), b.fromHost(HostTensor("f32", hb.shape, hb))
        lens = WL.lengths(24, 16, 300, seed=5)
        ids, cu = WL.token_batch(cfg, lens, seed=6)

        def forward(idx):
            parts = [ids[cu[i]:cu[i + 1]] for i in idx]
            sub = np.concatenate(parts).astype(np.int32)
            scu = np.concatenate([[0], np.cumsum([len(p) for p in parts])]).astype(np.int32)
            out = np.empty((len(idx), hw.shape[0]), np.float32)
            fused.forward_host(sub, scu, thw, thb, out=out)
            return out

        calls = {"n": 0}

        def worker(idx):
            calls["n"] += 1
            if rank == fault and calls["n"] == 1:
                os._exit(3)  # the rank leaves before this step launches anything
            return list(forward(idx))

        res = run_data_parallel_store([prompt_cost(int(L), layers=2) for L in lens], worker, rank, world, store, timeout_s=20.0)
        got = np.stack(res)
        want = forward(list(range(len(lens))))
        q.put((rank, float(np.abs(got - want).max()), bool((got.argmax(1) == want.argmax(1)).all())))
    except Exception as e:  # noqa: BLE001 — reported to the test
        q.put((rank, f"{type(e).__name__}: {e}", False))


def _run(fault):
    import torch.multiprocessing as mp
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_rank, args=(r, world, port, fault, q)) for r in range(world)]
    for p in ps:
        p.start()
    survivors = [r for r in range(world) if r != fault]
    got = dict((r, (e, a)) for r, e, a in (q.get(timeout=600) for _ in survivors))
    for r, p in enumerate(ps):
        p.join(timeout=120)
        assert p.exitcode == (3 if r == fault else 0), f"rank {r} exit code {p.exitcode}"
    return got


@pytest.mark.skipif(_gpus() < 2, reason="needs two GPUs")
@pytest.mark.parametrize("fault", [-1, 1])
def test_two_gpu_shards_with_and_without_a_dead_rank(fault):
    got = _run(fault)
    for r, (err, argmax_same) in got.items():
        assert not isinstance(err, str), f"rank {r}: {err}"
        assert err < 2e-3 and argmax_same, f"rank {r}: probabilities differ from one process by {err}"
