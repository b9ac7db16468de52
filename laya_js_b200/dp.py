"""Data-parallel serving over the GPUs of one box: prompts are independent, so
each rank holds a full weight replica and runs its own shard; only results
(class probabilities / logits) travel back, on the host. No collective runs
on the data path — ``torch.distributed`` (gloo or NCCL) carries the host-side
bookkeeping only.

- ``prompt_cost``: relative cost of one prompt of L tokens (linear layers ∝ L,
  global attention ∝ L², sliding ∝ L·window).
- ``lpt_shards``: longest-processing-time assignment of prompts to ranks.
- ``run_data_parallel``: every rank runs ``worker(indices)`` on its shard; a
  shard whose worker raises is reported to all ranks (a host-side all-gather
  of the outcome) and re-sharded over the ranks that succeeded, until every
  prompt has a result or no healthy rank is left.
"""
from __future__ import annotations

import heapq
from typing import Callable, Sequence


def prompt_cost(L: int, hidden: int = 768, intermediate: int = 1152, layers: int = 22, global_every: int = 3,
                window: int = 128) -> float:
    """FLOPs of one prompt through the encoder (the unit of load balancing)."""
    n_global = (layers + global_every - 1) // global_every
    n_local = layers - n_global
    linear = 2.0 * L * (hidden * 3 * hidden + hidden * hidden + hidden * 2 * intermediate + intermediate * hidden) * layers
    attn = 4.0 * hidden * (n_global * L * L + n_local * L * min(L, window + 1))
    return linear + attn


def lpt_shards(costs: Sequence[float], world: int) -> list[list[int]]:
    """Greedy longest-processing-time: biggest prompts first, each to the least-loaded rank."""
    if world < 1:
        raise ValueError("lpt_shards: world must be >= 1")
    heap = [(0.0, r) for r in range(world)]
    heapq.heapify(heap)
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda i: -costs[i]):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + float(costs[i]), r))
    for s in out:
        s.sort()
    return out


def run_data_parallel(costs: Sequence[float], worker: Callable[[list[int]], list], rank: int, world: int,
                      all_gather_object: Callable | None = None, max_rounds: int = 4) -> list:
    """Runs ``worker`` on this rank's shard and returns every prompt's result (on every rank).

    ``all_gather_object(obj) -> list`` exchanges one host object per rank
    (``torch.distributed.all_gather_object`` wrapped, or a fake in tests).
    A worker exception on a rank marks that rank unhealthy; its prompts are
    re-sharded over healthy ranks in the next round."""
    n = len(costs)
    results: list = [None] * n
    done = [False] * n
    healthy = list(range(world))
    if all_gather_object is None:
        if world != 1:
            raise ValueError("run_data_parallel: world > 1 needs all_gather_object")
        all_gather_object = lambda obj: [obj]
    pending = list(range(n))
    for _ in range(max_rounds):
        if not pending:
            break
        if not healthy:
            raise RuntimeError("run_data_parallel: no healthy rank left")
        shards = lpt_shards([costs[i] for i in pending], len(healthy))
        mine: list[int] = []
        if rank in healthy:
            mine = [pending[j] for j in shards[healthy.index(rank)]]
        try:
            out = ("ok", mine, worker(mine) if mine else [])
        except Exception as e:  # noqa: BLE001 — reported to every rank below
            out = ("error", mine, f"{type(e).__name__}: {e}")
        gathered = all_gather_object(out)
        failed = []
        for r, (status, idx, payload) in enumerate(gathered):
            if status == "ok":
                for i, v in zip(idx, payload):
                    results[i] = v
                    done[i] = True
            else:
                failed.append(r)
        healthy = [r for r in healthy if r not in failed]
        pending = [i for i in range(n) if not done[i]]
    if pending:
        raise RuntimeError(f"run_data_parallel: {len(pending)} prompts unfinished after {max_rounds} rounds")
    return results
