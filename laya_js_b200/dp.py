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
- ``run_data_parallel_store``: the same through a key-value store with rank 0
  coordinating, so that a rank that dies or hangs (which no collective
  survives) has its prompts re-run on the others after a timeout.
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


def run_data_parallel_store(costs: Sequence[float], worker: Callable[[list[int]], list], rank: int, world: int, store,
                            timeout_s: float = 60.0, max_rounds: int = 4, tag: str = "dp", poll_s: float = 0.005) -> list:
    """The same result as ``run_data_parallel``, also when a rank dies or hangs.

    A collective cannot outlive a dead peer, so the exchange goes through a
    key-value store (``torch.distributed.TCPStore`` or anything with
    ``set(key, bytes)``, ``get(key)`` and ``check([key]) -> bool``) hosted by
    rank 0, which also coordinates: each round it publishes the plan (LPT
    shards of the unfinished prompts over the ranks it still counts as
    healthy), every rank runs its part and publishes its outcome, and rank 0
    waits for each outcome up to ``timeout_s``. A rank whose worker raised,
    or whose outcome did not arrive in time (the process died, or hangs), is
    dropped and its prompts go to the others in the next round. Rank 0 then
    publishes every prompt's result (or the failure), waits (up to
    ``timeout_s``) until every rank not given up for lost has read it, and
    every rank returns it. Rank 0 must survive: it holds the store."""
    import pickle
    import time

    def key(*parts) -> str:
        return "/".join([tag, *map(str, parts)])

    def wait_key(k: str, deadline: float | None) -> bool:
        while not store.check([k]):
            if deadline is not None and time.monotonic() > deadline:
                return False
            time.sleep(poll_s)
        return True

    def run_part(mine: list[int]):
        try:
            return ("ok", mine, worker(mine) if mine else [])
        except Exception as e:  # noqa: BLE001 — reported to the coordinator
            return ("error", mine, f"{type(e).__name__}: {e}")

    n = len(costs)
    if rank != 0:
        for r in range(max_rounds):
            plan_key, final_key = key("plan", r), key("final")
            while not (store.check([plan_key]) or store.check([final_key])):
                time.sleep(poll_s)
            if store.check([final_key]):
                break
            plan = pickle.loads(store.get(plan_key))
            if rank in plan:
                store.set(key("res", r, rank), pickle.dumps(run_part(plan[rank])))
        wait_key(key("final"), None)
        status, payload = pickle.loads(store.get(key("final")))
        store.set(key("ack", rank), b"1")  # rank 0 may now take the store down
        if status != "ok":
            raise RuntimeError(payload)
        return payload

    results: list = [None] * n
    done = [False] * n
    healthy = list(range(world))
    pending = list(range(n))
    lost: set = set()  # ranks whose outcome never arrived (dead or hung)
    error = None
    for r in range(max_rounds):
        if not pending:
            break
        if not healthy:
            error = "run_data_parallel_store: no healthy rank left"
            break
        shards = lpt_shards([costs[i] for i in pending], len(healthy))
        plan = {h: [pending[j] for j in shards[k]] for k, h in enumerate(healthy)}
        store.set(key("plan", r), pickle.dumps(plan))
        outcomes = {0: run_part(plan[0])} if 0 in plan else {}
        deadline = time.monotonic() + timeout_s
        for h in healthy:
            if h == 0:
                continue
            k = key("res", r, h)
            outcomes[h] = pickle.loads(store.get(k)) if wait_key(k, deadline) else ("lost", plan[h], None)
        failed = []
        for h, (status, idx, payload) in outcomes.items():
            if status == "lost":
                lost.add(h)
            if status == "ok":
                for i, v in zip(idx, payload):
                    results[i] = v
                    done[i] = True
            else:
                failed.append(h)
        healthy = [h for h in healthy if h not in failed]
        pending = [i for i in range(n) if not done[i]]
    if error is None and pending:
        error = f"run_data_parallel_store: {len(pending)} prompts unfinished after {max_rounds} rounds"
    store.set(key("final"), pickle.dumps(("ok", results) if error is None else ("error", error)))
    # every rank that may still be alive reads the result before rank 0 (and the store) may go away
    deadline = time.monotonic() + timeout_s
    for h in range(1, world):
        if h not in lost:
            wait_key(key("ack", h), deadline)
    if error is not None:
        raise RuntimeError(error)
    return results
