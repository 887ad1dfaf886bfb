"""Multi-GPU partitioning of the two hot paths (one process per GPU).

Both paths shard without any data-path collective:

* dual GEMM: output columns are independent, so rank r owns the N-rows
  [r*N/P, (r+1)*N/P) of B1/B2 (and the matching scale atoms), A is
  replicated, and C[:, shard] stays on the rank.  Shards are multiples of 128
  rows so each rank's slice of the permuted scale tensor is a contiguous run
  of whole 128-row atom blocks;
* grouped GEMM: groups (experts) are independent; they are assigned to ranks
  by longest-processing-time bin packing on the cost M_g*N_g*K_g, and each
  C_g stays on its owner.
"""
from __future__ import annotations

import heapq


def n_shard(n_global: int, world: int, rank: int, align: int = 128) -> tuple[int, int]:
    """[start, stop) of rank's column shard; shards are `align`-row multiples
    except possibly the last (which takes the remainder)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    units = -(-n_global // align)
    base, extra = divmod(units, world)
    start_u = rank * base + min(rank, extra)
    stop_u = start_u + base + (1 if rank < extra else 0)
    return min(start_u * align, n_global), min(stop_u * align, n_global)


def lpt_assign(costs: list[float], world: int) -> list[list[int]]:
    """Longest-processing-time-first assignment of items to `world` bins.
    Returns per-rank lists of item indices (each list in ascending order)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0.0, r) for r in range(world)]
    bins: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(costs)), key=lambda i: (-costs[i], i)):
        load, r = heapq.heappop(heap)
        bins[r].append(i)
        heapq.heappush(heap, (load + costs[i], r))
    return [sorted(b) for b in bins]


def imbalance(costs: list[float], bins: list[list[int]]) -> float:
    """max bin load / mean bin load (1.0 = perfect)."""
    loads = [sum(costs[i] for i in b) for b in bins]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean > 0 else 1.0
