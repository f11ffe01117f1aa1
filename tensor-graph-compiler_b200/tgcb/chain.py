"""Static work lists for a chain of two SM-pair GEMMs run by one persistent launch.

The second GEMM of a chain reads the first one's output rows as its A operand (an MLP block:
``h = act(x @ W1 + b1)``, ``y = h @ W2 + b2``). In one launch the pairs of SMs work through
a fixed list of items each: item ``t < tiles1`` is output tile ``t`` of the first GEMM and
item ``tiles1 + t`` tile ``t`` of the second; a second-GEMM tile waits (on the device) until
every first-GEMM tile of its 256-row block is stored. Run as two launches, the second GEMM
starts only when the first one's last partial wave and its epilogue are done; in one launch a
pair that runs out of first-GEMM tiles goes on with second-GEMM tiles whose rows are ready.

The lists come from a list-scheduling simulation with a cost per tile linear in its k-blocks
(``k_blocks + TILE_OVERHEAD``): every first-GEMM tile in row-major order (so row blocks
complete in order), then every second-GEMM tile in row-major order, each to the pair that is
free first, a second-GEMM tile starting no earlier than its row block is stored. Taking
second-GEMM tiles early, as soon as their rows are ready, simulates a little shorter but
measured slower on B200 (MLP block: 214.5 us against 212.1 us for this order), so it is not
done. Every list this module returns has passed ``check``: each item appears exactly once and
the waits cannot form a cycle, whatever the real durations.
"""

from __future__ import annotations

import heapq
from collections import deque

from tgcb.errors import CodegenError

# Fixed time per tile in k-block units (tile setup, first loads, the share of the epilogue that
# does not overlap), fitted to the MLP block's measured tile times on B200: 15 us for 32
# k-blocks and 52 us for 128.
TILE_OVERHEAD = 7
# A first-GEMM tile's rows are in memory an epilogue after its MMAs finish (6.3 us for a
# 128 x 256 half-tile on B200, about 16 k-blocks of MMA time): the time a row block becomes
# readable lags the end of its last tile's MMAs by this much.
STORE_DELAY = 16


def tile_cost(k_blocks: int) -> int:
    return k_blocks + TILE_OVERHEAD


def _simulate(tiles1: int, tiles_n1: int, cost1: int, tiles2: int, tiles_n2: int, cost2: int,
              pairs: int) -> tuple[int, list[list[int]]]:
    rows = tiles1 // tiles_n1
    free = [(0, p) for p in range(pairs)]
    heapq.heapify(free)
    stored_at = [0] * rows
    lists: list[list[int]] = [[] for _ in range(pairs)]
    makespan = 0
    for i in range(tiles1):
        t, p = heapq.heappop(free)
        end = t + cost1
        r = i // tiles_n1
        stored_at[r] = max(stored_at[r], end + STORE_DELAY)
        lists[p].append(i)
        makespan = max(makespan, end)
        heapq.heappush(free, (end, p))
    for j in range(tiles2):
        t, p = heapq.heappop(free)
        end = max(t, stored_at[j // tiles_n2]) + cost2
        lists[p].append(tiles1 + j)
        makespan = max(makespan, end)
        heapq.heappush(free, (end, p))
    return makespan, lists


def check(lists: list[list[int]], tiles1: int, tiles_n1: int, tiles2: int, tiles_n2: int) -> None:
    """Raise CodegenError unless every item appears once and the waits form no cycle.

    The waits are: each item after the previous item of its pair, and each second-GEMM tile
    after every first-GEMM tile of its row block. Without a cycle, some pair can always make
    progress, so the launch finishes whatever the tile durations are.
    """
    total = tiles1 + tiles2
    seen = sorted(t for lst in lists for t in lst)
    if seen != list(range(total)):
        raise CodegenError("chain schedule does not list every tile exactly once")
    succ: list[list[int]] = [[] for _ in range(total)]
    indeg = [0] * total
    for lst in lists:
        for a, b in zip(lst, lst[1:]):
            succ[a].append(b)
            indeg[b] += 1
    rows = tiles1 // tiles_n1
    firsts = [[r * tiles_n1 + j for j in range(tiles_n1)] for r in range(rows)]
    for t in range(tiles2):
        r = t // tiles_n2
        for a in firsts[r]:
            succ[a].append(tiles1 + t)
            indeg[tiles1 + t] += 1
    queue = deque(i for i in range(total) if indeg[i] == 0)
    done = 0
    while queue:
        a = queue.popleft()
        done += 1
        for b in succ[a]:
            indeg[b] -= 1
            if indeg[b] == 0:
                queue.append(b)
    if done != total:
        raise CodegenError("chain schedule has waits that form a cycle")


def schedule(tiles1: int, tiles_n1: int, k_blocks1: int, tiles2: int, tiles_n2: int, k_blocks2: int,
             pairs: int) -> tuple[list[list[int]], float]:
    """Per-pair item lists for a chain and their simulated makespan (k-block units)."""
    if tiles1 % tiles_n1 or tiles2 % tiles_n2 or tiles1 // tiles_n1 != tiles2 // tiles_n2:
        raise CodegenError("chain GEMMs must cover the same row blocks")
    span, lists = _simulate(tiles1, tiles_n1, tile_cost(k_blocks1), tiles2, tiles_n2, tile_cost(k_blocks2), pairs)
    check(lists, tiles1, tiles_n1, tiles2, tiles_n2)
    return lists, span


def two_launch_makespan(tiles1: int, k_blocks1: int, tiles2: int, k_blocks2: int, pairs: int) -> float:
    """The same cost model for the two GEMMs as separate round-robin launches (the second
    starts when the first one's last rows are stored)."""
    waves1 = -(-tiles1 // pairs)
    waves2 = -(-tiles2 // pairs)
    return waves1 * tile_cost(k_blocks1) + STORE_DELAY + waves2 * tile_cost(k_blocks2)
