"""Static work lists for a chain of two SM-pair GEMMs run by one persistent launch.

The second GEMM of a chain reads the first one's output rows as its A operand (an MLP block:
``h = act(x @ W1 + b1)``, ``y = h @ W2 + b2``). In one launch the pairs of SMs work through
a fixed list of items each: item ``t < tiles1`` is output tile ``t`` of the first GEMM and
item ``tiles1 + t`` tile ``t`` of the second; a second-GEMM tile waits (on the device) until
every first-GEMM tile of its 256-row block is stored. Run as two launches, the second GEMM
starts only when the first one's last partial wave and its epilogue are done; in one launch a
pair that runs out of first-GEMM tiles goes on with second-GEMM tiles whose rows are ready.

The lists come from a simulation with a cost per tile linear in its k-blocks
(``k_blocks + TILE_OVERHEAD``), in which a second-GEMM tile starts no earlier than
``STORE_DELAY`` after the last first-GEMM tile of its row block ends. Two kinds of lists are
simulated and the one that ends first is kept (the balanced kind only with ``BALANCED``):

* greedy: every first-GEMM tile in row-major order, then every second-GEMM tile in row-major
  order, each to the pair that is free first;
* balanced: each pair is given a number of second-GEMM tiles (several splits of the
  second-GEMM tiles over the pairs are tried) and a quota of first-GEMM tiles that evens out
  the pairs' total work; first-GEMM tiles go in row-major order to the free pair among those
  with quota left, so row blocks still complete in order, and the second-GEMM tiles go in
  row-major order to the pairs' second-GEMM slots in the order the slots start. With two
  second-GEMM tiles for most pairs and one for the rest (the MLP block), the greedy lists give
  the pairs with one tile nothing to do for the last quarter of the launch; the balanced lists
  give them more first-GEMM tiles instead.

Every list this module returns has passed ``check``: each item appears exactly once and the
waits cannot form a cycle, whatever the real durations.
"""

from __future__ import annotations

import heapq
from collections import deque

from tgcb.errors import CodegenError

# Fixed time per tile in k-block units (tile setup and first loads that do not overlap the
# previous tile), fitted to the MLP block's tile times measured inside the chain launch on B200
# (%globaltimer stamps per tile): 12.9 us for 32 k-blocks and 48.5 us for 128.
TILE_OVERHEAD = 0.5
# A first-GEMM tile's rows are in memory an epilogue after its MMAs finish (about 7 us for a
# 128 x 256 half-tile with the GELU epilogue, 18 k-blocks of MMA time): the time a row block
# becomes readable lags the end of its last tile's MMAs by this much.
STORE_DELAY = 18
# Consider the balanced lists too (they simulate 2.7% shorter for the MLP block, but measured
# 0.3% slower on B200: 214.3 against 213.7 us, the same box, alternating runs), so off.
BALANCED = False


def tile_cost(k_blocks: int) -> float:
    return k_blocks + TILE_OVERHEAD


def _greedy(tiles1: int, tiles_n1: int, cost1: float, tiles2: int, tiles_n2: int, cost2: float,
            pairs: int) -> list[list[int]]:
    """First-GEMM tiles in row-major order, then second-GEMM tiles in row-major order, each to
    the pair that is free first (a second-GEMM tile no earlier than its rows are stored)."""
    rows = tiles1 // tiles_n1
    free = [(0.0, p) for p in range(pairs)]
    heapq.heapify(free)
    stored_at = [0.0] * rows
    lists: list[list[int]] = [[] for _ in range(pairs)]
    for i in range(tiles1):
        t, p = heapq.heappop(free)
        r = i // tiles_n1
        stored_at[r] = max(stored_at[r], t + cost1 + STORE_DELAY)
        lists[p].append(i)
        heapq.heappush(free, (t + cost1, p))
    for j in range(tiles2):
        t, p = heapq.heappop(free)
        lists[p].append(tiles1 + j)
        heapq.heappush(free, (max(t, stored_at[j // tiles_n2]) + cost2, p))
    return lists


def _deal_second(lists: list[list[int]], free: list[float], tiles1: int, tiles2: int, counts: list[int],
                 cost2: float) -> list[list[int]]:
    """Append the second-GEMM tiles in row-major order to the pairs' slots in the order the
    slots start (pair p has counts[p] slots, the first when its first-GEMM tiles end)."""
    slots = sorted((free[p] + k * cost2, p) for p in range(len(lists)) for k in range(counts[p]))
    for j, (_, p) in enumerate(slots):
        lists[p].append(tiles1 + j)
    return lists


def _balanced(tiles1: int, cost1: float, tiles2: int, cost2: float, counts: list[int]) -> list[list[int]]:
    """Lists in which pair p runs counts[p] second-GEMM tiles and a quota of first-GEMM tiles
    that evens out the pairs' total work (largest remainders get the leftover tiles)."""
    pairs = len(counts)
    target = (tiles1 * cost1 + tiles2 * cost2) / pairs
    raw = [max(0.0, (target - counts[p] * cost2) / cost1) for p in range(pairs)]
    scale = tiles1 / sum(raw)
    raw = [r * scale for r in raw]
    quota = [int(r) for r in raw]
    for p in sorted(range(pairs), key=lambda p: (quota[p] - raw[p], p))[: tiles1 - sum(quota)]:
        quota[p] += 1
    lists: list[list[int]] = [[] for _ in range(pairs)]
    free = [0.0] * pairs
    heap = [(0.0, p) for p in range(pairs) if quota[p] > 0]
    heapq.heapify(heap)
    for i in range(tiles1):
        t, p = heapq.heappop(heap)
        lists[p].append(i)
        free[p] = t + cost1
        quota[p] -= 1
        if quota[p]:
            heapq.heappush(heap, (free[p], p))
    return _deal_second(lists, free, tiles1, tiles2, counts, cost2)


def _splits(tiles2: int, pairs: int, most: int = 6):
    """Ways to give every pair b, b + 1, b + 2 or b + 3 second-GEMM tiles (b one below the even
    share, at most ``most`` pairs with b + 3), summing to tiles2, as per-pair counts (pairs with
    more tiles first)."""
    b = max(0, tiles2 // pairs - 1)
    rest = tiles2 - b * pairs  # tiles above b per pair, each pair taking 0-3 of them
    for n3 in range(most + 1):
        for n0 in range(pairs + 1):
            n2 = rest - 3 * n3 - (pairs - n3 - n0)
            n1 = pairs - n3 - n0 - n2
            if n1 >= 0 and n2 >= 0:
                yield [b + 3] * n3 + [b + 2] * n2 + [b + 1] * n1 + [b] * n0


def simulate(lists: list[list[int]], tiles1: int, tiles_n1: int, cost1: float, tiles2: int, tiles_n2: int,
             cost2: float) -> float:
    """Makespan of the lists: each pair runs its items in order; a second-GEMM tile starts no
    earlier than STORE_DELAY after the last first-GEMM tile of its row block ends. The lists
    must have passed ``check``."""
    rows = tiles1 // tiles_n1
    left = [tiles_n1] * rows
    stored = [0.0] * rows
    nxt = [0] * len(lists)
    free = [0.0] * len(lists)
    remaining = tiles1 + tiles2
    while remaining:
        moved = False
        for p, lst in enumerate(lists):
            while nxt[p] < len(lst):
                t = lst[nxt[p]]
                if t < tiles1:
                    free[p] += cost1
                    r = t // tiles_n1
                    left[r] -= 1
                    stored[r] = max(stored[r], free[p] + STORE_DELAY)
                else:
                    r = (t - tiles1) // tiles_n2
                    if left[r]:
                        break
                    free[p] = max(free[p], stored[r]) + cost2
                nxt[p] += 1
                remaining -= 1
                moved = True
        if not moved:
            raise CodegenError("chain schedule has waits that form a cycle")
    return max(free)


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
    c1, c2 = tile_cost(k_blocks1), tile_cost(k_blocks2)
    candidates = [_greedy(tiles1, tiles_n1, c1, tiles2, tiles_n2, c2, pairs)]
    if BALANCED and tiles1 >= pairs:
        candidates += [_balanced(tiles1, c1, tiles2, c2, counts) for counts in _splits(tiles2, pairs)]
    best = None
    for lists in candidates:
        check(lists, tiles1, tiles_n1, tiles2, tiles_n2)
        span = simulate(lists, tiles1, tiles_n1, c1, tiles2, tiles_n2, c2)
        if best is None or span < best[1]:
            best = (lists, span)
    return best


def two_launch_makespan(tiles1: int, k_blocks1: int, tiles2: int, k_blocks2: int, pairs: int) -> float:
    """The same cost model for the two GEMMs as separate round-robin launches (the second
    starts when the first one's last rows are stored)."""
    waves1 = -(-tiles1 // pairs)
    waves2 = -(-tiles2 // pairs)
    return waves1 * tile_cost(k_blocks1) + STORE_DELAY + waves2 * tile_cost(k_blocks2)
