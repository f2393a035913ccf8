"""CPU: a model check of the buffer reuse of the peer-memory sharded forward (``hffn_peer_pipeline_run``).

The issue loop of ``hffn_b200/csrc/peer.cu`` (``PeerPipeline::run``) is restated as operations with their
happens-before edges: program order on each rank's compute stream, the order of each copy stream, the event waits
(pulls after the barrier, the compute stream after the pulls and the deliveries it waits for, deliveries after the
compute) and the barrier (every rank's operations before barrier k happen before every rank's operations after it).
Every pair of accesses to one buffer region with a write among them must be ordered, and every consumer must come
after its producer, for world sizes 1 to 8 and streams of 1 to 7 batches."""
import itertools

import pytest

SLOTS, GATHERS = 3, 2


def schedule(world: int, count: int):
    """Operations (name, rank, accesses) and happens-before edges of one ``run`` of ``count`` batches.
    An access is (mode, region) with mode "r" or "w"; regions are tuples naming a rank's buffer rows."""
    ops, edges = [], []

    def op(name, rank, accesses):
        ops.append((name, rank, accesses))
        return len(ops) - 1

    last_compute = {r: None for r in range(world)}          # program order on each compute stream
    last_pull = {(r, j): None for r in range(world) for j in range(world)}
    last_push = {(r, j): None for r in range(world) for j in range(world)}
    pulled, delivered, computed = {}, {}, {}

    def on_compute(r, node):
        if last_compute[r] is not None:
            edges.append((last_compute[r], node))
        last_compute[r] = node

    for k in range(count + 3):
        g = k % GATHERS
        arrive = {}
        for r in range(world):
            if k < count:
                on_compute(r, op(("stage", k), r, [("w", ("gather", r, g, 0))]))
            if 1 <= k <= count:
                for j in range(1, world):
                    wait = op(("wait_pull", k - 1, j), r, [])
                    edges.append((pulled[(k - 1, r, j)], wait))
                    on_compute(r, wait)
            if k >= 3:
                for j in range(world):
                    wait = op(("wait_deliver", k - 3, j), r, [])
                    edges.append((delivered[(k - 3, r, j)], wait))
                    on_compute(r, wait)
            arrive[r] = op(("barrier_arrive", k), r, [])
            on_compute(r, arrive[r])
        barrier = op(("barrier", k), -1, [])
        for r in range(world):
            edges.append((arrive[r], barrier))
        for r in range(world):
            leave = op(("barrier_leave", k), r, [])
            edges.append((barrier, leave))
            on_compute(r, leave)
            if k < count:                                   # pulls of batch k, one copy stream per position
                for j in range(1, world):
                    owner = (r + j) % world
                    pull = op(("pull", k, j), r, [("r", ("gather", owner, g, 0)), ("w", ("gather", r, g, j))])
                    edges.append((leave, pull))
                    if last_pull[(r, j)] is not None:
                        edges.append((last_pull[(r, j)], pull))
                    last_pull[(r, j)] = pull
                    pulled[(k, r, j)] = pull
            if 1 <= k <= count:                             # the shard over batch k - 1, then its deliveries
                b, slot = (k - 1) % GATHERS, (k - 1) % SLOTS
                reads = [("r", ("gather", r, b, j)) for j in range(world)]
                writes = [("w", ("partial", r, b, j)) for j in range(world)]
                compute = op(("compute", k - 1), r, reads + writes)
                on_compute(r, compute)
                computed[(k - 1, r)] = compute
                for j in range(world):
                    owner = (r + j) % world
                    push = op(("deliver", k - 1, j), r, [("r", ("partial", r, b, j)), ("w", ("slot", owner, slot, r))])
                    edges.append((compute, push))
                    if last_push[(r, j)] is not None:
                        edges.append((last_push[(r, j)], push))
                    last_push[(r, j)] = push
                    delivered[(k - 1, r, j)] = push
            if k >= 3:
                slot = (k - 3) % SLOTS
                on_compute(r, op(("sum", k - 3), r, [("r", ("slot", r, slot, p)) for p in range(world)]))
    return ops, edges


def reachability(n, edges):
    succ = [[] for _ in range(n)]
    for a, b in edges:
        succ[a].append(b)
    order, seen = [], [False] * n
    for start in range(n):                                  # depth-first post-order of the graph
        if seen[start]:
            continue
        stack = [(start, iter(succ[start]))]
        seen[start] = True
        while stack:
            node, it = stack[-1]
            nxt = next(it, None)
            if nxt is None:
                order.append(node)
                stack.pop()
            elif not seen[nxt]:
                seen[nxt] = True
                stack.append((nxt, iter(succ[nxt])))
    reach = [0] * n
    for node in order:                                      # post-order: every successor is done first
        bits = 1 << node
        for s in succ[node]:
            bits |= reach[s]
        reach[node] = bits
    return reach


def before(reach, a, b):
    return a != b and (reach[a] >> b) & 1 == 1


@pytest.mark.parametrize("world,count", [(w, c) for w in (1, 2, 3, 4, 8) for c in (1, 2, 3, 4, 7)])
def test_every_conflict_is_ordered_and_every_consumer_follows_its_producer(world, count):
    ops, edges = schedule(world, count)
    reach = reachability(len(ops), edges)
    by_region: dict = {}
    for index, (_, _, accesses) in enumerate(ops):
        for mode, region in accesses:
            by_region.setdefault(region, []).append((index, mode))
    for region, accesses in by_region.items():
        for (a, ma), (b, mb) in itertools.combinations(accesses, 2):
            if "w" in (ma, mb) and a != b:
                assert before(reach, a, b) or before(reach, b, a), (world, count, region, ops[a][0], ops[b][0])
    # data dependencies: a batch's rows are read after they are written
    index = {(name, rank): i for i, (name, rank, _) in enumerate(ops)}
    for k in range(count):
        for r in range(world):
            compute = index[(("compute", k), r)]
            assert before(reach, index[(("stage", k), r)], compute)
            for j in range(1, world):
                assert before(reach, index[(("pull", k, j), r)], compute)
                assert before(reach, index[(("stage", k), (r + j) % world)], index[(("pull", k, j), r)])
            total = index[(("sum", k), r)]
            for p in range(world):                          # rank p delivered its partial for r's tokens
                j = (r - p) % world
                assert before(reach, index[(("deliver", k, j), p)], total)


def test_a_two_deep_slot_ring_would_race():
    """The check has teeth: with two receive slots instead of three, a delivery overwrites a slot its owner is
    still summing."""
    global SLOTS
    saved, SLOTS = SLOTS, 2
    try:
        ops, edges = schedule(2, 5)
        reach = reachability(len(ops), edges)
        races = 0
        by_region: dict = {}
        for i, (_, _, accesses) in enumerate(ops):
            for mode, region in accesses:
                by_region.setdefault(region, []).append((i, mode))
        for accesses in by_region.values():
            for (a, ma), (b, mb) in itertools.combinations(accesses, 2):
                if "w" in (ma, mb) and not (before(reach, a, b) or before(reach, b, a)):
                    races += 1
        assert races > 0
    finally:
        SLOTS = saved
