"""CPU: a model check of the buffer reuse of ``HostPipeline.run`` (``hffn_b200/pipeline.py``).

Batch k uses device buffers x[k % depth] and y[k % depth]. Its copy in runs on the copy-in stream, its kernels on
the compute stream, its copy out on the copy-out stream; events order them, and a buffer's reuse by batch k + depth
waits for the kernels (x) or the copy out (y) of batch k. Restated here as happens-before edges (stream order plus
the event waits, each wait taking the event's latest record at issue time), every conflicting pair of accesses must
be ordered and every batch must flow copy in -> kernels -> copy out, for depths 1 to 3 and up to 7 batches."""
import itertools

import pytest


def schedule(depth: int, count: int, wait_drained: bool = True):
    ops, edges = [], []
    last = {"in": None, "compute": None, "out": None}
    record = {}                                            # (event, buffer) -> op of its latest record

    def op(stream, name, accesses):
        ops.append((name, accesses))
        node = len(ops) - 1
        if last[stream] is not None:
            edges.append((last[stream], node))
        last[stream] = node
        return node

    def wait(stream, event, b):
        source = record.get((event, b))
        if source is not None:
            node = op(stream, ("wait", event, b), [])
            edges.append((source, node))

    for k in range(count):
        b = k % depth
        if k >= depth:
            wait("in", "computed", b)
            if wait_drained:
                wait("compute", "drained", b)
        record[("loaded", b)] = op("in", ("copy_in", k), [("w", ("x", b)), ("r", ("x_host", k))])
        wait("compute", "loaded", b)
        record[("computed", b)] = op("compute", ("kernels", k), [("r", ("x", b)), ("w", ("y", b))])
        wait("out", "computed", b)
        record[("drained", b)] = op("out", ("copy_out", k), [("r", ("y", b)), ("w", ("y_host", k))])
    return ops, edges


def closure(n, edges):
    succ = [[] for _ in range(n)]
    for a, b in edges:
        succ[a].append(b)
    reach = [0] * n
    for node in range(n - 1, -1, -1):                      # every edge points to a later-created node
        bits = 1 << node
        for s in succ[node]:
            bits |= reach[s]
        reach[node] = bits
    return reach


def unordered_conflicts(ops, reach):
    regions: dict = {}
    for i, (_, accesses) in enumerate(ops):
        for mode, region in accesses:
            regions.setdefault(region, []).append((i, mode))
    bad = []
    for region, accesses in regions.items():
        for (a, ma), (b, mb) in itertools.combinations(accesses, 2):
            if "w" in (ma, mb) and not ((reach[a] >> b) & 1 or (reach[b] >> a) & 1):
                bad.append((region, ops[a][0], ops[b][0]))
    return bad


@pytest.mark.parametrize("depth,count", [(d, c) for d in (1, 2, 3) for c in (1, 2, 3, 5, 7)])
def test_reuse_is_ordered_and_batches_flow(depth, count):
    ops, edges = schedule(depth, count)
    assert all(a < b for a, b in edges)
    reach = closure(len(ops), edges)
    assert unordered_conflicts(ops, reach) == []
    index = {name: i for i, (name, _) in enumerate(ops)}
    for k in range(count):
        assert (reach[index[("copy_in", k)]] >> index[("kernels", k)]) & 1
        assert (reach[index[("kernels", k)]] >> index[("copy_out", k)]) & 1


def test_without_the_wait_for_the_copy_out_the_output_buffer_races():
    ops, edges = schedule(2, 4, wait_drained=False)
    assert any(region[0] == "y" for region, _, _ in unordered_conflicts(ops, closure(len(ops), edges)))
