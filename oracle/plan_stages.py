"""CPU restatement of rakkan-mesh's planStages (internal/llm/plan.go:122-207)
and sortNodes (plan.go:103-113). Test infrastructure only: the tests check
the library's rk_plan_stages against it and against the reference's own
plan_test.go cases; nothing in the library calls it.

A node is (id, speed, free, fits) where fits(from, to) says whether layers
[from, to) fit it (stageNode.fits, plan.go:31-37). Returns a list of
(from, to, id) spans, or raises ValueError where the reference returns
ErrNoStages.
"""


def sort_nodes(nodes):
    """plan.go:103-113: speed descending, then free memory descending,
    then id ascending."""
    return sorted(nodes, key=lambda n: (-n[1], -n[2], n[0]))


def plan_stages(cost, nodes, stages):
    layers = len(cost)
    # Nodes that hold no single layer are dropped (plan.go:124-131).
    nodes = [n for n in nodes if any(n[3](i, i + 1) for i in range(layers))]
    nodes = sort_nodes(nodes)

    def longest(n, at, most):  # plan.go:134-140
        k = 0
        while k < most and n[3](at, at + k + 1):
            k += 1
        return k

    if stages <= 0:  # plan.go:141-156
        out, at = [], 0
        for n in nodes:
            if at == layers:
                break
            k = longest(n, at, layers - at)
            if k > 0:
                out.append((at, at + k, n[0]))
                at += k
        if at < layers or not out:
            raise ValueError("no stages")
        return out
    nodes = nodes[:min(stages, len(nodes), layers)]  # plan.go:157
    if not nodes:
        raise ValueError("no stages")
    s = [0] * (layers + 1)  # plan.go:163-166
    for i, c in enumerate(cost):
        s[i + 1] = s[i] + c

    def cut(bound):  # plan.go:167-187
        out, at = [], 0
        for j, n in enumerate(nodes):
            left = len(nodes) - j - 1
            k = 0
            while at + k < layers - left and n[3](at, at + k + 1) and (s[at + k + 1] - s[at]) / max(n[1], 1e-9) <= bound:
                k += 1
            if k == 0:
                return None
            out.append((at, at + k, n[0]))
            at += k
        return out if at >= layers else None

    bounds = sorted({(s[j] - s[i]) / max(n[1], 1e-9) for n in nodes for i in range(layers)
                     for j in range(i + 1, layers + 1)})  # plan.go:188-196
    # slices.BinarySearchFunc over "cut(b) succeeds" (plan.go:197-206): the
    # lower-bound search the reference does, which is the first cutting
    # bound only where cutting is monotone in the bound (capacities can
    # make it not; the search's answer is the reference's either way).
    i, j = 0, len(bounds)
    while i < j:
        h = (i + j) // 2
        if cut(bounds[h]) is None:
            i = h + 1
        else:
            j = h
    if i == len(bounds):
        raise ValueError("layers do not fit")
    return cut(bounds[i])
