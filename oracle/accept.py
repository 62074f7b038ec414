"""CPU restatement of the greedy acceptance walk (test infrastructure only).

Follows accept_batch (nanovllm/speculative/jetspec/serving_ops.py:55-90): greedy tokens
are the argmax of every node's logits row (numpy argmax: the first maximal index, NaN
ranking highest, as torch.argmax); child maps are filled in node order so that the last
sibling carrying a token wins (the rule the reference's child_maps preserve,
serving_ops.py:61-63); the path starts at the root and follows children while it holds
at most max_depth + 1 nodes; the correction is the greedy token of the last node.
"""
from __future__ import annotations

import numpy as np


def child_maps(tokens, parents):
    """children[n][token] = the last child of node n carrying that token."""
    children = [dict() for _ in tokens]
    for node, (token, parent) in enumerate(zip(tokens, parents)):
        if parent >= 0:
            children[parent][int(token)] = node
    return children


def accept_batch(logits, token_ids, parent_indices, depths, offsets, max_depth):
    """One result dict per request, as the reference's accept_batch returns."""
    logits = np.asarray(logits, dtype=np.float64)
    greedy_all = np.argmax(logits, axis=-1)
    results = []
    for r in range(len(offsets) - 1):
        lo, hi = int(offsets[r]), int(offsets[r + 1])
        tokens = [int(t) for t in token_ids[lo:hi]]
        parents = [int(t) for t in parent_indices[lo:hi]]
        depth = [int(t) for t in depths[lo:hi]]
        greedy = [int(g) for g in greedy_all[lo:hi]]
        children = child_maps(tokens, parents)
        path = [0]
        while len(path) <= max_depth:
            child = children[path[-1]].get(greedy[path[-1]])
            if child is None:
                break
            path.append(child)
        if [depth[node] for node in path] != list(range(len(path))):
            raise RuntimeError("accepted RoPE positions do not match canonical tail")
        correction = greedy[path[-1]]
        results.append({"path": path, "accepted_length": len(path) - 1,
                        "correction": correction,
                        "outputs": [tokens[node] for node in path[1:]] + [correction]})
    return results
