"""Host-side helpers for speculative verification over the paged cache.

Nothing here has a counterpart in the reference (it has no speculative
decoding); this is the integer bookkeeping around ``ops.tree_attention`` and
``ops.kv_move``:

* ``build_draft_tree``  — the EAGLE3-style static draft tree: node 0 is the
  root (the last sampled token, not yet in the cache), level l nodes have
  ``branching[l]`` children each. Truncation to ``max_nodes`` is
  deterministic: root, then the leftmost chain down to full depth, then the
  remaining nodes in breadth-first order. Nodes are numbered in BFS order of
  the full tree, so every parent precedes its children.
* ``ancestor_masks``    — one uint64 per node: bit i set iff node i is the node
  itself or one of its ancestors (the verification mask).
* ``chain_masks``       — the mask of a linear draft (n-gram / single chain).
* ``ngram_draft``       — prompt-lookup drafting: find the latest earlier
  occurrence of the trailing n-gram and propose the tokens that followed it.
* ``greedy_accept``     — walk the tree with the target model's argmax.
* ``compaction_moves``  — cache slot moves that pack an accepted path to
  consecutive positions after the committed context.
"""
from __future__ import annotations

import numpy as np

MAX_TREE_NODES = 64


def build_draft_tree(branching=(4, 3, 2, 1, 1, 1), max_nodes: int = MAX_TREE_NODES):
    """Return (parents, depths) int32 arrays of the truncated draft tree."""
    if max_nodes < 1 or max_nodes > MAX_TREE_NODES:
        raise ValueError(f"max_nodes must be in [1, {MAX_TREE_NODES}]")
    # Full tree in BFS order.
    parents = [-1]
    depths = [0]
    level = [0]
    for d, br in enumerate(branching):
        nxt = []
        for node in level:
            for _ in range(br):
                parents.append(node)
                depths.append(d + 1)
                nxt.append(len(parents) - 1)
        level = nxt
    n_full = len(parents)
    children = [[] for _ in range(n_full)]
    for i in range(1, n_full):
        children[parents[i]].append(i)
    keep = [0]
    # Leftmost chain to full depth.
    node = 0
    while children[node] and len(keep) < max_nodes:
        node = children[node][0]
        keep.append(node)
    chosen = set(keep)
    for i in range(1, n_full):
        if len(keep) >= max_nodes:
            break
        if i not in chosen:
            keep.append(i)
            chosen.add(i)
    keep.sort()  # BFS order of the full tree: parents first
    remap = {old: new for new, old in enumerate(keep)}
    out_par = np.array([-1 if parents[o] < 0 else remap[parents[o]] for o in keep], dtype=np.int32)
    out_dep = np.array([depths[o] for o in keep], dtype=np.int32)
    return out_par, out_dep


def ancestor_masks(parents: np.ndarray) -> np.ndarray:
    """uint64 per node: bits of the node and all its ancestors (parents < child)."""
    n = len(parents)
    if n > MAX_TREE_NODES:
        raise ValueError("at most 64 nodes fit a 64-bit mask")
    masks = np.zeros(n, dtype=np.uint64)
    for j in range(n):
        p = int(parents[j])
        if p >= j:
            raise ValueError("parents must precede children")
        masks[j] = np.uint64(1 << j) | (masks[p] if p >= 0 else np.uint64(0))
    return masks


def chain_masks(n: int) -> np.ndarray:
    """Masks of a linear draft of n tokens: row j sees rows 0..j."""
    if n > MAX_TREE_NODES:
        raise ValueError("at most 64 nodes")
    return np.array([(1 << (j + 1)) - 1 for j in range(n)], dtype=np.uint64)


def ngram_draft(tokens, num_draft: int = 8, max_n: int = 3, min_n: int = 1) -> list[int]:
    """Prompt-lookup draft: continue the latest earlier match of the last n-gram.

    Tries n = max_n .. min_n; returns up to num_draft tokens ([] if no match).
    """
    toks = list(tokens)
    L = len(toks)
    for n in range(max_n, min_n - 1, -1):
        if L <= n:
            continue
        tail = toks[L - n:]
        for start in range(L - n - 1, -1, -1):
            if toks[start:start + n] == tail:
                follow = toks[start + n:start + n + num_draft]
                if follow:
                    return follow
    return []


def greedy_accept(parents: np.ndarray, draft_tokens: np.ndarray,
                  target_argmax: np.ndarray) -> list[int]:
    """Accepted path (node indices, root first) under greedy verification.

    draft_tokens[j] is node j's token (root's entry unused); target_argmax[j]
    is the target model's argmax after node j.
    """
    n = len(parents)
    children = [[] for _ in range(n)]
    for j in range(1, n):
        children[int(parents[j])].append(j)
    path = [0]
    node = 0
    while True:
        want = int(target_argmax[node])
        nxt = next((c for c in children[node] if int(draft_tokens[c]) == want), None)
        if nxt is None:
            return path
        path.append(nxt)
        node = nxt


def compaction_moves(context_len: int, path: list[int], block_table: list[int],
                     block_size: int) -> tuple[list[int], list[int]]:
    """Slot moves packing path node path[k] (at position context_len+path[k])
    to position context_len+k. Nodes already in place are skipped."""
    src, dst = [], []
    for k, node in enumerate(path):
        if node == k:
            continue
        ps, pd = context_len + node, context_len + k
        src.append(block_table[ps // block_size] * block_size + ps % block_size)
        dst.append(block_table[pd // block_size] * block_size + pd % block_size)
    return src, dst
