"""Draft-tree topology helpers (host side), mirroring QAttention's ``src/tree_mask.py``.

Same names, arguments and results as the reference (file:line there):
  num_tree_nodes / build_tree / ancestors   src/tree_mask.py:78-126
  build_pruned_tree                          src/tree_mask.py:129-214
  sample_balanced_tree_nodes                 src/tree_mask.py:219-296
  tree_attention_mask(_n/_pruned)            src/tree_mask.py:301-386
  full_sequence_mask                         src/tree_mask.py:389-420
  verify_tree_mask                           src/tree_mask.py:436-494
The complete-tree builders are vectorised with numpy (parent(i) = (i-1)//b in
BFS order); the random builders consume the generator in the reference's
order so a seeded ``numpy.random.Generator`` yields the same tree.

``kernel_parents`` converts a ``-1``-rooted parent array to the kernel's
convention (root self-loop), as the reference's callers do
(scripts/benchmark_micro.py:283-285).
"""
from __future__ import annotations

import numpy as np

EAGLE_PRUNING_PROBABILITY = 0.3
EAGLE_PRUNING_DEPTH_SCALE = 1.05


def num_tree_nodes(branching_factor: int, depth: int) -> int:
    """Nodes of a complete b-ary tree of the given depth (d+1 for a chain)."""
    b, d = branching_factor, depth
    if b == 1:
        return d + 1
    return (b ** (d + 1) - 1) // (b - 1)


def build_tree(branching_factor: int, depth: int) -> list[int]:
    """BFS parent array of a complete b-ary tree; ``parent[0] = -1``."""
    b, d = branching_factor, depth
    if b <= 0:
        raise ValueError(f"branching_factor must be >= 1, got {b}")
    if d < 0:
        raise ValueError(f"depth must be >= 0, got {d}")
    n = num_tree_nodes(b, d)
    par = np.empty(n, dtype=np.int64)
    par[0] = -1
    par[1:] = (np.arange(1, n, dtype=np.int64) - 1) // b
    return par.tolist()


def ancestors(node: int, parent_array: list[int]) -> set[int]:
    """Ancestors of ``node`` including itself (path to the root)."""
    out: set[int] = set()
    cur = node
    while cur != -1:
        out.add(cur)
        cur = parent_array[cur]
    return out


def _mask_from_parents(parent: np.ndarray) -> np.ndarray:
    """mask[i, j] = j is on the root path of i, by repeated parent lookup on all rows at once."""
    n = parent.shape[0]
    mask = np.zeros((n, n), dtype=bool)
    rows = np.arange(n)
    cur = np.arange(n)
    alive = np.ones(n, dtype=bool)
    while alive.any():
        mask[rows[alive], cur[alive]] = True
        nxt = np.where(alive, parent[np.where(alive, cur, 0)], -1)
        alive = nxt >= 0
        cur = np.where(alive, nxt, 0)
    return mask


def tree_attention_mask(branching_factor: int, depth: int) -> np.ndarray:
    """``[N, N]`` bool mask of the complete tree: True iff j in ancestors(i)."""
    return _mask_from_parents(np.asarray(build_tree(branching_factor, depth), dtype=np.int64))


def tree_attention_mask_n(branching_factor: int, N: int) -> np.ndarray:
    """Ancestor mask of the first ``N`` BFS nodes of a b-ary tree."""
    parent = np.empty(N, dtype=np.int64)
    if N:
        parent[0] = -1
        parent[1:] = (np.arange(1, N, dtype=np.int64) - 1) // branching_factor
    return _mask_from_parents(parent)


def tree_attention_mask_pruned(parent_array: list[int]) -> np.ndarray:
    """Ancestor mask of an explicit (possibly pruned) tree, ``parent[root] = -1``."""
    return _mask_from_parents(np.asarray(parent_array, dtype=np.int64))


def full_sequence_mask(ctx_len: int, branching_factor: int, depth: int) -> np.ndarray:
    """Mask of ``[context | tree]``: causal context, tree rows see all context + ancestors."""
    N = num_tree_nodes(branching_factor, depth)
    total = ctx_len + N
    mask = np.zeros((total, total), dtype=bool)
    mask[:ctx_len, :ctx_len] = np.tril(np.ones((ctx_len, ctx_len), dtype=bool))
    mask[ctx_len:, :ctx_len] = True
    mask[ctx_len:, ctx_len:] = tree_attention_mask(branching_factor, depth)
    return mask


def kernel_parents(parent_array) -> np.ndarray:
    """int32 parents with the root as a self-loop (the kernel's convention)."""
    p = np.asarray(parent_array, dtype=np.int64).copy()
    roots = p < 0
    p[roots] = np.nonzero(roots)[0]
    return p.astype(np.int32)


def build_pruned_tree(
    branching_factor: int,
    max_depth: int,
    target_nodes: int | None = None,
    pruning_prob: float = EAGLE_PRUNING_PROBABILITY,
    pruning_depth_scale: float = EAGLE_PRUNING_DEPTH_SCALE,
    rng: np.random.Generator | None = None,
) -> list[int]:
    """EAGLE-like pruned tree in BFS order (``parent[0] = -1``).

    Level by level, each frontier node below ``max_depth`` keeps each of its
    ``b`` potential children with probability ``1 - min(p * s**depth, 0.95)``
    (a chain always keeps its one child); stops once ``target_nodes`` is
    reached. Draws ``b`` uniforms per expanded node, in frontier order.
    """
    if rng is None:
        rng = np.random.default_rng()
    parent: list[int] = [-1]
    frontier: list[tuple[int, int]] = [(0, 0)]
    while frontier:
        nxt: list[tuple[int, int]] = []
        hit = False
        for node, depth in frontier:
            if depth >= max_depth:
                continue
            if branching_factor == 1:
                kids = 1
            else:
                p = min(pruning_prob * (pruning_depth_scale ** depth), 0.95)
                kids = sum(rng.random() > p for _ in range(branching_factor))
            for _ in range(kids):
                nxt.append((len(parent), depth + 1))
                parent.append(node)
            if target_nodes is not None and len(parent) >= target_nodes:
                hit = True
                break
        frontier = nxt
        if hit:
            break
    return parent


def sample_balanced_tree_nodes(
    branching_factor: int,
    max_depth: int,
    num_nodes: int,
    rng: np.random.Generator | None = None,
) -> list[int]:
    """Random BFS-connected subset of a complete tree with about ``num_nodes`` nodes.

    If the complete tree has at most 1.2x ``num_nodes`` nodes, its first
    ``num_nodes`` BFS nodes are returned. Otherwise children (BFS index
    ``node*b + k``) are kept level by level with probability
    ``min(1, remaining / (children + 1))``; kept nodes are renumbered by BFS rank.
    """
    if rng is None:
        rng = np.random.default_rng()
    b = branching_factor
    full = build_tree(b, max_depth)
    n_full = len(full)
    if n_full <= num_nodes * 1.2:
        return full[:num_nodes]
    kept = {0}
    frontier = [0]
    while len(kept) < num_nodes and frontier:
        nxt = []
        for node in frontier:
            remaining = num_nodes - len(kept)
            children = sum(1 for k in range(1, b + 1) if node * b + k < n_full)
            keep_p = min(1.0, remaining / (children + 1)) if (children > 0 and remaining > 0) else 0.0
            for k in range(1, b + 1):
                child = node * b + k
                if child < n_full and len(kept) < num_nodes:
                    if rng.random() < keep_p:
                        kept.add(child)
                        nxt.append(child)
        frontier = nxt
    order = sorted(kept)
    rank = {n: i for i, n in enumerate(order)}
    return [-1 if full[n] == -1 else rank[full[n]] for n in order]


def _node_depths(parent: np.ndarray) -> np.ndarray:
    depth = np.zeros(parent.shape[0], dtype=np.int64)
    for i in range(parent.shape[0]):  # BFS order: parent precedes child
        depth[i] = 0 if parent[i] < 0 else depth[parent[i]] + 1
    return depth


def verify_tree_mask(branching_factor: int, depth: int, verbose: bool = True) -> bool:
    """Structural checks: reflexive, exact ancestor sets, no sibling edges, row sum = depth+1."""
    parent = build_tree(branching_factor, depth)
    mask = tree_attention_mask(branching_factor, depth)
    n = len(parent)
    ok = bool(np.all(np.diag(mask)))
    for i in range(n):
        exp = np.zeros(n, dtype=bool)
        exp[list(ancestors(i, parent))] = True
        ok &= bool(np.array_equal(mask[i], exp))
    ok &= bool(np.array_equal(mask.sum(1), _node_depths(np.asarray(parent)) + 1))
    if verbose:
        print(f"[verify_tree_mask] b={branching_factor} d={depth} N={n}  ->  {'PASS' if ok else 'FAIL'}")
    return ok
