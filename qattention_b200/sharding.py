"""Batch sharding of independent draft trees across the GPUs of one node.

Trees (sequences) never attend to each other, so a packed batch splits by
tree with no exchange on the hot path: rank r owns a contiguous range of
trees, runs the ancestor pass (or the whole verify attention) on its own
GPU, and one collective after the step gathers the outputs to a destination
rank. The reference parallelises the same batch axis inside one launch (its
grid is ``(B*H, ceil(max_seqlen / BLOCK_M))``, src/ragged_attn.py:1147);
here the batch axis is also the axis across GPUs.

Functions:
  shard_trees(cu_seqlens, world_size, rank)     which trees/tokens rank owns
  local_inputs(Q, K, V, cu_seqlens, shard)      views of a global packed batch
  sharded_ragged_attention_with_lse(...)        the rank's pass on its trees
  gather_outputs(O, LSE, shard, ...)            one gather of O and LSE to dst

The gather uses whatever backend the process group runs (NCCL on GPUs, gloo
for CPU tests); uneven shards are padded to the largest shard for the
collective and trimmed on the destination.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List, Optional, Sequence, Tuple

import torch


@dataclass(frozen=True)
class TreeShard:
    """A rank's contiguous range of trees in a packed batch.

    ``tree_lo:tree_hi`` index the batch, ``tok_lo:tok_hi`` the packed token
    axis; ``cu_local`` is the shard's own int32 ``cu_seqlens`` (starting at 0,
    on the CPU) and ``tokens_per_rank`` the token count of every rank's shard,
    which the gather needs.
    """

    rank: int
    world_size: int
    tree_lo: int
    tree_hi: int
    tok_lo: int
    tok_hi: int
    cu_local: torch.Tensor
    tokens_per_rank: Tuple[int, ...]

    @property
    def num_trees(self) -> int:
        return self.tree_hi - self.tree_lo

    @property
    def num_tokens(self) -> int:
        return self.tok_hi - self.tok_lo

    @property
    def max_seqlen(self) -> int:
        if self.num_trees == 0:
            return 0
        return int((self.cu_local[1:] - self.cu_local[:-1]).max())


def _split_points(cu: Sequence[int], world_size: int) -> List[int]:
    """Tree boundaries that split the batch into `world_size` contiguous groups of
    near-equal token counts (equal trees give equal tree counts).

    Boundary k is the tree index whose start offset is closest to k/world_size of
    the tokens, kept monotone, so every rank gets a contiguous range (possibly
    empty when there are fewer trees than ranks).
    """
    B = len(cu) - 1
    total = cu[-1]
    pts = [0]
    for k in range(1, world_size):
        if total == 0:
            target_tree = (k * B) // world_size
        else:
            goal = total * k / world_size
            # first tree start at or past the goal, then the nearer of it and the one before
            j = next((i for i in range(B + 1) if cu[i] >= goal), B)
            if j > 0 and goal - cu[j - 1] < cu[j] - goal:
                j -= 1
            target_tree = j
        pts.append(max(pts[-1], min(B, target_tree)))
    pts.append(B)
    return pts


def shard_trees(cu_seqlens: torch.Tensor, world_size: int, rank: int) -> TreeShard:
    """The contiguous range of trees (and packed tokens) that `rank` owns."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"rank {rank} out of range for world_size {world_size}")
    cu = [int(x) for x in cu_seqlens.detach().cpu().tolist()]
    if len(cu) < 1 or cu[0] != 0 or any(cu[i + 1] < cu[i] for i in range(len(cu) - 1)):
        raise ValueError("cu_seqlens must start at 0 and be non-decreasing")
    pts = _split_points(cu, world_size)
    lo, hi = pts[rank], pts[rank + 1]
    cu_local = torch.tensor([c - cu[lo] for c in cu[lo:hi + 1]], dtype=torch.int32)
    tokens = tuple(cu[pts[r + 1]] - cu[pts[r]] for r in range(world_size))
    return TreeShard(rank, world_size, lo, hi, cu[lo], cu[hi], cu_local, tokens)


def local_inputs(Q: torch.Tensor, K: torch.Tensor, V: torch.Tensor, shard: TreeShard):
    """Views (no copies) of a global packed ``[T, H, D]`` batch restricted to the shard."""
    s = slice(shard.tok_lo, shard.tok_hi)
    return Q[s], K[s], V[s]


def sharded_ragged_attention_with_lse(Q_local: torch.Tensor, K_local: torch.Tensor, V_local: torch.Tensor,
                                      shard: TreeShard, branching_factor: int, max_depth: int):
    """The rank's ancestor pass over its own trees: ``ragged_attention_with_lse`` on the shard.

    ``Q_local`` etc. hold only this rank's tokens (``shard.num_tokens`` rows, on this
    rank's GPU). Returns (O_local, LSE_local). An empty shard returns empty tensors.
    """
    from .ragged_attn import ragged_attention_with_lse

    if shard.num_trees == 0:
        T, H, D = 0, Q_local.shape[1], Q_local.shape[2]
        return (torch.empty(T, H, D, dtype=Q_local.dtype, device=Q_local.device),
                torch.empty(T, H, dtype=torch.float32, device=Q_local.device))
    cu_dev = shard.cu_local.to(Q_local.device, non_blocking=True)
    return ragged_attention_with_lse(Q_local, K_local, V_local, cu_dev, branching_factor, max_depth,
                                     max_seqlen=shard.max_seqlen)


def gather_outputs(O_local: torch.Tensor, LSE_local: Optional[torch.Tensor], shard: TreeShard,
                   dst: int = 0, group=None) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
    """Gathers every rank's (O, LSE) into the global packed batch on rank `dst`.

    One collective per tensor (``torch.distributed.gather`` over the shards padded
    to the largest one). Returns the full ``[T, H, D]`` O and ``[T, H]`` LSE on
    `dst` and (None, None) elsewhere. With world_size 1 it returns the inputs.
    """
    import torch.distributed as dist

    if shard.world_size == 1:
        return O_local, LSE_local
    pad = max(shard.tokens_per_rank)
    outs = []
    for t in (O_local, LSE_local):
        if t is None:
            outs.append(None)
            continue
        buf = torch.zeros((pad,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
        buf[: t.shape[0]].copy_(t)
        parts = [torch.empty_like(buf) for _ in range(shard.world_size)] if shard.rank == dst else None
        dist.gather(buf, parts, dst=dst, group=group)
        if shard.rank == dst:
            outs.append(torch.cat([p[:n] for p, n in zip(parts, shard.tokens_per_rank)], 0))
        else:
            outs.append(None)
    return outs[0], outs[1]
