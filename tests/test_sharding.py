"""Batch sharding by tree (host logic) and the output gather over gloo ranks on CPU."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from qattention_b200 import sharding


def _cu(lens):
    return torch.tensor([0] + list(torch.tensor(lens).cumsum(0).tolist()), dtype=torch.int32)


@pytest.mark.parametrize("ws", [1, 2, 4, 8])
def test_equal_trees_split_evenly(ws):
    cu = _cu([1023] * 16)
    shards = [sharding.shard_trees(cu, ws, r) for r in range(ws)]
    assert [s.num_trees for s in shards] == [16 // ws] * ws
    assert shards[0].tok_lo == 0 and shards[-1].tok_hi == 16 * 1023
    for a, b in zip(shards, shards[1:]):
        assert a.tree_hi == b.tree_lo and a.tok_hi == b.tok_lo
    for s in shards:
        assert s.cu_local[0] == 0 and int(s.cu_local[-1]) == s.num_tokens
        assert s.max_seqlen == 1023
        assert sum(s.tokens_per_rank) == 16 * 1023


def test_ragged_trees_cover_every_token_once():
    lens = [5, 300, 17, 1023, 1, 64, 64, 900, 2]
    cu = _cu(lens)
    for ws in (1, 2, 3, 4, 8, 12):
        shards = [sharding.shard_trees(cu, ws, r) for r in range(ws)]
        covered = []
        for s in shards:
            covered += list(range(s.tree_lo, s.tree_hi))
            assert torch.equal(s.cu_local, cu[s.tree_lo:s.tree_hi + 1] - cu[s.tree_lo])
        assert covered == list(range(len(lens)))
        if ws <= len(lens):
            # near-equal token counts: no shard exceeds the even share by more than the largest tree
            assert max(s.num_tokens for s in shards) <= sum(lens) / ws + max(lens)


def test_fewer_trees_than_ranks_leaves_empty_shards():
    cu = _cu([7, 7])
    shards = [sharding.shard_trees(cu, 4, r) for r in range(4)]
    assert sum(s.num_trees for s in shards) == 2
    assert all(s.num_trees in (0, 1) for s in shards)
    assert sum(s.num_tokens for s in shards) == 14


def test_rejects_bad_arguments():
    with pytest.raises(ValueError):
        sharding.shard_trees(_cu([3, 3]), 2, 2)
    with pytest.raises(ValueError):
        sharding.shard_trees(torch.tensor([1, 4], dtype=torch.int32), 1, 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gather_worker(rank, ws, port, lens, q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=ws)
    try:
        cu = _cu(lens)
        T = int(cu[-1])
        g = torch.Generator().manual_seed(0)
        O_all = torch.randn(T, 3, 8, generator=g).half()
        L_all = torch.randn(T, 3, generator=g)
        sh = sharding.shard_trees(cu, ws, rank)
        O, L = sharding.gather_outputs(O_all[sh.tok_lo:sh.tok_hi].clone(), L_all[sh.tok_lo:sh.tok_hi].clone(),
                                       sh, dst=0)
        if rank == 0:
            q.put(bool(torch.equal(O, O_all) and torch.equal(L, L_all)))
        else:
            q.put(O is None and L is None)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("lens", [[11] * 4, [5, 30, 2, 19, 1]])
def test_gather_outputs_two_gloo_ranks(lens):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_gather_worker, args=(r, 2, port, lens, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert all(q.get(timeout=5) for _ in procs)
