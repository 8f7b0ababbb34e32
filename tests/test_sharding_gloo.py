"""CPU: the multi-GPU host logic -- sequences partitioned across ranks, each
rank decoding its own page pool with no collective on the data path --
checked with world_size 2 over gloo (the oracle stands in for the GPU
kernel, which these CPU tests never launch)."""
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from slm_turbo_b200.sharding import partition_sequences, shard_kv_heads

HQ, KV, D, BS = 8, 2, 64, 16
LENGTHS = [5, 130, 17, 64, 1, 99, 33, 250, 16, 48, 0, 77]


def _seq_inputs(i, L):
    """Per-sequence data from a per-sequence seed: independent of sharding."""
    g = torch.Generator().manual_seed(1000 + i)
    k = torch.randn(L, KV, D, generator=g).half()
    v = torch.randn(L, KV, D, generator=g).half()
    q = torch.randn(HQ, D, generator=g).half()
    return k, v, q


def _decode_pool(indices, pool_seed):
    """Build one rank's pool (blocks permuted by the rank's own seed), store
    its sequences with the quantizer and decode them."""
    lens = [LENGTHS[i] for i in indices]
    nblk = [max(1, (L + BS - 1) // BS) for L in lens]
    perm = torch.randperm(sum(nblk), generator=torch.Generator().manual_seed(pool_seed))
    bt = torch.zeros(len(indices), max(nblk), dtype=torch.int32)
    o = 0
    for r, n in enumerate(nblk):
        bt[r, :n] = perm[o:o + n].to(torch.int32)
        o += n
    cache = np.zeros((sum(nblk), BS, KV, D + 8), dtype=np.uint8)
    qs = []
    for r, i in enumerate(indices):
        k, v, q = _seq_inputs(i, lens[r])
        slots = torch.tensor([int(bt[r, t // BS]) * BS + t % BS for t in range(lens[r])], dtype=torch.int64)
        if lens[r]:
            oracle.kv_store(k, v, cache, slots)
        qs.append(q)
    q = torch.stack(qs)
    return oracle.paged_decode(q, cache, bt, torch.tensor(lens, dtype=torch.int32), BS, KV)


def _rank_main(rank, world, port, out_path):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        parts = partition_sequences(LENGTHS, world)
        mine = parts[rank]
        out = _decode_pool(mine, pool_seed=77 + rank)
        gathered = [None] * world
        dist.all_gather_object(gathered, (mine, out))
        # step time is the max over ranks (the bench reports that)
        t = torch.tensor([float(1 + rank)], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            np.savez(out_path, t_max=t.item(),
                     **{f"idx{r}": np.asarray(g[0], dtype=np.int64) for r, g in enumerate(gathered)},
                     **{f"out{r}": g[1] for r, g in enumerate(gathered)})
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_partition_covers_every_sequence_once_and_balances():
    for world in (1, 2, 3, 8):
        parts = partition_sequences(LENGTHS, world)
        flat = sorted(i for p in parts for i in p)
        assert flat == list(range(len(LENGTHS)))
        loads = [sum(LENGTHS[i] for i in p) for p in parts]
        assert max(loads) - min(loads) <= max(LENGTHS)
        assert parts == partition_sequences(LENGTHS, world)  # deterministic


def test_shard_kv_heads():
    assert [list(shard_kv_heads(8, 4, r)) for r in range(4)] == [[0, 1], [2, 3], [4, 5], [6, 7]]
    with pytest.raises(ValueError):
        shard_kv_heads(8, 3, 0)


def test_two_ranks_over_gloo_match_single_process(tmp_path):
    oracle.lib()  # build the checker once, before the ranks start
    out_path = tmp_path / "gathered.npz"
    mp.spawn(_rank_main, args=(2, _free_port(), str(out_path)), nprocs=2, join=True)
    got = np.load(out_path)
    assert got["t_max"] == 2.0
    want = _decode_pool(list(range(len(LENGTHS))), pool_seed=5)
    seen = set()
    for r in range(2):
        idx, out = got[f"idx{r}"], got[f"out{r}"]
        assert out.shape == (len(idx), HQ, D)
        for row, i in enumerate(idx):
            np.testing.assert_allclose(out[row], want[i], rtol=1e-6, atol=1e-7)
            seen.add(int(i))
    assert seen == set(range(len(LENGTHS)))
