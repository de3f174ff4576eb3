"""Host side of the multi-GPU path, on CPU: world_size-2 gloo ranks running
the product's exchange code (scratchtape_b200.shard).

The kNN key set is split with shard_range; each rank finds its shard's best
128 per query (the oracle stands in for the device scan, whose list format
oracle.pack_keys restates), exchanges the lists with shard.gather_lists (the
product all-gather, rank order) and merges them with the oracle's restatement
of k_merge_parts: the result must be the oracle's top-k over the whole set,
so a gather that drops, reorders or mis-shapes a rank's list fails.  The
local-SGD average runs shard.average_params itself and must give every rank
the sum over ranks divided by the rank count, bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle


def test_shard_range_partitions():
    from scratchtape_b200.shard import shard_range  # loads the library; makes no device call
    for n in (1, 7, 128, 1000, 2 ** 20 + 3):
        for world in (1, 2, 3, 4, 8):
            got = [shard_range(n, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            assert all(lo <= hi for lo, hi in got)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from scratchtape_b200 import shard
    rng = np.random.default_rng(5)
    n, d, nq, k = 3001, 64, 6, 128
    keys = rng.standard_normal((n, d)).astype(np.float32)
    codes, scales, _ = oracle.quantize_rows(keys, 2)
    q = rng.standard_normal((nq, d)).astype(np.float32)
    lo, hi = shard.shard_range(n, world, rank)
    s, i = oracle.knn_topk(codes[lo:hi], scales[lo:hi], q, k, mode="dot", threads=1)
    i = np.where(i >= 0, i + lo, -1)
    local = torch.from_numpy(oracle.pack_keys(s.astype(np.float32), i).view(np.int64))
    gathered = shard.gather_lists(local)
    ok_shape = tuple(gathered.shape) == (world, nq, k)
    ok_own = bool(torch.equal(gathered[rank], local))
    merged = oracle.merge_keys(gathered.numpy().view(np.uint64), k)
    # the model average, through the product function
    base = np.random.default_rng(100 + rank).standard_normal(1001).astype(np.float32)
    flat = torch.from_numpy(base.copy())
    shard.average_params(flat)
    allp = [np.random.default_rng(100 + r).standard_normal(1001).astype(np.float32) for r in range(world)]
    want_avg = allp[0].copy()
    for p in allp[1:]:
        want_avg = want_avg + p
    want_avg = want_avg / np.float32(world)
    ok_avg = bool(np.array_equal(flat.numpy().view(np.uint32), want_avg.view(np.uint32)))
    if rank == 0:
        ws, wi = oracle.knn_topk(codes, scales, q, k, mode="dot", threads=1)
        want = oracle.pack_keys(ws.astype(np.float32), wi)
        ok_knn = bool(np.array_equal(merged, want)) and ok_shape and ok_own
        with open(result_path, "w") as f:
            f.write("%d %d" % (ok_knn, ok_avg))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gloo_sharded_knn_exchange_and_average(tmp_path, world):
    path = str(tmp_path / "res.txt")
    mp.start_processes(_worker, args=(world, _free_port(), path), nprocs=world, start_method="spawn", join=True)
    ok_knn, ok_avg = open(path).read().split()
    assert ok_knn == "1", "gathered and merged top-k differs from the global top-k"
    assert ok_avg == "1", "local-SGD average (shard.average_params) wrong"
