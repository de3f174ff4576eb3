"""Host side of the multi-GPU path, on CPU: world_size-2 gloo ranks.

The kNN key set is split with shard_range; each rank finds its shard's best
128 per query (the oracle stands in for the device scan), packs them as the
device does (order-preserving f32 score bits << 32 | 0xFFFFFFFF - global
index), all-gathers over gloo and merges; the result must be the oracle's
top-k over the whole set.  The local-SGD average must give every rank the
mean of the ranks' parameters.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle


def _shard_range(n, world, rank):
    from scratchtape_b200.shard import shard_range  # loads the library; makes no device call
    return shard_range(n, world, rank)


def test_shard_range_partitions():
    for n in (1, 7, 128, 1000, 2 ** 20 + 3):
        for world in (1, 2, 3, 4, 8):
            got = [_shard_range(n, world, r) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(got, got[1:]))
            assert all(lo <= hi for lo, hi in got)


def _pack(scores, ids):
    u = np.asarray(scores, np.float32).view(np.uint32).astype(np.uint64)
    o = np.where(u & 0x80000000, ~u & 0xFFFFFFFF, u | 0x80000000)
    keys = (o << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.asarray(ids, np.uint64))
    return np.where(np.asarray(ids) >= 0, keys, 0).astype(np.uint64)


def _merge(lists, k):
    allk = np.concatenate(lists, axis=1)
    return np.sort(allk, axis=1)[:, ::-1][:, :k]


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
    rng = np.random.default_rng(5)
    n, d, nq, k = 3001, 64, 6, 128
    keys = rng.standard_normal((n, d)).astype(np.float32)
    codes, scales, _ = oracle.quantize_rows(keys, 2)
    q = rng.standard_normal((nq, d)).astype(np.float32)
    lo, hi = _shard_range(n, world, rank)
    s, i = oracle.knn_topk(codes[lo:hi], scales[lo:hi], q, k, mode="dot", threads=1)
    i = np.where(i >= 0, i + lo, -1)
    local = torch.from_numpy(_pack(s.astype(np.float32), i).view(np.int64))
    gathered = [torch.empty_like(local) for _ in range(world)]
    dist.all_gather(gathered, local)
    merged = _merge([g.numpy().view(np.uint64) for g in gathered], k)
    # average
    flat = torch.full((10,), float(rank + 1))
    dist.all_reduce(flat, op=dist.ReduceOp.SUM)
    flat.mul_(1.0 / world)
    if rank == 0:
        ws, wi = oracle.knn_topk(codes, scales, q, k, mode="dot", threads=1)
        want = _pack(ws.astype(np.float32), wi)
        ok_knn = bool(np.array_equal(merged, want))
        ok_avg = bool(torch.allclose(flat, torch.full((10,), (world + 1) / 2.0)))
        with open(result_path, "w") as f:
            f.write("%d %d" % (ok_knn, ok_avg))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_gloo_sharded_knn_merge_and_average(tmp_path, world):
    path = str(tmp_path / "res.txt")
    mp.start_processes(_worker, args=(world, _free_port(), path), nprocs=world, start_method="spawn", join=True)
    ok_knn, ok_avg = open(path).read().split()
    assert ok_knn == "1", "sharded top-k merge differs from the global top-k"
    assert ok_avg == "1", "local-SGD average wrong"
