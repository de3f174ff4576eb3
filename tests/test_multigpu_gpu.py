"""Multi-GPU paths on 2 GPUs (skipped with fewer): NCCL ranks, one per GPU.

* kNN keys sharded over the ranks (each rank makes its own shard with the
  counter-based generator), local scans, all-gather of the best-128 lists,
  merge: identical, bit for bit, to one scan of the whole key set.
* attention heads split over ranks: each rank's heads identical to the
  single-GPU result for the same heads.
* local-SGD average over NCCL.
* the same search and average through the C ABI (st_knn_search_sharded,
  st_avg_params on a communicator made by st_nccl_comm_init): identical to
  the torch.distributed route.
* a C-ABI search large enough for the sampling stages (the keys-in-TMEM scan
  with 300 queries, the narrow scan with 20), whose stages' best-128 lists
  are merged across the ranks before seeding: identical, bit for bit, to one
  scan of all keys.
"""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, result_path):
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    import scratchtape_b200.knn as K
    from scratchtape_b200 import shard
    from scratchtape_b200.attention import attention_fwd
    n, d, nq = 200_003, 256, 300
    lo, hi = shard.shard_range(n, world, rank)
    codes, scales = K.synth_keys(hi - lo, d, seed=11, first_key=lo)
    g = torch.Generator(device="cuda").manual_seed(1)
    q = torch.randn((nq, d), device="cuda", generator=g)
    s, i = shard.knn_search_sharded(codes, scales, q, lo, k=128, mode="dot")
    comm = shard.NcclComm()
    s_abi, i_abi = shard.knn_search_sharded(codes, scales, q, lo, k=128, mode="dot", comm=comm)
    flat = torch.full((1000,), float(rank + 1), device="cuda")
    shard.average_params(flat)
    gp = torch.Generator(device="cuda").manual_seed(50 + rank)
    p_torch = torch.randn(100_003, device="cuda", generator=gp)
    p_abi = p_torch.clone()
    shard.average_params(p_torch)
    shard.average_params(p_abi, comm=comm)
    # 2.6 M keys per rank: both sampling stages' seeds cross the ranks
    n2 = 5_200_001
    lo2, hi2 = shard.shard_range(n2, world, rank)
    c2, sc2 = K.synth_keys(hi2 - lo2, d, seed=13, first_key=lo2)
    seeded = []
    for nq2 in (300, 20):
        q2 = torch.randn((nq2, d), device="cuda", generator=g)
        seeded.append((q2, shard.knn_search_sharded(c2, sc2, q2, lo2, k=128, mode="dot", comm=comm)))
    torch.cuda.synchronize()
    del c2, sc2
    comm.close()
    ok_abi = torch.equal(s_abi, s) and torch.equal(i_abi, i) and torch.equal(p_abi, p_torch)
    # heads: this rank's slice of 16 heads
    gh = torch.Generator(device="cuda").manual_seed(2)
    qh, kh, vh = (torch.randn((16, 128, 64), device="cuda", generator=gh).half() / 8 for _ in range(3))
    h0, h1 = shard.shard_range(16, world, rank)
    o_part, _ = attention_fwd(qh[h0:h1], kh[h0:h1], vh[h0:h1], 0.125)
    o_all, _ = attention_fwd(qh, kh, vh, 0.125)
    ok_heads = torch.equal(o_part, o_all[h0:h1])
    oks = torch.tensor([int(ok_heads), int(torch.allclose(flat, torch.full_like(flat, (world + 1) / 2))),
                        int(ok_abi)], device="cuda")
    dist.all_reduce(oks, op=dist.ReduceOp.MIN)
    if rank == 0:
        ac, asc = K.synth_keys(n, d, seed=11)
        ws, wi = K.search(ac, asc, q, k=128, mode="dot")
        ok_knn = torch.equal(wi, i) and torch.equal(ws, s)
        ac2, asc2 = K.synth_keys(n2, d, seed=13)
        ok_seeded = True
        for q2, (s2, i2) in seeded:
            ws2, wi2 = K.search(ac2, asc2, q2, k=128, mode="dot")
            ok_seeded = ok_seeded and torch.equal(wi2, i2) and torch.equal(ws2, s2)
        with open(result_path, "w") as f:
            f.write("%d %d %d %d %d" % (int(ok_knn), int(oks[0].item()), int(oks[1].item()), int(oks[2].item()),
                                        int(ok_seeded)))
    dist.barrier()
    dist.destroy_process_group()


def test_two_gpu_sharded_paths(tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    path = str(tmp_path / "res.txt")
    mp.start_processes(_worker, args=(2, _free_port(), path), nprocs=2, start_method="spawn", join=True)
    ok_knn, ok_heads, ok_avg, ok_abi, ok_seeded = open(path).read().split()
    assert ok_knn == "1", "sharded kNN differs from the single-GPU scan"
    assert ok_heads == "1", "head-sharded attention differs"
    assert ok_avg == "1", "NCCL parameter average wrong"
    assert ok_abi == "1", "the C-ABI route (st_knn_search_sharded / st_avg_params) differs from the torch route"
    assert ok_seeded == "1", "the sharded search with seeds shared across ranks differs from the single-GPU scan"
