"""Work that splits across GPUs: one process per GPU, torch.distributed (NCCL
on NVLink) for the exchange.

Only the naturally partitioned parts of the path are sharded:

* kNN keys: rank r holds keys [first, first + count) of
  the global key set, scans them with ``index_base = first`` and produces its
  best 128 per query as sortable 64-bit keys; one all-gather exchanges those
  lists (nq x 128 x 8 bytes per rank) and every rank merges the world's lists.
  Exact: the global best k of a query is contained in the union of the
  per-shard best k.  This replaces, across GPUs, the reference's in-device
  merge of part lists (k_merge_parts, src/gpu_step/knn.rs:661-715).
* attention heads: the batch x heads dimension is split; heads
  are independent, so there is no exchange.
* model replicas: local SGD -- every ``sync_every`` steps the flat
  parameters are averaged over ranks (DeviceParams::average_models,
  src/gpu_step/mod.rs:182-195, across GPUs instead of inside one).

The single GEMMs of configs[0] and [1] do not shard: replicas only.
"""
import torch
import torch.distributed as dist

from . import knn


def shard_range(n_total: int, world: int, rank: int):
    """[lo, hi) of an even split of n_total items (the last shard may be short or empty)."""
    per = (n_total + world - 1) // world
    lo = min(n_total, rank * per)
    hi = min(n_total, lo + per)
    return lo, hi


def knn_search_sharded(codes: torch.Tensor, scales: torch.Tensor, queries: torch.Tensor, first: int, k: int = 128,
                       mode: str = "dot", prec: str = "exact", group=None, work=None):
    """Best k of every query over all ranks' keys.  codes/scales: this rank's
    shard, whose first key has global index ``first``.  Returns (scores, ids)
    on every rank; ids are global key indices."""
    world = dist.get_world_size(group)
    nq = queries.shape[0]
    if work is None:
        work = (torch.empty((nq, knn.KMAX), dtype=torch.int64, device=queries.device),
                torch.empty((world, nq, knn.KMAX), dtype=torch.int64, device=queries.device),
                torch.empty((nq, knn.KMAX), dtype=torch.int64, device=queries.device))
    local, gathered, merged = work
    knn.topk_keys(codes, scales, queries, mode=mode, prec=prec, index_base=first, out=local)
    dist.all_gather_into_tensor(gathered, local, group=group)
    knn.merge_keys(gathered, nq, out=merged)
    return knn.decode(merged, queries, k, mode=mode, prec=prec)


def average_params(flat: torch.Tensor, group=None):
    """Local-SGD model average: every rank's flat parameters become the mean
    over ranks (one all-reduce)."""
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    flat.mul_(1.0 / dist.get_world_size(group))
    return flat
