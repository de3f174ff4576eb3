"""Work that splits across GPUs: one process per GPU, NCCL over NVLink for the
exchange.

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

Two routes to the same exchanges.  With a ``NcclComm`` (a communicator made
through the library's C ABI) the search and the average are single library
calls -- st_knn_search_sharded and st_avg_params, which run the scan, NCCL and
the merge on the caller's stream -- the route a host without Python takes.
Without one they go through torch.distributed's process group.

The single GEMMs of configs[0] and [1] do not shard: replicas only.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _native as N
from . import knn
from .device import handle, ptr


def shard_range(n_total: int, world: int, rank: int):
    """[lo, hi) of an even split of n_total items (the last shard may be short or empty)."""
    per = (n_total + world - 1) // world
    lo = min(n_total, rank * per)
    hi = min(n_total, lo + per)
    return lo, hi


class NcclComm:
    """An NCCL communicator over the ranks of a torch.distributed group, made by
    the library (st_nccl_unique_id on rank 0, the id broadcast over the group,
    st_nccl_comm_init on every rank).  ``ptr`` is the ncclComm_t the C ABI
    takes.  Every rank of the group must construct it together."""

    def __init__(self, group=None, device=None):
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        dev = torch.cuda.current_device() if device is None else torch.device(device).index
        uid = (ctypes.c_uint8 * 128)()
        if self.rank == 0:
            N.check(None, N.lib.st_nccl_unique_id(uid))
        box = [bytes(uid)]
        dist.broadcast_object_list(box, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        uid = (ctypes.c_uint8 * 128).from_buffer_copy(box[0])
        comm = ctypes.c_void_p()
        N.check(None, N.lib.st_nccl_comm_init(self.world, self.rank, uid, dev, ctypes.byref(comm)))
        self.ptr = comm
        self.device = dev

    def close(self):
        if self.ptr:
            N.lib.st_nccl_comm_destroy(self.ptr)
            self.ptr = None


def gather_lists(local: torch.Tensor, group=None, out=None):
    """The all-gather of the kNN exchange: every rank's [nq, 128] best-128
    list (int64 view of the sortable u64 keys) stacked in rank order into
    [world, nq, 128] on every rank."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world,) + tuple(local.shape), dtype=local.dtype, device=local.device)
    if local.is_cuda:
        dist.all_gather_into_tensor(out, local, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), local, group=group)
    return out


def knn_search_sharded(codes: torch.Tensor, scales: torch.Tensor, queries: torch.Tensor, first: int, k: int = 128,
                       mode: str = "dot", prec: str = "exact", group=None, work=None, comm: NcclComm = None,
                       out=None):
    """Best k of every query over all ranks' keys.  codes/scales: this rank's
    shard, whose first key has global index ``first``.  Returns (scores, ids)
    on every rank; ids are global key indices.  With ``comm`` the whole search
    is one st_knn_search_sharded call; otherwise the scan, merge and decode are
    library calls around a torch.distributed all-gather."""
    nq = queries.shape[0]
    if comm is not None:
        dev = queries.device
        scores, ids = out if out is not None else (torch.empty((nq, k), dtype=torch.float32, device=dev),
                                                   torch.empty((nq, k), dtype=torch.int64, device=dev))
        q = queries.contiguous()
        handle(dev).call("st_knn_search_sharded", ptr(codes), ptr(scales), codes.shape[0], q.shape[1], ptr(q), nq,
                         k, knn.MODES[mode], knn.PRECS[prec], first, comm.ptr, ptr(scores), ptr(ids))
        return scores, ids
    world = dist.get_world_size(group)
    if work is None:
        work = (torch.empty((nq, knn.KMAX), dtype=torch.int64, device=queries.device),
                torch.empty((world, nq, knn.KMAX), dtype=torch.int64, device=queries.device),
                torch.empty((nq, knn.KMAX), dtype=torch.int64, device=queries.device))
    local, gathered, merged = work
    knn.topk_keys(codes, scales, queries, mode=mode, prec=prec, index_base=first, out=local)
    gather_lists(local, group, out=gathered)
    knn.merge_keys(gathered, nq, out=merged)
    return knn.decode(merged, queries, k, mode=mode, prec=prec)


def average_params(flat: torch.Tensor, group=None, comm: NcclComm = None):
    """Local-SGD model average: every rank's flat parameters become the sum
    over ranks divided by the rank count (one all-reduce), as the reference
    divides its sum of models (mod.rs:261-275).  With ``comm``: st_avg_params."""
    if comm is not None:
        handle(flat.device).call("st_avg_params", ptr(flat), flat.numel(), comm.ptr)
        return flat
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    flat.div_(float(dist.get_world_size(group)))
    return flat
