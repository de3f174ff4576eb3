// st_comm.cu -- the multi-GPU exchanges of the path, in the C ABI: one
// process per GPU, NCCL over NVLink / NVSwitch.
//
// * st_avg_params: the local-SGD model average across GPUs -- what
//   DeviceParams::average_models (src/gpu_step/mod.rs:182-195, kernel
//   k_average_models :261-275) does across the K models held on one device,
//   here across ranks: an in-place ncclAllReduce (sum) of the flat parameters,
//   then p / world, divided as the reference divides its sum.
// * st_knn_search_sharded: a kNN search over a key set split by rows across
//   ranks -- each rank scans its shard (st_knn_topk_keys with index_base = its
//   first global row), one ncclAllGather exchanges the per-query best-128
//   lists (nq x 128 x 8 bytes per rank), and every rank merges the world's
//   lists (st_knn_merge_keys) and decodes them.  Exact: a query's global best k
//   lie in the union of the shards' best k.  This is k_merge_parts
//   (src/gpu_step/knn.rs:661-715) across GPUs instead of across one GPU's
//   key parts.  The scans that seed their per-query thresholds from samples
//   of the keys share each sampling stage's lists (an ncclAllGather of nq x 128
//   x 8 bytes per rank and a merge, twice): the 128th best of the union of the
//   ranks' samples bounds the global 128th best from below, so each rank
//   filters as tightly as one GPU holding every key would.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, preferring a copy the
// process has already loaded -- e.g. torch's -- so a communicator made by the
// host and the calls made here go through the same library).  The library
// therefore loads, and everything else in it works, on a machine without
// NCCL; these entry points then return ST_NCCL_ERROR.  A communicator is
// passed as an opaque pointer (an ncclComm_t); hosts without an NCCL binding
// of their own make one with st_nccl_unique_id + st_nccl_comm_init.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "st_internal.h"

st_status st_divide_by(st_handle *h, float *p, int64_t n, float by);

namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRank) comm_init_rank = nullptr;
    decltype(&ncclCommDestroy) comm_destroy = nullptr;
    decltype(&ncclCommCount) comm_count = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
    bool ok = false;
    std::string why;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);  // the process's own copy, if loaded
        if (!lib) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
        if (!lib) lib = dlopen("libnccl.so", RTLD_NOW | RTLD_LOCAL);
        if (!lib) {
            api.why = "libnccl.so.2 not found";
            return;
        }
        auto sym = [&](const char *name) { return dlsym(lib, name); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.comm_count = reinterpret_cast<decltype(api.comm_count)>(sym("ncclCommCount"));
        api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(sym("ncclAllReduce"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.comm_count && api.all_reduce &&
                 api.all_gather && api.error_string;
        if (!api.ok) api.why = "libnccl.so.2 lacks an expected symbol";
    });
    return api;
}

#define ST_CHECK_NCCL(h, call)                                                                                  \
    do {                                                                                                        \
        ncclResult_t r_ = (call);                                                                               \
        if (r_ != ncclSuccess) return (h)->fail(ST_NCCL_ERROR, "%s: %s", #call, nccl().error_string(r_)); \
    } while (0)

constexpr int64_t KLIST = 128;  // entries per query in a best-128 list

// The handle's seed exchange during a sharded scan: a sampling stage's merged
// best-128 lists (nq x 128 sortable keys) are all-gathered and merged into the
// best 128 of every rank's sample, in place, on the handle's stream.
struct SeedExchange {
    ncclComm_t comm;
    int world;
    uint64_t *gathered;  // [world][nq][128]
};
st_status merge_seeds(st_handle *h, uint64_t *seed_lists, int64_t nq, void *ctx) {
    const SeedExchange *x = static_cast<const SeedExchange *>(ctx);
    ST_CHECK_NCCL(h, nccl().all_gather(seed_lists, x->gathered, static_cast<size_t>(nq) * KLIST, ncclUint64, x->comm,
                                       h->stream));
    return st_knn_merge_keys(h, x->gathered, x->world, nq * KLIST, nq, seed_lists);
}

// Clears the handle's seed exchange when the sharded call returns.
struct ExchangeScope {
    st_handle *h;
    ExchangeScope(st_handle *hh, SeedExchange *x) : h(hh) {
        h->seed_exchange = merge_seeds;
        h->seed_ctx = x;
    }
    ~ExchangeScope() {
        h->seed_exchange = nullptr;
        h->seed_ctx = nullptr;
    }
};

}  // namespace

extern "C" st_status st_nccl_unique_id(uint8_t *out) {
    if (!out) return ST_INVALID_ARG;
    const NcclApi &api = nccl();
    if (!api.ok) return ST_NCCL_ERROR;
    ncclUniqueId id;
    if (api.get_unique_id(&id) != ncclSuccess) return ST_NCCL_ERROR;
    memcpy(out, id.internal, NCCL_UNIQUE_ID_BYTES);
    return ST_OK;
}

extern "C" st_status st_nccl_comm_init(int32_t nranks, int32_t rank, const uint8_t *unique_id, int32_t device,
                                       void **comm_out) {
    if (!unique_id || !comm_out || nranks < 1 || rank < 0 || rank >= nranks) return ST_INVALID_ARG;
    *comm_out = nullptr;
    const NcclApi &api = nccl();
    if (!api.ok) return ST_NCCL_ERROR;
    if (cudaSetDevice(device) != cudaSuccess) return ST_CUDA_ERROR;
    ncclUniqueId id;
    memcpy(id.internal, unique_id, NCCL_UNIQUE_ID_BYTES);
    ncclComm_t c = nullptr;
    if (api.comm_init_rank(&c, nranks, id, rank) != ncclSuccess) return ST_NCCL_ERROR;
    *comm_out = c;
    return ST_OK;
}

extern "C" st_status st_nccl_comm_destroy(void *comm) {
    if (!comm) return ST_INVALID_ARG;
    const NcclApi &api = nccl();
    if (!api.ok) return ST_NCCL_ERROR;
    return api.comm_destroy(static_cast<ncclComm_t>(comm)) == ncclSuccess ? ST_OK : ST_NCCL_ERROR;
}

extern "C" st_status st_avg_params(st_handle *h, float *p, int64_t n, void *comm) {
    if (!h) return ST_INVALID_ARG;
    if (!p || n < 1 || !comm) return h->fail(ST_INVALID_ARG, "st_avg_params: null pointer or n < 1");
    const NcclApi &api = nccl();
    if (!api.ok) return h->fail(ST_NCCL_ERROR, "st_avg_params: %s", api.why.c_str());
    cudaSetDevice(h->device);
    ncclComm_t c = static_cast<ncclComm_t>(comm);
    int world = 0;
    ST_CHECK_NCCL(h, api.comm_count(c, &world));
    if (world == 1) return ST_OK;
    ST_CHECK_NCCL(h, api.all_reduce(p, p, static_cast<size_t>(n), ncclFloat32, ncclSum, c, h->stream));
    return st_divide_by(h, p, n, static_cast<float>(world));
}

extern "C" st_status st_knn_search_sharded(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_local,
                                           int32_t dim, const float *queries, int64_t nq, int32_t k, int32_t mode,
                                           int32_t prec, int64_t index_base, void *comm, float *out_scores,
                                           int64_t *out_ids) {
    const char *who = "st_knn_search_sharded";
    if (!h) return ST_INVALID_ARG;
    if (!comm || !queries || !out_scores || !out_ids || nq < 1 || n_local < 0 || k < 1 || k > KLIST ||
        index_base < 0)
        return h->fail(ST_INVALID_ARG, "%s: bad arguments", who);
    const NcclApi &api = nccl();
    if (!api.ok) return h->fail(ST_NCCL_ERROR, "%s: %s", who, api.why.c_str());
    cudaSetDevice(h->device);
    ncclComm_t c = static_cast<ncclComm_t>(comm);
    int world = 0;
    ST_CHECK_NCCL(h, api.comm_count(c, &world));
    const size_t list_bytes = sizeof(uint64_t) * static_cast<size_t>(nq) * KLIST;
    uint8_t *buf = static_cast<uint8_t *>(st_scratch(h, SLOT_COMM, list_bytes * (world + 3)));
    if (!buf) return ST_NO_MEMORY;
    uint64_t *local = reinterpret_cast<uint64_t *>(buf);
    uint64_t *gathered = reinterpret_cast<uint64_t *>(buf + list_bytes);
    uint64_t *merged = reinterpret_cast<uint64_t *>(buf + list_bytes * (world + 1));
    st_status s;
    // The scans that seed their thresholds from samples share the seeds: every rank
    // takes the same two exchanges (the gathered buffer holds them while the local
    // scan runs; a rank with an empty shard contributes empty lists -- key 0 ranks
    // below every real key).
    const bool seeded = world > 1 && st_knn_seeded_route(dim, nq, mode, prec);
    SeedExchange x{c, world, gathered};
    if (n_local > 0) {
        if (seeded) {
            ExchangeScope scope(h, &x);
            s = st_knn_topk_keys(h, codes, scales, n_local, dim, queries, nq, mode, prec, index_base, local);
        } else {
            s = st_knn_topk_keys(h, codes, scales, n_local, dim, queries, nq, mode, prec, index_base, local);
        }
        if (s != ST_OK) return s;
    } else {
        ST_CHECK_CUDA(h, cudaMemsetAsync(local, 0, list_bytes, h->stream));
        if (seeded) {
            uint64_t *seed = reinterpret_cast<uint64_t *>(buf + list_bytes * (world + 2));
            for (int stage = 0; stage < 2; stage++) {
                ST_CHECK_CUDA(h, cudaMemsetAsync(seed, 0, list_bytes, h->stream));
                s = merge_seeds(h, seed, nq, &x);
                if (s != ST_OK) return s;
            }
        }
    }
    ST_CHECK_NCCL(h, api.all_gather(local, gathered, static_cast<size_t>(nq) * KLIST, ncclUint64, c, h->stream));
    s = st_knn_merge_keys(h, gathered, world, nq * KLIST, nq, merged);
    if (s != ST_OK) return s;
    return st_knn_decode(h, merged, queries, nq, dim, k, mode, prec, out_scores, out_ids);
}
