// st_internal.h -- handle state and host helpers shared by the .cu files.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdarg>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <string>

#include "../../include/st_b200.h"

// Scratch slots of the handle's pool (one buffer each, grown on demand).
enum StScratchSlot {
    SLOT_SPLITK = 0,  // split-k partial sums
    SLOT_HOST_A,      // device copies for the host-buffer entry points
    SLOT_HOST_B,
    SLOT_HOST_C,
    SLOT_KNN_CAND,    // kNN candidate lists
    SLOT_KNN_PART,    // kNN per-split partial top-k lists
    SLOT_KNN_Q,       // kNN quantised queries
    SLOT_KNN_MISC,
    SLOT_STEP,        // LayerNorm parameter-gradient partials
    SLOT_STEP_ROWS,   // per-row cross-entropy losses
    SLOT_COLSUM,      // column-sum partials of the GEMM epilogue
    SLOT_GROUP,       // grouped GEMM: ticket / finished-tile / split counters
    SLOT_KNN_UNITS,   // kNN unit-table scans: the device copy of the unit tables
    SLOT_MLP_PART,    // fused MLP step: per-block partial products
    SLOT_MLP_CTL,     // fused MLP step: per-block arrival / departure counters
    SLOT_COMM,        // sharded kNN search: local, gathered and merged best-128 lists
    SLOT_X3,          // TF32X3: the operands split into TF32 parts, concatenated along k
    SLOT_COUNT
};

struct st_handle {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    int *d_status = nullptr;  // device status word written by bounded waits
    void *slot_ptr[SLOT_COUNT] = {};
    size_t slot_bytes[SLOT_COUNT] = {};
    int64_t launches = 0;
    const char *last_kernel = "";
    int num_sms = 148;
    void *group_ctl = nullptr;   // grouped GEMM counters: where they were last zeroed, and how many bytes
    size_t group_ctl_bytes = 0;
    void *mlp_ctl = nullptr;     // fused MLP step counters: where they were last zeroed, and how many bytes
    size_t mlp_ctl_bytes = 0;
    // Set by the sharded kNN search for the duration of its local scan: after each of
    // the two sampling stages the scan calls it on the stage's merged best-128 lists
    // (nq rows of 128 sortable keys, zeros where the stage did not run on this rank),
    // which it replaces by the merge of every rank's lists -- the best 128 of the union
    // of the ranks' samples, from which the next stage's thresholds are seeded.
    st_status (*seed_exchange)(st_handle *h, uint64_t *seed_lists, int64_t nq, void *ctx) = nullptr;
    void *seed_ctx = nullptr;

    st_status fail(st_status s, const char *fmt, ...) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        err = buf;
        return s;
    }
};

#define ST_CHECK_CUDA(h, call)                                                                           \
    do {                                                                                                 \
        cudaError_t e_ = (call);                                                                         \
        if (e_ != cudaSuccess) return (h)->fail(ST_CUDA_ERROR, "%s: %s", #call, cudaGetErrorString(e_)); \
    } while (0)

// Checks the launch that was just enqueued and counts it.
st_status st_after_launch(st_handle *h, const char *what);

// Launches `kern` on h's stream programmatically dependent on the previous
// kernel there: the launch may overlap that kernel's tail, so `kern` must
// execute griddepcontrol.wait before it touches global memory.
template <typename... KArgs, typename... Args>
cudaError_t st_launch_dependent(st_handle *h, void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = h->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

// Returns a device buffer of at least `bytes` for `slot` (grows the slot;
// growth synchronises the stream).  nullptr on failure (h->err set).
void *st_scratch(st_handle *h, int slot, size_t bytes);

// cuTensorMapEncodeTiled, resolved through the runtime (no libcuda link).
PFN_cuTensorMapEncodeTiled_v12000 st_encode_fn();

// A 4-D tiled tensor map over fp32/f16/... rows: dims {cols, rows, grp, outer},
// byte strides {ld, inner, stride}, box {box_cols, box_rows, 1, 1}, 128-byte
// swizzle, zero fill out of bounds.
bool st_make_map_4d(CUtensorMap *map, CUtensorMapDataType dtype, int elem_bytes, const void *base, uint64_t cols,
                    uint64_t rows, uint64_t grp, uint64_t outer, uint64_t ld_elems, uint64_t inner_elems,
                    uint64_t stride_elems, uint32_t box_cols, uint32_t box_rows, CUtensorMapSwizzle swz,
                    std::string *why);

// Whether a kNN scan of nq queries at this dim / mode / precision runs the two
// threshold-seeding stages (and so calls h->seed_exchange exactly twice).
bool st_knn_seeded_route(int32_t dim, int64_t nq, int32_t mode, int32_t prec);
