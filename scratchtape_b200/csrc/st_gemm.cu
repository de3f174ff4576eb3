// st_gemm.cu -- the matmul family: NN / NT / TN, batched, head views,
// epilogue, deterministic split-k.
//
// Reference: gpu_step::matmul (src/gpu_step/matmul.rs:86-299): MatRef
// addressing (:31-60), Epilogue (:66-79), split-k summed in a fixed order
// (:246-299); CPU semantics of NdArray::matmul (src/tensor.rs:248-276).
//
// Two kernels:
//  * k_gemm_tf32: tcgen05 kind::tf32.  One 128 x BN output tile per CTA,
//    operands streamed by TMA into 128-byte-swizzled shared memory, a
//    STAGES-deep mbarrier ring, the accumulator in TMEM, one thread issuing
//    the MMAs.  NT/TN need no transpose: a stored-transposed operand is
//    loaded as it lies and described to the tensor core as MN-major.
//  * k_gemm_exact: SIMT, each output a k-ascending chain of f32 multiply then
//    add starting from 0 (no FMA) -- the same bits as NdArray::matmul.
#include <algorithm>
#include <cstring>
#include <mutex>

#include "st_internal.h"
#include "st_ptx.cuh"

namespace {

constexpr int BM = 128;
constexpr int BK = 32;  // f32 elements per k block = one 128-byte swizzle row

struct Operand {  // element (z, r, c) of a logical [rows, cols] matrix
    const float *ptr;  // element type: f32, or f16 / bf16 (esize 2; only TMA reads those)
    int64_t off, stride, inner, ld;
    int grp, trans;
    int esize = 4;
    CUtensorMapDataType tdt = CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
};

struct GemmArgs {
    int M, N, K;
    int batch, splits, kb_per_split;
    int a_grp, a_outer, b_grp, b_outer;  // TMA batch coordinates: z%grp (if grp>1), z/grp (if outer)
    float *c;
    int64_t c_off, c_stride, c_inner, c_ld;
    int c_grp;
    const float *bias;
    int64_t bias_off, bias_stride;
    const float *mask;
    int64_t mask_off;
    const float *residual;
    int64_t residual_off;
    int relu, accumulate;
    int vec;  // out/mask/residual rows 16-byte aligned with N % 4 == 0: float4 epilogue
    int tma_store;   // no split-k and a TMA-describable out: epilogue through TMA stores
    int tma_aux;     // with tma_store: mask / residual tiles loaded by TMA (maps tmM / tmR)
    int c_outer;     // out has a batch stride (TMA batch coordinate z / c_grp)
    float *partial;  // split-k partials, [batch*splits][M][N]
    float *cs_part;  // Epilogue::col_sum inside the GEMM: per-split column sums of b, [splits][N] (or null)
    float *cs_dst;   // ... added into cs_dst[cs_off + col] by k_splitk_reduce
    int64_t cs_off;
    int *status;
};

__device__ __forceinline__ int64_t out_index(const GemmArgs &g, int z, int row, int col) {
    return g.c_off + static_cast<int64_t>(z / g.c_grp) * g.c_stride + static_cast<int64_t>(z % g.c_grp) * g.c_inner +
           static_cast<int64_t>(row) * g.c_ld + col;
}

// A float4 read of the output buffer that the compiler may not hoist out of
// its guarding branch: a plain load there is "safe" to speculate (the same
// thread stores to the address later), and speculating it turned every
// epilogue step into a wait on cold DRAM even when nothing accumulates.
__device__ __forceinline__ float4 load_guarded(const float *p) {
    float4 v;
    asm volatile("ld.global.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "l"(p));
    return v;
}
__device__ __forceinline__ float load_guarded1(const float *p) {
    float v;
    asm volatile("ld.global.f32 %0, [%1];" : "=f"(v) : "l"(p));
    return v;
}

// Epilogue order of the reference: + bias, ReLU, mask, + residual, + out.
// mask and residual share out's layout relative to their own offsets
// (src/gpu_step/matmul.rs:925-931).
__device__ __forceinline__ float epilogue(const GemmArgs &g, int z, int64_t oi, int col, float v) {
    if (g.bias) v = v + g.bias[g.bias_off + static_cast<int64_t>(z) * g.bias_stride + col];
    if (g.relu) v = fmaxf(v, 0.0f);
    if (g.mask && !(g.mask[g.mask_off + oi - g.c_off] > 0.0f)) v = 0.0f;
    if (g.residual) v = v + g.residual[g.residual_off + oi - g.c_off];
    if (g.accumulate) v = v + load_guarded1(g.c + oi);
    return v;
}

template <int BN, int STAGES>
struct Cfg {
    static constexpr int A_BYTES = BM * BK * 4;
    static constexpr int B_BYTES = BN * BK * 4;
    static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
    static constexpr int SMEM = STAGES * STAGE_BYTES + 1024 + 256;
    static constexpr int TMEM_COLS = BN;  // f32 accumulator, one column per output column
};

// Epilogue of one CTA tile, run by 4 warps; warp q owns TMEM lanes (tile
// rows) 32q..32q+31.  Each 32x32 TMEM chunk (thread = row after tcgen05.ld)
// is transposed through shared memory so that global traffic is row-major
// and coalesced.  The staging tile reuses the operand ring: once acc_full
// has fired every stage has been consumed by the tensor core.

// float4 path: 32 x 32 tile, 16-byte chunks XOR-swizzled by row so both the
// row-wise writes and the 4-rows-per-pass reads are free of bank conflicts;
// lane = (row within pass, 4-column chunk); all extra loads are issued before
// any arithmetic so their latencies overlap.
template <int BN>
__device__ __forceinline__ void epilogue_vec(const GemmArgs &g, uint8_t *smem, uint32_t tmem, int q, int lane, int m0,
                                             int n0, int z, bool have) {
    float *tile = reinterpret_cast<float *>(smem) + q * 1024;
    const int sub = lane >> 3, ch = lane & 7;
    const bool split_out = g.splits > 1;
    const int64_t zbase = g.c_off + static_cast<int64_t>(z / g.c_grp) * g.c_stride +
                          static_cast<int64_t>(z % g.c_grp) * g.c_inner;
    const float *bias_z = g.bias ? g.bias + g.bias_off + static_cast<int64_t>(z) * g.bias_stride : nullptr;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        st::tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);
        st::tmem_ld_wait();
#pragma unroll
        for (int c = 0; c < 8; c++) {
            float4 w = have ? make_float4(__uint_as_float(r[4 * c]), __uint_as_float(r[4 * c + 1]),
                                          __uint_as_float(r[4 * c + 2]), __uint_as_float(r[4 * c + 3]))
                            : make_float4(0.f, 0.f, 0.f, 0.f);
            *reinterpret_cast<float4 *>(tile + lane * 32 + ((c ^ (lane & 7)) << 2)) = w;
        }
        __syncwarp();
        float4 v[8];
#pragma unroll
        for (int it = 0; it < 8; it++) {
            const int rr = it * 4 + sub;
            v[it] = *reinterpret_cast<const float4 *>(tile + rr * 32 + ((ch ^ (rr & 7)) << 2));
        }
        __syncwarp();
        const int col = n0 + c0 + ch * 4;
        if (col >= g.N) continue;  // N % 4 == 0: a chunk is all in or all out
        const int row0 = m0 + q * 32 + sub;
        if (split_out) {
            float *dst = g.partial + (static_cast<int64_t>(blockIdx.z) * g.M + row0) * g.N + col;
#pragma unroll
            for (int it = 0; it < 8; it++)
                if (row0 + it * 4 < g.M) *reinterpret_cast<float4 *>(dst + static_cast<int64_t>(it) * 4 * g.N) = v[it];
            continue;
        }
        float4 mk[8], rs[8], ac[8];
#pragma unroll
        for (int it = 0; it < 8; it++) {
            mk[it] = make_float4(1.f, 1.f, 1.f, 1.f);
            rs[it] = make_float4(0.f, 0.f, 0.f, 0.f);
            ac[it] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        if (g.mask || g.residual || g.accumulate) {
#pragma unroll
            for (int it = 0; it < 8; it++) {
                const int row = row0 + it * 4;
                if (row >= g.M) break;
                const int64_t rel = static_cast<int64_t>(row) * g.c_ld + col + (zbase - g.c_off);
                if (g.mask) mk[it] = __ldg(reinterpret_cast<const float4 *>(g.mask + g.mask_off + rel));
                if (g.residual) rs[it] = __ldg(reinterpret_cast<const float4 *>(g.residual + g.residual_off + rel));
                if (g.accumulate) ac[it] = load_guarded(g.c + g.c_off + rel);
            }
        }
        float4 bz = make_float4(0.f, 0.f, 0.f, 0.f);
        if (bias_z) bz = make_float4(bias_z[col], bias_z[col + 1], bias_z[col + 2], bias_z[col + 3]);
#pragma unroll
        for (int it = 0; it < 8; it++) {
            const int row = row0 + it * 4;
            if (row >= g.M) break;
            float o[4] = {v[it].x, v[it].y, v[it].z, v[it].w};
            const float b4[4] = {bz.x, bz.y, bz.z, bz.w};
            const float m4[4] = {mk[it].x, mk[it].y, mk[it].z, mk[it].w};
            const float r4[4] = {rs[it].x, rs[it].y, rs[it].z, rs[it].w};
            const float a4[4] = {ac[it].x, ac[it].y, ac[it].z, ac[it].w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                float x = o[j];
                if (bias_z) x = x + b4[j];
                if (g.relu) x = fmaxf(x, 0.0f);
                if (g.mask && !(m4[j] > 0.0f)) x = 0.0f;
                if (g.residual) x = x + r4[j];
                if (g.accumulate) x = x + a4[j];
                o[j] = x;
            }
            *reinterpret_cast<float4 *>(g.c + zbase + static_cast<int64_t>(row) * g.c_ld + col) =
                make_float4(o[0], o[1], o[2], o[3]);
        }
    }
}

// TMA-store path: thread = tile row (its TMEM lane); the epilogue runs in
// registers on 32 columns at a time (bias broadcast, ReLU, and the thread's
// own row of mask / residual / out), the result goes to a 128-byte-swizzled
// 32x32 box in this warp's staging area (two boxes, alternating), and lane 0
// hands the box to a TMA store.  The store engine clips rows and columns that
// fall outside out.
// Mask / residual tiles by TMA: per warp two 8 KB buffers (mask box, then
// residual box, 32 rows x 32 columns each, 128-byte swizzled) and two
// mbarriers; the box of chunk i+1 is in flight while chunk i is processed.
struct EpiAux {
    const CUtensorMap *mask, *residual;  // null: that operand is not loaded by TMA
    uint8_t *buf;                        // this warp's 16 KB
    uint64_t *bar;                       // this warp's 2 mbarriers
};

// AUX: mask / residual come from `aux` (compiled out when false, so the plain
// epilogue carries none of that code).
template <bool AUX = false>
__device__ __forceinline__ void epilogue_tma(const GemmArgs &g, const CUtensorMap *tmC, uint8_t *stage, uint32_t tmem,
                                             int q, int lane, int m0, int n0, int z, bool have, int BN,
                                             uint64_t *acc_release = nullptr, const EpiAux *aux = nullptr) {
    const int row = m0 + q * 32 + lane;
    const bool rin = row < g.M;
    const int64_t zbase = g.c_off + static_cast<int64_t>(z / g.c_grp) * g.c_stride +
                          static_cast<int64_t>(z % g.c_grp) * g.c_inner;
    const float *bias_z = g.bias ? g.bias + g.bias_off + static_cast<int64_t>(z) * g.bias_stride : nullptr;
    const int cz2 = g.c_grp > 1 ? z % g.c_grp : 0, cz3 = g.c_outer ? z / g.c_grp : 0;
    constexpr bool tma_aux = AUX;
    const bool row_loads = rin && ((!tma_aux && (g.mask || g.residual)) || g.accumulate);
    const uint32_t aux_bytes = tma_aux ? 4096u * ((aux->mask ? 1u : 0u) + (aux->residual ? 1u : 0u)) : 0u;
    auto aux_issue = [&](int i, int c) {  // lane 0: the boxes of chunk i (columns n0 + c ..)
        uint8_t *b = aux->buf + (i & 1) * 8192;
        st::mbar_arrive_expect_tx(&aux->bar[i & 1], aux_bytes);
        if (aux->mask) st::tma_load_4d(b, aux->mask, &aux->bar[i & 1], n0 + c, m0 + q * 32, cz2, cz3);
        if (aux->residual) st::tma_load_4d(b + 4096, aux->residual, &aux->bar[i & 1], n0 + c, m0 + q * 32, cz2, cz3);
    };
    if (tma_aux && lane == 0) aux_issue(0, 0);
    int it = 0;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32, ++it) {
        if (n0 + c0 >= g.N) break;
        if (tma_aux && lane == 0 && c0 + 32 < BN && n0 + c0 + 32 < g.N) aux_issue(it + 1, c0 + 32);
        uint32_t r[32];
        st::tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);
        st::tmem_ld_wait();
        if (acc_release && (c0 + 32 >= BN || n0 + c0 + 32 >= g.N)) {  // last TMEM read of this warp
            st::tc_fence_before();
            __syncwarp();
            if (lane == 0) st::mbar_arrive(acc_release);
        }
        float x[32];
#pragma unroll
        for (int j = 0; j < 32; j++) x[j] = have ? __uint_as_float(r[j]) : 0.0f;
        if (bias_z) {
#pragma unroll
            for (int j4 = 0; j4 < 8; j4++) {
                const int col = n0 + c0 + 4 * j4;
                if (col < g.N) {  // scalar loads: a batch's bias row need not be 16-byte aligned
                    x[4 * j4] += __ldg(bias_z + col);
                    x[4 * j4 + 1] += __ldg(bias_z + col + 1);
                    x[4 * j4 + 2] += __ldg(bias_z + col + 2);
                    x[4 * j4 + 3] += __ldg(bias_z + col + 3);
                }
            }
        }
        if (g.relu) {
#pragma unroll
            for (int j = 0; j < 32; j++) x[j] = fmaxf(x[j], 0.0f);
        }
        if (tma_aux) {
            const bool ok = st::mbar_wait(&aux->bar[it & 1], (it >> 1) & 1, g.status, st::DEV_TIMEOUT_FULL);
            const uint8_t *b = aux->buf + (it & 1) * 8192;
            if (ok) {
#pragma unroll
                for (int j4 = 0; j4 < 8; j4++) {
                    if (aux->mask) {
                        const float4 m = *reinterpret_cast<const float4 *>(b + st::sw128_offset(lane, j4));
                        if (!(m.x > 0.0f)) x[4 * j4] = 0.0f;
                        if (!(m.y > 0.0f)) x[4 * j4 + 1] = 0.0f;
                        if (!(m.z > 0.0f)) x[4 * j4 + 2] = 0.0f;
                        if (!(m.w > 0.0f)) x[4 * j4 + 3] = 0.0f;
                    }
                    if (aux->residual) {
                        const float4 rr = *reinterpret_cast<const float4 *>(b + 4096 + st::sw128_offset(lane, j4));
                        x[4 * j4] = x[4 * j4] + rr.x;
                        x[4 * j4 + 1] = x[4 * j4 + 1] + rr.y;
                        x[4 * j4 + 2] = x[4 * j4 + 2] + rr.z;
                        x[4 * j4 + 3] = x[4 * j4 + 3] + rr.w;
                    }
                }
            }
        }
        if (row_loads) {
            const int64_t rel0 = static_cast<int64_t>(row) * g.c_ld + (zbase - g.c_off);
#pragma unroll
            for (int j4 = 0; j4 < 8; j4++) {
                const int col = n0 + c0 + 4 * j4;
                if (col >= g.N) break;
                const int64_t rel = rel0 + col;
                float v[4] = {x[4 * j4], x[4 * j4 + 1], x[4 * j4 + 2], x[4 * j4 + 3]};
                if (g.mask && !tma_aux) {
                    const float4 m = __ldg(reinterpret_cast<const float4 *>(g.mask + g.mask_off + rel));
                    if (!(m.x > 0.0f)) v[0] = 0.0f;
                    if (!(m.y > 0.0f)) v[1] = 0.0f;
                    if (!(m.z > 0.0f)) v[2] = 0.0f;
                    if (!(m.w > 0.0f)) v[3] = 0.0f;
                }
                if (g.residual && !tma_aux) {
                    const float4 rr = __ldg(reinterpret_cast<const float4 *>(g.residual + g.residual_off + rel));
                    v[0] = v[0] + rr.x;
                    v[1] = v[1] + rr.y;
                    v[2] = v[2] + rr.z;
                    v[3] = v[3] + rr.w;
                }
                if (g.accumulate) {
                    const float4 a = load_guarded(g.c + g.c_off + rel);
                    v[0] = v[0] + a.x;
                    v[1] = v[1] + a.y;
                    v[2] = v[2] + a.z;
                    v[3] = v[3] + a.w;
                }
                x[4 * j4] = v[0];
                x[4 * j4 + 1] = v[1];
                x[4 * j4 + 2] = v[2];
                x[4 * j4 + 3] = v[3];
            }
        }
        uint8_t *buf = stage + (it & 1) * 4096;
        if (it >= 2) {
            if (lane == 0) st::bulk_wait_read<1>();  // the store that last used buf has read it
            __syncwarp();
        }
#pragma unroll
        for (int j = 0; j < 8; j++)
            *reinterpret_cast<float4 *>(buf + st::sw128_offset(lane, j)) =
                make_float4(x[4 * j], x[4 * j + 1], x[4 * j + 2], x[4 * j + 3]);
        st::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
            st::tma_store_4d(tmC, buf, n0 + c0, m0 + q * 32, cz2, cz3);
            st::bulk_commit();
        }
    }
    if (lane == 0) st::bulk_wait_all();
    __syncwarp();
}

// Scalar path for layouts that are not 16-byte aligned: lane = column.
template <int BN>
__device__ __forceinline__ void epilogue_scalar(const GemmArgs &g, uint8_t *smem, uint32_t tmem, int q, int lane,
                                                int m0, int n0, int z, bool have) {
    float *tile = reinterpret_cast<float *>(smem) + q * (32 * 33);
    const bool split_out = g.splits > 1;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 32) {
        uint32_t r[32];
        st::tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);
        st::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 32; j++) tile[lane * 33 + j] = have ? __uint_as_float(r[j]) : 0.0f;
        __syncwarp();
        const int col = n0 + c0 + lane;
        if (col < g.N) {
#pragma unroll 4
            for (int rr = 0; rr < 32; rr++) {
                const int row = m0 + q * 32 + rr;
                if (row >= g.M) break;
                const float v = tile[rr * 33 + lane];
                if (split_out) {
                    g.partial[(static_cast<int64_t>(blockIdx.z) * g.M + row) * g.N + col] = v;
                } else {
                    const int64_t oi = out_index(g, z, row, col);
                    g.c[oi] = epilogue(g, z, oi, col, v);
                }
            }
        }
        __syncwarp();
    }
}

// One CTA of the tensor-core GEMM.  AB: operand type -- 0 f32 (kind::tf32,
// 32 elements per 128-byte k row), 1 f16 / 2 bf16 (kind::f16, 64 elements per
// k row).  A k block is one 128-byte swizzled row per tile row either way, so
// the stage layout, the four MMAs per k block and the K-major descriptors are
// shared; MN-major 16-bit tiles are 64-element (128-byte) rows along MN, k in
// rows, 64-wide MN atoms one 64-row TMA box (8 KB) apart.
template <int BN, int STAGES, bool A_MN, bool B_MN, int AB>
__device__ __forceinline__ void gemm_cta(const CUtensorMap &tmA, const CUtensorMap &tmB, const CUtensorMap &tmC,
                                         const CUtensorMap &tmM, const CUtensorMap &tmR, const GemmArgs &g) {
    using C = Cfg<BN, STAGES>;
    constexpr int BKE = AB ? 64 : BK;      // elements per k block
    constexpr int MNW = AB ? 64 : 32;      // MN-major box width (elements)
    constexpr int MNBOX = MNW * BKE * (AB ? 2 : 4);  // bytes of one MN-major box
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + STAGES * C::STAGE_BYTES);
    uint64_t *empty = full + STAGES;
    uint64_t *acc_full = empty + STAGES;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    uint64_t *aux_bar = acc_full + 2;  // [4 epilogue warps][2]

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int z = blockIdx.z / g.splits, split = blockIdx.z % g.splits;
    const int kb_total = (g.K + BKE - 1) / BKE;
    const int kb_begin = split * g.kb_per_split;
    const int nkb = max(0, min(kb_total, kb_begin + g.kb_per_split) - kb_begin);
    // column sums of b (Epilogue::col_sum) by the epilogue warps of the first row of tiles, from the b tiles
    // the ring stages anyway: row-major f32 b, 128 columns, one 32-column box per epilogue warp
    constexpr bool CS_FORM = AB == 0 && B_MN && BN == 128;
    const bool csum = CS_FORM && g.cs_part != nullptr && blockIdx.y == 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; s++) {
            st::mbar_init(&full[s], 1);
            st::mbar_init(&empty[s], csum ? 5 : 1);  // + one arrival per column-summing warp
        }
        st::mbar_init(acc_full, 1);
        for (int b = 0; b < 8; b++) st::mbar_init(&aux_bar[b], 1);
        st::fence_mbar_init();
    }
    if (warp == 1) {
        st::tmem_alloc(tmem_slot, C::TMEM_COLS);
        st::tmem_relinquish();
    }
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // everything above overlaps the previous kernel's tail; no global memory
    // is touched before it has completed
    st::grid_dep_wait();

    if (warp == 0) {
        if (lane == 0) {  // TMA producer
            st::tma_prefetch_desc(&tmA);
            st::tma_prefetch_desc(&tmB);
            const int ca2 = g.a_grp > 1 ? z % g.a_grp : 0, ca3 = g.a_outer ? z / g.a_grp : 0;
            const int cb2 = g.b_grp > 1 ? z % g.b_grp : 0, cb3 = g.b_outer ? z / g.b_grp : 0;
            for (int i = 0; i < nkb; i++) {
                const int s = i % STAGES;
                if (i >= STAGES && !st::mbar_wait(&empty[s], ((i / STAGES) - 1) & 1, g.status, st::DEV_TIMEOUT_EMPTY))
                    break;
                st::mbar_arrive_expect_tx(&full[s], C::STAGE_BYTES);
                const int kc = (kb_begin + i) * BKE;
                uint8_t *sa = smem + s * C::STAGE_BYTES;
                uint8_t *sb = sa + C::A_BYTES;
                if (!A_MN) {
                    st::tma_load_4d(sa, &tmA, &full[s], kc, m0, ca2, ca3);
                } else {
#pragma unroll
                    for (int j = 0; j < BM / MNW; j++)
                        st::tma_load_4d(sa + j * MNBOX, &tmA, &full[s], m0 + MNW * j, kc, ca2, ca3);
                }
                if (!B_MN) {
                    st::tma_load_4d(sb, &tmB, &full[s], kc, n0, cb2, cb3);
                } else {
#pragma unroll
                    for (int j = 0; j < BN / MNW; j++)
                        st::tma_load_4d(sb + j * MNBOX, &tmB, &full[s], n0 + MNW * j, kc, cb2, cb3);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // MMA issuer
            constexpr uint32_t idesc = st::idesc_make(1, AB ? AB - 1 : 2, A_MN, B_MN, BM, BN);
            for (int i = 0; i < nkb; i++) {
                const int s = i % STAGES;
                if (!st::mbar_wait(&full[s], (i / STAGES) & 1, g.status, st::DEV_TIMEOUT_FULL)) break;
                st::tc_fence_after();
                const uint32_t sa = st::smem_u32(smem + s * C::STAGE_BYTES);
                const uint32_t sb = sa + C::A_BYTES;
#pragma unroll
                for (int kk = 0; kk < 4; kk++) {
                    // K-major (128B swizzle): advance 32 bytes (8 tf32 or 16
                    // f16) along the swizzled row; 8-row groups 1024 bytes apart.
                    // MN-major tf32 (128B swizzle on a 32B base): advance 8 k rows
                    // (1024 bytes); 4-row atoms 512 bytes apart; 32-wide MN
                    // chunks (one TMA box each) 4096 bytes apart.
                    // MN-major 16-bit (128B swizzle): advance 16 k rows (2048
                    // bytes); 8-row atoms 1024 bytes apart; 64-wide MN chunks 8 KB apart.
                    uint64_t ad, bd;
                    if (AB) {
                        ad = A_MN ? st::sdesc_make(sa + kk * 2048, MNBOX, 1024, st::LAYOUT_SW128)
                                  : st::sdesc_sw128(sa + kk * 32, 16, 1024);
                        bd = B_MN ? st::sdesc_make(sb + kk * 2048, MNBOX, 1024, st::LAYOUT_SW128)
                                  : st::sdesc_sw128(sb + kk * 32, 16, 1024);
                        st::umma_f16(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                    } else {
                        ad = A_MN ? st::sdesc_make(sa + kk * 1024, 4096, 512, st::LAYOUT_SW128_BASE32B)
                                  : st::sdesc_sw128(sa + kk * 32, 16, 1024);
                        bd = B_MN ? st::sdesc_make(sb + kk * 1024, 4096, 512, st::LAYOUT_SW128_BASE32B)
                                  : st::sdesc_sw128(sb + kk * 32, 16, 1024);
                        st::umma_tf32(tmem, ad, bd, idesc, (i > 0 || kk > 0) ? 1u : 0u);
                    }
                }
                st::umma_commit(&empty[s]);
            }
            st::umma_commit(acc_full);
        }
    } else {  // warps 2..5: epilogue; warp w reads TMEM lanes 32*(w%4) ..
        const int q = warp & 3;
        if (CS_FORM && csum) {
            // this thread's column (box q, column lane) of every staged b tile, k ascending; the 32-byte
            // atoms of box row r sit at atom (column / 8) ^ (r % 4) (the 32-byte-atom 128-byte swizzle)
            float acc = 0.0f;
            for (int i = 0; i < nkb; i++) {
                const int s = i % STAGES;
                if (!st::mbar_wait(&full[s], (i / STAGES) & 1, g.status, st::DEV_TIMEOUT_FULL)) break;
                const float *box = reinterpret_cast<const float *>(smem + s * C::STAGE_BYTES + C::A_BYTES + q * MNBOX);
#pragma unroll 8
                for (int r = 0; r < 32; r++) acc = __fadd_rn(acc, box[r * 32 + ((((lane >> 3) ^ (r & 3)) << 3) | (lane & 7))]);
                __syncwarp();
                if (lane == 0) st::mbar_arrive(&empty[s]);
            }
            const int col = n0 + q * 32 + lane;
            if (col < g.N) g.cs_part[static_cast<int64_t>(split) * g.N + col] = acc;
        }
        const bool ok = st::mbar_wait(acc_full, 0, g.status, st::DEV_TIMEOUT_ACC);
        st::tc_fence_after();
        st::grid_dep_launch();  // the MMAs are done: let the next kernel start its prologue
        if (g.tma_store) {
            // the operand ring is free once acc_full has fired: store boxes in
            // its first 32 KB, mask / residual boxes in the next 64 KB
            if (g.tma_aux) {
                const EpiAux aux{g.mask ? &tmM : nullptr, g.residual ? &tmR : nullptr, smem + 32768 + q * 16384,
                                 aux_bar + 2 * q};
                epilogue_tma<true>(g, &tmC, smem + q * 8192, tmem, q, lane, m0, n0, z, ok && nkb > 0, BN, nullptr,
                                   &aux);
            } else {
                epilogue_tma<false>(g, &tmC, smem + q * 8192, tmem, q, lane, m0, n0, z, ok && nkb > 0, BN);
            }
        } else if (g.vec) {
            epilogue_vec<BN>(g, smem, tmem, q, lane, m0, n0, z, ok && nkb > 0);
        } else {
            epilogue_scalar<BN>(g, smem, tmem, q, lane, m0, n0, z, ok && nkb > 0);
        }
    }
    st::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, C::TMEM_COLS);
    }
}

template <int BN, int STAGES, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(192, 2)
    k_gemm_tf32(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmM,
                const __grid_constant__ CUtensorMap tmR, const GemmArgs g) {
    gemm_cta<BN, STAGES, A_MN, B_MN, 0>(tmA, tmB, tmC, tmM, tmR, g);
}

// The same CTA on f16 (AB 1) or bf16 (AB 2) operands: kind::f16, f32 accumulate.
template <int BN, int STAGES, bool A_MN, bool B_MN, int AB>
__global__ void __launch_bounds__(192, 2)
    k_gemm_f16(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmM,
               const __grid_constant__ CUtensorMap tmR, const GemmArgs g) {
    gemm_cta<BN, STAGES, A_MN, B_MN, AB>(tmA, tmB, tmC, tmM, tmR, g);
}

// Sums split-k partials in split order, then applies the epilogue.  Thread
// (z, row, 4-column group); coalesced along the row.  Partials are fetched
// eight splits at a time before any addition, so their latencies overlap;
// the additions stay in split order.
__global__ void k_splitk_reduce(const GemmArgs g) {
    st::grid_dep_wait();
    st::grid_dep_launch();
    const int groups = (g.N + 3) / 4;
    const int z = blockIdx.z;
    const int64_t mn = static_cast<int64_t>(g.M) * g.N;
    const bool vec = (g.N % 4 == 0);
    for (int row = blockIdx.y; row < g.M; row += gridDim.y) {
        for (int gi = blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += gridDim.x * blockDim.x) {
            const int col0 = gi * 4;
            const float *p = g.partial + static_cast<int64_t>(z) * g.splits * mn + static_cast<int64_t>(row) * g.N + col0;
            float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (vec) {
                for (int sp0 = 0; sp0 < g.splits; sp0 += 8) {
                    float4 v[8];
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        v[j] = (sp0 + j < g.splits) ? __ldcg(reinterpret_cast<const float4 *>(p + (sp0 + j) * mn))
                                                    : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        if (sp0 + j >= g.splits) break;
                        s[0] = __fadd_rn(s[0], v[j].x);
                        s[1] = __fadd_rn(s[1], v[j].y);
                        s[2] = __fadd_rn(s[2], v[j].z);
                        s[3] = __fadd_rn(s[3], v[j].w);
                    }
                }
            } else {
                for (int sp = 0; sp < g.splits; sp++)
                    for (int j = 0; j < 4; j++)
                        if (col0 + j < g.N) s[j] = __fadd_rn(s[j], p[sp * mn + j]);
            }
            for (int j = 0; j < 4; j++) {
                const int col = col0 + j;
                if (col >= g.N) break;
                const int64_t oi = out_index(g, z, row, col);
                g.c[oi] = epilogue(g, z, oi, col, s[j]);
            }
        }
    }
    if (g.cs_part && z == 0 && blockIdx.y == 0) {  // the GEMM's column sums of b, splits in order
        for (int gi = blockIdx.x * blockDim.x + threadIdx.x; gi < groups; gi += gridDim.x * blockDim.x) {
            float s[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int sp0 = 0; sp0 < g.splits; sp0 += 8) {  // 32 loads in flight, then the additions in split order
                float v[8][4];
#pragma unroll
                for (int u = 0; u < 8; u++)
#pragma unroll
                    for (int j = 0; j < 4; j++)
                        v[u][j] = (sp0 + u < g.splits && gi * 4 + j < g.N)
                                      ? __ldcg(g.cs_part + static_cast<int64_t>(sp0 + u) * g.N + gi * 4 + j)
                                      : 0.0f;
#pragma unroll
                for (int u = 0; u < 8; u++)
                    if (sp0 + u < g.splits)
#pragma unroll
                        for (int j = 0; j < 4; j++) s[j] = __fadd_rn(s[j], v[u][j]);
            }
            for (int j = 0; j < 4; j++) {
                const int col = gi * 4 + j;
                if (col >= g.N) break;
                g.cs_dst[g.cs_off + col] = __fadd_rn(g.cs_dst[g.cs_off + col], s[j]);
            }
        }
    }
}

#include "st_gemm_group.cuh"

__device__ __forceinline__ float load_op(const Operand &o, int z, int r, int c) {
    const int64_t base = o.off + static_cast<int64_t>(z / o.grp) * o.stride + static_cast<int64_t>(z % o.grp) * o.inner;
    return o.trans ? o.ptr[base + static_cast<int64_t>(c) * o.ld + r] : o.ptr[base + static_cast<int64_t>(r) * o.ld + c];
}

// Bit-exact SIMT matmul: 64x64 tile per 256 threads, 4x4 outputs per thread,
// each output accumulated as acc = acc + a*b (separately rounded) over k
// ascending, from +0.
constexpr int EX_T = 64, EX_K = 16;
__global__ void __launch_bounds__(256) k_gemm_exact(const Operand A, const Operand B, const GemmArgs g) {
    __shared__ float As[EX_K][EX_T + 4];
    __shared__ float Bs[EX_K][EX_T + 4];
    const int z = blockIdx.z;
    const int m0 = blockIdx.y * EX_T, n0 = blockIdx.x * EX_T;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4];
#pragma unroll
    for (int i = 0; i < 4; i++)
#pragma unroll
        for (int j = 0; j < 4; j++) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < g.K; k0 += EX_K) {
        for (int e = threadIdx.x; e < EX_K * EX_T; e += 256) {
            const int kk = e / EX_T, mm = e % EX_T;
            const int kg = k0 + kk;
            As[kk][mm] = (m0 + mm < g.M && kg < g.K) ? load_op(A, z, m0 + mm, kg) : 0.0f;
            Bs[kk][mm] = (n0 + mm < g.N && kg < g.K) ? load_op(B, z, kg, n0 + mm) : 0.0f;
        }
        __syncthreads();
        const int kmax = min(EX_K, g.K - k0);
        for (int kk = 0; kk < kmax; kk++) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = As[kk][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; j++) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int j = 0; j < 4; j++) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i], b[j]));
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int row = m0 + ty * 4 + i;
        if (row >= g.M) continue;
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const int col = n0 + tx * 4 + j;
            if (col >= g.N) continue;
            const int64_t oi = out_index(g, z, row, col);
            g.c[oi] = epilogue(g, z, oi, col, acc[i][j]);
        }
    }
}

// Column sums of b[z] (logical [k, n]) over k, added into col_sum: the
// Epilogue::col_sum bias gradient (src/gpu_step/matmul.rs:75-78), k ascending.
__global__ void k_col_sum(const Operand B, int K, int N, int batch, float *dst, int64_t off, int64_t stride) {
    const int64_t total = static_cast<int64_t>(batch) * N;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int z = static_cast<int>(i / N), col = static_cast<int>(i % N);
        float s = 0.0f;
        for (int k = 0; k < K; k++) s = __fadd_rn(s, load_op(B, z, k, col));
        float *d = dst + off + static_cast<int64_t>(z) * stride + col;
        *d = __fadd_rn(*d, s);
    }
}

// Column sums in two fixed-order passes, for many rows: pass 1 sums rows
// [chunk * rpc, (chunk + 1) * rpc) of each column of b[z] in k order; pass 2
// adds the chunk sums in chunk order into col_sum.  Grid of pass 1:
// (column blocks, chunks, batch).
__global__ void k_col_sum_part(const Operand B, int K, int N, int64_t rpc, float *part) {
    const int col = blockIdx.x * blockDim.x + threadIdx.x;
    const int chunk = blockIdx.y, z = blockIdx.z;
    if (col >= N) return;
    const int64_t k0 = chunk * rpc, k1 = k0 + rpc < K ? k0 + rpc : static_cast<int64_t>(K);
    float s = 0.0f;
    for (int64_t k = k0; k < k1; k++) s = __fadd_rn(s, load_op(B, z, static_cast<int>(k), col));
    part[(static_cast<int64_t>(z) * gridDim.y + chunk) * N + col] = s;
}
// k_col_sum_part for a row-major B whose rows are 16-byte aligned.  Block
// (64, COL_GROUPS): thread (q, g) sums column quad blockIdx.x * 64 + q over
// rows k0 + g, k0 + g + COL_GROUPS, ... of the chunk (adjacent groups read
// adjacent rows), COL_UNROLL 16-byte loads in flight, additions in row order;
// the groups are then added in group order.
constexpr int COL_QUADS = 64, COL_GROUPS = 4, COL_UNROLL = 8;
__global__ void __launch_bounds__(COL_QUADS *COL_GROUPS)
    k_col_sum_part4(const Operand B, int K, int N, int64_t rpc, float *part) {
    __shared__ float4 red[COL_GROUPS][COL_QUADS];
    st::grid_dep_wait();  // launched programmatically dependent (st_launch_dependent)
    st::grid_dep_launch();
    const int q = blockIdx.x * COL_QUADS + threadIdx.x;  // column quad
    const int g = threadIdx.y;
    const int chunk = blockIdx.y, z = blockIdx.z;
    const int64_t k0 = chunk * rpc, k1 = k0 + rpc < K ? k0 + rpc : static_cast<int64_t>(K);
    float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (4 * q < N) {
        const int64_t base =
            B.off + static_cast<int64_t>(z / B.grp) * B.stride + static_cast<int64_t>(z % B.grp) * B.inner;
        const float *col = B.ptr + base + 4 * static_cast<int64_t>(q);
        int64_t k = k0 + g;
        for (; k + (COL_UNROLL - 1) * COL_GROUPS < k1; k += COL_UNROLL * COL_GROUPS) {
            float4 v[COL_UNROLL];
#pragma unroll
            for (int u = 0; u < COL_UNROLL; u++)
                v[u] = *reinterpret_cast<const float4 *>(col + (k + u * COL_GROUPS) * B.ld);
#pragma unroll
            for (int u = 0; u < COL_UNROLL; u++) {
                s.x = __fadd_rn(s.x, v[u].x);
                s.y = __fadd_rn(s.y, v[u].y);
                s.z = __fadd_rn(s.z, v[u].z);
                s.w = __fadd_rn(s.w, v[u].w);
            }
        }
        for (; k < k1; k += COL_GROUPS) {
            const float4 v = *reinterpret_cast<const float4 *>(col + k * B.ld);
            s.x = __fadd_rn(s.x, v.x);
            s.y = __fadd_rn(s.y, v.y);
            s.z = __fadd_rn(s.z, v.z);
            s.w = __fadd_rn(s.w, v.w);
        }
    }
    red[g][threadIdx.x] = s;
    __syncthreads();
    if (g == 0 && 4 * q < N) {
#pragma unroll
        for (int j = 1; j < COL_GROUPS; j++) {
            const float4 v = red[j][threadIdx.x];
            s.x = __fadd_rn(s.x, v.x);
            s.y = __fadd_rn(s.y, v.y);
            s.z = __fadd_rn(s.z, v.z);
            s.w = __fadd_rn(s.w, v.w);
        }
        *reinterpret_cast<float4 *>(part + (static_cast<int64_t>(z) * gridDim.y + chunk) * N + 4 * q) = s;
    }
}

// k_col_sum_fin over many chunks: block of COLF_WARPS warps per 32 columns
// (lane = column, coalesced), warp w adds chunks w, w + COLF_WARPS, ... in
// order with eight loads in flight (256 chunks: one round trip), then the
// warps' sums are added in a fixed tree (warp w + h into w, h = 16, 8, .., 1).
constexpr int COLF_WARPS = 32;
__global__ void __launch_bounds__(COLF_WARPS * 32)
    k_col_sum_fin32(const float *part, int chunks, int N, float *dst, int64_t off, int64_t stride) {
    __shared__ float red[COLF_WARPS][32];
    st::grid_dep_wait();  // launched programmatically dependent (st_launch_dependent)
    st::grid_dep_launch();
    const int lane = threadIdx.x & 31, w = threadIdx.x / 32;
    const int col = blockIdx.x * 32 + lane, z = blockIdx.y;
    float s = 0.0f;
    if (col < N) {
        const float *p = part + static_cast<int64_t>(z) * chunks * N + col;
        int c = w;
        for (; c + 7 * COLF_WARPS < chunks; c += 8 * COLF_WARPS) {
            float v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = p[static_cast<int64_t>(c + u * COLF_WARPS) * N];
#pragma unroll
            for (int u = 0; u < 8; u++) s = __fadd_rn(s, v[u]);
        }
        for (; c < chunks; c += COLF_WARPS) s = __fadd_rn(s, p[static_cast<int64_t>(c) * N]);
    }
    red[w][lane] = s;
    __syncthreads();
#pragma unroll
    for (int h = COLF_WARPS / 2; h > 0; h >>= 1) {
        if (w < h) red[w][lane] = __fadd_rn(red[w][lane], red[w + h][lane]);
        __syncthreads();
    }
    if (w == 0 && col < N) {
        float *d = dst + off + static_cast<int64_t>(z) * stride + col;
        *d = __fadd_rn(*d, red[0][lane]);
    }
}

// one warp per (z, column): lanes take chunks lane, lane + 32, ..., then a
// fixed butterfly
__global__ void k_col_sum_fin(const float *part, int chunks, int N, int batch, float *dst, int64_t off,
                              int64_t stride) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (i >= static_cast<int64_t>(batch) * N) return;
    const int z = static_cast<int>(i / N), col = static_cast<int>(i % N);
    float s = 0.0f;
    for (int c = lane; c < chunks; c += 32) s = __fadd_rn(s, part[(static_cast<int64_t>(z) * chunks + c) * N + col]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
    if (lane == 0) {
        float *d = dst + off + static_cast<int64_t>(z) * stride + col;
        *d = __fadd_rn(*d, s);
    }
}

// Launches `kern` so that it may begin while the previous kernel on the
// stream finishes (the kernel waits for it with grid_dep_wait).
template <typename K, typename... Args>
st_status launch_pdl(st_handle *h, K kern, dim3 grid, dim3 block, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = 0;
    cfg.stream = h->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ST_CHECK_CUDA(h, cudaLaunchKernelEx(&cfg, kern, args...));
    return ST_OK;
}

template <int BN, int STAGES, bool A_MN, bool B_MN, int AB>
st_status launch_tf32(st_handle *h, const CUtensorMap &ma, const CUtensorMap &mb, const CUtensorMap &mc,
                      const CUtensorMap &mm, const CUtensorMap &mr, const GemmArgs &g, dim3 grid) {
    using C = Cfg<BN, STAGES>;
    auto kern = AB ? k_gemm_f16<BN, STAGES, A_MN, B_MN, AB> : k_gemm_tf32<BN, STAGES, A_MN, B_MN>;
    static bool attr_done = false;  // per instantiation
    if (!attr_done) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM));
        attr_done = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(192);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = h->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // may start before the previous kernel ends
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ST_CHECK_CUDA(h, cudaLaunchKernelEx(&cfg, kern, ma, mb, mc, mm, mr, g));
    return st_after_launch(h, AB ? "k_gemm_f16" : "k_gemm_tf32");
}

template <int BN, int STAGES, int AB = 0>
st_status dispatch_tf32(st_handle *h, bool a_mn, bool b_mn, const CUtensorMap &ma, const CUtensorMap &mb,
                        const CUtensorMap &mc, const CUtensorMap &mm, const CUtensorMap &mr, const GemmArgs &g,
                        dim3 grid) {
    if (!a_mn && !b_mn) return launch_tf32<BN, STAGES, false, false, AB>(h, ma, mb, mc, mm, mr, g, grid);
    if (!a_mn && b_mn) return launch_tf32<BN, STAGES, false, true, AB>(h, ma, mb, mc, mm, mr, g, grid);
    if (a_mn && !b_mn) return launch_tf32<BN, STAGES, true, false, AB>(h, ma, mb, mc, mm, mr, g, grid);
    return launch_tf32<BN, STAGES, true, true, AB>(h, ma, mb, mc, mm, mr, g, grid);
}

Operand to_operand(const st_mat *m, int64_t packed_ld) {
    Operand o;
    o.ptr = static_cast<const float *>(m->ptr);
    o.off = m->off;
    o.stride = m->stride;
    o.inner = m->inner;
    o.ld = m->ld ? m->ld : packed_ld;
    o.grp = m->group > 0 ? m->group : 1;
    o.trans = m->trans;
    o.esize = m->dtype == ST_F32 ? 4 : 2;
    o.tdt = m->dtype == ST_F16    ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
            : m->dtype == ST_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                  : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    return o;
}

// Tensor map for an operand stored as [srows, scols] (scols contiguous).
bool operand_map(CUtensorMap *map, const Operand &o, int64_t batch, int64_t srows, int64_t scols, uint32_t box_cols,
                 uint32_t box_rows, CUtensorMapSwizzle swz, std::string *why) {
    const void *base = reinterpret_cast<const char *>(o.ptr) + o.off * o.esize;
    const int64_t outer = (o.stride != 0) ? (batch + o.grp - 1) / o.grp : 1;
    const int64_t grp = o.grp > 1 ? std::min<int64_t>(o.grp, batch) : 1;
    const uint64_t filler = static_cast<uint64_t>(o.ld) * srows;  // any valid stride for extent-1 dims
    const uint64_t inner = grp > 1 ? static_cast<uint64_t>(o.inner) : filler;
    const uint64_t stride = o.stride != 0 ? static_cast<uint64_t>(o.stride) : filler;
    return st_make_map_4d(map, o.tdt, o.esize, base, scols, srows, grp, outer, o.ld, inner, stride, box_cols, box_rows,
                          swz, why);
}

}  // namespace

// Epilogue::col_sum: col_sum[z][col] += the sum over k of b[z][:, col], in a
// fixed order (per-chunk partials, then the chunks in order).
st_status launch_col_sum(st_handle *h, const Operand &B, int64_t batch, int64_t k, int64_t n, const st_epilogue &e) {
    GemmArgs g{};
    g.K = static_cast<int>(k);
    g.N = static_cast<int>(n);
    g.batch = static_cast<int>(batch);
    const bool quad = !B.trans && n % 4 == 0 && B.ld % 4 == 0 &&
                      (reinterpret_cast<uintptr_t>(B.ptr + B.off) % 16) == 0 &&
                      (batch == 1 || (B.stride % 4 == 0 && (B.grp == 1 || B.inner % 4 == 0)));
    if (quad) {
        // B's rows 16-byte aligned: chunks of 32 rows (one round of loads
        // per thread), 64 column quads per block
        int64_t rpc = 32;
        if ((k + rpc - 1) / rpc > 65535) rpc = (k + 65534) / 65535;
        const int64_t chunks = std::max<int64_t>(1, (k + rpc - 1) / rpc);
        float *part = static_cast<float *>(st_scratch(h, SLOT_COLSUM, sizeof(float) * batch * chunks * n));
        if (!part) return ST_NO_MEMORY;
        dim3 grid(static_cast<unsigned>((n / 4 + COL_QUADS - 1) / COL_QUADS), static_cast<unsigned>(chunks),
                  static_cast<unsigned>(batch));
        ST_CHECK_CUDA(h, st_launch_dependent(h, k_col_sum_part4, grid, dim3(COL_QUADS, COL_GROUPS), 0, B, g.K, g.N,
                                             rpc, part));
        st_status s = st_after_launch(h, "k_col_sum_part4");
        if (s != ST_OK) return s;
        ST_CHECK_CUDA(h, st_launch_dependent(h, k_col_sum_fin32,
                                             dim3(static_cast<unsigned>((n + 31) / 32), static_cast<unsigned>(batch)),
                                             dim3(COLF_WARPS * 32), 0, part, static_cast<int>(chunks), g.N, e.col_sum,
                                             e.col_sum_off, e.col_sum_stride));
        s = st_after_launch(h, "k_col_sum_fin32");
        if (s != ST_OK) return s;
    } else {
        // one column per thread, chunks of >= 64 rows, so that batch * column
        // blocks * chunks fills the GPU
        const int64_t col_blocks = (n + 127) / 128;
        int64_t chunks = std::max<int64_t>(
            1, std::min<int64_t>((k + 63) / 64, (4LL * h->num_sms) / (col_blocks * batch) + 1));
        chunks = std::min<int64_t>(chunks, 65535);
        const int64_t rpc = std::max<int64_t>(1, (k + chunks - 1) / chunks);
        chunks = std::max<int64_t>(1, (k + rpc - 1) / rpc);
        float *part = static_cast<float *>(st_scratch(h, SLOT_COLSUM, sizeof(float) * batch * chunks * n));
        if (!part) return ST_NO_MEMORY;
        dim3 grid(static_cast<unsigned>(col_blocks), static_cast<unsigned>(chunks), static_cast<unsigned>(batch));
        k_col_sum_part<<<grid, 128, 0, h->stream>>>(B, g.K, g.N, rpc, part);
        st_status s = st_after_launch(h, "k_col_sum_part");
        if (s != ST_OK) return s;
        const int64_t fin_blocks = (batch * n + 7) / 8;
        if (fin_blocks > (1LL << 31) - 1) return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm: col_sum too wide");
        k_col_sum_fin<<<static_cast<unsigned>(fin_blocks), 256, 0, h->stream>>>(
            part, static_cast<int>(chunks), g.N, g.batch, e.col_sum, e.col_sum_off, e.col_sum_stride);
        s = st_after_launch(h, "k_col_sum_fin");
        if (s != ST_OK) return s;
    }
    return ST_OK;
}

static bool fits_i32(int64_t v) { return v >= 0 && v < (1ll << 31); }

// ---- TF32X3: three TF32 products that together carry an f32 product -----
//
// x = hi + lo with hi = x rounded to TF32 (cvt.rna.tf32.f32) and lo = the
// remainder, rounded to TF32 the same way (x - hi is exact in f32), so both
// reach the tensor core with their low 13 bits already zero.  Then
//   a b = a_hi b_hi + a_hi b_lo + a_lo b_hi + a_lo b_lo,
// and the last term is below 2^-22 of |a| |b|: a GEMM with K' = 3K over the
// operands concatenated along k -- A' = [a_hi  a_hi  a_lo], B' = [b_hi; b_lo;
// b_hi] -- is the f32 product to about 2^-21, on the TF32 tensor cores, with
// the TF32 kernel, its split-k and its epilogue unchanged.

__device__ __forceinline__ float tf32_rna(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// The stored [srows, scols] matrix of every batch item of `src`, copied into
// dst with its k axis (the columns if kcols, else the rows) three times as
// long: copy j of each element is hi, or lo where j == lo_copy.
__global__ void k_split3(const Operand src, int64_t srows, int64_t scols, int batch, int kcols, int lo_copy,
                         float *dst, int64_t dld, int64_t dstride) {
    const int64_t per = srows * scols, total = per * batch;
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total; i += step) {
        const int z = static_cast<int>(i / per);
        const int64_t e = i % per, r = e / scols, c = e % scols;
        const float x = src.ptr[src.off + static_cast<int64_t>(z / src.grp) * src.stride +
                                static_cast<int64_t>(z % src.grp) * src.inner + r * src.ld + c];
        const float hi = tf32_rna(x), lo = tf32_rna(x - hi);
        float *d = dst + z * dstride;
#pragma unroll
        for (int j = 0; j < 3; j++) {
            const float v = j == lo_copy ? lo : hi;
            if (kcols) d[r * dld + c + j * scols] = v;
            else d[(r + j * srows) * dld + c] = v;
        }
    }
}

st_status gemm_tf32x3(st_handle *h, const st_mat *a, const st_mat *b, const st_mat *out, int64_t batch, int64_t m,
                      int64_t k, int64_t n, const st_epilogue *epi) {
    if (a->dtype != ST_F32 || b->dtype != ST_F32 || out->dtype != ST_F32)
        return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm: ST_PREC_TF32X3 takes f32 operands");
    if (3 * k >= (1ll << 31)) return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm: k too large for TF32X3");
    cudaSetDevice(h->device);
    const Operand A = to_operand(a, a->trans ? m : k);
    const Operand B = to_operand(b, b->trans ? k : n);
    auto r4 = [](int64_t v) { return (v + 3) / 4 * 4; };
    // A' logical [m, 3k]: stored [m, 3k] or (trans) [3k, m]; B' logical [3k, n]: stored [3k, n] or (trans) [n, 3k]
    const int64_t a_ld = a->trans ? r4(m) : r4(3 * k), a_rows = a->trans ? 3 * k : m;
    const int64_t b_ld = b->trans ? r4(3 * k) : r4(n), b_rows = b->trans ? n : 3 * k;
    const int64_t a_str = a_rows * a_ld, b_str = b_rows * b_ld;
    float *buf = static_cast<float *>(st_scratch(h, SLOT_X3, sizeof(float) * batch * (a_str + b_str)));
    if (!buf) return ST_NO_MEMORY;
    float *a3 = buf, *b3 = buf + batch * a_str;
    auto split = [&](const Operand &src, int64_t srows, int64_t scols, bool kcols, int lo_copy, float *dst,
                     int64_t dld, int64_t dstr) {
        const int64_t total = srows * scols * batch;
        const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 16LL * h->num_sms));
        k_split3<<<blocks, 256, 0, h->stream>>>(src, srows, scols, static_cast<int>(batch), kcols ? 1 : 0, lo_copy,
                                                dst, dld, dstr);
        return st_after_launch(h, "k_split3");
    };
    // A' = [hi hi lo] along k: k is A's stored columns unless A is stored transposed
    st_status s = a->trans ? split(A, k, m, false, 2, a3, a_ld, a_str) : split(A, m, k, true, 2, a3, a_ld, a_str);
    if (s != ST_OK) return s;
    // B' = [hi; lo; hi] along k: k is B's stored rows unless B is stored transposed
    s = b->trans ? split(B, n, k, true, 1, b3, b_ld, b_str) : split(B, k, n, false, 1, b3, b_ld, b_str);
    if (s != ST_OK) return s;
    st_epilogue e{};
    if (epi) e = *epi;
    if (e.col_sum) {  // the column sums of the original b
        s = launch_col_sum(h, B, batch, k, n, e);
        if (s != ST_OK) return s;
        e.col_sum = nullptr;
    }
    const st_mat a2{a3, 0, a_str, 0, a_ld, 1, a->trans, ST_F32, 0};
    const st_mat b2{b3, 0, b_str, 0, b_ld, 1, b->trans, ST_F32, 0};
    return st_gemm(h, &a2, &b2, out, batch, m, 3 * k, n, &e, ST_PREC_TF32);
}

extern "C" st_status st_gemm(st_handle *h, const st_mat *a, const st_mat *b, const st_mat *out, int64_t batch,
                             int64_t m, int64_t k, int64_t n, const st_epilogue *epi, st_precision prec) {
    if (!h) return ST_INVALID_ARG;
    if (!a || !b || !out || !a->ptr || !b->ptr || !out->ptr) return h->fail(ST_INVALID_ARG, "st_gemm: null operand");
    if (batch < 1 || m < 1 || n < 1 || k < 0 || !fits_i32(m) || !fits_i32(n) || !fits_i32(k) || batch > 65535)
        return h->fail(ST_INVALID_ARG, "st_gemm: bad shape batch=%lld m=%lld k=%lld n=%lld", (long long)batch,
                       (long long)m, (long long)k, (long long)n);
    if (out->trans) return h->fail(ST_INVALID_ARG, "st_gemm: out must be stored row-major (trans = 0)");
    auto ab_of = [](int dt) { return dt == ST_F16 ? 1 : dt == ST_BF16 ? 2 : dt == ST_F32 ? 0 : -1; };
    const int ab = ab_of(a->dtype);
    if (out->dtype != ST_F32 || ab < 0 || ab_of(b->dtype) != ab)
        return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm: a and b must both be f32, f16 or bf16, out f32");
    if (a->off < 0 || b->off < 0 || out->off < 0 || a->ld < 0 || b->ld < 0 || out->ld < 0)
        return h->fail(ST_INVALID_ARG, "st_gemm: negative offset or ld");
    if (prec != ST_PREC_F32_EXACT && prec != ST_PREC_TF32 && prec != ST_PREC_F16 && prec != ST_PREC_TF32X3)
        return h->fail(ST_INVALID_ARG, "st_gemm: unknown precision");
    if (prec == ST_PREC_TF32X3) {
        if (k == 0) prec = ST_PREC_TF32;  // nothing to split: the epilogue alone
        else return gemm_tf32x3(h, a, b, out, batch, m, k, n, epi);
    }
    if ((ab != 0) != (prec == ST_PREC_F16))
        return h->fail(ST_INVALID_ARG, "st_gemm: ST_PREC_F16 goes with f16 / bf16 operands, the others with f32");
    if (ab && epi && epi->col_sum)
        return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm: col_sum needs f32 operands");
    cudaSetDevice(h->device);

    const Operand A = to_operand(a, a->trans ? m : k);
    const Operand B = to_operand(b, b->trans ? k : n);
    st_epilogue e{};
    if (epi) e = *epi;

    GemmArgs g{};
    g.M = static_cast<int>(m);
    g.N = static_cast<int>(n);
    g.K = static_cast<int>(k);
    g.batch = static_cast<int>(batch);
    g.splits = 1;
    g.c = static_cast<float *>(out->ptr);
    g.c_off = out->off;
    g.c_stride = out->stride;
    g.c_inner = out->inner;
    g.c_ld = out->ld ? out->ld : n;
    g.c_grp = out->group > 0 ? out->group : 1;
    g.bias = e.bias;
    g.bias_off = e.bias_off;
    g.bias_stride = e.bias_stride;
    g.mask = e.mask;
    g.mask_off = e.mask_off;
    g.residual = e.residual;
    g.residual_off = e.residual_off;
    g.relu = e.relu;
    g.accumulate = e.accumulate;
    g.status = h->d_status;
    {
        auto al16 = [](const void *p, int64_t off) {
            return (reinterpret_cast<uintptr_t>(p) + static_cast<uintptr_t>(off) * 4) % 16 == 0;
        };
        bool v = (n % 4 == 0) && (g.c_ld % 4 == 0) && al16(g.c, g.c_off);
        if (batch > 1) v = v && (g.c_stride % 4 == 0) && (g.c_grp == 1 || g.c_inner % 4 == 0);
        if (g.mask) v = v && al16(g.mask, g.mask_off);
        if (g.residual) v = v && al16(g.residual, g.residual_off);
        g.vec = v ? 1 : 0;
    }

    bool use_tc = (prec == ST_PREC_TF32 || prec == ST_PREC_F16) && k >= 1;
    const int bke = ab ? 64 : BK;  // elements per 128-byte k row
    const uint32_t mnw = ab ? 64 : 32;
    CUtensorMap ma, mb;
    std::string why;
    const bool a_mn = a->trans != 0, b_mn = b->trans == 0;
    // Tile width: 128 when the grid already fills the GPU, or when it is so
    // small that split-k carries the parallelism (fewer re-reads of A);
    // otherwise 64, which doubles the CTAs.
    const int64_t m_tiles = (m + BM - 1) / BM;
    const int64_t tiles128 = m_tiles * ((n + 127) / 128) * batch;
    int BN = (n > 64 && (tiles128 >= h->num_sms || tiles128 * 8 <= h->num_sms)) ? 128 : 64;
    // f32 operands: 256 wide when 128-wide tiles need more than one wave of two CTAs per SM and 256-wide ones
    // fit in one (half the MMA instructions per flop; a 2-stage ring keeps two CTAs per SM)
    const int64_t tiles256 = m_tiles * ((n + 255) / 256) * batch;
    if (!ab && n > 256 && tiles128 > 2 * h->num_sms && tiles256 <= 2 * h->num_sms) BN = 256;
    if (use_tc) {
        // A: logical [m, k]; stored [m, k] (K-major) or [k, m] (MN-major).
        // K-major tiles: 128-byte swizzle.  MN-major tf32 tiles: 128-byte
        // swizzle of 32-byte chunks (the layout the tensor core reads for
        // 32-bit MN-major operands).
        // 16-bit MN-major tiles: 128-byte swizzle of 64-element rows.
        const CUtensorMapSwizzle kmaj = CU_TENSOR_MAP_SWIZZLE_128B,
                                 mnmaj = ab ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
        const uint32_t kb = static_cast<uint32_t>(bke);
        bool okA = a_mn ? operand_map(&ma, A, batch, k, m, mnw, kb, mnmaj, &why)
                        : operand_map(&ma, A, batch, m, k, kb, BM, kmaj, &why);
        bool okB = okA && (b_mn ? operand_map(&mb, B, batch, k, n, mnw, kb, mnmaj, &why)
                                : operand_map(&mb, B, batch, n, k, kb, static_cast<uint32_t>(BN), kmaj, &why));
        use_tc = okA && okB;
    }
    if (use_tc && m_tiles > 65535) use_tc = false;
    if (ab && !use_tc)
        return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm: f16 / bf16 operands need a TMA-describable layout (%s)",
                       why.empty() ? "m too large" : why.c_str());
    if (use_tc) {
        g.a_grp = A.grp > 1 ? static_cast<int>(std::min<int64_t>(A.grp, batch)) : 1;
        g.a_outer = A.stride != 0;
        g.b_grp = B.grp > 1 ? static_cast<int>(std::min<int64_t>(B.grp, batch)) : 1;
        g.b_outer = B.stride != 0;
        if (A.grp > 1) g.a_grp = A.grp;
        if (B.grp > 1) g.b_grp = B.grp;
        const int kb_total = static_cast<int>((k + bke - 1) / bke);
        const int64_t tiles = m_tiles * ((n + BN - 1) / BN) * batch;
        // Split k only when the tiles fill less than half the GPU, keeping
        // at least 4 k blocks (128) per split; up to two CTAs per SM (one CTA
        // streams operands at about half the rate two do).
        int splits = 1;
        if (tiles * 2 <= h->num_sms && kb_total >= 8) {
            splits = static_cast<int>(std::min<int64_t>(std::min<int64_t>(2 * h->num_sms / tiles, kb_total / 4), 32));
            splits = std::max(splits, 1);
        }
        int kbps = (kb_total + splits - 1) / splits;
        splits = (kb_total + kbps - 1) / kbps;
        if (batch * splits > 65535) {
            splits = 1;
            kbps = kb_total;
        }
        g.splits = splits;
        g.kb_per_split = kbps;
        if (splits > 1) {
            g.partial = static_cast<float *>(st_scratch(h, SLOT_SPLITK, sizeof(float) * batch * splits * m * n));
            if (!g.partial) return ST_NO_MEMORY;
        }
        // Epilogue::col_sum: inside the GEMM when it splits k over 128-wide tiles of a row-major f32 b (the
        // first row of tiles adds up the b tiles it stages; k_splitk_reduce adds the splits in order), else
        // by its own two launches
        if (e.col_sum && !ab && b_mn && splits > 1 && BN == 128 && batch == 1) {
            g.cs_part = static_cast<float *>(st_scratch(h, SLOT_COLSUM, sizeof(float) * splits * n));
            if (!g.cs_part) return ST_NO_MEMORY;
            g.cs_dst = e.col_sum;
            g.cs_off = e.col_sum_off;
        } else if (e.col_sum) {
            const st_status cs = launch_col_sum(h, B, batch, k, n, e);
            if (cs != ST_OK) return cs;
        }
        // epilogue through TMA stores when there is no split-k and out is
        // TMA-describable (16-byte aligned start and rows)
        CUtensorMap mc;
        std::memset(&mc, 0, sizeof mc);
        g.c_outer = out->stride != 0;
        if (splits == 1 && g.vec && (batch == 1 || out->stride != 0)) {
            const Operand Cm = to_operand(out, n);
            g.tma_store = operand_map(&mc, Cm, batch, m, n, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B, nullptr) ? 1 : 0;
        }
        // mask / residual (out's layout at their own offsets) by TMA as well
        CUtensorMap mm, mr;
        std::memset(&mm, 0, sizeof mm);
        std::memset(&mr, 0, sizeof mr);
        if (g.tma_store && (g.mask || g.residual)) {
            auto aux_map = [&](CUtensorMap *map, const float *ptr, int64_t off) {
                Operand o = to_operand(out, n);
                o.ptr = ptr;
                o.off = off;
                return operand_map(map, o, batch, m, n, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B, nullptr);
            };
            g.tma_aux = (!g.mask || aux_map(&mm, g.mask, g.mask_off)) &&
                        (!g.residual || aux_map(&mr, g.residual, g.residual_off)) ? 1 : 0;
        }
        dim3 grid(static_cast<unsigned>((n + BN - 1) / BN), static_cast<unsigned>(m_tiles),
                  static_cast<unsigned>(batch * splits));
        st_status s;
        if (ab == 1)
            s = BN == 64 ? dispatch_tf32<64, 4, 1>(h, a_mn, b_mn, ma, mb, mc, mm, mr, g, grid)
                         : dispatch_tf32<128, 3, 1>(h, a_mn, b_mn, ma, mb, mc, mm, mr, g, grid);
        else if (ab == 2)
            s = BN == 64 ? dispatch_tf32<64, 4, 2>(h, a_mn, b_mn, ma, mb, mc, mm, mr, g, grid)
                         : dispatch_tf32<128, 3, 2>(h, a_mn, b_mn, ma, mb, mc, mm, mr, g, grid);
        else
            s = BN == 64    ? dispatch_tf32<64, 4>(h, a_mn, b_mn, ma, mb, mc, mm, mr, g, grid)
                : BN == 256 ? dispatch_tf32<256, 2>(h, a_mn, b_mn, ma, mb, mc, mm, mr, g, grid)
                            : dispatch_tf32<128, 3>(h, a_mn, b_mn, ma, mb, mc, mm, mr, g, grid);
        if (s != ST_OK) return s;
        if (splits > 1) {
            const int groups = static_cast<int>((n + 3) / 4);
            const int threads = groups >= 128 ? 128 : 32 * ((groups + 31) / 32);
            dim3 rgrid(static_cast<unsigned>((groups + threads - 1) / threads), static_cast<unsigned>(std::min<int64_t>(m, 65535)),
                       static_cast<unsigned>(batch));
            st_status rs = launch_pdl(h, k_splitk_reduce, rgrid, dim3(threads), g);
            if (rs != ST_OK) return rs;
            return st_after_launch(h, "k_splitk_reduce");
        }
        return ST_OK;
    }
    if (e.col_sum) {
        const st_status cs = launch_col_sum(h, B, batch, k, n, e);
        if (cs != ST_OK) return cs;
    }
    dim3 grid(static_cast<unsigned>((n + EX_T - 1) / EX_T), static_cast<unsigned>((m + EX_T - 1) / EX_T),
              static_cast<unsigned>(batch));
    if (grid.y > 65535) return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm: m too large for the exact kernel");
    k_gemm_exact<<<grid, 256, 0, h->stream>>>(A, B, g);
    return st_after_launch(h, "k_gemm_exact");
}

extern "C" st_status st_matmul_host(st_handle *h, const float *a, const float *b, float *out, int64_t m, int64_t k,
                                    int64_t n, int32_t ta, int32_t tb, st_precision prec) {
    if (!h) return ST_INVALID_ARG;
    if (!a || !b || !out) return h->fail(ST_INVALID_ARG, "st_matmul_host: null buffer");
    if (m < 1 || n < 1 || k < 0) return h->fail(ST_INVALID_ARG, "st_matmul_host: bad shape");
    cudaSetDevice(h->device);
    const size_t ab = sizeof(float) * m * k, bb = sizeof(float) * k * n, cb = sizeof(float) * m * n;
    float *da = static_cast<float *>(st_scratch(h, SLOT_HOST_A, ab));
    float *db = static_cast<float *>(st_scratch(h, SLOT_HOST_B, bb));
    float *dc = static_cast<float *>(st_scratch(h, SLOT_HOST_C, cb));
    if (!da || !db || !dc) return ST_NO_MEMORY;
    if (ab) ST_CHECK_CUDA(h, cudaMemcpyAsync(da, a, ab, cudaMemcpyHostToDevice, h->stream));
    if (bb) ST_CHECK_CUDA(h, cudaMemcpyAsync(db, b, bb, cudaMemcpyHostToDevice, h->stream));
    st_mat A{da, 0, 0, 0, 0, 1, ta, ST_F32, 0};
    st_mat B{db, 0, 0, 0, 0, 1, tb, ST_F32, 0};
    st_mat C{dc, 0, 0, 0, 0, 1, 0, ST_F32, 0};
    st_status s = st_gemm(h, &A, &B, &C, 1, m, k, n, nullptr, prec);
    if (s != ST_OK) return s;
    ST_CHECK_CUDA(h, cudaMemcpyAsync(out, dc, cb, cudaMemcpyDeviceToHost, h->stream));
    return st_sync(h);
}

// ---------------------------------------------------------------------------
// st_gemm_tf32_fixed_scratch: the TF32 GEMM for callers that cannot let this
// library allocate device memory.
//
// st_gemm keeps its split-k partial sums in the handle's scratch pool, which
// grows with cudaMalloc the first time a larger problem comes along.  Some
// callers cannot accept that: a host program that has already carved the
// GPU's memory into its own pools and lends none to plug-ins, or a
// latency-critical loop in which a cudaMalloc / cudaFree (which may
// synchronise the whole device) would stall it.  This entry point computes the
// same result as st_gemm with ST_PREC_TF32 but takes its partial sums from one
// array compiled into the library, so the call itself never allocates.
//
// The array is FIXED_SCRATCH_FLOATS floats (8 MiB); every GPU that loads the
// library holds it until the process exits.  All calls share it, and it keeps
// whatever the last call left in it, so two calls that overlap on the GPU (on
// different streams, or from different host threads) race on it.  Nothing in
// it has to start at zero: every split writes each element of its partial
// before the reduction reads it.
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t FIXED_SCRATCH_FLOATS = 2 * 1024 * 1024;      // 8 MiB of f32 partial sums
constexpr int64_t FIXED_MAX_OUTPUT = FIXED_SCRATCH_FLOATS / 2;  // room for at least two splits

static __device__ __align__(256) float g_fixed_partials[FIXED_SCRATCH_FLOATS];

constexpr int FIXED_MAX_DEVICES = 64;
float *g_fixed_ptr[FIXED_MAX_DEVICES] = {};
std::mutex g_fixed_mu;

// The device address of g_fixed_partials on `device` (which must be current).
// Looked up once per device; in host code the symbol itself is only a host
// stand-in and must never be handed to a kernel.
float *fixed_scratch(int device) {
    if (device < 0 || device >= FIXED_MAX_DEVICES) return nullptr;
    std::lock_guard<std::mutex> lock(g_fixed_mu);
    if (!g_fixed_ptr[device]) {
        void *p = nullptr;
        if (cudaGetSymbolAddress(&p, g_fixed_partials) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        g_fixed_ptr[device] = static_cast<float *>(p);
    }
    return g_fixed_ptr[device];
}

}  // namespace

extern "C" st_status st_gemm_tf32_fixed_scratch(st_handle *h, const st_mat *a, const st_mat *b, const st_mat *out,
                                                int64_t batch, int64_t m, int64_t k, int64_t n,
                                                const st_epilogue *epi) {
    if (!h || !a || !b || !out || !a->ptr || !b->ptr || !out->ptr) return ST_INVALID_ARG;
    if (batch < 1 || m < 1 || n < 1 || k < 1 || !fits_i32(m) || !fits_i32(n) || !fits_i32(k) || batch > 65535)
        return ST_INVALID_ARG;
    if (out->trans || a->off < 0 || b->off < 0 || out->off < 0 || a->ld < 0 || b->ld < 0 || out->ld < 0)
        return ST_INVALID_ARG;
    if (a->dtype != ST_F32 || b->dtype != ST_F32 || out->dtype != ST_F32) return ST_UNSUPPORTED_SHAPE;
    if (batch * m * n > FIXED_MAX_OUTPUT) return ST_UNSUPPORTED_SHAPE;  // output beyond the fixed scratch
    if (cudaSetDevice(h->device) != cudaSuccess) return ST_CUDA_ERROR;
    float *scratch = fixed_scratch(h->device);
    if (!scratch) return ST_CUDA_ERROR;

    const Operand A = to_operand(a, a->trans ? m : k);
    const Operand B = to_operand(b, b->trans ? k : n);
    st_epilogue e{};
    if (epi) e = *epi;
    GemmArgs g{};
    g.M = static_cast<int>(m);
    g.N = static_cast<int>(n);
    g.K = static_cast<int>(k);
    g.batch = static_cast<int>(batch);
    g.c = static_cast<float *>(out->ptr);
    g.c_off = out->off;
    g.c_stride = out->stride;
    g.c_inner = out->inner;
    g.c_ld = out->ld ? out->ld : n;
    g.c_grp = out->group > 0 ? out->group : 1;
    g.bias = e.bias;
    g.bias_off = e.bias_off;
    g.bias_stride = e.bias_stride;
    g.mask = e.mask;
    g.mask_off = e.mask_off;
    g.residual = e.residual;
    g.residual_off = e.residual_off;
    g.relu = e.relu;
    g.accumulate = e.accumulate;
    g.status = h->d_status;
    {
        auto al16 = [](const void *p, int64_t off) {
            return (reinterpret_cast<uintptr_t>(p) + static_cast<uintptr_t>(off) * 4) % 16 == 0;
        };
        bool v = (n % 4 == 0) && (g.c_ld % 4 == 0) && al16(g.c, g.c_off);
        if (batch > 1) v = v && (g.c_stride % 4 == 0) && (g.c_grp == 1 || g.c_inner % 4 == 0);
        if (g.mask) v = v && al16(g.mask, g.mask_off);
        if (g.residual) v = v && al16(g.residual, g.residual_off);
        g.vec = v ? 1 : 0;
    }

    const int64_t m_tiles = (m + BM - 1) / BM;
    if (m_tiles > 65535) return ST_UNSUPPORTED_SHAPE;
    const int64_t tiles128 = m_tiles * ((n + 127) / 128) * batch;
    const int BN = (n > 64 && (tiles128 >= h->num_sms || tiles128 * 8 <= h->num_sms)) ? 128 : 64;
    const bool a_mn = a->trans != 0, b_mn = b->trans == 0;
    CUtensorMap ma, mb;
    const CUtensorMapSwizzle kmaj = CU_TENSOR_MAP_SWIZZLE_128B, mnmaj = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
    const bool okA = a_mn ? operand_map(&ma, A, batch, k, m, 32, 32, mnmaj, nullptr)
                          : operand_map(&ma, A, batch, m, k, 32, BM, kmaj, nullptr);
    const bool okB = okA && (b_mn ? operand_map(&mb, B, batch, k, n, 32, 32, mnmaj, nullptr)
                                  : operand_map(&mb, B, batch, n, k, 32, static_cast<uint32_t>(BN), kmaj, nullptr));
    if (!okA || !okB) return ST_UNSUPPORTED_SHAPE;  // needs TMA-describable (16-byte aligned) operands
    g.a_grp = A.grp > 1 ? A.grp : 1;
    g.a_outer = A.stride != 0;
    g.b_grp = B.grp > 1 ? B.grp : 1;
    g.b_outer = B.stride != 0;

    // The split plan of st_gemm, capped so the partials fit the fixed array.
    const int kb_total = static_cast<int>((k + BK - 1) / BK);
    const int64_t tiles = m_tiles * ((n + BN - 1) / BN) * batch;
    int splits = 1;
    if (tiles * 2 <= h->num_sms && kb_total >= 8)
        splits = static_cast<int>(std::min<int64_t>(std::min<int64_t>(h->num_sms / tiles, kb_total / 4), 16));
    splits = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(splits, FIXED_SCRATCH_FLOATS / (batch * m * n))));
    int kbps = (kb_total + splits - 1) / splits;
    splits = (kb_total + kbps - 1) / kbps;
    if (batch * splits > 65535) {
        splits = 1;
        kbps = kb_total;
    }
    g.splits = splits;
    g.kb_per_split = kbps;
    g.partial = splits > 1 ? scratch : nullptr;

    if (e.col_sum) {
        const int64_t total = batch * n;
        const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
        k_col_sum<<<blocks, 256, 0, h->stream>>>(B, g.K, g.N, g.batch, e.col_sum, e.col_sum_off, e.col_sum_stride);
        if (cudaGetLastError() != cudaSuccess) return ST_CUDA_ERROR;
    }
    dim3 grid(static_cast<unsigned>((n + BN - 1) / BN), static_cast<unsigned>(m_tiles),
              static_cast<unsigned>(batch * splits));
    CUtensorMap mc, mm, mr;  // the fixed-scratch path keeps the register-staged epilogue (tma_store = 0)
    std::memset(&mc, 0, sizeof mc);
    std::memset(&mm, 0, sizeof mm);
    std::memset(&mr, 0, sizeof mr);
    const st_status s = BN == 64 ? dispatch_tf32<64, 4>(h, a_mn, b_mn, ma, mb, mc, mm, mr, g, grid)
                                 : dispatch_tf32<128, 3>(h, a_mn, b_mn, ma, mb, mc, mm, mr, g, grid);
    if (s != ST_OK) return s;
    if (splits > 1) {
        const int groups = static_cast<int>((n + 3) / 4);
        const int threads = groups >= 128 ? 128 : 32 * ((groups + 31) / 32);
        dim3 rgrid(static_cast<unsigned>((groups + threads - 1) / threads),
                   static_cast<unsigned>(std::min<int64_t>(m, 65535)), static_cast<unsigned>(batch));
        k_splitk_reduce<<<rgrid, threads, 0, h->stream>>>(g);
        if (cudaGetLastError() != cudaSuccess) return ST_CUDA_ERROR;
    }
    return ST_OK;
}

// ---- grouped GEMM ----------------------------------------------------------

extern "C" st_status st_gemm_group(st_handle *h, const st_group_gemm *gemms, int32_t count) {
    if (!h) return ST_INVALID_ARG;
    if (!gemms || count < 1 || count > GRP_MAX) return h->fail(ST_INVALID_ARG, "st_gemm_group: 1..%d GEMMs", GRP_MAX);
    cudaSetDevice(h->device);
    static GroupPlan plan;  // host staging of the kernel parameter (large: built in place)
    static std::mutex plan_mu;
    std::lock_guard<std::mutex> lock(plan_mu);
    std::memset(&plan, 0, sizeof plan);
    plan.count = count;
    plan.status = h->d_status;
    int tasks = 0, split_tiles = 0;
    int64_t part_floats = 0;
    for (int i = 0; i < count; i++) {
        const st_group_gemm &q = gemms[i];
        GroupGemm &G = plan.gemm[i];
        GroupMaps &MP = plan.maps[i];
        const int64_t m = q.m, k = q.k, n = q.n;
        if (!q.a.ptr || !q.b.ptr || !q.out.ptr || m < 1 || k < 1 || n < 1 || !fits_i32(m) || !fits_i32(n) ||
            !fits_i32(k) || q.out.trans || q.a.off < 0 || q.b.off < 0 || q.out.off < 0 || q.a.ld < 0 || q.b.ld < 0 ||
            q.out.ld < 0 || (q.after >> i) != 0)
            return h->fail(ST_INVALID_ARG, "st_gemm_group: bad GEMM %d", i);
        if (q.a.dtype != ST_F32 || q.b.dtype != ST_F32 || q.out.dtype != ST_F32 || (q.epi && q.epi->col_sum))
            return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm_group: GEMM %d: f32 operands, no col_sum", i);
        st_epilogue e{};
        if (q.epi) e = *q.epi;
        GemmArgs &g = G.g;
        g.M = static_cast<int>(m);
        g.N = static_cast<int>(n);
        g.K = static_cast<int>(k);
        g.batch = 1;
        g.splits = 1;
        g.c = static_cast<float *>(q.out.ptr);
        g.c_off = q.out.off;
        g.c_ld = q.out.ld ? q.out.ld : n;
        g.c_grp = 1;
        g.bias = e.bias;
        g.bias_off = e.bias_off;
        g.mask = e.mask;
        g.mask_off = e.mask_off;
        g.residual = e.residual;
        g.residual_off = e.residual_off;
        g.relu = e.relu;
        g.accumulate = e.accumulate;
        g.status = h->d_status;
        auto al16 = [](const void *p, int64_t off) {
            return (reinterpret_cast<uintptr_t>(p) + static_cast<uintptr_t>(off) * 4) % 16 == 0;
        };
        g.vec = (n % 4 == 0) && (g.c_ld % 4 == 0) && al16(g.c, g.c_off) && (!g.mask || al16(g.mask, g.mask_off)) &&
                (!g.residual || al16(g.residual, g.residual_off));
        if (!g.vec) return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm_group: GEMM %d: output rows not 16-byte aligned", i);
        g.tma_store = 1;
        const Operand A = to_operand(&q.a, q.a.trans ? m : k);
        const Operand B = to_operand(&q.b, q.b.trans ? k : n);
        G.a_mn = q.a.trans != 0;
        G.b_mn = q.b.trans == 0;
        const int64_t m_tiles = (m + BM - 1) / BM;
        const int64_t tiles128 = m_tiles * ((n + 127) / 128);
        G.bn = (n > 64 && (tiles128 >= h->num_sms || tiles128 * 8 <= h->num_sms)) ? 128 : 64;
        const CUtensorMapSwizzle kmaj = CU_TENSOR_MAP_SWIZZLE_128B, mnmaj = CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B;
        const bool ok = (G.a_mn ? operand_map(&MP.tmA, A, 1, k, m, 32, 32, mnmaj, nullptr)
                                : operand_map(&MP.tmA, A, 1, m, k, 32, BM, kmaj, nullptr)) &&
                        (G.b_mn ? operand_map(&MP.tmB, B, 1, k, n, 32, 32, mnmaj, nullptr)
                                : operand_map(&MP.tmB, B, 1, n, k, 32, static_cast<uint32_t>(G.bn), kmaj, nullptr)) &&
                        operand_map(&MP.tmC, to_operand(&q.out, n), 1, m, n, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B,
                                    nullptr);
        if (!ok) return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm_group: GEMM %d is not TMA-describable", i);
        G.m_tiles = static_cast<int>(m_tiles);
        G.n_tiles = static_cast<int>((n + G.bn - 1) / G.bn);
        const int tiles = G.m_tiles * G.n_tiles;
        const int kb_total = static_cast<int>((k + BK - 1) / BK);
        // split k as st_gemm does (while the tiles fill less than half the GPU, >= 4 k blocks per split, up to
        // two CTAs per SM), so every GEMM's sums are the same, bit for bit
        int splits = 1;
        if (tiles * 2 <= h->num_sms && kb_total >= 8)
            splits = std::max(1, std::min(std::min(2 * h->num_sms / tiles, kb_total / 4), 32));
        G.kb_per_split = (kb_total + splits - 1) / splits;
        G.splits = (kb_total + G.kb_per_split - 1) / G.kb_per_split;
        // a split GEMM's tiles are summed by red_parts reduction tasks each (row bands of 16 rows)
        G.red_parts = G.splits > 1 ? BM / 16 : 0;
        G.need = G.splits > 1 ? tiles * G.red_parts : tiles;
        G.task_begin = tasks;
        tasks += tiles * G.splits + tiles * G.red_parts;
        G.tile_begin = split_tiles;
        if (G.splits > 1) {
            split_tiles += tiles;
            g.partial = reinterpret_cast<float *>(part_floats);  // offset for now; based below
            part_floats += static_cast<int64_t>(G.splits) * m * n;
        }
        G.after = q.after;
    }
    plan.tasks = tasks;
    float *part = nullptr;
    if (part_floats > 0) {
        part = static_cast<float *>(st_scratch(h, SLOT_SPLITK, sizeof(float) * part_floats));
        if (!part) return ST_NO_MEMORY;
    }
    for (int i = 0; i < count; i++) {
        GroupGemm &G = plan.gemm[i];
        if (G.splits == 1) continue;
        GroupMaps &MP = plan.maps[i];
        G.g.partial = part + reinterpret_cast<intptr_t>(G.g.partial);
        Operand P{};
        P.ptr = G.g.partial;
        P.ld = G.g.N;
        P.grp = G.splits;
        P.inner = static_cast<int64_t>(G.g.M) * G.g.N;
        if (!operand_map(&MP.tmP, P, G.splits, G.g.M, G.g.N, 32, 32, CU_TENSOR_MAP_SWIZZLE_128B, nullptr))
            return h->fail(ST_UNSUPPORTED_SHAPE, "st_gemm_group: partials of GEMM %d not TMA-describable", i);
    }
    // the counters are left at zero by every launch (the last CTA resets them);
    // they are zeroed here only when their memory is new
    plan.ctl_words = CTL_TILES + split_tiles;
    const size_t ctl_bytes = sizeof(unsigned int) * plan.ctl_words;
    plan.ctl = static_cast<unsigned int *>(st_scratch(h, SLOT_GROUP, ctl_bytes));
    if (!plan.ctl) return ST_NO_MEMORY;
    if (plan.ctl != h->group_ctl || ctl_bytes > h->group_ctl_bytes) {
        ST_CHECK_CUDA(h, cudaMemsetAsync(plan.ctl, 0, ctl_bytes, h->stream));
        h->group_ctl = plan.ctl;
        h->group_ctl_bytes = ctl_bytes;
    }
    static bool attr_set[64] = {};
    if (h->device >= 0 && h->device < 64 && !attr_set[h->device]) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_gemm_group, cudaFuncAttributeMaxDynamicSharedMemorySize, GRP_SMEM));
        attr_set[h->device] = true;
    }
    const int grid = std::min(2 * h->num_sms, tasks);  // two CTAs per SM
    k_gemm_group<<<grid, GRP_THREADS, GRP_SMEM, h->stream>>>(plan);
    return st_after_launch(h, "k_gemm_group");
}
