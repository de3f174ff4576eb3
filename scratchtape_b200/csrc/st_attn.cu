// st_attn.cu -- fused causal attention, forward and backward, per head.
//
// Reference: the attention of TransformerBlock::forward_full
// (src/nn.rs:646-671) and of DeviceTape::block_forward / backward
// (src/gpu_step/tape.rs:481-484, :349-375):
//   S = (Q K^T) * scale, causal mask (-inf above the diagonal, src/nn.rs:396-407),
//   P = softmax(S) (row max taken after masking, masked entries exactly 0),
//   O = P V;
// backward (src/tape.rs:90-112 for the two batched matmuls, the softmax
// backward of src/gpu_step/rows.rs:117-123):
//   dV = P^T dO, dP = dO V^T, dS = P * (dP - rowsum(dO * O)) * scale,
//   dQ = dS K, dK = dS^T Q.
//
// B200 design.  A head of up to 128 rows fits one tile, so one CTA (8 warps,
// two threads per row) does a whole head with no online rescaling: Q, K, V (and
// dO) are staged once in 128-byte-swizzled shared memory (16 KB each at
// d = 64), every contraction is a tcgen05 kind::f16 MMA with f32
// accumulation in TMEM, and every transposed operand (K^T, V as an N-major
// B, P^T, dS^T, Q and K as N-major B) is expressed by the shared-memory
// descriptor alone -- nothing is ever transposed in memory.  Softmax runs
// in registers on the TMEM rows; P and dS go to shared memory as f16, the
// A operand of the next MMA.  The forward writes O (f16) and the row
// log-sum-exp (f32) the backward needs.
#include <cuda_fp16.h>

#include "st_internal.h"
#include "st_ptx.cuh"

namespace {

constexpr int AT = 128;               // rows per head tile (max t)
constexpr int AD = 64;                // head width
constexpr int TILE = AT * AD * 2;     // one [128 x 64] f16 operand: 16 KB
constexpr int PT = AT * AT * 2;       // one [128 x 128] f16 operand: 32 KB
constexpr int ATHREADS = 256;  // two threads per row

struct AttnArgs {
    const __half *q, *k, *v, *o, *dout;
    __half *out, *dq, *dk, *dv;
    float *lse;
    int bh, t;
    float scale;
    int causal;
    int *status;
};

// Bounded wait on a barrier that the MMA thread's commit completes.
__device__ __forceinline__ bool await(uint64_t *bar, uint32_t parity, int *status) {
    if (st::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = st::globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (st::mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if ((i & 7u) == 0 && st::globaltimer() - t0 > st::WAIT_LIMIT_NS) {
            st::set_status(status, st::DEV_TIMEOUT_ACC);
            return false;
        }
    }
}

// Half `half` (32 of the 64 columns) of row r (< t, else zeros) of a [t, 64]
// f16 head into a swizzled 16 KB tile.
__device__ __forceinline__ void stage_half_rows(uint8_t *dst, const __half *src, int r, int half, int t) {
    const uint4 *s = reinterpret_cast<const uint4 *>(src + static_cast<int64_t>(r) * AD);
#pragma unroll
    for (int c = 4 * half; c < 4 * half + 4; c++) {
        const uint4 v = r < t ? __ldg(s + c) : make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4 *>(dst + st::sw128_offset(r, c)) = v;
    }
}

// 16 f32 values -> 8 packed f16 pairs.
__device__ __forceinline__ void pack16(const float (&x)[16], uint32_t (&o)[8]) {
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const __half2 h = __floats2half2_rn(x[2 * i], x[2 * i + 1]);
        o[i] = *reinterpret_cast<const uint32_t *>(&h);
    }
}

// Columns [c0, c0+16) of row r of a [128 x 128] f16 operand tile (two 64-column
// 128-byte-swizzled halves of 16 KB).
__device__ __forceinline__ void put16(uint8_t *tile, int r, int c0, const uint32_t (&o)[8]) {
    uint8_t *half = tile + (c0 >> 6) * (PT / 2);
    const int piece = (c0 & 63) >> 3;
    *reinterpret_cast<uint4 *>(half + st::sw128_offset(r, piece)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4 *>(half + st::sw128_offset(r, piece + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
}

// K-major operand descriptor: [rows x 64] chunk at `base`, k step kk (16 elements).
__device__ __forceinline__ uint64_t kmaj(uint32_t base, int kk) { return st::sdesc_sw128(base + kk * 32, 16, 1024); }
// K-major descriptor into a [128 x 128] tile: k step kk of 8 (64 columns per half).
__device__ __forceinline__ uint64_t kmaj128(uint32_t base, int kk) {
    return st::sdesc_sw128(base + (kk >> 2) * (PT / 2) + (kk & 3) * 32, 16, 1024);
}
// MN-major operand descriptor: rows are K, 64-element (128-byte) rows along
// MN; k step kk covers rows 16kk..16kk+15; MN atoms (64 wide) mn_stride apart.
__device__ __forceinline__ uint64_t mnmaj(uint32_t base, int kk, uint32_t mn_stride) {
    return st::sdesc_make(base + kk * 2048, mn_stride, 1024, st::LAYOUT_SW128);
}

// e^x for the softmax numerators, as 2^(x * log2 e) on the SFU: P is rounded
// to f16 right after, so its ~2 ulp f32 error is far below what is kept.
__device__ __forceinline__ float fast_exp(float x) { return exp2f(x * 1.4426950408889634f); }

// Threads r and r + 128 share row r % 128: thread r < 128 owns columns
// [0, 64) of the row, thread r + 128 columns [64, 128) (warps w and w + 4 read
// the same TMEM lanes).  Row reductions combine the two halves through `red`.
__global__ void __launch_bounds__(ATHREADS, 1) k_attn_fwd(const AttnArgs g) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem, *sK = smem + TILE, *sV = smem + 2 * TILE, *sP = smem + 3 * TILE;
    float *red = reinterpret_cast<float *>(sP + PT);  // [2][128]
    uint64_t *bar = reinterpret_cast<uint64_t *>(red + 2 * AT);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 2);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int r = tid & (AT - 1), half = tid >> 7;
    const int64_t head = static_cast<int64_t>(blockIdx.x) * g.t * AD;

    if (tid == 0) {
        st::mbar_init(&bar[0], 1);
        st::mbar_init(&bar[1], 1);
        st::fence_mbar_init();
    }
    if (warp == 0) {
        st::tmem_alloc(tslot, 256);
        st::tmem_relinquish();
    }
    stage_half_rows(sQ, g.q + head, r, half, g.t);
    stage_half_rows(sK, g.k + head, r, half, g.t);
    stage_half_rows(sV, g.v + head, r, half, g.t);
    st::fence_proxy_async_smem();
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t tmem = *tslot, tS = tmem, tO = tmem + 128;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;

    if (tid == 0) {  // S = Q K^T
        constexpr uint32_t id = st::idesc_make(1, 0, false, false, AT, AT);
        const uint32_t q = st::smem_u32(sQ), k = st::smem_u32(sK);
#pragma unroll
        for (int kk = 0; kk < AD / 16; kk++) st::umma_f16(tS, kmaj(q, kk), kmaj(k, kk), id, kk > 0 ? 1u : 0u);
        st::umma_commit(&bar[0]);
    }
    bool ok = await(&bar[0], 0, g.status);
    st::tc_fence_after();

    // softmax of row r over this thread's 64 columns: masked max, exchange,
    // p = exp(s - max) as f16 into sP, partial sums, exchange
    const int lim = r < g.t ? (g.causal ? r + 1 : g.t) : 0;  // columns < lim are visible
    const int cbase = half * 64;
    uint32_t x[64];
    st::tmem_ld32(tS + lane_base + cbase, *reinterpret_cast<uint32_t(*)[32]>(&x[0]));
    st::tmem_ld32(tS + lane_base + cbase + 32, *reinterpret_cast<uint32_t(*)[32]>(&x[32]));
    st::tmem_ld_wait();
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < 64; j++)
        if (cbase + j < lim) m = fmaxf(m, __uint_as_float(x[j]) * g.scale);
    red[half * AT + r] = m;
    __syncthreads();
    m = fmaxf(m, red[(half ^ 1) * AT + r]);
    float l = 0.0f;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        float p[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const int col = cbase + 16 * c + j;
            p[j] = col < lim ? fast_exp(__uint_as_float(x[16 * c + j]) * g.scale - m) : 0.0f;
            l += p[j];
        }
        uint32_t o[8];
        pack16(p, o);
        put16(sP, r, cbase + 16 * c, o);
    }
    __syncthreads();  // every thread has read red (max) before it is reused for sums
    red[half * AT + r] = l;
    st::fence_proxy_async_smem();
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    l += red[(half ^ 1) * AT + r];
    if (half == 0 && r < g.t) g.lse[static_cast<int64_t>(blockIdx.x) * g.t + r] = lim > 0 ? m + logf(l) : -INFINITY;

    if (tid == 0) {  // O = P V   (V: B operand, N = d contiguous -> MN-major)
        constexpr uint32_t id = st::idesc_make(1, 0, false, true, AT, AD);
        const uint32_t p = st::smem_u32(sP), v = st::smem_u32(sV);
#pragma unroll
        for (int kk = 0; kk < AT / 16; kk++) st::umma_f16(tO, kmaj128(p, kk), mnmaj(v, kk, TILE), id, kk > 0 ? 1u : 0u);
        st::umma_commit(&bar[1]);
    }
    ok = await(&bar[1], 0, g.status) && ok;
    st::tc_fence_after();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll 1
    for (int c0 = half * (AD / 2); c0 < (half + 1) * (AD / 2); c0 += 16) {
        uint32_t y16[16];
        st::tmem_ld16(tO + lane_base + c0, y16);
        st::tmem_ld_wait();
        float y[16];
#pragma unroll
        for (int j = 0; j < 16; j++) y[j] = __uint_as_float(y16[j]) * inv;
        uint32_t o[8];
        pack16(y, o);
        if (r < g.t && ok) {
            uint4 *dst = reinterpret_cast<uint4 *>(g.out + head + static_cast<int64_t>(r) * AD + c0);
            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
        }
    }
    st::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, 256);
    }
}

__global__ void __launch_bounds__(ATHREADS, 1) k_attn_bwd(const AttnArgs g) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem, *sK = smem + TILE, *sV = smem + 2 * TILE, *sO = smem + 3 * TILE;  // sO holds dO
    uint8_t *sP = smem + 4 * TILE, *sS = sP + PT;                                          // P, dS
    float *red = reinterpret_cast<float *>(sS + PT);                                       // [2][128]
    uint64_t *bar = reinterpret_cast<uint64_t *>(red + 2 * AT);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 2);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int r = tid & (AT - 1), half = tid >> 7;
    const int64_t head = static_cast<int64_t>(blockIdx.x) * g.t * AD;

    if (tid == 0) {
        st::mbar_init(&bar[0], 1);
        st::mbar_init(&bar[1], 1);
        st::fence_mbar_init();
    }
    if (warp == 0) {
        st::tmem_alloc(tslot, 512);
        st::tmem_relinquish();
    }
    stage_half_rows(sQ, g.q + head, r, half, g.t);
    stage_half_rows(sK, g.k + head, r, half, g.t);
    stage_half_rows(sV, g.v + head, r, half, g.t);
    stage_half_rows(sO, g.dout + head, r, half, g.t);
    // D_r = sum_d dO[r,d] * O[r,d], this thread's 32 of the 64 d, then exchanged
    float dsum = 0.0f;
    if (r < g.t) {
        const uint4 *po = reinterpret_cast<const uint4 *>(g.o + head + static_cast<int64_t>(r) * AD) + 4 * half;
        const uint4 *pd = reinterpret_cast<const uint4 *>(g.dout + head + static_cast<int64_t>(r) * AD) + 4 * half;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 a = __ldg(po + c), b = __ldg(pd + c);
            const uint32_t av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 fa = __half22float2(*reinterpret_cast<const __half2 *>(&av[i]));
                const float2 fb = __half22float2(*reinterpret_cast<const __half2 *>(&bv[i]));
                dsum = fmaf(fa.x, fb.x, dsum);
                dsum = fmaf(fa.y, fb.y, dsum);
            }
        }
    }
    red[half * AT + r] = dsum;
    const float lse = r < g.t ? g.lse[static_cast<int64_t>(blockIdx.x) * g.t + r] : 0.0f;
    st::fence_proxy_async_smem();
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    dsum = red[0 * AT + r] + red[1 * AT + r];  // same order in both halves
    const uint32_t tmem = *tslot;
    const uint32_t tS = tmem, tdP = tmem + 128, tdV = tmem + 256, tdK = tmem + 320, tdQ = tmem + 384;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;

    if (tid == 0) {  // S = Q K^T, dP = dO V^T
        constexpr uint32_t id = st::idesc_make(1, 0, false, false, AT, AT);
        const uint32_t q = st::smem_u32(sQ), k = st::smem_u32(sK), v = st::smem_u32(sV), d = st::smem_u32(sO);
#pragma unroll
        for (int kk = 0; kk < AD / 16; kk++) {
            st::umma_f16(tS, kmaj(q, kk), kmaj(k, kk), id, kk > 0 ? 1u : 0u);
            st::umma_f16(tdP, kmaj(d, kk), kmaj(v, kk), id, kk > 0 ? 1u : 0u);
        }
        st::umma_commit(&bar[0]);
    }
    bool ok = await(&bar[0], 0, g.status);
    st::tc_fence_after();

    // P = exp(scale*S - lse) (masked: 0) and dS = scale * P * (dP - D), both f16
    const int lim = r < g.t ? (g.causal ? r + 1 : g.t) : 0;
#pragma unroll 1
    for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 16) {
        uint32_t xs[16], xd[16];
        st::tmem_ld16(tS + lane_base + c0, xs);
        st::tmem_ld16(tdP + lane_base + c0, xd);
        st::tmem_ld_wait();
        float p[16], ds[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const bool vis = c0 + j < lim;
            p[j] = vis ? fast_exp(__uint_as_float(xs[j]) * g.scale - lse) : 0.0f;
            ds[j] = p[j] * (__uint_as_float(xd[j]) - dsum) * g.scale;
        }
        uint32_t o[8];
        pack16(p, o);
        put16(sP, r, c0, o);
        pack16(ds, o);
        put16(sS, r, c0, o);
    }
    st::fence_proxy_async_smem();
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();

    if (tid == 0) {
        // dV = P^T dO and dK = dS^T Q: A = P^T / dS^T (stored [i][j]: MN-major, M = j),
        // B = dO / Q (stored [i][d]: MN-major, N = d), K = i
        constexpr uint32_t id_tt = st::idesc_make(1, 0, true, true, AT, AD);
        // dQ = dS K: A = dS (K-major, K = j), B = K (stored [j][d]: MN-major, N = d)
        constexpr uint32_t id_nt = st::idesc_make(1, 0, false, true, AT, AD);
        const uint32_t p = st::smem_u32(sP), s = st::smem_u32(sS), q = st::smem_u32(sQ), k = st::smem_u32(sK),
                       d = st::smem_u32(sO);
#pragma unroll
        for (int kk = 0; kk < AT / 16; kk++) {
            st::umma_f16(tdV, mnmaj(p, kk, PT / 2), mnmaj(d, kk, TILE), id_tt, kk > 0 ? 1u : 0u);
            st::umma_f16(tdK, mnmaj(s, kk, PT / 2), mnmaj(q, kk, TILE), id_tt, kk > 0 ? 1u : 0u);
            st::umma_f16(tdQ, kmaj128(s, kk), mnmaj(k, kk, TILE), id_nt, kk > 0 ? 1u : 0u);
        }
        st::umma_commit(&bar[1]);
    }
    ok = await(&bar[1], 0, g.status) && ok;
    st::tc_fence_after();
    // row r of dV, dK (rows = keys) and dQ (rows = queries), this thread's 32 columns
#pragma unroll
    for (int w = 0; w < 3; w++) {
        __half *dst_t = w == 0 ? g.dv : w == 1 ? g.dk : g.dq;
        const uint32_t src = w == 0 ? tdV : w == 1 ? tdK : tdQ;
#pragma unroll
        for (int c0 = half * (AD / 2); c0 < (half + 1) * (AD / 2); c0 += 16) {
            uint32_t x[16];
            st::tmem_ld16(src + lane_base + c0, x);
            st::tmem_ld_wait();
            float y[16];
#pragma unroll
            for (int j = 0; j < 16; j++) y[j] = __uint_as_float(x[j]);
            uint32_t o[8];
            pack16(y, o);
            if (r < g.t && ok) {
                uint4 *dst = reinterpret_cast<uint4 *>(dst_t + head + static_cast<int64_t>(r) * AD + c0);
                dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
                dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
            }
        }
    }
    st::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, 512);
    }
}

constexpr int FWD_SMEM = 3 * TILE + PT + 2 * AT * 4 + 64 + 1024;
constexpr int BWD_SMEM = 4 * TILE + 2 * PT + 2 * AT * 4 + 64 + 1024;

st_status check(st_handle *h, const void *q, const void *k, const void *v, int64_t bh, int64_t t, int64_t d,
                const char *who) {
    if (!q || !k || !v) return h->fail(ST_INVALID_ARG, "%s: null buffer", who);
    if (bh < 1 || bh > (1 << 30) || t < 1) return h->fail(ST_INVALID_ARG, "%s: bad bh / t", who);
    if (t > AT || d != AD)
        return h->fail(ST_UNSUPPORTED_SHAPE, "%s: the fused kernel takes t <= %d and d = %d (got t=%lld d=%lld)", who, AT,
                       AD, (long long)t, (long long)d);
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15u)
        return h->fail(ST_INVALID_ARG, "%s: q, k, v must be 16-byte aligned", who);
    return ST_OK;
}

}  // namespace

extern "C" st_status st_attn_fwd(st_handle *h, const void *q, const void *k, const void *v, void *o, float *lse,
                                 int64_t bh, int64_t t, int64_t d, float scale, int32_t causal) {
    if (!h) return ST_INVALID_ARG;
    st_status s = check(h, q, k, v, bh, t, d, "st_attn_fwd");
    if (s != ST_OK) return s;
    if (!o || !lse || (reinterpret_cast<uintptr_t>(o) & 15u)) return h->fail(ST_INVALID_ARG, "st_attn_fwd: bad output");
    cudaSetDevice(h->device);
    static bool attr = false;
    if (!attr) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_attn_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, FWD_SMEM));
        attr = true;
    }
    AttnArgs g{};
    g.q = static_cast<const __half *>(q);
    g.k = static_cast<const __half *>(k);
    g.v = static_cast<const __half *>(v);
    g.out = static_cast<__half *>(o);
    g.lse = lse;
    g.bh = static_cast<int>(bh);
    g.t = static_cast<int>(t);
    g.scale = scale;
    g.causal = causal;
    g.status = h->d_status;
    k_attn_fwd<<<static_cast<unsigned>(bh), ATHREADS, FWD_SMEM, h->stream>>>(g);
    return st_after_launch(h, "k_attn_fwd");
}

extern "C" st_status st_attn_bwd(st_handle *h, const void *q, const void *k, const void *v, const void *o,
                                 const void *dout, const float *lse, void *dq, void *dk, void *dv, int64_t bh, int64_t t,
                                 int64_t d, float scale, int32_t causal) {
    if (!h) return ST_INVALID_ARG;
    st_status s = check(h, q, k, v, bh, t, d, "st_attn_bwd");
    if (s != ST_OK) return s;
    if (!o || !dout || !lse || !dq || !dk || !dv ||
        ((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(dout) | reinterpret_cast<uintptr_t>(dq) |
          reinterpret_cast<uintptr_t>(dk) | reinterpret_cast<uintptr_t>(dv)) & 15u))
        return h->fail(ST_INVALID_ARG, "st_attn_bwd: null or unaligned buffer");
    cudaSetDevice(h->device);
    static bool attr = false;
    if (!attr) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_attn_bwd, cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM));
        attr = true;
    }
    AttnArgs g{};
    g.q = static_cast<const __half *>(q);
    g.k = static_cast<const __half *>(k);
    g.v = static_cast<const __half *>(v);
    g.o = static_cast<const __half *>(o);
    g.dout = static_cast<const __half *>(dout);
    g.dq = static_cast<__half *>(dq);
    g.dk = static_cast<__half *>(dk);
    g.dv = static_cast<__half *>(dv);
    g.lse = const_cast<float *>(lse);
    g.bh = static_cast<int>(bh);
    g.t = static_cast<int>(t);
    g.scale = scale;
    g.causal = causal;
    g.status = h->d_status;
    k_attn_bwd<<<static_cast<unsigned>(bh), ATHREADS, BWD_SMEM, h->stream>>>(g);
    return st_after_launch(h, "k_attn_bwd");
}
