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

// Where row r of head z of a tensor lives: element (z / heads) * bstride +
// (z % heads) * hstride + r * rstride of its base.  Per-head tensors
// [bh, t, 64] use heads = 1, bstride = t * 64, rstride = 64; the packed
// layouts of the transformer step (fused QKV [B*T, 3*H*64], merged O
// [B*T, H*64]) use heads = H, hstride = 64, bstride = t * rstride.
struct RowMap {
    int64_t bstride, hstride, rstride;
    __device__ __forceinline__ int64_t at(int z, int heads, int r) const {
        return static_cast<int64_t>(z / heads) * bstride + static_cast<int64_t>(z % heads) * hstride +
               static_cast<int64_t>(r) * rstride;
    }
};

struct AttnArgs {
    const void *q, *k, *v, *o, *dout;  // f16, or f32 when the kernel's F32 flag is set
    void *out, *dq, *dk, *dv;
    float *lse;
    RowMap mq, mo;  // q/k/v/dq/dk/dv rows; o/dout/out rows
    int bh, t, heads;
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

// Half `half` (32 of the 64 columns) of row r (zeros when !live) into a
// swizzled 16 KB f16 tile; F32 sources are rounded to f16 on the way.
template <bool F32>
__device__ __forceinline__ void stage_half_rows(uint8_t *dst, const void *base, int64_t off, int r, int half,
                                                bool live) {
    if (F32) {
        const float4 *s = reinterpret_cast<const float4 *>(static_cast<const float *>(base) + off) + 8 * half;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            uint4 v = make_uint4(0u, 0u, 0u, 0u);
            if (live) {
                const float4 a = __ldg(s + 2 * c), b = __ldg(s + 2 * c + 1);
                const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
                const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
                v = make_uint4(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1),
                               *reinterpret_cast<const uint32_t *>(&h2), *reinterpret_cast<const uint32_t *>(&h3));
            }
            *reinterpret_cast<uint4 *>(dst + st::sw128_offset(r, 4 * half + c)) = v;
        }
    } else {
        const uint4 *s = reinterpret_cast<const uint4 *>(static_cast<const __half *>(base) + off) + 4 * half;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 v = live ? __ldg(s + c) : make_uint4(0u, 0u, 0u, 0u);
            *reinterpret_cast<uint4 *>(dst + st::sw128_offset(r, 4 * half + c)) = v;
        }
    }
}

// 16 consecutive output values at element `off` of `base` (f16 or f32).
template <bool F32>
__device__ __forceinline__ void store16(void *base, int64_t off, const float (&y)[16]) {
    if (F32) {
        float4 *d = reinterpret_cast<float4 *>(static_cast<float *>(base) + off);
#pragma unroll
        for (int i = 0; i < 4; i++) d[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
    } else {
        uint32_t o[8];
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const __half2 h = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
            o[i] = *reinterpret_cast<const uint32_t *>(&h);
        }
        uint4 *d = reinterpret_cast<uint4 *>(static_cast<__half *>(base) + off);
        d[0] = make_uint4(o[0], o[1], o[2], o[3]);
        d[1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
}

// sum over this thread's 32 columns of a[i] * b[i] (f16 or f32 rows)
template <bool F32>
__device__ __forceinline__ float dot_half(const void *a, const void *b, int64_t off, int half) {
    float acc = 0.0f;
    if (F32) {
        const float4 *pa = reinterpret_cast<const float4 *>(static_cast<const float *>(a) + off) + 8 * half;
        const float4 *pb = reinterpret_cast<const float4 *>(static_cast<const float *>(b) + off) + 8 * half;
#pragma unroll
        for (int c = 0; c < 8; c++) {
            const float4 x = __ldg(pa + c), y = __ldg(pb + c);
            acc = fmaf(x.x, y.x, acc);
            acc = fmaf(x.y, y.y, acc);
            acc = fmaf(x.z, y.z, acc);
            acc = fmaf(x.w, y.w, acc);
        }
    } else {
        const uint4 *pa = reinterpret_cast<const uint4 *>(static_cast<const __half *>(a) + off) + 4 * half;
        const uint4 *pb = reinterpret_cast<const uint4 *>(static_cast<const __half *>(b) + off) + 4 * half;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const uint4 x = __ldg(pa + c), y = __ldg(pb + c);
            const uint32_t xv[4] = {x.x, x.y, x.z, x.w}, yv[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 fa = __half22float2(*reinterpret_cast<const __half2 *>(&xv[i]));
                const float2 fb = __half22float2(*reinterpret_cast<const __half2 *>(&yv[i]));
                acc = fmaf(fa.x, fb.x, acc);
                acc = fmaf(fa.y, fb.y, acc);
            }
        }
    }
    return acc;
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
template <bool F32>
__global__ void __launch_bounds__(ATHREADS, 1) k_attn_fwd(const AttnArgs g) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem, *sK = smem + TILE, *sV = smem + 2 * TILE, *sP = smem + 3 * TILE;
    float *red = reinterpret_cast<float *>(sP + PT);  // [2][128]
    uint64_t *bar = reinterpret_cast<uint64_t *>(red + 2 * AT);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 2);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int r = tid & (AT - 1), half = tid >> 7;
    const int64_t rq = g.mq.at(blockIdx.x, g.heads, r), ro = g.mo.at(blockIdx.x, g.heads, r);
    const bool live = r < g.t;

    if (tid == 0) {
        st::mbar_init(&bar[0], 1);
        st::mbar_init(&bar[1], 1);
        st::fence_mbar_init();
    }
    if (warp == 0) {
        st::tmem_alloc(tslot, 256);
        st::tmem_relinquish();
    }
    stage_half_rows<F32>(sQ, g.q, rq, r, half, live);
    stage_half_rows<F32>(sK, g.k, rq, r, half, live);
    stage_half_rows<F32>(sV, g.v, rq, r, half, live);
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
        if (live && ok) store16<F32>(g.out, ro + c0, y);
    }
    st::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, 256);
    }
}

template <bool F32>
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
    const int64_t rq = g.mq.at(blockIdx.x, g.heads, r), ro = g.mo.at(blockIdx.x, g.heads, r);
    const bool live = r < g.t;

    if (tid == 0) {
        st::mbar_init(&bar[0], 1);
        st::mbar_init(&bar[1], 1);
        st::fence_mbar_init();
    }
    if (warp == 0) {
        st::tmem_alloc(tslot, 512);
        st::tmem_relinquish();
    }
    stage_half_rows<F32>(sQ, g.q, rq, r, half, live);
    stage_half_rows<F32>(sK, g.k, rq, r, half, live);
    stage_half_rows<F32>(sV, g.v, rq, r, half, live);
    stage_half_rows<F32>(sO, g.dout, ro, r, half, live);
    // D_r = sum_d dO[r,d] * O[r,d], this thread's 32 of the 64 d, then exchanged
    const float dsum_half = live ? dot_half<F32>(g.o, g.dout, ro, half) : 0.0f;
    float dsum = dsum_half;
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
        void *dst_t = w == 0 ? g.dv : w == 1 ? g.dk : g.dq;
        const uint32_t src = w == 0 ? tdV : w == 1 ? tdK : tdQ;
#pragma unroll
        for (int c0 = half * (AD / 2); c0 < (half + 1) * (AD / 2); c0 += 16) {
            uint32_t x[16];
            st::tmem_ld16(src + lane_base + c0, x);
            st::tmem_ld_wait();
            float y[16];
#pragma unroll
            for (int j = 0; j < 16; j++) y[j] = __uint_as_float(x[j]);
            if (live && ok) store16<F32>(dst_t, rq + c0, y);
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

template <bool F32>
st_status launch_fwd(st_handle *h, const AttnArgs &g) {
    static bool attr = false;
    if (!attr) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_attn_fwd<F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, FWD_SMEM));
        attr = true;
    }
    k_attn_fwd<F32><<<static_cast<unsigned>(g.bh), ATHREADS, FWD_SMEM, h->stream>>>(g);
    return st_after_launch(h, "k_attn_fwd");
}

template <bool F32>
st_status launch_bwd(st_handle *h, const AttnArgs &g) {
    static bool attr = false;
    if (!attr) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_attn_bwd<F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM));
        attr = true;
    }
    k_attn_bwd<F32><<<static_cast<unsigned>(g.bh), ATHREADS, BWD_SMEM, h->stream>>>(g);
    return st_after_launch(h, "k_attn_bwd");
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace

extern "C" st_status st_attn_fwd(st_handle *h, const void *q, const void *k, const void *v, void *o, float *lse,
                                 int64_t bh, int64_t t, int64_t d, float scale, int32_t causal) {
    if (!h) return ST_INVALID_ARG;
    st_status s = check(h, q, k, v, bh, t, d, "st_attn_fwd");
    if (s != ST_OK) return s;
    if (!o || !lse || !al16(o)) return h->fail(ST_INVALID_ARG, "st_attn_fwd: bad output");
    cudaSetDevice(h->device);
    AttnArgs g{};
    g.q = q;
    g.k = k;
    g.v = v;
    g.out = o;
    g.lse = lse;
    g.mq = RowMap{t * AD, 0, AD};
    g.mo = g.mq;
    g.bh = static_cast<int>(bh);
    g.t = static_cast<int>(t);
    g.heads = 1;
    g.scale = scale;
    g.causal = causal;
    g.status = h->d_status;
    return launch_fwd<false>(h, g);
}

extern "C" st_status st_attn_bwd(st_handle *h, const void *q, const void *k, const void *v, const void *o,
                                 const void *dout, const float *lse, void *dq, void *dk, void *dv, int64_t bh, int64_t t,
                                 int64_t d, float scale, int32_t causal) {
    if (!h) return ST_INVALID_ARG;
    st_status s = check(h, q, k, v, bh, t, d, "st_attn_bwd");
    if (s != ST_OK) return s;
    if (!o || !dout || !lse || !dq || !dk || !dv || !al16(o) || !al16(dout) || !al16(dq) || !al16(dk) || !al16(dv))
        return h->fail(ST_INVALID_ARG, "st_attn_bwd: null or unaligned buffer");
    cudaSetDevice(h->device);
    AttnArgs g{};
    g.q = q;
    g.k = k;
    g.v = v;
    g.o = o;
    g.dout = dout;
    g.dq = dq;
    g.dk = dk;
    g.dv = dv;
    g.lse = const_cast<float *>(lse);
    g.mq = RowMap{t * AD, 0, AD};
    g.mo = g.mq;
    g.bh = static_cast<int>(bh);
    g.t = static_cast<int>(t);
    g.heads = 1;
    g.scale = scale;
    g.causal = causal;
    g.status = h->d_status;
    return launch_bwd<false>(h, g);
}

extern "C" st_status st_attn_fwd_packed(st_handle *h, const float *qkv, float *o, float *lse, int64_t batch,
                                        int64_t heads, int64_t t, int64_t d, float scale, int32_t causal) {
    if (!h) return ST_INVALID_ARG;
    if (batch < 1 || heads < 1 || batch * heads > (1 << 30)) return h->fail(ST_INVALID_ARG, "st_attn_fwd_packed: bad shape");
    st_status s = check(h, qkv, qkv, qkv, batch * heads, t, d, "st_attn_fwd_packed");
    if (s != ST_OK) return s;
    if (!o || !lse || !al16(o)) return h->fail(ST_INVALID_ARG, "st_attn_fwd_packed: bad output");
    cudaSetDevice(h->device);
    const int64_t width = heads * AD;
    AttnArgs g{};
    g.q = qkv;
    g.k = qkv + width;
    g.v = qkv + 2 * width;
    g.out = o;
    g.lse = lse;
    g.mq = RowMap{t * 3 * width, AD, 3 * width};
    g.mo = RowMap{t * width, AD, width};
    g.bh = static_cast<int>(batch * heads);
    g.t = static_cast<int>(t);
    g.heads = static_cast<int>(heads);
    g.scale = scale;
    g.causal = causal;
    g.status = h->d_status;
    return launch_fwd<true>(h, g);
}

extern "C" st_status st_attn_bwd_packed(st_handle *h, const float *qkv, const float *o, const float *dout,
                                        const float *lse, float *dqkv, int64_t batch, int64_t heads, int64_t t,
                                        int64_t d, float scale, int32_t causal) {
    if (!h) return ST_INVALID_ARG;
    if (batch < 1 || heads < 1 || batch * heads > (1 << 30)) return h->fail(ST_INVALID_ARG, "st_attn_bwd_packed: bad shape");
    st_status s = check(h, qkv, qkv, qkv, batch * heads, t, d, "st_attn_bwd_packed");
    if (s != ST_OK) return s;
    if (!o || !dout || !lse || !dqkv || !al16(o) || !al16(dout) || !al16(dqkv))
        return h->fail(ST_INVALID_ARG, "st_attn_bwd_packed: null or unaligned buffer");
    cudaSetDevice(h->device);
    const int64_t width = heads * AD;
    AttnArgs g{};
    g.q = qkv;
    g.k = qkv + width;
    g.v = qkv + 2 * width;
    g.o = o;
    g.dout = dout;
    g.dq = dqkv;
    g.dk = dqkv + width;
    g.dv = dqkv + 2 * width;
    g.lse = const_cast<float *>(lse);
    g.mq = RowMap{t * 3 * width, AD, 3 * width};
    g.mo = RowMap{t * width, AD, width};
    g.bh = static_cast<int>(batch * heads);
    g.t = static_cast<int>(t);
    g.heads = static_cast<int>(heads);
    g.scale = scale;
    g.causal = causal;
    g.status = h->d_status;
    return launch_bwd<true>(h, g);
}
