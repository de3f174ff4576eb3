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

constexpr int AT = 128;               // rows per query / key tile
constexpr int AMAXT = 256;            // longest sequence (the reference's MAX_SEQ)
constexpr int AD = 64;                // head width
constexpr int TILE = AT * AD * 2;     // one [128 x 64] f16 operand: 16 KB
constexpr int PT = AT * AT * 2;       // one [128 x 128] f16 operand: 32 KB
constexpr int ATHREADS = 256;  // two threads per row (thread-loaded operands, f32 layouts, many heads)
constexpr int ATHREADS4 = 512;  // four threads per row (TMA-loaded f16 heads, at most one CTA per SM)

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
    int one;  // softmax1 (forward): a phantom zero logit in every row's denominator
    int tma;  // f16 per-head inputs: operand tiles by TMA (maps tq, tk, tv[, to, tdo]) instead of thread loads
    int *status;
};

// The tensor maps of the TMA-staged forward and backward: per-head f16
// tensors [bh, t, 64] as {64 columns, t rows, bh heads}, boxes of 128 rows,
// 128-byte swizzle (the layout the thread-loaded tiles use), zero fill past t.
struct HeadMaps {
    CUtensorMap q, k, v, o, dout;
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

// Up to N [128 x 64] row ranges into 128-byte-swizzled f16 tiles: source i
// is rows row0[i] .. row0[i] + 127 of head z of src[i] (row map map[i]) into
// dst[i] (a null dst skips the source).  Every thread issues its loads of all
// the sources before any store, so one global round trip covers them all;
// rows at and beyond t are zero, and f32 sources are rounded to f16 on the way.
template <int N>
struct Tiles {
    uint8_t *dst[N];
    const void *src[N];
    RowMap map[N];
    int row0[N];
};

template <bool F32, int N>
__device__ __forceinline__ void stage_tiles(const Tiles<N> &s, int z, int heads, int t) {
    constexpr int PER = AT * 8 / ATHREADS;  // 16-byte f16 pieces per thread per tile
    constexpr int W = F32 ? 2 : 1;          // 16-byte loads per piece
    uint4 raw[N][PER][W];
#pragma unroll
    for (int i = 0; i < N; i++) {
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int p = threadIdx.x + j * ATHREADS, r = p >> 3, c = p & 7;
            const int gr = s.row0[i] + r;
#pragma unroll
            for (int w = 0; w < W; w++) raw[i][j][w] = make_uint4(0u, 0u, 0u, 0u);
            if (s.dst[i] && gr < t) {
                const int64_t off = s.map[i].at(z, heads, gr) + 8 * c;
                if (F32) {
                    const uint4 *q = reinterpret_cast<const uint4 *>(static_cast<const float *>(s.src[i]) + off);
                    raw[i][j][0] = __ldg(q);
                    raw[i][j][W - 1] = __ldg(q + (W - 1));
                } else {
                    raw[i][j][0] = __ldg(reinterpret_cast<const uint4 *>(static_cast<const __half *>(s.src[i]) + off));
                }
            }
        }
    }
#pragma unroll
    for (int i = 0; i < N; i++) {
        if (!s.dst[i]) continue;
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int p = threadIdx.x + j * ATHREADS;
            uint4 v = raw[i][j][0];
            if (F32) {
                const uint4 a = raw[i][j][0], b = raw[i][j][W - 1];
                const __half2 h0 = __floats2half2_rn(__uint_as_float(a.x), __uint_as_float(a.y));
                const __half2 h1 = __floats2half2_rn(__uint_as_float(a.z), __uint_as_float(a.w));
                const __half2 h2 = __floats2half2_rn(__uint_as_float(b.x), __uint_as_float(b.y));
                const __half2 h3 = __floats2half2_rn(__uint_as_float(b.z), __uint_as_float(b.w));
                v = make_uint4(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1),
                               *reinterpret_cast<const uint32_t *>(&h2), *reinterpret_cast<const uint32_t *>(&h3));
            }
            *reinterpret_cast<uint4 *>(s.dst[i] + st::sw128_offset(p >> 3, p & 7)) = v;
        }
    }
}

// The forward's Q (128 rows from q0), K and V (TK rows from 0, zero from kc
// on) with every thread's loads of all three issued before any store.
template <bool F32, int TK>
__device__ __forceinline__ void stage_qkv(uint8_t *sq, uint8_t *sk, uint8_t *sv, const AttnArgs &g, int z, int q0,
                                          int kc) {
    constexpr int PQ = AT * 8 / ATHREADS, PK = TK * 8 / ATHREADS;
    uint4 v[PQ + 2 * PK];
    auto load = [&](const void *base, int row, int c) {
        if (F32) {
            const float4 *src = reinterpret_cast<const float4 *>(static_cast<const float *>(base) +
                                                                 g.mq.at(z, g.heads, row) + 8 * c);
            const float4 a = __ldg(src), b = __ldg(src + 1);
            const __half2 h0 = __floats2half2_rn(a.x, a.y), h1 = __floats2half2_rn(a.z, a.w);
            const __half2 h2 = __floats2half2_rn(b.x, b.y), h3 = __floats2half2_rn(b.z, b.w);
            return make_uint4(*reinterpret_cast<const uint32_t *>(&h0), *reinterpret_cast<const uint32_t *>(&h1),
                              *reinterpret_cast<const uint32_t *>(&h2), *reinterpret_cast<const uint32_t *>(&h3));
        }
        return __ldg(reinterpret_cast<const uint4 *>(static_cast<const __half *>(base) + g.mq.at(z, g.heads, row)) +
                     c);
    };
#pragma unroll
    for (int i = 0; i < PQ; i++) {
        const int p = threadIdx.x + i * ATHREADS, r = p >> 3, c = p & 7;
        v[i] = q0 + r < g.t ? load(g.q, q0 + r, c) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < PK; i++) {
        const int p = threadIdx.x + i * ATHREADS, r = p >> 3, c = p & 7;
        v[PQ + i] = r < kc ? load(g.k, r, c) : make_uint4(0u, 0u, 0u, 0u);
        v[PQ + PK + i] = r < kc ? load(g.v, r, c) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int i = 0; i < PQ; i++) {
        const int p = threadIdx.x + i * ATHREADS;
        *reinterpret_cast<uint4 *>(sq + st::sw128_offset(p >> 3, p & 7)) = v[i];
    }
#pragma unroll
    for (int i = 0; i < PK; i++) {
        const int p = threadIdx.x + i * ATHREADS;
        *reinterpret_cast<uint4 *>(sk + st::sw128_offset(p >> 3, p & 7)) = v[PQ + i];
        *reinterpret_cast<uint4 *>(sv + st::sw128_offset(p >> 3, p & 7)) = v[PQ + PK + i];
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

// Columns [c0, c0+16) of row r of a [128 x 64n] f16 operand tile (n 64-column
// 128-byte-swizzled blocks of 16 KB).
__device__ __forceinline__ void put16(uint8_t *tile, int r, int c0, const uint32_t (&o)[8]) {
    uint8_t *blk = tile + (c0 >> 6) * (PT / 2);
    const int piece = (c0 & 63) >> 3;
    *reinterpret_cast<uint4 *>(blk + st::sw128_offset(r, piece)) = make_uint4(o[0], o[1], o[2], o[3]);
    *reinterpret_cast<uint4 *>(blk + st::sw128_offset(r, piece + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
}

// K-major operand descriptor: [rows x 64] chunk at `base`, k step kk (16 elements).
__device__ __forceinline__ uint64_t kmaj(uint32_t base, int kk) { return st::sdesc_sw128(base + kk * 32, 16, 1024); }
// K-major descriptor into a [128 x 64n] tile of 64-column blocks: k step kk (16 columns).
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

// Shared-memory layout of the forward for TK staged key rows (128 or 256).
template <int TK>
struct FwdSmem {
    static constexpr int Q = 0, K = TILE, V = K + TK * 128, P = V + TK * 128;
    static constexpr int RED = P + AT * TK * 2;  // [4][128] f32
    static constexpr int BAR = RED + 4 * AT * 4;
    static constexpr int SIZE = BAR + 64 + 1024;
    static constexpr uint32_t TMEM = TK == 128 ? 256 : 512;  // S (TK columns) + O (64)
};

// Forward.  CTA = (head z = blockIdx.x, query tile blockIdx.y of 128 rows): S = Q K^T over every
// key the tile sees (at most TK = 256 columns, so a row's scores fit one TMEM
// row and need no online rescaling), the masked softmax (or softmax1) of
// scale * S in registers, P as f16 into shared memory, O = P V.  The NTH / 128
// threads r, r + 128, ... share row r: each takes an equal share of the row's
// key columns (warps w, w + 4, ... read the same TMEM lanes); row reductions
// go through `red`.  NTH = 512 (four threads per row) only with TMA-loaded
// f16 operands and TK = 128.
template <bool F32, int TK, int NTH = ATHREADS>
__global__ void __launch_bounds__(NTH, (TK == 128 && NTH == ATHREADS) ? 2 : 1)
    k_attn_fwd(const AttnArgs g, const __grid_constant__ HeadMaps tm) {
    static_assert(NTH == ATHREADS || (NTH == ATHREADS4 && TK == AT && !F32), "four threads per row: f16, TK 128");
    constexpr int NG = NTH / AT;  // threads per row
    using L = FwdSmem<TK>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sQ = smem + L::Q, *sK = smem + L::K, *sV = smem + L::V, *sP = smem + L::P;
    float *red = reinterpret_cast<float *>(smem + L::RED);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + L::BAR);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 2);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int r = tid & (AT - 1), half = tid >> 7;  // half: this thread's share of the row (0 .. NG - 1)
    const int z = blockIdx.x, q0 = blockIdx.y * AT, gr = q0 + r;
    const int kc = g.causal ? min(g.t, q0 + AT) : g.t;  // keys this tile sees
    const int kc16 = (kc + 15) & ~15;                      // the MMAs' N / K extent over keys
    const int64_t ro = g.mo.at(z, g.heads, gr < g.t ? gr : 0);
    const bool live = gr < g.t;

    const bool tma = !F32 && g.tma;
    if (tid == 0) {
        st::mbar_init(&bar[0], 1);
        st::mbar_init(&bar[1], 1);
        st::mbar_init(&bar[3], 1);
        st::fence_mbar_init();
    }
    if (warp == 0) {
        st::tmem_alloc(tslot, L::TMEM);
        st::tmem_relinquish();
    }
    // everything above overlaps the previous kernel's tail (programmatic dependent launch); no global
    // memory is read before it has completed
    st::grid_dep_wait();
    st::grid_dep_launch();
    if (tid == 0) {
        if (tma) {  // Q, and K, V in 128-row boxes up to the last key this tile sees
            const int nkb = (kc + AT - 1) / AT;
            st::mbar_arrive_expect_tx(&bar[3], static_cast<uint32_t>(TILE * (1 + 2 * nkb)));
            st::tma_load_4d(sQ, &tm.q, &bar[3], 0, q0, z, 0);
            for (int b = 0; b < nkb; b++) {
                st::tma_load_4d(sK + b * TILE, &tm.k, &bar[3], 0, b * AT, z, 0);
                st::tma_load_4d(sV + b * TILE, &tm.v, &bar[3], 0, b * AT, z, 0);
            }
        }
    }
    if constexpr (NTH == ATHREADS) {
        if (!tma) stage_qkv<F32, TK>(sQ, sK, sV, g, z, q0, kc);
    }
    st::fence_proxy_async_smem();
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t tmem = *tslot, tS = tmem, tO = tmem + TK;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;

    if (tid == 0) {  // S = Q K^T over kc16 keys
        if (!tma || await(&bar[3], 0, g.status)) {
            const uint32_t id = st::idesc_make(1, 0, false, false, AT, kc16);
            const uint32_t q = st::smem_u32(sQ), k = st::smem_u32(sK);
#pragma unroll
            for (int kk = 0; kk < AD / 16; kk++) st::umma_f16(tS, kmaj(q, kk), kmaj(k, kk), id, kk > 0 ? 1u : 0u);
        }
        st::umma_commit(&bar[0]);
    }
    bool ok = await(&bar[0], 0, g.status);
    st::tc_fence_after();

    const int lim = live ? (g.causal ? gr + 1 : g.t) : 0;  // columns < lim are visible
    float m = -INFINITY, l = 0.0f;
    if constexpr (TK == AT) {
        // up to 128 key columns: share h of the row takes columns CW h .. CW h + CW - 1
        // in registers (one TMEM read); columns at and past kc16 are masked
        constexpr int CW = AT / NG;
        const int cbase = half * CW;
        uint32_t x[CW];
#pragma unroll
        for (int c = 0; c < CW / 32; c++)
            st::tmem_ld32(tS + lane_base + cbase + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(&x[32 * c]));
        st::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < CW; j++)
            if (cbase + j < lim) m = fmaxf(m, __uint_as_float(x[j]) * g.scale);
        red[half * AT + r] = m;
        __syncthreads();
#pragma unroll
        for (int o = 0; o < NG; o++) m = fmaxf(m, red[o * AT + r]);
        if (g.one) m = fmaxf(m, 0.0f);  // softmax1 shifts by max(row max, 0)
#pragma unroll
        for (int c = 0; c < CW / 16; c++) {
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
    } else {
        // up to 256 columns: the row's kc16 columns split in two 16-aligned
        // halves, read from TMEM twice (max, then exponentials)
        const int cw = ((kc16 >> 1) + 15) & ~15;
        const int c_lo = half ? cw : 0, c_hi = half ? kc16 : cw;
#pragma unroll 1
        for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
            uint32_t x[16];
            st::tmem_ld16(tS + lane_base + c0, x);
            st::tmem_ld_wait();
#pragma unroll
            for (int j = 0; j < 16; j++)
                if (c0 + j < lim) m = fmaxf(m, __uint_as_float(x[j]) * g.scale);
        }
        red[half * AT + r] = m;
        __syncthreads();
        m = fmaxf(m, red[(half ^ 1) * AT + r]);
        if (g.one) m = fmaxf(m, 0.0f);  // softmax1 shifts by max(row max, 0)
#pragma unroll 1
        for (int c0 = c_lo; c0 < c_hi; c0 += 16) {
            uint32_t x[16];
            st::tmem_ld16(tS + lane_base + c0, x);
            st::tmem_ld_wait();
            float p[16];
#pragma unroll
            for (int j = 0; j < 16; j++) {
                p[j] = c0 + j < lim ? fast_exp(__uint_as_float(x[j]) * g.scale - m) : 0.0f;
                l += p[j];
            }
            uint32_t o[8];
            pack16(p, o);
            put16(sP, r, c0, o);
        }
    }
    __syncthreads();  // every thread has read red (max) before it is reused for sums
    red[half * AT + r] = l;
    st::fence_proxy_async_smem();
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    l = 0.0f;  // the shares' sums in share order: the same value on every thread of the row
#pragma unroll
    for (int o = 0; o < NG; o++) l += red[o * AT + r];
    if (g.one && lim > 0) l += fast_exp(-m);  // softmax1's phantom zero logit
    if (half == 0 && live) g.lse[static_cast<int64_t>(z) * g.t + gr] = lim > 0 ? m + logf(l) : -INFINITY;

    if (tid == 0) {  // O = P V   (V: B operand, N = d contiguous -> MN-major), K = kc16 keys
        constexpr uint32_t id = st::idesc_make(1, 0, false, true, AT, AD);
        const uint32_t p = st::smem_u32(sP), v = st::smem_u32(sV);
        for (int kk = 0; kk < kc16 / 16; kk++)
            st::umma_f16(tO, kmaj128(p, kk), mnmaj(v, kk, TILE), id, kk > 0 ? 1u : 0u);
        st::umma_commit(&bar[1]);
    }
    ok = await(&bar[1], 0, g.status) && ok;
    st::tc_fence_after();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll 1
    for (int c0 = half * (AD / NG); c0 < (half + 1) * (AD / NG); c0 += 16) {
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
        st::tmem_dealloc(tmem, L::TMEM);
    }
}

// Backward shared memory: two [128 x 64] operand pairs and two [128 x 128] f16 tiles.
constexpr int B_Q = 0, B_DO = TILE, B_K = 2 * TILE, B_V = 3 * TILE, B_P = 4 * TILE, B_S = B_P + PT;
constexpr int B_RED = B_S + PT, B_BAR = B_RED + 4 * AT * 4;
constexpr int BWD_SMEM = B_BAR + 64 + 1024;

// dot_half's sum for f16 rows held in 128-byte-swizzled tiles: row r, the
// NP 8-column pieces from piece NP h on, in the same order as dot_half (so
// with NP = 4 the same bits).
template <int NP>
__device__ __forceinline__ float dot_tiles(const uint8_t *ta, const uint8_t *tb, int r, int h) {
    float acc = 0.0f;
#pragma unroll
    for (int c = 0; c < NP; c++) {
        const uint4 x = *reinterpret_cast<const uint4 *>(ta + st::sw128_offset(r, NP * h + c));
        const uint4 y = *reinterpret_cast<const uint4 *>(tb + st::sw128_offset(r, NP * h + c));
        const uint32_t xv[4] = {x.x, x.y, x.z, x.w}, yv[4] = {y.x, y.y, y.z, y.w};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const float2 fa = __half22float2(*reinterpret_cast<const __half2 *>(&xv[i]));
            const float2 fb = __half22float2(*reinterpret_cast<const __half2 *>(&yv[i]));
            acc = fmaf(fa.x, fb.x, acc);
            acc = fmaf(fa.y, fb.y, acc);
        }
    }
    return acc;
}

// Stages key tile kt (K, V; none when kt < 0) and query tile qt (Q, dO; none
// when qt < 0), and for a query tile computes D_r = sum_d dO[r,d] O[r,d]
// (both halves of the row, the same order on both threads) and the row's
// log-sum-exp.  f16 inputs take one global round trip for everything: O is
// staged too, into the P tile's space (free until bwd_scores writes P), and D
// is read from shared memory; with g.tma the tiles come by TMA (one mbarrier,
// `tbar`, phase `tph`).  f32 inputs take one round trip per pair of tiles (to
// bound registers) and D from the f32 rows in memory.  False when the TMA
// wait ran out (the status word says so).
template <bool F32, int NTH>
__device__ __forceinline__ bool bwd_stage(const AttnArgs &g, const HeadMaps &tm, uint64_t *tbar, uint32_t &tph,
                                          uint8_t *smem, float *red, int z, int qt, int kt, float &dsum, float &lse) {
    constexpr int NG = NTH / AT;
    const int r = threadIdx.x & (AT - 1), half = threadIdx.x >> 7, gr = qt * AT + r;
    const bool qrow = qt >= 0 && gr < g.t;
    lse = qrow ? g.lse[static_cast<int64_t>(z) * g.t + gr] : 0.0f;
    uint8_t *kd = kt >= 0 ? smem + B_K : nullptr, *vd = kt >= 0 ? smem + B_V : nullptr;
    uint8_t *qd = qt >= 0 ? smem + B_Q : nullptr, *dd = qt >= 0 ? smem + B_DO : nullptr;
    bool ok = true;
    if (!F32 && g.tma) {
        if (threadIdx.x == 0) {
            st::mbar_arrive_expect_tx(tbar, static_cast<uint32_t>(TILE * ((kt >= 0 ? 2 : 0) + (qt >= 0 ? 3 : 0))));
            if (kt >= 0) {
                st::tma_load_4d(kd, &tm.k, tbar, 0, kt * AT, z, 0);
                st::tma_load_4d(vd, &tm.v, tbar, 0, kt * AT, z, 0);
            }
            if (qt >= 0) {
                st::tma_load_4d(qd, &tm.q, tbar, 0, qt * AT, z, 0);
                st::tma_load_4d(dd, &tm.dout, tbar, 0, qt * AT, z, 0);
                st::tma_load_4d(smem + B_P, &tm.o, tbar, 0, qt * AT, z, 0);
            }
        }
        ok = await(tbar, tph, g.status);
        tph ^= 1u;
    } else if constexpr (NTH != ATHREADS) {
        // four threads per row is launched only with the tensor maps
    } else if (F32) {
        if (kt >= 0) stage_tiles<true, 2>(Tiles<2>{{kd, vd}, {g.k, g.v}, {g.mq, g.mq}, {kt * AT, kt * AT}}, z, g.heads, g.t);
        if (qt >= 0)
            stage_tiles<true, 2>(Tiles<2>{{qd, dd}, {g.q, g.dout}, {g.mq, g.mo}, {qt * AT, qt * AT}}, z, g.heads, g.t);
    } else {
        stage_tiles<false, 5>(Tiles<5>{{kd, vd, qd, dd, qt >= 0 ? smem + B_P : nullptr},
                                       {g.k, g.v, g.q, g.dout, g.o},
                                       {g.mq, g.mq, g.mq, g.mo, g.mo},
                                       {kt * AT, kt * AT, qt * AT, qt * AT, qt * AT}},
                              z, g.heads, g.t);
    }
    if (qt < 0) return ok;
    float part;
    if constexpr (F32) {
        part = qrow ? dot_half<true>(g.o, g.dout, g.mo.at(z, g.heads, gr), half) : 0.0f;
    } else {
        __syncthreads();  // O and dO tiles complete
        part = qrow ? dot_tiles<8 / NG>(smem + B_P, smem + B_DO, r, half) : 0.0f;
    }
    red[half * AT + r] = part;
    __syncthreads();
    dsum = 0.0f;  // the shares in share order: the same value on every thread of the row
#pragma unroll
    for (int o = 0; o < NG; o++) dsum += red[o * AT + r];
    __syncthreads();  // red and the staged O are read before either is reused
    return ok;
}

// S = Q K^T and dP = dO V^T of one (query tile, key tile) pair, then P =
// exp(scale S - lse) and dS = scale P (dP - D) (masked entries 0) as f16
// tiles in shared memory (P only when want_p).  Rows are queries.
template <bool F32, int NTH>
__device__ __forceinline__ bool bwd_scores(const AttnArgs &g, uint8_t *smem, uint32_t tmem, uint64_t *bar,
                                           uint32_t &phase, int qt, int kt, float dsum, float lse, bool want_p) {
    const int tid = threadIdx.x, warp = tid >> 5, r = tid & (AT - 1), half = tid >> 7;
    const uint32_t tS = tmem, tdP = tmem + 128;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    if (tid == 0) {
        constexpr uint32_t id = st::idesc_make(1, 0, false, false, AT, AT);
        const uint32_t q = st::smem_u32(smem + B_Q), k = st::smem_u32(smem + B_K), v = st::smem_u32(smem + B_V),
                       d = st::smem_u32(smem + B_DO);
#pragma unroll
        for (int kk = 0; kk < AD / 16; kk++) {
            st::umma_f16(tS, kmaj(q, kk), kmaj(k, kk), id, kk > 0 ? 1u : 0u);
            st::umma_f16(tdP, kmaj(d, kk), kmaj(v, kk), id, kk > 0 ? 1u : 0u);
        }
        st::umma_commit(&bar[0]);
    }
    const bool ok = await(&bar[0], phase, g.status);
    phase ^= 1u;
    st::tc_fence_after();
    const int gr = qt * AT + r;
    // key column c of this tile is key kt*128 + c; visible iff < t and (causal) <= gr
    const int lim = gr < g.t ? min(g.t, g.causal ? gr + 1 : g.t) - kt * AT : 0;
    constexpr int CW = AT / (NTH / AT);  // this thread's share of the key columns
#pragma unroll 1
    for (int c0 = half * CW; c0 < half * CW + CW; c0 += 16) {
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
        if (want_p) {
            pack16(p, o);
            put16(smem + B_P, r, c0, o);
        }
        pack16(ds, o);
        put16(smem + B_S, r, c0, o);
    }
    st::fence_proxy_async_smem();
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    return ok;
}

// Backward.  Two kinds of CTA per head (blockIdx.x = head; blockIdx.y <
// ntile: key tile kt = blockIdx.y, else query tile qt = blockIdx.y - ntile;
// a sequence of one tile has one CTA per head, which does both):
//  * key tile kt: dV = sum over query tiles of P^T dO, dK = sum of dS^T Q
//    (accumulated in TMEM across the query tiles that see the keys);
//  * query tile qt: dQ = sum over the key tiles it sees of dS K.
// Both recompute S and dP from Q, K, V, dO and the forward's log-sum-exp
// (D = rowsum(dO O) gives the softmax backward for softmax and softmax1
// alike).  Every transposed operand is a shared-memory descriptor.
template <bool F32, int NTH = ATHREADS>
__global__ void __launch_bounds__(NTH, 1) k_attn_bwd(const AttnArgs g, const __grid_constant__ HeadMaps tm) {
    static_assert(NTH == ATHREADS || (NTH == ATHREADS4 && !F32), "four threads per row: f16 heads");
    constexpr int NG = NTH / AT;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *red = reinterpret_cast<float *>(smem + B_RED);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + B_BAR);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 2);
    const int tid = threadIdx.x, warp = tid >> 5, r = tid & (AT - 1), half = tid >> 7;
    const int z = blockIdx.x, ntile = (g.t + AT - 1) / AT;
    const bool key_role = static_cast<int>(blockIdx.y) < ntile;
    const int tile = key_role ? blockIdx.y : blockIdx.y - ntile;

    if (tid == 0) {
        st::mbar_init(&bar[0], 1);
        st::mbar_init(&bar[1], 1);
        st::mbar_init(&bar[3], 1);
        st::fence_mbar_init();
    }
    if (warp == 0) {
        st::tmem_alloc(tslot, 512);
        st::tmem_relinquish();
    }
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t tmem = *tslot, tA = tmem + 256, tB = tmem + 320;  // dV / dQ, dK
    const uint32_t tQ = tmem + 384;                                   // dQ of a one-tile sequence
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint32_t ph0 = 0, ph1 = 0, ph3 = 0;
    bool ok = true;
    st::grid_dep_wait();  // the prologue above overlaps the previous kernel's tail
    st::grid_dep_launch();
    if (key_role) {
        const int kt = tile;
        bool first = true;
        for (int qt = g.causal ? kt : 0; qt < ntile && ok; qt++) {
            float dsum, lse;
            ok = bwd_stage<F32, NTH>(g, tm, &bar[3], ph3, smem, red, z, qt, first ? kt : -1, dsum, lse) && ok;
            st::fence_proxy_async_smem();
            st::tc_fence_before();
            __syncthreads();
            st::tc_fence_after();
            ok = bwd_scores<F32, NTH>(g, smem, tmem, bar, ph0, qt, kt, dsum, lse, true) && ok;
            if (tid == 0) {
                // dV += P^T dO, dK += dS^T Q: A = P^T / dS^T (stored [query][key]: MN-major, M = key),
                // B = dO / Q (stored [query][d]: MN-major, N = d), K = the tile's 128 queries
                constexpr uint32_t id_tt = st::idesc_make(1, 0, true, true, AT, AD);
                const uint32_t p = st::smem_u32(smem + B_P), s = st::smem_u32(smem + B_S),
                               q = st::smem_u32(smem + B_Q), d = st::smem_u32(smem + B_DO);
#pragma unroll
                for (int kk = 0; kk < AT / 16; kk++) {
                    const uint32_t acc = (first && kk == 0) ? 0u : 1u;
                    st::umma_f16(tA, mnmaj(p, kk, PT / 2), mnmaj(d, kk, TILE), id_tt, acc);
                    st::umma_f16(tB, mnmaj(s, kk, PT / 2), mnmaj(q, kk, TILE), id_tt, acc);
                }
                if (ntile == 1) {
                    // one tile of keys and queries: this CTA also has everything dQ = dS K needs
                    constexpr uint32_t id_nt = st::idesc_make(1, 0, false, true, AT, AD);
                    const uint32_t k = st::smem_u32(smem + B_K);
#pragma unroll
                    for (int kk = 0; kk < AT / 16; kk++)
                        st::umma_f16(tQ, kmaj128(s, kk), mnmaj(k, kk, TILE), id_nt, kk > 0 ? 1u : 0u);
                }
                st::umma_commit(&bar[1]);
            }
            // the next query tile restages Q, dO, P and dS: these MMAs must be done
            ok = await(&bar[1], ph1, g.status) && ok;
            ph1 ^= 1u;
            st::tc_fence_after();
            first = false;
        }
        const int gk = kt * AT + r;
        const int64_t rk = g.mq.at(z, g.heads, gk < g.t ? gk : 0);
        for (int w = 0; w < (ntile == 1 ? 3 : 2); w++) {
            void *dst_t = w == 0 ? g.dv : w == 1 ? g.dk : g.dq;
            const uint32_t src = w == 0 ? tA : w == 1 ? tB : tQ;
#pragma unroll
            for (int c0 = half * (AD / NG); c0 < (half + 1) * (AD / NG); c0 += 16) {
                uint32_t x[16];
                st::tmem_ld16(src + lane_base + c0, x);
                st::tmem_ld_wait();
                float y[16];
#pragma unroll
                for (int j = 0; j < 16; j++) y[j] = __uint_as_float(x[j]);
                if (gk < g.t && ok) store16<F32>(dst_t, rk + c0, y);
            }
        }
    } else {
        const int qt = tile;
        float dsum, lse;
        ok = bwd_stage<F32, NTH>(g, tm, &bar[3], ph3, smem, red, z, qt, 0, dsum, lse);  // the queries with key tile 0
        const int last = g.causal ? qt : ntile - 1;
        for (int kt = 0; kt <= last && ok; kt++) {
            if (kt > 0) {
                float unused0, unused1;
                ok = bwd_stage<F32, NTH>(g, tm, &bar[3], ph3, smem, red, z, -1, kt, unused0, unused1) && ok;
            }
            st::fence_proxy_async_smem();
            st::tc_fence_before();
            __syncthreads();
            st::tc_fence_after();
            ok = bwd_scores<F32, NTH>(g, smem, tmem, bar, ph0, qt, kt, dsum, lse, false) && ok;
            if (tid == 0) {
                // dQ += dS K: A = dS (K-major, K = key), B = K (stored [key][d]: MN-major, N = d)
                constexpr uint32_t id_nt = st::idesc_make(1, 0, false, true, AT, AD);
                const uint32_t s = st::smem_u32(smem + B_S), k = st::smem_u32(smem + B_K);
#pragma unroll
                for (int kk = 0; kk < AT / 16; kk++)
                    st::umma_f16(tA, kmaj128(s, kk), mnmaj(k, kk, TILE), id_nt, (kt == 0 && kk == 0) ? 0u : 1u);
                st::umma_commit(&bar[1]);
            }
            ok = await(&bar[1], ph1, g.status) && ok;  // K and dS are restaged by the next key tile
            ph1 ^= 1u;
            st::tc_fence_after();
        }
        const int gq = qt * AT + r;
        const int64_t rq = g.mq.at(z, g.heads, gq < g.t ? gq : 0);
#pragma unroll
        for (int c0 = half * (AD / NG); c0 < (half + 1) * (AD / NG); c0 += 16) {
            uint32_t x[16];
            st::tmem_ld16(tA + lane_base + c0, x);
            st::tmem_ld_wait();
            float y[16];
#pragma unroll
            for (int j = 0; j < 16; j++) y[j] = __uint_as_float(x[j]);
            if (gq < g.t && ok) store16<F32>(g.dq, rq + c0, y);
        }
    }
    st::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, 512);
    }
}

// Compact backward for one-tile sequences (t <= 128) when the heads are more
// than the SMs: 98 KB of shared memory and 256 TMEM columns, so two CTAs fit
// on an SM and the grid runs in one wave instead of two.  The same arithmetic
// as k_attn_bwd (the same bits): after S = Q K^T and dP = dO V^T,
//  1. dS = scale P (dP - D) -> the one [128 x 128] f16 tile X; dK = dS^T Q and
//     dQ = dS K accumulate into dP's TMEM columns (dP is read by then);
//  2. once those MMAs have read X, P = exp(scale S - lse) -> X (recomputed from
//     S, which is still in TMEM); dV = P^T dO accumulates into S's columns.
// Shared memory: Q, dO, K, V (16 KB each), X (32 KB, where the f16 path also
// stages O for D), the row-reduction scratch and the barriers.
constexpr int C_X = B_P, C_RED = C_X + PT, C_BAR = C_RED + 2 * AT * 4;
constexpr int CBWD_SMEM = C_BAR + 64 + 1024;

// One pass over this thread's 64 key columns of S (and dP): dS (want_ds) or
// P as f16 into X, with k_attn_bwd's formulas.
__device__ __forceinline__ void tile_pass(const AttnArgs &g, uint8_t *x, uint32_t tS, uint32_t tdP, int r, int half,
                                          int lim, float dsum, float lse, bool want_ds) {
    const uint32_t lane_base = static_cast<uint32_t>(r & ~31) << 16;
#pragma unroll 1
    for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 16) {
        uint32_t xs[16], xd[16];
        st::tmem_ld16(tS + lane_base + c0, xs);
        if (want_ds) st::tmem_ld16(tdP + lane_base + c0, xd);
        st::tmem_ld_wait();
        float p[16];
#pragma unroll
        for (int j = 0; j < 16; j++) {
            const bool vis = c0 + j < lim;
            p[j] = vis ? fast_exp(__uint_as_float(xs[j]) * g.scale - lse) : 0.0f;
            if (want_ds) p[j] = p[j] * (__uint_as_float(xd[j]) - dsum) * g.scale;
        }
        uint32_t o[8];
        pack16(p, o);
        put16(x, r, c0, o);
    }
    st::fence_proxy_async_smem();
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
}

template <bool F32>
__global__ void __launch_bounds__(ATHREADS, 2) k_attn_bwd1(const AttnArgs g, const __grid_constant__ HeadMaps tm) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *red = reinterpret_cast<float *>(smem + C_RED);
    uint64_t *bar = reinterpret_cast<uint64_t *>(smem + C_BAR);
    uint32_t *tslot = reinterpret_cast<uint32_t *>(bar + 2);
    const int tid = threadIdx.x, warp = tid >> 5, r = tid & (AT - 1), half = tid >> 7;
    const int z = blockIdx.x;
    if (tid == 0) {
        st::mbar_init(&bar[0], 1);
        st::mbar_init(&bar[1], 1);
        st::mbar_init(&bar[3], 1);
        st::fence_mbar_init();
    }
    if (warp == 0) {
        st::tmem_alloc(tslot, 256);
        st::tmem_relinquish();
    }
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t tmem = *tslot, tS = tmem, tdP = tmem + 128;
    const uint32_t tdV = tmem, tdK = tmem + 128, tdQ = tmem + 192;  // into S's and dP's columns once they are read
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    st::grid_dep_wait();  // the prologue above overlaps the previous kernel's tail
    st::grid_dep_launch();

    uint32_t ph3 = 0;
    float dsum, lse;
    bool ok = bwd_stage<F32, ATHREADS>(g, tm, &bar[3], ph3, smem, red, z, 0, 0, dsum, lse);  // X holds O (f16)
    st::fence_proxy_async_smem();
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t q = st::smem_u32(smem + B_Q), k = st::smem_u32(smem + B_K), v = st::smem_u32(smem + B_V),
                   d = st::smem_u32(smem + B_DO), x = st::smem_u32(smem + C_X);
    if (tid == 0) {  // S = Q K^T, dP = dO V^T
        constexpr uint32_t id = st::idesc_make(1, 0, false, false, AT, AT);
#pragma unroll
        for (int kk = 0; kk < AD / 16; kk++) {
            st::umma_f16(tS, kmaj(q, kk), kmaj(k, kk), id, kk > 0 ? 1u : 0u);
            st::umma_f16(tdP, kmaj(d, kk), kmaj(v, kk), id, kk > 0 ? 1u : 0u);
        }
        st::umma_commit(&bar[0]);
    }
    ok = await(&bar[0], 0, g.status) && ok;
    st::tc_fence_after();
    const int lim = r < g.t ? min(g.t, g.causal ? r + 1 : g.t) : 0;
    tile_pass(g, smem + C_X, tS, tdP, r, half, lim, dsum, lse, true);
    if (tid == 0) {  // dK = dS^T Q, dQ = dS K
        constexpr uint32_t id_tt = st::idesc_make(1, 0, true, true, AT, AD);
        constexpr uint32_t id_nt = st::idesc_make(1, 0, false, true, AT, AD);
#pragma unroll
        for (int kk = 0; kk < AT / 16; kk++) {
            st::umma_f16(tdK, mnmaj(x, kk, PT / 2), mnmaj(q, kk, TILE), id_tt, kk > 0 ? 1u : 0u);
            st::umma_f16(tdQ, kmaj128(x, kk), mnmaj(k, kk, TILE), id_nt, kk > 0 ? 1u : 0u);
        }
        st::umma_commit(&bar[1]);
    }
    ok = await(&bar[1], 0, g.status) && ok;  // X is read: P may replace dS
    st::tc_fence_after();
    tile_pass(g, smem + C_X, tS, tdP, r, half, lim, dsum, lse, false);
    if (tid == 0) {  // dV = P^T dO
        constexpr uint32_t id_tt = st::idesc_make(1, 0, true, true, AT, AD);
#pragma unroll
        for (int kk = 0; kk < AT / 16; kk++)
            st::umma_f16(tdV, mnmaj(x, kk, PT / 2), mnmaj(d, kk, TILE), id_tt, kk > 0 ? 1u : 0u);
        st::umma_commit(&bar[0]);
    }
    ok = await(&bar[0], 1, g.status) && ok;
    st::tc_fence_after();
    const int64_t rk = g.mq.at(z, g.heads, r < g.t ? r : 0);
    for (int w = 0; w < 3; w++) {
        void *dst_t = w == 0 ? g.dv : w == 1 ? g.dk : g.dq;
        const uint32_t src = w == 0 ? tdV : w == 1 ? tdK : tdQ;
#pragma unroll
        for (int c0 = half * (AD / 2); c0 < (half + 1) * (AD / 2); c0 += 16) {
            uint32_t y16[16];
            st::tmem_ld16(src + lane_base + c0, y16);
            st::tmem_ld_wait();
            float y[16];
#pragma unroll
            for (int j = 0; j < 16; j++) y[j] = __uint_as_float(y16[j]);
            if (r < g.t && ok) store16<F32>(dst_t, rk + c0, y);
        }
    }
    st::tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, 256);
    }
}

st_status check(st_handle *h, const void *q, const void *k, const void *v, int64_t bh, int64_t t, int64_t d,
                const char *who) {
    if (!q || !k || !v) return h->fail(ST_INVALID_ARG, "%s: null buffer", who);
    if (bh < 1 || bh > (1 << 30) || t < 1) return h->fail(ST_INVALID_ARG, "%s: bad bh / t", who);
    if (t > AMAXT || d != AD)
        return h->fail(ST_UNSUPPORTED_SHAPE, "%s: the fused kernel takes t <= %d and d = %d (got t=%lld d=%lld)", who,
                       AMAXT, AD, (long long)t, (long long)d);
    if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15u)
        return h->fail(ST_INVALID_ARG, "%s: q, k, v must be 16-byte aligned", who);
    return ST_OK;
}

// Launches an attention kernel programmatically dependent on the previous
// kernel of the stream: its prologue (barriers, TMEM) may run while that
// kernel finishes; every global read follows griddepcontrol.wait.
template <typename K>
cudaError_t launch_dependent(st_handle *h, K kern, dim3 grid, int threads, int smem, const AttnArgs &g,
                             const HeadMaps &tm) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(static_cast<unsigned>(threads));
    cfg.dynamicSmemBytes = static_cast<size_t>(smem);
    cfg.stream = h->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, g, tm);
}

// The 128-key forward fits two CTAs per SM (82 KB of shared memory, 256 TMEM
// columns, 128 registers a thread): with more CTAs than SMs every one is
// resident in one wave.  With at most one per SM the launch asks for more than
// half an SM's shared memory, so the CTAs spread over the SMs instead of
// pairing up on half of them.
constexpr int FWD_SPREAD_SMEM = 120 * 1024;

// With at most one CTA per SM and TMA-loaded f16 heads of one tile, the
// forward runs four threads per row (k_attn_fwd<false, 128, 512>).
template <bool F32, int TK>
st_status launch_fwd_tk(st_handle *h, const AttnArgs &g, const HeadMaps &tm) {
    constexpr int spread = TK == 128 && FwdSmem<TK>::SIZE < FWD_SPREAD_SMEM ? FWD_SPREAD_SMEM : FwdSmem<TK>::SIZE;
    static bool attr = false;
    if (!attr) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_attn_fwd<F32, TK>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              spread));
        if constexpr (!F32 && TK == AT)
            ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_attn_fwd<false, AT, ATHREADS4>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize, spread));
        attr = true;
    }
    const dim3 grid(static_cast<unsigned>(g.bh), static_cast<unsigned>((g.t + AT - 1) / AT));
    const int64_t ctas = static_cast<int64_t>(grid.x) * grid.y;
    const int smem = ctas > h->num_sms ? FwdSmem<TK>::SIZE : spread;
    if constexpr (!F32 && TK == AT) {
        if (g.tma && ctas <= h->num_sms) {
            ST_CHECK_CUDA(h, launch_dependent(h, k_attn_fwd<false, AT, ATHREADS4>, grid, ATHREADS4, smem, g, tm));
            return st_after_launch(h, "k_attn_fwd");
        }
    }
    ST_CHECK_CUDA(h, launch_dependent(h, k_attn_fwd<F32, TK>, grid, ATHREADS, smem, g, tm));
    return st_after_launch(h, "k_attn_fwd");
}

template <bool F32>
st_status launch_fwd(st_handle *h, const AttnArgs &g, const HeadMaps &tm) {
    return g.t <= AT ? launch_fwd_tk<F32, AT>(h, g, tm) : launch_fwd_tk<F32, AMAXT>(h, g, tm);
}

// With at most one CTA per SM and TMA-loaded f16 heads the backward runs
// four threads per row (k_attn_bwd<false, 512>).
template <bool F32>
st_status launch_bwd(st_handle *h, const AttnArgs &g, const HeadMaps &tm) {
    static bool attr = false;
    if (!attr) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_attn_bwd<F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM));
        if constexpr (!F32)
            ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_attn_bwd<false, ATHREADS4>,
                                                  cudaFuncAttributeMaxDynamicSharedMemorySize, BWD_SMEM));
        attr = true;
    }
    const int ntile = (g.t + AT - 1) / AT;
    const dim3 grid(static_cast<unsigned>(g.bh), static_cast<unsigned>(ntile == 1 ? 1 : 2 * ntile));
    if (ntile == 1 && g.bh > h->num_sms) {  // one-tile heads beyond one per SM: the compact form, two per SM
        static bool attr1 = false;
        if (!attr1) {
            ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_attn_bwd1<F32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                  CBWD_SMEM));
            attr1 = true;
        }
        ST_CHECK_CUDA(h, launch_dependent(h, k_attn_bwd1<F32>, grid, ATHREADS, CBWD_SMEM, g, tm));
        return st_after_launch(h, "k_attn_bwd1");
    }
    if constexpr (!F32) {
        if (g.tma && static_cast<int64_t>(grid.x) * grid.y <= h->num_sms) {
            ST_CHECK_CUDA(h, launch_dependent(h, k_attn_bwd<false, ATHREADS4>, grid, ATHREADS4, BWD_SMEM, g, tm));
            return st_after_launch(h, "k_attn_bwd");
        }
    }
    ST_CHECK_CUDA(h, launch_dependent(h, k_attn_bwd<F32>, grid, ATHREADS, BWD_SMEM, g, tm));
    return st_after_launch(h, "k_attn_bwd");
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// The map of one per-head f16 tensor [bh, t, 64] (see HeadMaps); false when
// the driver refuses it, and the kernels then stage with thread loads.
bool head_map(CUtensorMap *m, const void *base, int64_t bh, int64_t t) {
    return st_make_map_4d(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, base, AD, static_cast<uint64_t>(t),
                          static_cast<uint64_t>(bh), 1, AD, static_cast<uint64_t>(t * AD),
                          static_cast<uint64_t>(bh * t * AD), AD, AT, CU_TENSOR_MAP_SWIZZLE_128B, nullptr);
}

}  // namespace

extern "C" st_status st_attn_fwd(st_handle *h, const void *q, const void *k, const void *v, void *o, float *lse,
                                 int64_t bh, int64_t t, int64_t d, float scale, int32_t causal, int32_t one) {
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
    g.one = one;
    g.status = h->d_status;
    HeadMaps tm{};
    g.tma = head_map(&tm.q, q, bh, t) && head_map(&tm.k, k, bh, t) && head_map(&tm.v, v, bh, t);
    return launch_fwd<false>(h, g, tm);
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
    HeadMaps tm{};
    g.tma = head_map(&tm.q, q, bh, t) && head_map(&tm.k, k, bh, t) && head_map(&tm.v, v, bh, t) &&
            head_map(&tm.o, o, bh, t) && head_map(&tm.dout, dout, bh, t);
    return launch_bwd<false>(h, g, tm);
}

extern "C" st_status st_attn_fwd_packed(st_handle *h, const float *qkv, float *o, float *lse, int64_t batch,
                                        int64_t heads, int64_t t, int64_t d, float scale, int32_t causal,
                                        int32_t one) {
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
    g.one = one;
    g.status = h->d_status;
    return launch_fwd<true>(h, g, HeadMaps{});
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
    return launch_bwd<true>(h, g, HeadMaps{});
}
