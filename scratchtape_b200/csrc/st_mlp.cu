// st_mlp.cu -- one Linear -> ReLU -> Linear layer (no bias), forward and
// backward, as one tcgen05 kernel plus one fixed-order reduction.
//
// The six TF32 GEMMs of the layer (src/tape.rs:505-510 for the MatMul arm,
// :530-534 for ReLU's mask; the C2 configuration of the MLP step):
//   H  = relu(X W1)          [M, F]     Y  = H W2        [M, D]
//   dH = (dY W2^T) * (H > 0) [M, F]     dX = dH W1^T     [M, D]
//   dW2 = H^T dY             [F, D]     dW1 = X^T dH     [D, F]
// with D = 128.  CTA (cc, rb) owns 128 tokens (rb) and 128 columns of F (cc);
// everything it needs of H and dH it makes itself, so the six products chain
// through TMEM and shared memory instead of through global memory:
//   P1  acc_H = X_rb W1[:, cc],  acc_G = dY_rb W2[cc, :]^T   (K = D, streamed)
//   E1  H = relu(acc_H), dH = acc_G * (H > 0): back into TMEM (the A operand of
//       P2), transposed into shared memory (an operand of P3), and to H / dH
//   P2  Y_p = H W2[cc, :],  dX_p = dH W1[:, cc]^T           (A from TMEM)
//   P3  dW2_p = H^T dY_rb,  dW1_p = X_rb^T dH               (K = 128 tokens)
//   E2  the four partial products to a scratch buffer
// Y and dX are sums over the F / 128 column blocks, dW1 and dW2 over the
// M / 128 token blocks: k_mlp_reduce adds the partials in block order, so the
// results are deterministic.
//
// Roles (320 threads): warp 0 issues TMA loads (16 loads of 32 KB: 8 for P1,
// 4 for P2, 4 for P3), warp 1 issues the MMAs, warps 2..9 are the epilogue
// (warp w reads TMEM lanes 32 (w % 4).. and one half of the columns).  Load
// slots: three 32 KB ring slots, plus, during P1 only, the four slots of the
// 128 KB that later holds H^T and dH^T.  TMEM: [0,128) acc_H then dW2_p,
// [128,256) acc_G then dW1_p, [256,384) Y_p, [384,512) dX_p.
#include "st_internal.h"
#include "st_ptx.cuh"

#include <algorithm>

namespace {

constexpr int MT = 128;   // tokens per CTA (MMA M, TMEM lanes)
constexpr int CT = 128;   // F columns per CTA
constexpr int DM = 128;   // D (model width)
constexpr int KB = 32;    // f32 per 128-byte row: one k block
constexpr int SLOT = 32768;
constexpr int NRING = 3;           // slots outside the H^T / dH^T region
constexpr int NSLOT = NRING + 4;   // + the four slots of that region (P1 only)
constexpr int TILE = MT * CT * 4;  // 64 KB
constexpr int OFF_HT = 0;          // H^T  [token block][c][token % 32], K-major 128B swizzle
constexpr int OFF_DHT = TILE;      // dH^T, the same layout
constexpr int OFF_RING = 2 * TILE;
constexpr int OFF_BAR = OFF_RING + NRING * SLOT;
constexpr int SMEM = OFF_BAR + 256 + 1024;  // barriers, then slack for 1024-byte alignment
constexpr int NEPI = 256;
constexpr int THREADS = 64 + NEPI;
constexpr int N_LOADS = 16;
static_assert(SMEM <= 232448, "MLP step kernel exceeds the sm_100 shared-memory limit");

struct MlpArgs {
    float *h, *dh;  // [M, F] outputs, or null
    float *part;    // Y_p [F/128][M][D], dX_p [F/128][M][D], dW2_p [M/128][F][D], dW1_p [M/128][D][F]
    int m, f;
    int *status;
};

struct MlpMaps {
    CUtensorMap xk, dyk;  // X, dY [M, D]: boxes 32 x 128 rows, 128B swizzle (K-major A)
    CUtensorMap xn, dyn;  // X, dY: boxes 32 x 32 rows, 128B swizzle with 32B atoms (MN-major)
    CUtensorMap w1n, w1k; // W1 [D, F]: 32 x 32 MN-major / 32 x 128 K-major
    CUtensorMap w2k, w2n; // W2 [F, D]: 32 x 128 K-major / 32 x 32 MN-major
};

// Load e's slot and how many loads used that slot before it: loads 0..6 take
// slots 0..6 once; loads 7.. cycle through ring slots 0..2.
__device__ __forceinline__ void slot_of(int e, int &slot, int &use) {
    if (e < NSLOT) {
        slot = e, use = 0;
    } else {
        slot = (e - NSLOT) % NRING, use = 1 + (e - NSLOT) / NRING;
    }
}
__device__ __forceinline__ uint8_t *slot_ptr(uint8_t *smem, int slot) {
    return slot < NRING ? smem + OFF_RING + slot * SLOT : smem + OFF_HT + (slot - NRING) * SLOT;
}

__device__ __forceinline__ uint64_t kdesc(uint32_t a) { return st::sdesc_sw128(a, 16, 1024); }
__device__ __forceinline__ uint64_t ndesc(uint32_t a) { return st::sdesc_make(a, 4096, 512, st::LAYOUT_SW128_BASE32B); }

__device__ __forceinline__ void st_v4(float *p, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
    *reinterpret_cast<float4 *>(p) = make_float4(__uint_as_float(a), __uint_as_float(b), __uint_as_float(c),
                                                 __uint_as_float(d));
}
__device__ __forceinline__ void st_row32(float *p, const uint32_t (&r)[32]) {
#pragma unroll
    for (int i = 0; i < 8; i++) st_v4(p + 4 * i, r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]);
}

__global__ void __launch_bounds__(THREADS, 1) k_mlp_step(const __grid_constant__ MlpMaps mp, const MlpArgs g) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *full = bars, *empty = bars + NSLOT;
    uint64_t *acc1 = bars + 2 * NSLOT, *hs_ready = acc1 + 1, *acc2 = acc1 + 2, *acc3 = acc1 + 3;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc1 + 4);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cc = blockIdx.x, rb = blockIdx.y;
    const int c0 = cc * CT, t0 = rb * MT;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NSLOT; s++) {
            st::mbar_init(&full[s], 1);
            st::mbar_init(&empty[s], 1);
        }
        st::mbar_init(acc1, 1);
        st::mbar_init(hs_ready, NEPI);
        st::mbar_init(acc2, 1);
        st::mbar_init(acc3, 1);
        st::fence_mbar_init();
    }
    if (warp == 1) {
        st::tmem_alloc(tmem_slot, 512);
        st::tmem_relinquish();
    }
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    st::grid_dep_wait();

    if (warp == 0) {
        if (lane == 0) {  // ------------------------------------------------ TMA
            st::tma_prefetch_desc(&mp.xk);
            st::tma_prefetch_desc(&mp.dyk);
            st::tma_prefetch_desc(&mp.w1n);
            st::tma_prefetch_desc(&mp.w2k);
            for (int e = 0; e < N_LOADS; e++) {
                int s, use;
                slot_of(e, s, use);
                if (use > 0 && !st::mbar_wait(&empty[s], (use - 1) & 1, g.status, st::DEV_TIMEOUT_EMPTY)) break;
                st::mbar_arrive_expect_tx(&full[s], SLOT);
                uint8_t *a = slot_ptr(smem, s), *b = a + SLOT / 2;
                if (e < 8) {
                    const int k = (e >> 1) * KB;  // D columns
                    if ((e & 1) == 0) {           // acc_H: A = X (K-major), B = W1[k.., c0..] (MN-major)
                        st::tma_load_4d(a, &mp.xk, &full[s], k, t0, 0, 0);
#pragma unroll
                        for (int j = 0; j < 4; j++) st::tma_load_4d(b + 4096 * j, &mp.w1n, &full[s], c0 + 32 * j, k, 0, 0);
                    } else {                      // acc_G: A = dY (K-major), B = W2[c0.., k..] (K-major)
                        st::tma_load_4d(a, &mp.dyk, &full[s], k, t0, 0, 0);
                        st::tma_load_4d(b, &mp.w2k, &full[s], k, c0, 0, 0);
                    }
                } else if (e < 12) {
                    const int k = c0 + (e - 8) * KB;  // F columns
                    // Y_p: B = W2[k.., :] (MN-major); dX_p: B = W1[:, k..] (K-major)
#pragma unroll
                    for (int j = 0; j < 4; j++) st::tma_load_4d(a + 4096 * j, &mp.w2n, &full[s], 32 * j, k, 0, 0);
                    st::tma_load_4d(b, &mp.w1k, &full[s], k, 0, 0, 0);
                } else {
                    const int k = t0 + (e - 12) * KB;  // tokens
                    // dW2_p: B = dY[k.., :] (MN-major); dW1_p: A = X[k.., :]^T (MN-major)
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        st::tma_load_4d(a + 4096 * j, &mp.dyn, &full[s], 32 * j, k, 0, 0);
                        st::tma_load_4d(b + 4096 * j, &mp.xn, &full[s], 32 * j, k, 0, 0);
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {  // ------------------------------------------------ MMA
            constexpr uint32_t ID_KK = st::idesc_make(1, 2, false, false, MT, CT);
            constexpr uint32_t ID_KN = st::idesc_make(1, 2, false, true, MT, CT);
            constexpr uint32_t ID_NK = st::idesc_make(1, 2, true, false, MT, CT);
            const uint32_t tH = tmem, tG = tmem + 128, tY = tmem + 256, tDX = tmem + 384;
            const uint32_t sHT = st::smem_u32(smem + OFF_HT), sDHT = st::smem_u32(smem + OFF_DHT);
            for (int e = 0; e < N_LOADS; e++) {
                int s, use;
                slot_of(e, s, use);
                if (e == 8) {  // P2 reads H and dH from TMEM
                    if (!st::mbar_wait(hs_ready, 0, g.status, st::DEV_TIMEOUT_ACC)) break;
                    st::tc_fence_after();
                }
                if (!st::mbar_wait(&full[s], use & 1, g.status, st::DEV_TIMEOUT_FULL)) break;
                st::tc_fence_after();
                const uint32_t sa = st::smem_u32(slot_ptr(smem, s)), sb = sa + SLOT / 2;
                if (e < 8) {
                    const int kb = e >> 1;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                        if ((e & 1) == 0) st::umma_tf32(tH, kdesc(sa + 32 * kk), ndesc(sb + 1024 * kk), ID_KN, acc);
                        else st::umma_tf32(tG, kdesc(sa + 32 * kk), kdesc(sb + 32 * kk), ID_KK, acc);
                    }
                } else if (e < 12) {
                    const int kb = e - 8;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                        const uint32_t col = static_cast<uint32_t>(KB * kb + 8 * kk);
                        st::umma_tf32_ts(tY, tH + col, ndesc(sa + 1024 * kk), ID_KN, acc);
                        st::umma_tf32_ts(tDX, tG + col, kdesc(sb + 32 * kk), ID_KK, acc);
                    }
                } else {
                    const int kb = e - 12;
#pragma unroll
                    for (int kk = 0; kk < 4; kk++) {
                        const uint32_t acc = (kb > 0 || kk > 0) ? 1u : 0u;
                        const uint32_t ko = static_cast<uint32_t>(kb * (TILE / 4) + 32 * kk);
                        st::umma_tf32(tH, kdesc(sHT + ko), ndesc(sa + 1024 * kk), ID_KN, acc);   // dW2_p [c][d]
                        st::umma_tf32(tG, ndesc(sb + 1024 * kk), kdesc(sDHT + ko), ID_NK, acc);  // dW1_p [d][c]
                    }
                }
                st::umma_commit(&empty[s]);
                if (e == 7) st::umma_commit(acc1);
                if (e == 11) {
                    // P3 accumulates into the columns P2 reads as A: wait for P2
                    st::umma_commit(acc2);
                    if (!st::mbar_wait(acc2, 0, g.status, st::DEV_TIMEOUT_ACC)) break;
                    st::tc_fence_after();
                }
                if (e == N_LOADS - 1) st::umma_commit(acc3);
            }
        }
    } else {  // -------------------------------------------------------- epilogue
        const int q = warp & 3, half = (warp - 2) >> 2;
        const int row = q * 32 + lane;
        const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
        // E1: H and dH.  acc1 also means every P1 load has been consumed, so
        // the H^T / dH^T region (P1's extra load slots) is free to write.
        bool ok = st::mbar_wait(acc1, 0, g.status, st::DEV_TIMEOUT_ACC);
        st::tc_fence_after();
        if (ok) {
#pragma unroll 1
            for (int j = 0; j < 2; j++) {
                const int col = half * 64 + j * 32;
                uint32_t hr[32], gr[32];
                st::tmem_ld32(tmem + lanes + col, hr);
                st::tmem_ld32(tmem + lanes + 128 + col, gr);
                st::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const float h = fmaxf(__uint_as_float(hr[i]), 0.0f);
                    const float dh = h > 0.0f ? __uint_as_float(gr[i]) : 0.0f;
                    hr[i] = __float_as_uint(h);
                    gr[i] = __float_as_uint(dh);
                }
                st::tmem_st32(tmem + lanes + col, hr);
                st::tmem_st32(tmem + lanes + 128 + col, gr);
                // transposed: row c of token block q holds tokens 32q.. of column c
                uint8_t *ht = smem + OFF_HT + q * (TILE / 4), *dht = smem + OFF_DHT + q * (TILE / 4);
                const uint32_t within = static_cast<uint32_t>(lane & 3) * 4u;
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    const uint32_t off =
                        st::sw128_offset(static_cast<uint32_t>(col + i), static_cast<uint32_t>(lane >> 2)) + within;
                    *reinterpret_cast<uint32_t *>(ht + off) = hr[i];
                    *reinterpret_cast<uint32_t *>(dht + off) = gr[i];
                }
                const int64_t gi = static_cast<int64_t>(t0 + row) * g.f + c0 + col;
                if (g.h) st_row32(g.h + gi, hr);
                if (g.dh) st_row32(g.dh + gi, gr);
            }
        }
        st::tmem_st_wait();
        st::fence_proxy_async_smem();
        st::tc_fence_before();
        st::mbar_arrive(hs_ready);

        // E2: the partial products
        const int ncc = g.f / CT;
        float *yp = g.part;
        float *xp = yp + static_cast<int64_t>(ncc) * g.m * DM;
        float *w2p = xp + static_cast<int64_t>(ncc) * g.m * DM;
        float *w1p = w2p + static_cast<int64_t>(g.m / MT) * g.f * DM;
        ok = ok && st::mbar_wait(acc2, 0, g.status, st::DEV_TIMEOUT_ACC);
        st::tc_fence_after();
        if (ok) {
            float *y_row = yp + (static_cast<int64_t>(cc) * g.m + t0 + row) * DM;
            float *x_row = xp + (static_cast<int64_t>(cc) * g.m + t0 + row) * DM;
#pragma unroll 1
            for (int j = 0; j < 2; j++) {
                const int col = half * 64 + j * 32;
                uint32_t r[32], u[32];
                st::tmem_ld32(tmem + lanes + 256 + col, r);
                st::tmem_ld32(tmem + lanes + 384 + col, u);
                st::tmem_ld_wait();
                st_row32(y_row + col, r);
                st_row32(x_row + col, u);
            }
        }
        ok = ok && st::mbar_wait(acc3, 0, g.status, st::DEV_TIMEOUT_ACC);
        st::tc_fence_after();
        if (ok) {
            float *w2_row = w2p + (static_cast<int64_t>(rb) * g.f + c0 + row) * DM;  // lane = c, columns = d
            float *w1_row = w1p + (static_cast<int64_t>(rb) * DM + row) * g.f + c0;  // lane = d, columns = c
#pragma unroll 1
            for (int j = 0; j < 2; j++) {
                const int col = half * 64 + j * 32;
                uint32_t r[32], u[32];
                st::tmem_ld32(tmem + lanes + col, r);
                st::tmem_ld32(tmem + lanes + 128 + col, u);
                st::tmem_ld_wait();
                st_row32(w2_row + col, r);
                st_row32(w1_row + col, u);
            }
        }
        st::grid_dep_launch();
    }
    st::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, 512);
    }
}

// Y = sum of the F/128 partials, dX likewise; dW2 and dW1 = sums of the
// M/128 partials; each output float4 adds its partials in block order.
__global__ void __launch_bounds__(256) k_mlp_reduce(const float *part, float *y, float *dx, float *dw1, float *dw2,
                                                    int m, int f) {
    st::grid_dep_wait();
    const int ncc = f / CT, nrb = m / MT;
    const int64_t ny = static_cast<int64_t>(m) * DM / 4, nw = static_cast<int64_t>(f) * DM / 4;
    const float4 *yp = reinterpret_cast<const float4 *>(part), *xp = yp + ncc * ny, *w2p = xp + ncc * ny,
                 *w1p = w2p + nrb * nw;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < 2 * ny + 2 * nw;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float4 *src;
        float4 *dst;
        int n;
        int64_t stride;
        if (i < ny) {
            src = yp + i, dst = reinterpret_cast<float4 *>(y) + i, n = ncc, stride = ny;
        } else if (i < 2 * ny) {
            src = xp + (i - ny), dst = reinterpret_cast<float4 *>(dx) + (i - ny), n = ncc, stride = ny;
        } else if (i < 2 * ny + nw) {
            src = w2p + (i - 2 * ny), dst = reinterpret_cast<float4 *>(dw2) + (i - 2 * ny), n = nrb, stride = nw;
        } else {
            src = w1p + (i - 2 * ny - nw), dst = reinterpret_cast<float4 *>(dw1) + (i - 2 * ny - nw), n = nrb,
            stride = nw;
        }
        float4 s = __ldcg(src);
        int k = 1;
        for (; k + 8 <= n; k += 8) {
            float4 v[8];
#pragma unroll
            for (int u = 0; u < 8; u++) v[u] = __ldcg(src + (k + u) * stride);
#pragma unroll
            for (int u = 0; u < 8; u++) s.x += v[u].x, s.y += v[u].y, s.z += v[u].z, s.w += v[u].w;
        }
        for (; k < n; k++) {
            const float4 v = __ldcg(src + k * stride);
            s.x += v.x, s.y += v.y, s.z += v.z, s.w += v.w;
        }
        *dst = s;
    }
}

bool map2d(CUtensorMap *map, const float *base, uint64_t cols, uint64_t rows, uint32_t box_rows, bool mn,
           std::string *why) {
    return st_make_map_4d(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, cols, rows, 1, 1, cols, rows * cols,
                          rows * cols, 32, box_rows,
                          mn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B, why);
}

bool aligned16(const void *p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace

extern "C" st_status st_mlp_step_tf32(st_handle *h, const float *x, const float *w1, const float *w2, const float *dy,
                                      float *hout, float *y, float *dhout, float *dx, float *dw1, float *dw2, int64_t m,
                                      int64_t d, int64_t f) {
    const char *who = "st_mlp_step_tf32";
    if (!h) return ST_INVALID_ARG;
    if (!x || !w1 || !w2 || !dy || !y || !dx || !dw1 || !dw2 || m < 1 || d < 1 || f < 1)
        return h->fail(ST_INVALID_ARG, "%s: null buffer or empty shape", who);
    if (d != DM || m % MT != 0 || f % CT != 0 || m > (1 << 24) || f > (1 << 16))
        return h->fail(ST_UNSUPPORTED_SHAPE, "%s: needs d == 128, m and f multiples of 128 (got m %lld d %lld f %lld)",
                       who, (long long)m, (long long)d, (long long)f);
    const void *ptrs[10] = {x, w1, w2, dy, hout, y, dhout, dx, dw1, dw2};
    for (const void *p : ptrs)
        if (p && !aligned16(p)) return h->fail(ST_UNSUPPORTED_SHAPE, "%s: buffers must be 16-byte aligned", who);
    cudaSetDevice(h->device);
    MlpMaps mp;
    std::string why;
    if (!map2d(&mp.xk, x, DM, m, 128, false, &why) || !map2d(&mp.dyk, dy, DM, m, 128, false, &why) ||
        !map2d(&mp.xn, x, DM, m, 32, true, &why) || !map2d(&mp.dyn, dy, DM, m, 32, true, &why) ||
        !map2d(&mp.w1n, w1, f, DM, 32, true, &why) || !map2d(&mp.w1k, w1, f, DM, 128, false, &why) ||
        !map2d(&mp.w2k, w2, DM, f, 128, false, &why) || !map2d(&mp.w2n, w2, DM, f, 32, true, &why))
        return h->fail(ST_UNSUPPORTED_SHAPE, "%s: %s", who, why.c_str());
    const int64_t part_floats = 2 * (f / CT) * m * DM + 2 * (m / MT) * f * DM;
    float *part = static_cast<float *>(st_scratch(h, SLOT_MLP_PART, sizeof(float) * part_floats));
    if (!part) return ST_NO_MEMORY;
    MlpArgs g{hout, dhout, part, static_cast<int>(m), static_cast<int>(f), h->d_status};

    static bool attr_done = false;
    if (!attr_done) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_mlp_step, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        attr_done = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(f / CT), static_cast<unsigned>(m / MT));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM;
    cfg.stream = h->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ST_CHECK_CUDA(h, cudaLaunchKernelEx(&cfg, k_mlp_step, mp, g));
    st_status s = st_after_launch(h, "k_mlp_step");
    if (s != ST_OK) return s;
    const int64_t items = 2 * (m * DM / 4) + 2 * (f * DM / 4);
    cfg.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>((items + 255) / 256, 8LL * h->num_sms)));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    ST_CHECK_CUDA(h, cudaLaunchKernelEx(&cfg, k_mlp_reduce, static_cast<const float *>(part), y, dx, dw1, dw2,
                                        static_cast<int>(m), static_cast<int>(f)));
    return st_after_launch(h, "k_mlp_reduce");
}
