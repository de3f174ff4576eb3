// st_mlp.cu -- one Linear -> ReLU -> Linear layer (no bias), forward and
// backward, as one tcgen05 kernel whose CTAs also add up each other's partial
// products in a fixed order.
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
//       P2) and, transposed, into shared memory (an operand of P3)
//   P2  Y_p = H W2[cc, :],  dX_p = dH W1[:, cc]^T           (A from TMEM)
//   P3  dW2_p = H^T dY_rb,  dW1_p = X_rb^T dH               (K = 128 tokens)
//   E3  H and dH to global memory from their transposed shared-memory tiles
//       (while P2 runs)
//   E2  the four partial products to a scratch buffer (Y_p, dX_p while P3 runs)
//   R1  Y and dX: the ncc = F/128 CTAs of a token block each sum 128/ncc rows
//       over the block's ncc partials
//   R2  dW2 and dW1: the nrb = M/128 CTAs of a column block each sum 256/nrb
//       of its columns over the block's nrb partials
// R1 and R2 wait (bounded) on per-block arrival counters, so the launch is
// cooperative (every CTA resident); every output is summed in one fixed
// block order, so the results are deterministic.
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
constexpr int R1_ITEMS = 8, R1_K = 4;  // Y / dX reduction: items per thread per pass, partials per load round
constexpr int R2_K = 32;               // dW reduction: partials per load round
static_assert(SMEM <= 232448, "MLP step kernel exceeds the sm_100 shared-memory limit");

struct MlpArgs {
    float *h, *dh;  // [M, F] outputs, or null
    float *y, *dx, *dw1, *dw2;
    unsigned *ctl;  // [M/128] arrivals, [M/128] departures per token block; the same per column block; abort
    float *part;    // Y_p, dX_p [F/128][M/128] tiles; dW2_p, dW1_p [M/128][F/128] tiles (128 x 128, column-major)
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

// Barrier of the 256 epilogue threads only (warps 2..9).
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, %0;" ::"n"(NEPI) : "memory"); }

// epi_bar that also returns whether `v` holds in every epilogue thread, so
// that branches holding further barriers are taken by all of them or none.
__device__ __forceinline__ bool epi_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(static_cast<uint32_t>(v)), "n"(NEPI)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ unsigned ld_acquire(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// With `ok` (the same in every epilogue thread), thread `et` == 0 spins
// (bounded) until *ctr >= need -- the CTAs it waits for are resident with it
// (cooperative launch) -- and shares the outcome with the other epilogue
// threads.  On expiry: the status word and the abort flag.
__device__ bool wait_count(const MlpArgs &g, const unsigned *ctr, unsigned need, int et, bool ok_in) {
    __shared__ int s_ok;
    if (et == 0) {
        int ok = ok_in ? 1 : 0;
        const unsigned *abort_flag = g.ctl + 2 * (g.m / MT) + 2 * (g.f / CT);
        const uint64_t t0 = st::globaltimer();
#pragma unroll 1
        for (uint32_t i = 0; ok; ++i) {
            if (ld_acquire(ctr) >= need) break;
            if (ld_acquire(abort_flag)) {
                ok = 0;
                break;
            }
            __nanosleep(64);
            if ((i & 15u) == 0 && st::globaltimer() - t0 > st::WAIT_LIMIT_NS) {
                st::set_status(g.status, st::DEV_TIMEOUT_FULL);
                atomicExch(const_cast<unsigned *>(abort_flag), 1u);
                ok = 0;
                break;
            }
        }
        s_ok = ok;
    }
    epi_bar();
    return s_ok != 0;
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
        const int q = warp & 3, half = (warp - 2) >> 2, ew = warp - 2;
        const int row = q * 32 + lane;
        const int et = threadIdx.x - 64;  // 0..255
        const uint32_t lanes = static_cast<uint32_t>(q * 32) << 16;
        const int ncc = g.f / CT, nrb = g.m / MT;
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
            }
        }
        st::tmem_st_wait();
        st::fence_proxy_async_smem();
        st::tc_fence_before();
        st::mbar_arrive(hs_ready);
        ok = epi_all(ok);  // the H^T / dH^T tiles are complete

        // E3: H and dH out of their transposed shared-memory tiles while P2
        // runs (the tiles are final; P3 only reads them): lane = column, so
        // each store is one 128-byte line
        if (ok && (g.h || g.dh)) {
#pragma unroll 1
            for (int tt = 0; tt < MT / 8; tt++) {
                const int t = ew * (MT / 8) + tt;
                const uint32_t tin = static_cast<uint32_t>(t & 31);
                const uint8_t *ht = smem + OFF_HT + (t >> 5) * (TILE / 4);
                const int64_t gi = static_cast<int64_t>(t0 + t) * g.f + c0 + lane;
#pragma unroll
                for (int ch = 0; ch < CT / 32; ch++) {
                    const uint32_t off =
                        st::sw128_offset(static_cast<uint32_t>(ch * 32 + lane), tin >> 2) + (tin & 3u) * 4u;
                    if (g.h) g.h[gi + ch * 32] = *reinterpret_cast<const float *>(ht + off);
                    if (g.dh) g.dh[gi + ch * 32] = *reinterpret_cast<const float *>(ht + TILE + off);
                }
            }
        }

        // E2: the partial products, each 128 x 128 tile column-major (element
        // (lane, column) at column * 128 + lane), so a warp's store of one
        // column is one full 128-byte line
        float *yp = g.part;
        float *xp = yp + static_cast<int64_t>(ncc) * nrb * (MT * CT);
        float *w2p = xp + static_cast<int64_t>(ncc) * nrb * (MT * CT);
        float *w1p = w2p + static_cast<int64_t>(ncc) * nrb * (MT * CT);
        ok = ok && st::mbar_wait(acc2, 0, g.status, st::DEV_TIMEOUT_ACC);
        st::tc_fence_after();
        if (ok) {
            float *yt = yp + static_cast<int64_t>(cc * nrb + rb) * (MT * CT) + row;
            float *xt = xp + static_cast<int64_t>(cc * nrb + rb) * (MT * CT) + row;
#pragma unroll 1
            for (int j = 0; j < 2; j++) {
                const int col = half * 64 + j * 32;
                uint32_t r[32], u[32];
                st::tmem_ld32(tmem + lanes + 256 + col, r);
                st::tmem_ld32(tmem + lanes + 384 + col, u);
                st::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    yt[(col + i) * MT] = __uint_as_float(r[i]);
                    xt[(col + i) * MT] = __uint_as_float(u[i]);
                }
            }
        }
        __threadfence();
        ok = epi_all(ok);
        if (et == 0 && ok) atomicAdd(g.ctl + rb, 1u);
        ok = ok && st::mbar_wait(acc3, 0, g.status, st::DEV_TIMEOUT_ACC);
        st::tc_fence_after();
        if (ok) {
            float *w2t = w2p + static_cast<int64_t>(rb * ncc + cc) * (MT * CT) + row;  // lane = c, columns = d
            float *w1t = w1p + static_cast<int64_t>(rb * ncc + cc) * (MT * CT) + row;  // lane = d, columns = c
#pragma unroll 1
            for (int j = 0; j < 2; j++) {
                const int col = half * 64 + j * 32;
                uint32_t r[32], u[32];
                st::tmem_ld32(tmem + lanes + col, r);
                st::tmem_ld32(tmem + lanes + 128 + col, u);
                st::tmem_ld_wait();
#pragma unroll
                for (int i = 0; i < 32; i++) {
                    w2t[(col + i) * MT] = __uint_as_float(r[i]);
                    w1t[(col + i) * MT] = __uint_as_float(u[i]);
                }
            }
        }
        __threadfence();
        ok = epi_all(ok);
        if (et == 0 && ok) atomicAdd(g.ctl + 2 * nrb + cc, 1u);

        // R1: rows [r0, r0 + R) of this token block's Y and dX, each the sum
        // of its ncc partials in column-block order; staged row-major in the
        // (now free) shared memory and written out a row at a time
        float *stage = reinterpret_cast<float *>(smem);
        ok = wait_count(g, g.ctl + rb, static_cast<unsigned>(ncc), et, ok);
        if (ok) {
            const int q0 = cc * (MT / 4) / ncc, q1 = (cc + 1) * (MT / 4) / ncc, nq4 = q1 - q0;
            const int items = 2 * CT * nq4;
            const int64_t step4 = static_cast<int64_t>(nrb) * (MT * CT) / 4;
            // R1_ITEMS items per thread per pass, R1_K partials per load round,
            // every load of a round in flight before the first addition
            for (int i0 = 0; i0 < items; i0 += R1_ITEMS * NEPI) {
                const float4 *p[R1_ITEMS];
                float4 a[R1_ITEMS];
#pragma unroll
                for (int j = 0; j < R1_ITEMS; j++) {
                    const int i = min(i0 + j * NEPI + et, items - 1);
                    const int o = i / (CT * nq4), rem = i % (CT * nq4), c = rem / nq4, qq = rem % nq4;
                    p[j] = reinterpret_cast<const float4 *>((o ? xp : yp) + static_cast<int64_t>(rb) * (MT * CT) +
                                                            c * MT + 4 * (q0 + qq));
                    a[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                }
                for (int k0 = 0; k0 < ncc; k0 += R1_K) {
                    float4 v[R1_ITEMS][R1_K];
#pragma unroll
                    for (int j = 0; j < R1_ITEMS; j++)
#pragma unroll
                        for (int k = 0; k < R1_K; k++)
                            v[j][k] = k0 + k < ncc ? __ldcg(p[j] + (k0 + k) * step4) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int j = 0; j < R1_ITEMS; j++)
#pragma unroll
                        for (int k = 0; k < R1_K; k++)
                            if (k0 + k < ncc) a[j].x += v[j][k].x, a[j].y += v[j][k].y, a[j].z += v[j][k].z, a[j].w += v[j][k].w;
                }
#pragma unroll
                for (int j = 0; j < R1_ITEMS; j++) {
                    const int i = i0 + j * NEPI + et;
                    if (i >= items) continue;
                    const int o = i / (CT * nq4), rem = i % (CT * nq4), c = rem / nq4, qq = rem % nq4;
                    float *sr = stage + (o * MT + 4 * qq) * (CT + 4) + c;
                    sr[0] = a[j].x, sr[CT + 4] = a[j].y, sr[2 * (CT + 4)] = a[j].z, sr[3 * (CT + 4)] = a[j].w;
                }
            }
            epi_bar();
            const int rows = 4 * nq4;
            for (int i = et; i < 2 * rows * (DM / 4); i += NEPI) {
                const int o = i / (rows * (DM / 4)), rem = i % (rows * (DM / 4)), r = rem / (DM / 4), c4 = rem % (DM / 4);
                const float *sr = stage + (o * MT + r) * (CT + 4) + 4 * c4;
                float *dst = (o ? g.dx : g.y) + static_cast<int64_t>(t0 + 4 * q0 + r) * DM + 4 * c4;
                *reinterpret_cast<float4 *>(dst) = make_float4(sr[0], sr[1], sr[2], sr[3]);
            }
            epi_bar();
            if (et == 0 && atomicAdd(g.ctl + nrb + rb, 1u) == static_cast<unsigned>(ncc - 1)) {
                atomicExch(g.ctl + rb, 0u);  // every CTA of this token block is past its wait
                atomicExch(g.ctl + nrb + rb, 0u);
            }
        }

        // R2: columns [u0, u1) of this column block's dW2 (units 0..127 = its
        // d columns) and dW1 (units 128..255 = its c columns), each the sum of
        // its nrb partials in token-block order
        ok = wait_count(g, g.ctl + 2 * nrb + cc, static_cast<unsigned>(nrb), et, ok);
        if (ok) {
            const int u0 = rb * 256 / nrb, u1 = (rb + 1) * 256 / nrb, nu = u1 - u0;
            const int64_t step = static_cast<int64_t>(ncc) * (MT * CT);
            for (int i = et; i < nu * (MT / 4); i += NEPI) {
                const int ul = i / (MT / 4), r4 = (i % (MT / 4)) * 4, u = u0 + ul;
                const float *base = (u < DM ? w2p : w1p) + static_cast<int64_t>(cc) * (MT * CT) + (u & 127) * MT + r4;
                const float4 *p = reinterpret_cast<const float4 *>(base);
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
                for (int k0 = 0; k0 < nrb; k0 += R2_K) {  // R2_K loads in flight, then their sums in order
                    float4 v[R2_K];
#pragma unroll
                    for (int t = 0; t < R2_K; t++)
                        v[t] = k0 + t < nrb ? __ldcg(p + (k0 + t) * (step / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int t = 0; t < R2_K; t++)
                        if (k0 + t < nrb) a.x += v[t].x, a.y += v[t].y, a.z += v[t].z, a.w += v[t].w;
                }
                float *sr = stage + r4 * (nu + 1) + ul;
                sr[0] = a.x, sr[nu + 1] = a.y, sr[2 * (nu + 1)] = a.z, sr[3 * (nu + 1)] = a.w;
            }
            epi_bar();
            for (int i = et; i < MT * nu; i += NEPI) {
                const int r = i / nu, ul = i % nu, u = u0 + ul;
                const float v = stage[r * (nu + 1) + ul];
                if (u < DM) g.dw2[static_cast<int64_t>(c0 + r) * DM + u] = v;   // row c, column d
                else g.dw1[static_cast<int64_t>(r) * g.f + c0 + (u - DM)] = v;   // row d, column c
            }
            epi_bar();
            if (et == 0 && atomicAdd(g.ctl + 2 * nrb + ncc + cc, 1u) == static_cast<unsigned>(nrb - 1)) {
                atomicExch(g.ctl + 2 * nrb + cc, 0u);
                atomicExch(g.ctl + 2 * nrb + ncc + cc, 0u);
            }
        }
    }
    st::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, 512);
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
    // every CTA of the grid must be resident at once: CTAs wait for the
    // partial products of the other CTAs of their token and column blocks
    const int64_t ctas = (m / MT) * (f / CT);
    if (ctas > h->num_sms)
        return h->fail(ST_UNSUPPORTED_SHAPE, "%s: (m/128)*(f/128) = %lld CTAs exceeds the %d SMs", who,
                       (long long)ctas, h->num_sms);
    const int64_t part_floats = 4 * ctas * MT * CT;
    float *part = static_cast<float *>(st_scratch(h, SLOT_MLP_PART, sizeof(float) * part_floats));
    if (!part) return ST_NO_MEMORY;
    // the counters are left at zero by every launch (the last CTA out of each
    // group resets its pair); they are zeroed here only when their memory is new
    const size_t ctl_bytes = sizeof(unsigned) * (2 * (m / MT) + 2 * (f / CT) + 1);
    unsigned *ctl = static_cast<unsigned *>(st_scratch(h, SLOT_MLP_CTL, ctl_bytes));
    if (!ctl) return ST_NO_MEMORY;
    if (ctl != h->mlp_ctl || ctl_bytes > h->mlp_ctl_bytes) {
        ST_CHECK_CUDA(h, cudaMemsetAsync(ctl, 0, h->slot_bytes[SLOT_MLP_CTL], h->stream));
        h->mlp_ctl = ctl;
        h->mlp_ctl_bytes = h->slot_bytes[SLOT_MLP_CTL];
    }
    MlpArgs g{hout, dhout, y, dx, dw1, dw2, ctl, part, static_cast<int>(m), static_cast<int>(f), h->d_status};

    static bool attr_set[64] = {};
    if (h->device >= 0 && h->device < 64 && !attr_set[h->device]) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_mlp_step, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM));
        attr_set[h->device] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(f / CT), static_cast<unsigned>(m / MT));
    cfg.blockDim = dim3(THREADS);
    cfg.dynamicSmemBytes = SMEM;
    cfg.stream = h->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    ST_CHECK_CUDA(h, cudaLaunchKernelEx(&cfg, k_mlp_step, mp, g));
    return st_after_launch(h, "k_mlp_step");
}
