// st_knn.cu -- the kNN memory's 2-bit key scan, fused with top-k selection.
//
// Reference: KnnStore (src/gpu_step/knn.rs).  Keys are stored as the
// reference stores them (knn.rs:190-221): per key, d/4 bytes of 2-bit codes u
// packed low bits first, and one f32 scale; the dequantised key is
// k[i] = (u_i - 1.5) * scale (k_dequant, knn.rs:630-643).  A search returns,
// per query, the k best keys by
//   DOT: q.k, largest first, or
//   L2:  |k|^2 - 2 q.k + |q|^2 clamped at 0, smallest first (knn.rs:5,
//        :522-532, :855),
// ties broken by the lower key index.  Two arithmetics:
//   EXACT:  c_i = 2u_i - 3 in {-3,-1,1,3} is exact in f16.  Each query is
//           scaled by a power of two 2^e (max|q| into [2^14, 2^15)) and split
//           into f16 hi + lo parts (~22 significant bits); the tensor core
//           accumulates hi.c + lo.c in f32 and the epilogue multiplies by
//           scale/2.  Error ~2^-22 of sum|q_i||k_i|.
//   F16REF: the reference's numerics: query and dequantised key rounded to
//           f16 (knn.rs:403-411, :630-643), products accumulated in f32.
//
// k_knn_scan is one persistent CTA per SM.  A unit of work is (block of 128
// queries, contiguous key split); a CTA loops over units round-robin, so the
// 32-odd CTAs that share a key split run together and share it through L2.
// Per CTA:
//   warps 5-8 (producers): load the unit's queries (f32 -> f16 hi/lo,
//     128-byte swizzled, K-major) once; then per 256-key tile load the 2-bit
//     codes from HBM and expand them in registers (byte -> prmt selector LUT)
//     into f16 K-major swizzled shared memory, 64 dims per stage; per-key
//     factors (scale/2, |k|^2) go to a small double buffer.
//   warp 4 (one thread): tcgen05.mma kind::f16, M=128 queries x N=256 keys
//     x K=16, accumulating in TMEM; two 256-column accumulators (all 512
//     columns) so the epilogue of tile t overlaps the MMAs of tile t+1.
//   warps 0-3 (epilogue): thread = query = TMEM lane.  tcgen05.ld 32 columns
//     at a time, score = f(dot, key factors), and a running threshold: a key
//     enters the query's candidate buffer (global, 1024 entries) only when it
//     is at least as good as the current 128th best.  A full buffer is cut
//     back to its best 128 by a warp-cooperative exact select (bitwise
//     radix over 64-bit keys); at the end of a unit the best 128 are written
//     out.  Inserts are rare after the first tiles, so the scan runs at the
//     tensor core's pace.
// k_knn_merge then merges the per-split lists of each query (exact: the
// global best k is inside the union of the per-split best k), and
// k_knn_decode turns 64-bit keys back into scores and indices.
//
// A candidate is one 64-bit key: (order-preserving bits of the score << 32)
// | (0xFFFFFFFF - key index), so "larger key" = better score, then lower index.
// Scores inside the kernel are "larger is better" in every mode; L2 uses
// 2 q.k - |k|^2 and adds |q|^2 only when decoding.
#include <cuda_fp16.h>

#include <algorithm>
#include <vector>

#include "st_internal.h"
#include "st_ptx.cuh"

namespace {

constexpr int KQ = 128;          // queries per unit (MMA M = TMEM lanes)
constexpr int KT = 256;          // keys per tile (MMA N)
constexpr int KSTAGES = 2;       // 64-dim key stages in flight
constexpr int KTOP = 128;        // best entries kept per query and unit
constexpr int KCAP = 1024;       // candidate buffer entries per query
constexpr int KMAXD = 256;
constexpr int QCH_BYTES = KQ * 128;  // one 64-dim chunk of 128 queries, f16
constexpr int KCH_BYTES = KT * 128;  // one 64-dim chunk of 256 keys, f16
constexpr int Q_BYTES = 2 * (KMAXD / 64) * QCH_BYTES;  // hi and lo limbs
constexpr int OFF_K = Q_BYTES;
constexpr int OFF_KF = OFF_K + KSTAGES * KCH_BYTES;        // [2][256] f32: scale/2
constexpr int OFF_KN = OFF_KF + 2 * KT * 4;                // [2][256] f32: |k|^2
constexpr int OFF_LUT = OFF_KN + 2 * KT * 4;               // [256] u32 prmt selectors
constexpr int OFF_SLOT = OFF_LUT + 256 * 4;                // [NEPI][16] f32: scores of a step with hits
constexpr int OFF_BAR = OFF_SLOT + 256 * 16 * 4;
constexpr int NBARS = 2 * KSTAGES + 2 + 2 + 2 + 3;        // full, empty, accf, acce, kfr, qfull, qfree, fin
constexpr int OFF_MISC = OFF_BAR + NBARS * 8;              // tmem slot, abort flag
constexpr int KNN_SMEM = OFF_MISC + 16 + 1024;             // + alignment slack
constexpr int NEPI = 256;                                  // epilogue threads: warps 0-7
constexpr int NPROD = 256;                                 // producer threads: warps 8-15, one key row each
constexpr int MMA_WARP = (NEPI + NPROD) / 32;              // warp 16: TMEM owner, MMA issuer
constexpr int KNN_THREADS = NEPI + NPROD + 32;             // 17 warps
constexpr uint32_t TMEM_COLS = 512;

static_assert(KNN_SMEM <= 232448, "kNN scan shared memory exceeds the sm_100 limit");

enum { MODE_DOT = 0, MODE_L2 = 1 };
enum { PREC_EXACT = 0, PREC_F16REF = 1 };

struct ScanArgs {
    const uint8_t *codes;  // [n_keys, d/4]
    const float *scales;   // [n_keys]
    const float *q;        // [nq, d]
    int64_t n_keys;
    int d, nq, nq_pad, nqb, splits;
    int64_t tiles_per_split;
    uint32_t index_base;
    uint64_t *cbuf;      // [gridDim.x * NEPI][KCAP]
    uint64_t *unit_out;  // [splits * 2][nq_pad][KTOP]: one list per (split, column half)
    const int64_t *ranges;  // masked scans: [nq][2] global key range [lo, hi) per query, or null
    int64_t always;         // masked scans: keys below this global index are visible to every query
    // unit-table scans (IVF): unit u scans store rows unit_keys[2u] .. unit_keys[2u + 1] for the queries
    // unit_q[u * KQ + r] (-1: an empty row), writing row r's list to output list unit_list[u * KQ + r];
    // null: the units are (query block, key split)
    const int *unit_q;
    const int *unit_list;
    const int64_t *unit_keys;
    int n_units;
    // [nq] order-preserving bits of the best 128th score any list of the
    // query has reached (0: none yet), shared by every unit of the query
    uint32_t *gthr;
    int *status;
};

__device__ __forceinline__ uint32_t ord_f32(float f) {
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float unord_f32(uint32_t o) {
    return __uint_as_float((o & 0x80000000u) ? (o & 0x7fffffffu) : ~o);
}
// A published threshold's bits back to a score (0: none published).
__device__ __forceinline__ float thr_of(uint32_t v) { return v == 0u ? -INFINITY : unord_f32(v); }
// A candidate key: score bits above (0xffffffff - index), so that equal scores
// rank the lower index first; -0 is stored as +0 (s + 0 = +0 for s = -0), the
// two being one score.
__device__ __forceinline__ uint64_t make_key(float s, uint32_t idx) {
    return (static_cast<uint64_t>(ord_f32(s + 0.0f)) << 32) | static_cast<uint64_t>(0xffffffffu - idx);
}

// Power-of-two exponent e with max|q| * 2^e in [2^14, 2^15) (0 for an all-zero
// query), clamped so that 2^e and 2^(e-1) are normal floats.
__device__ __forceinline__ int query_exp(float maxabs) {
    if (!(maxabs > 0.0f)) return 0;
    const int biased = static_cast<int>((__float_as_uint(maxabs) >> 23) & 0xff);
    const int ex = biased == 0 ? -126 : biased - 126;  // maxabs < 2^ex
    return max(-100, min(100, 15 - ex));
}
__device__ __forceinline__ float pow2f(int e) { return __uint_as_float(static_cast<uint32_t>(e + 127) << 23); }

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Bounded mbarrier wait shared by every role of the scan: gives up after the
// time limit, or at once when another thread of the CTA has given up.
__device__ __forceinline__ bool kwait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status,
                                      int code) {
    if (st::mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = st::globaltimer();
    for (uint32_t i = 1;; ++i) {
        if (st::mbar_try_wait_sleep(bar, parity, 20000u)) return true;
        if ((i & 7u) == 0) {
            if (*abort_flag) return false;
            if (st::globaltimer() - t0 > st::WAIT_LIMIT_NS) {
                *abort_flag = 1;
                st::set_status(status, code);
                return false;
            }
        }
    }
}

// 16 consecutive f32 from shared memory (16-byte aligned address).
__device__ __forceinline__ void lds_f32x16(uint32_t addr, float (&v)[16]) {
#pragma unroll
    for (int i = 0; i < 4; i++)
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(v[4 * i]), "=f"(v[4 * i + 1]), "=f"(v[4 * i + 2]), "=f"(v[4 * i + 3])
                     : "r"(addr + 16 * i));
}

// A threshold T over the warp's 1024 keys (v[i] of lane l is entry i*32+l;
// absent entries are 0 and never counted) with exactly k keys >= T: the
// largest prefix with #{v >= prefix} >= k, found bit by bit from the top and
// stopped as soon as the count is exactly k (keys are distinct, so the full
// 64-bit search ends at the k-th largest key, where the count is k).
__device__ __forceinline__ uint64_t warp_select_threshold(const uint64_t (&v)[32], int k) {
    // the leading bits that every non-zero entry shares are the prefix's: the search
    // starts below them (entries are distinct, so with more than k of them some bit differs)
    uint64_t a = ~0ull, o = 0ull;
#pragma unroll
    for (int i = 0; i < 32; i++)
        if (v[i] != 0ull) {
            a &= v[i];
            o |= v[i];
        }
    const uint64_t all = (static_cast<uint64_t>(__reduce_and_sync(0xffffffffu, static_cast<uint32_t>(a >> 32))) << 32) |
                         __reduce_and_sync(0xffffffffu, static_cast<uint32_t>(a));
    const uint64_t any = (static_cast<uint64_t>(__reduce_or_sync(0xffffffffu, static_cast<uint32_t>(o >> 32))) << 32) |
                         __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(o));
    const uint64_t diff = all ^ any;
    if (diff == 0ull) return all;
    const int top = 63 - __clzll(static_cast<long long>(diff));
    uint64_t prefix = all & ~((2ull << top) - 1ull);
#pragma unroll 1
    for (int bit = top; bit >= 0; --bit) {
        const uint64_t cand = prefix | (1ull << bit);
        unsigned c = 0;
#pragma unroll
        for (int i = 0; i < 32; i++) c += v[i] >= cand ? 1u : 0u;
        c = __reduce_add_sync(0xffffffffu, c);
        if (c >= static_cast<unsigned>(k)) {
            prefix = cand;
            if (c == static_cast<unsigned>(k)) break;
        }
    }
    return prefix;
}

// For every lane of this warp flagged in `need`: load its candidate buffer
// (cnt entries), keep its best KTOP (all, if fewer), and write them either
// back to the buffer front (dst_rows == nullptr) or to the lane's output row.
// Updates the lane's count and threshold.
__device__ void warp_compact(unsigned need, uint64_t *my_buf, int &cnt, float &thr, uint64_t *my_out, bool final) {
    const int lane = threadIdx.x & 31;
    __syncwarp();  // every lane's buffer writes are visible to the others
    while (need) {
        const int L = __ffs(need) - 1;
        need &= need - 1;
        const int n = __shfl_sync(0xffffffffu, cnt, L);
        const uint64_t *src = reinterpret_cast<const uint64_t *>(
            __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(my_buf), L));
        uint64_t *dst = final ? reinterpret_cast<uint64_t *>(
                                    __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(my_out), L))
                              : const_cast<uint64_t *>(src);
        uint64_t v[32];
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const int idx = i * 32 + lane;
            v[i] = idx < n ? __ldcg(src + idx) : 0ull;
        }
        const uint64_t T = n > KTOP ? warp_select_threshold(v, KTOP) : 0ull;
        __syncwarp();
        int base = 0;
        const unsigned lt = (1u << lane) - 1u;
#pragma unroll
        for (int i = 0; i < 32; i++) {
            const bool keep = v[i] != 0ull && v[i] >= T;
            const unsigned m = __ballot_sync(0xffffffffu, keep);
            if (keep) dst[base + __popc(m & lt)] = v[i];
            base += __popc(m);
        }
        if (final)
            for (int p = base + lane; p < KTOP; p += 32) dst[p] = 0ull;
        __syncwarp();
        if (lane == L) {
            cnt = base;
            if (n > KTOP) thr = unord_f32(static_cast<uint32_t>(T >> 32));
        }
    }
}

__device__ __forceinline__ void key_tile_range(const ScanArgs &g, int split, int64_t &k0, int64_t &k1) {
    k0 = static_cast<int64_t>(split) * g.tiles_per_split * KT;
    k1 = min(g.n_keys, k0 + g.tiles_per_split * KT);
}
// A unit's key rows, the query of each of its rows and the list that row writes.
__device__ __forceinline__ void unit_key_range(const ScanArgs &g, int unit, int64_t &k0, int64_t &k1) {
    if (g.unit_q) {
        k0 = g.unit_keys[2 * static_cast<int64_t>(unit)];
        k1 = g.unit_keys[2 * static_cast<int64_t>(unit) + 1];
    } else {
        key_tile_range(g, unit / g.nqb, k0, k1);
    }
}
__device__ __forceinline__ int unit_query(const ScanArgs &g, int unit, int r) {
    return g.unit_q ? g.unit_q[static_cast<int64_t>(unit) * KQ + r] : (unit % g.nqb) * KQ + r;
}
__device__ __forceinline__ int unit_out_list(const ScanArgs &g, int unit, int r) {
    return g.unit_q ? g.unit_list[static_cast<int64_t>(unit) * KQ + r] : unit / g.nqb;
}

// Codes (d/4 bytes, zero-padded to 64) and scale of key `key` when it lies
// below k1; zeros otherwise.
__device__ __forceinline__ void load_key_codes(const ScanArgs &g, int64_t key, int64_t k1, int nchunks, uint4 (&cw)[4],
                                               float &sk) {
    const bool in = key < k1;
    const uint4 *src = reinterpret_cast<const uint4 *>(g.codes + key * (g.d / 4));
#pragma unroll
    for (int j = 0; j < 4; j++) cw[j] = (in && j < nchunks) ? __ldg(src + j) : make_uint4(0u, 0u, 0u, 0u);
    sk = in ? __ldg(g.scales + key) : 0.0f;
}

// Bits of the 16 global key indices [i0, i0 + 16) that lie in [lo, hi).
__device__ __forceinline__ uint32_t range_bits(int64_t i0, int64_t lo, int64_t hi) {
    const int64_t a = lo > i0 ? lo : i0, b = hi < i0 + 16 ? hi : i0 + 16;
    if (a >= b) return 0u;
    const int n = static_cast<int>(b - a), s0 = static_cast<int>(a - i0);
    return (n >= 32 ? 0xffffffffu : ((1u << n) - 1u)) << s0;
}

template <int MODE, int PREC, bool MASKED>
__global__ void __launch_bounds__(KNN_THREADS, 1) k_knn_scan(const ScanArgs g) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *kf = reinterpret_cast<float *>(smem + OFF_KF);
    float *kn = reinterpret_cast<float *>(smem + OFF_KN);
    uint32_t *lut = reinterpret_cast<uint32_t *>(smem + OFF_LUT);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + OFF_BAR);
    uint64_t *full = bars, *empty = bars + KSTAGES, *accf = bars + 2 * KSTAGES, *acce = accf + 2, *kfr = acce + 2;
    uint64_t *qfull = kfr + 2, *qfree = qfull + 1, *fin = qfree + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_MISC + 4);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nchunks = g.d / 64;
    const int units = g.unit_q ? g.n_units : g.nqb * g.splits;

    if (threadIdx.x == 0) {
        for (int s = 0; s < KSTAGES; s++) {
            st::mbar_init(&full[s], NPROD);
            st::mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; b++) {
            st::mbar_init(&accf[b], 1);
            st::mbar_init(&acce[b], NEPI);
            st::mbar_init(&kfr[b], NPROD);
        }
        st::mbar_init(qfull, NPROD);
        st::mbar_init(qfree, 1);
        st::mbar_init(fin, 1);
        *abort_flag = 0;
        st::fence_mbar_init();
    }
    if (warp == MMA_WARP) {
        st::tmem_alloc(tmem_slot, TMEM_COLS);
        st::tmem_relinquish();
    }
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp >= NEPI / 32 && warp < MMA_WARP) {
        // ------------------------------------------------------------ producers
        const int pt = threadIdx.x - NEPI;  // 0..255: key row of every tile
        const int pw = pt >> 5;
        {  // byte of four codes -> two prmt selectors (codes 0,1 | codes 2,3)
            const int x = pt;
            uint32_t sel[2];
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const uint32_t u0 = (x >> (4 * h)) & 3u, u1 = (x >> (4 * h + 2)) & 3u;
                sel[h] = (2u * u0) | ((2u * u0 + 1u) << 4) | ((2u * u1) << 8) | ((2u * u1 + 1u) << 12);
            }
            lut[x] = sel[0] | (sel[1] << 16);
        }
        asm volatile("bar.sync 1, %0;" ::"n"(NPROD) : "memory");
        uint32_t lc = 0, gt = 0, ui = 0;
        bool ok = true;
        for (int unit = blockIdx.x; unit < units && ok; unit += gridDim.x, ++ui) {
            // queries of this unit: row r, lane = 8 dims
            if (ui > 0 && !kwait(qfree, (ui - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) break;
            for (int r = pw; r < KQ; r += NPROD / 32) {
                const int qi = unit_query(g, unit, r);
                float x[8];
                const bool live = qi >= 0 && qi < g.nq && lane * 8 < g.d;
                if (live) {
                    const float4 *src = reinterpret_cast<const float4 *>(g.q + static_cast<int64_t>(qi) * g.d + lane * 8);
                    const float4 a = __ldg(src), b = __ldg(src + 1);
                    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
                    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
                } else {
#pragma unroll
                    for (int i = 0; i < 8; i++) x[i] = 0.0f;
                }
                float m = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; i++) m = fmaxf(m, fabsf(x[i]));
                m = warp_max(m);
                const float sc = PREC == PREC_EXACT ? pow2f(query_exp(m)) : 1.0f;
                uint32_t hi[4], lo[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float a = x[2 * i] * sc, b = x[2 * i + 1] * sc;
                    const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
                    const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
                    hi[i] = static_cast<uint32_t>(__half_as_ushort(ha)) | (static_cast<uint32_t>(__half_as_ushort(hb)) << 16);
                    lo[i] = static_cast<uint32_t>(__half_as_ushort(la)) | (static_cast<uint32_t>(__half_as_ushort(lb)) << 16);
                }
                if (lane * 8 < g.d) {
                    const int j = lane >> 3, c = lane & 7;
                    const uint32_t off = st::sw128_offset(r, c);
                    *reinterpret_cast<uint4 *>(smem + j * QCH_BYTES + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
                    if (PREC == PREC_EXACT)
                        *reinterpret_cast<uint4 *>(smem + (nchunks + j) * QCH_BYTES + off) =
                            make_uint4(lo[0], lo[1], lo[2], lo[3]);
                }
            }
            st::fence_proxy_async_smem();
            st::mbar_arrive(qfull);

            int64_t k0, k1;
            unit_key_range(g, unit, k0, k1);
            uint4 nx_cw[4];
            float nx_sk;
            load_key_codes(g, k0 + pt, k1, nchunks, nx_cw, nx_sk);
            for (int64_t tb = k0; tb < k1 && ok; tb += KT, ++gt) {
                const uint32_t b = gt & 1u, use = gt >> 1;
                // this thread's key (row pt); the next tile's codes are loaded
                // now, so their latency hides behind this tile
                uint4 cw[4];
#pragma unroll
                for (int j = 0; j < 4; j++) cw[j] = nx_cw[j];
                const float sk = nx_sk;
                const bool kin = tb + pt < k1;
                load_key_codes(g, tb + KT + pt, k1, nchunks, nx_cw, nx_sk);
                int c3 = 0;  // codes with |2u-3| = 3: the two bits of u are equal
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const uint32_t w[4] = {cw[j].x, cw[j].y, cw[j].z, cw[j].w};
#pragma unroll
                    for (int t = 0; t < 4; t++) c3 += __popc(~(w[t] ^ (w[t] >> 1)) & 0x55555555u);
                }
                // zero-filled words (absent dims) count as equal bits: take them out
                const int n3 = kin ? c3 - 64 * (4 - nchunks) : 0;
                // value table: f16 of code u at bytes 2u, 2u+1 of {thi:tlo}
                uint32_t tlo, thi;
                if (PREC == PREC_EXACT) {
                    tlo = 0xBC00C200u;  // -1.0 | -3.0
                    thi = 0x42003C00u;  // 3.0 | 1.0
                } else {
                    const uint32_t v0 = __half_as_ushort(__float2half_rn(-1.5f * sk));
                    const uint32_t v1 = __half_as_ushort(__float2half_rn(-0.5f * sk));
                    const uint32_t v2 = __half_as_ushort(__float2half_rn(0.5f * sk));
                    const uint32_t v3 = __half_as_ushort(__float2half_rn(1.5f * sk));
                    tlo = v0 | (v1 << 16);
                    thi = v2 | (v3 << 16);
                }
                for (int j = 0; j < nchunks; j++, ++lc) {
                    const uint32_t s = lc % KSTAGES;
                    if (lc >= KSTAGES &&
                        !kwait(&empty[s], ((lc / KSTAGES) - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    uint8_t *stage = smem + OFF_K + s * KCH_BYTES;
                    uint4 cj = cw[0];
                    if (j == 1) cj = cw[1];
                    if (j == 2) cj = cw[2];
                    if (j == 3) cj = cw[3];
                    const uint32_t w[4] = {cj.x, cj.y, cj.z, cj.w};
#pragma unroll
                    for (int c = 0; c < 8; c++) {
                        const uint32_t half16 = (w[c >> 1] >> (16 * (c & 1))) & 0xffffu;
                        const uint32_t s0 = lut[half16 & 0xffu], s1 = lut[half16 >> 8];
                        uint4 o;
                        o.x = __byte_perm(tlo, thi, s0 & 0xffffu);
                        o.y = __byte_perm(tlo, thi, s0 >> 16);
                        o.z = __byte_perm(tlo, thi, s1 & 0xffffu);
                        o.w = __byte_perm(tlo, thi, s1 >> 16);
                        *reinterpret_cast<uint4 *>(stage + st::sw128_offset(pt, c)) = o;
                    }
                    st::fence_proxy_async_smem();
                    st::mbar_arrive(&full[s]);
                }
                if (!ok) break;
                // per-key factors of this tile, once the epilogue is done with buffer b
                if (use > 0 && !kwait(&acce[b], (use - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_EMPTY)) {
                    ok = false;
                    break;
                }
                float f, nrm;
                if (PREC == PREC_EXACT) {
                    f = 0.5f * sk;
                    nrm = f * f * static_cast<float>(g.d + 8 * n3);
                } else {
                    const float h1 = __half2float(__float2half_rn(0.5f * sk));
                    const float h3 = __half2float(__float2half_rn(1.5f * sk));
                    f = 1.0f;
                    nrm = static_cast<float>(g.d - n3) * (h1 * h1) + static_cast<float>(n3) * (h3 * h3);
                }
                kf[b * KT + pt] = f;
                kn[b * KT + pt] = nrm;
                st::mbar_arrive(&kfr[b]);
            }
        }
    } else if (warp == MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = st::idesc_make(1, 0, false, false, KQ, KT);
            uint32_t lc = 0, gt = 0, ui = 0;
            bool ok = true;
            for (int unit = blockIdx.x; unit < units && ok; unit += gridDim.x, ++ui) {
                if (!kwait(qfull, ui & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) break;
                st::tc_fence_after();
                int64_t k0, k1;
                unit_key_range(g, unit, k0, k1);
                for (int64_t tb = k0; tb < k1 && ok; tb += KT, ++gt) {
                    const uint32_t b = gt & 1u, use = gt >> 1;
                    if (use > 0 && !kwait(&acce[b], (use - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    st::tc_fence_after();
                    const uint32_t acc = tmem + b * KT;
                    for (int j = 0; j < nchunks; j++, ++lc) {
                        const uint32_t s = lc % KSTAGES;
                        if (!kwait(&full[s], (lc / KSTAGES) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) {
                            ok = false;
                            break;
                        }
                        st::tc_fence_after();
                        const uint32_t sb = st::smem_u32(smem + OFF_K + s * KCH_BYTES);
                        const uint32_t sq = st::smem_u32(smem + j * QCH_BYTES);
                        const uint32_t sl = st::smem_u32(smem + (nchunks + j) * QCH_BYTES);
#pragma unroll
                        for (int kk = 0; kk < 4; kk++) {
                            const uint64_t bd = st::sdesc_sw128(sb + kk * 32, 16, 1024);
                            st::umma_f16(acc, st::sdesc_sw128(sq + kk * 32, 16, 1024), bd, idesc,
                                         (j > 0 || kk > 0) ? 1u : 0u);
                            if (PREC == PREC_EXACT) st::umma_f16(acc, st::sdesc_sw128(sl + kk * 32, 16, 1024), bd, idesc, 1u);
                        }
                        st::umma_commit(&empty[s]);
                    }
                    if (!ok) break;
                    st::umma_commit(&accf[b]);
                }
                st::umma_commit(qfree);
            }
            // wait for every MMA issued above before the TMEM is released
            st::umma_commit(fin);
            kwait(fin, 0, abort_flag, g.status, st::DEV_TIMEOUT_ACC);
        }
    } else if (warp < NEPI / 32) {
        // ------------------------------------------------------------ epilogue
        // Warp w reads TMEM lanes 32*(w%4).. (its 32 queries) and owns half
        // w/4 of every tile's columns; each (query, half) keeps its own
        // candidate buffer, threshold and output list.
        const int row = (warp & 3) * 32 + lane;  // TMEM lane = query row within the unit
        const int half = warp >> 2;
        uint64_t *my_buf = g.cbuf + (static_cast<int64_t>(blockIdx.x) * NEPI + threadIdx.x) * KCAP;
        const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
        float *my_slot = reinterpret_cast<float *>(smem + OFF_SLOT) + threadIdx.x * 16;
        uint32_t gt = 0;
        bool ok = true;
        for (int unit = blockIdx.x; unit < units && ok; unit += gridDim.x) {
            const int qi = unit_query(g, unit, row);
            const bool qlive = qi >= 0 && qi < g.nq;
            // search_masked (src/gpu_step/knn.rs:280-291): key j visible iff
            // j < always or lo <= j < hi
            int64_t mlo = 0, mhi = 0;
            if (MASKED && qlive) {
                mlo = g.ranges[2 * static_cast<int64_t>(qi)];
                mhi = g.ranges[2 * static_cast<int64_t>(qi) + 1];
            }
            float qf = 0.0f;  // 2^(e-1): L2's |k|^2 term in the query's scaled units
            if (MODE == MODE_L2 && PREC == PREC_EXACT && qlive) {
                const float4 *src = reinterpret_cast<const float4 *>(g.q + static_cast<int64_t>(qi) * g.d);
                float m = 0.0f;
                for (int i = 0; i < g.d / 4; i++) {
                    const float4 a = __ldg(src + i);
                    m = fmaxf(m, fmaxf(fmaxf(fabsf(a.x), fabsf(a.y)), fmaxf(fabsf(a.z), fabsf(a.w))));
                }
                qf = pow2f(query_exp(m) - 1);
            }
            int cnt = 0;
            float thr = -INFINITY;  // this list's 128th best
            // The 128th best of any list of the query bounds its final 128th
            // best from below, so keys under the best one published cannot
            // place: read one tile ahead of use, published at each compaction.
            float pubd = -INFINITY;
            uint32_t pub = qlive ? __ldcg(g.gthr + qi) : 0u;
            int64_t k0, k1;
            unit_key_range(g, unit, k0, k1);
            for (int64_t tb = k0; tb < k1; tb += KT, ++gt) {
                const uint32_t b = gt & 1u, use = gt >> 1;
                const float teff = fmaxf(thr, thr_of(pub));
                if (qlive) pub = __ldcg(g.gthr + qi);
                if (!kwait(&accf[b], use & 1u, abort_flag, g.status, st::DEV_TIMEOUT_ACC) ||
                    !kwait(&kfr[b], use & 1u, abort_flag, g.status, st::DEV_TIMEOUT_ACC)) {
                    ok = false;
                    break;
                }
                st::tc_fence_after();
                const int col_lo = half * (KT / 2);
                const int ncols = static_cast<int>(k1 - tb < KT ? k1 - tb : KT) - col_lo;  // may be <= 0
                const uint32_t kfb = st::smem_u32(kf + b * KT), knb = st::smem_u32(kn + b * KT);
                // 16 columns at a time: scores into registers, one pass mask,
                // and the (rare) inserts only when this lane has a hit -- no
                // per-key branch on the common path
#pragma unroll 1
                for (int c0 = 0; c0 < ncols && c0 < KT / 2; c0 += 16) {
                    const int col = col_lo + c0;
                    uint32_t r[16];
                    st::tmem_ld16(tmem + lane_base + b * KT + col, r);
                    float f[16], nk[16];
                    if (PREC == PREC_EXACT) lds_f32x16(kfb + 4 * col, f);
                    if (MODE == MODE_L2) lds_f32x16(knb + 4 * col, nk);
                    st::tmem_ld_wait();
                    float sc[16];
                    uint32_t pass = 0;
#pragma unroll
                    for (int jj = 0; jj < 16; jj++) {
                        const float dot = __uint_as_float(r[jj]);
                        if (MODE == MODE_DOT) {
                            sc[jj] = PREC == PREC_EXACT ? dot * f[jj] : dot;
                        } else {
                            sc[jj] = PREC == PREC_EXACT ? fmaf(-nk[jj], qf, dot * f[jj]) : fmaf(2.0f, dot, -nk[jj]);
                        }
                        pass |= (sc[jj] >= teff ? 1u : 0u) << jj;
                    }
                    const int lim = ncols - c0;
                    if (lim < 16) pass &= (1u << lim) - 1u;
                    if (!qlive) pass = 0;
                    if (MASKED) {
                        const int64_t i0 = static_cast<int64_t>(g.index_base) + tb + col;
                        pass &= range_bits(i0, mlo, mhi) | range_bits(i0, 0, g.always);
                    }
                    if (pass) {
                        // stage the 16 scores in this thread's slot, then visit only the hits
                        const uint32_t idx0 = g.index_base + static_cast<uint32_t>(tb) + static_cast<uint32_t>(col);
#pragma unroll
                        for (int i = 0; i < 4; i++)
                            *reinterpret_cast<float4 *>(my_slot + 4 * i) =
                                make_float4(sc[4 * i], sc[4 * i + 1], sc[4 * i + 2], sc[4 * i + 3]);
                        do {
                            const int jj = __ffs(pass) - 1;
                            pass &= pass - 1;
                            my_buf[cnt] = make_key(my_slot[jj], idx0 + static_cast<uint32_t>(jj));
                            cnt++;
                        } while (pass);
                    }
                }
                st::tc_fence_before();
                st::mbar_arrive(&acce[b]);
                const unsigned need = __ballot_sync(0xffffffffu, cnt > KCAP - KT / 2);
                if (need) {
                    warp_compact(need, my_buf, cnt, thr, nullptr, false);
                    if (qlive && thr > pubd) {
                        atomicMax(g.gthr + qi, ord_f32(thr));
                        pubd = thr;
                    }
                }
            }
            if (!ok) break;
            const int list = qlive ? unit_out_list(g, unit, row) : 0;
            uint64_t *my_out = g.unit_out + ((static_cast<int64_t>(list) * 2 + half) * g.nq_pad + (qlive ? qi : 0)) * KTOP;
            const unsigned need = __ballot_sync(0xffffffffu, qlive);
            if (need) warp_compact(need, my_buf, cnt, thr, my_out, true);
            if (qlive && thr > pubd) atomicMax(g.gthr + qi, ord_f32(thr));
        }
    }

    st::tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, TMEM_COLS);
    }
}

// Merge: out[q] = the best KTOP of lists l < n_lists, entries
// lists[l * list_stride + q * KTOP + r], sorted best first (0 = empty).
// One 256-thread CTA per query: an exact 8-bit-digit radix select of the
// KTOP-th largest key, a gather of the keys at or above it, a rank sort.
// With gridDim.y = G > 1, block (q, y) merges only lists y * ceil(n/G) .. and
// writes its best KTOP to out[(y * gridDim.x + q) * KTOP]: the first stage of a
// two-stage merge whose second stage merges those G lists.
__global__ void __launch_bounds__(256) k_knn_merge(const uint64_t *lists, int64_t n_lists, int64_t list_stride,
                                                   uint64_t *out) {
    __shared__ int hist[256];
    __shared__ uint64_t sel[KTOP];
    __shared__ int s_digit, s_need, s_count;
    const int64_t q = blockIdx.x;
    if (gridDim.y > 1) {
        const int64_t per = (n_lists + gridDim.y - 1) / gridDim.y;
        const int64_t l0 = blockIdx.y * per;
        n_lists = l0 < n_lists ? (n_lists - l0 < per ? n_lists - l0 : per) : 0;
        lists += l0 * list_stride;
        out += static_cast<int64_t>(blockIdx.y) * gridDim.x * KTOP;
    }
    const int64_t total = n_lists * KTOP;
    auto at = [&](int64_t i) { return __ldg(lists + (i / KTOP) * list_stride + q * KTOP + (i % KTOP)); };
    uint64_t prefix = 0, mask = 0;
    int need = KTOP;
    bool all = false;
    for (int pass = 7; pass >= 0; --pass) {
        for (int i = threadIdx.x; i < 256; i += blockDim.x) hist[i] = 0;
        __syncthreads();
        for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
            const uint64_t v = at(i);
            if (v != 0ull && (v & mask) == prefix) atomicAdd(&hist[(v >> (8 * pass)) & 0xff], 1);
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int acc = 0, d = -1;
            for (int b = 255; b >= 0; --b) {
                if (acc + hist[b] >= need) {
                    d = b;
                    break;
                }
                acc += hist[b];
            }
            s_digit = d;
            s_need = d >= 0 ? need - acc : need;
        }
        __syncthreads();
        if (s_digit < 0) {  // fewer than `need` candidates left: keep every nonzero key at or above the prefix
            all = true;
            break;
        }
        prefix |= static_cast<uint64_t>(s_digit) << (8 * pass);
        mask |= 0xffull << (8 * pass);
        need = s_need;
        __syncthreads();
    }
    // T: the KTOP-th largest (or, with fewer candidates, the smallest admissible prefix)
    const uint64_t T = all ? (prefix == 0 ? 1ull : prefix) : prefix;
    if (threadIdx.x == 0) s_count = 0;
    for (int i = threadIdx.x; i < KTOP; i += blockDim.x) sel[i] = 0ull;
    __syncthreads();
    for (int64_t i = threadIdx.x; i < total; i += blockDim.x) {
        const uint64_t v = at(i);
        if (v != 0ull && v >= T) {
            const int p = atomicAdd(&s_count, 1);
            if (p < KTOP) sel[p] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x < KTOP) {
        const uint64_t v = sel[threadIdx.x];
        int rank = 0;
        for (int j = 0; j < KTOP; j++) rank += sel[j] > v ? 1 : 0;
        // zeros all have the same rank; place them after the real keys
        if (v == 0ull) {
            int zeros_before = 0;
            for (int j = 0; j < threadIdx.x; j++) zeros_before += sel[j] == 0ull ? 1 : 0;
            rank += zeros_before;
        }
        out[q * KTOP + rank] = v;
    }
}

// The same merge with every candidate of the block's query in registers (at
// most 256 MR of them): the 8-bit digit passes start at the first byte where
// the candidates differ, count into a shared histogram that one warp scans in
// parallel, and read no global memory after the first load.
constexpr int MR = 32;  // candidates per thread: 64 lists of 128
__global__ void __launch_bounds__(256) k_knn_merge_reg(const uint64_t *lists, int64_t n_lists, int64_t list_stride,
                                                       uint64_t *out) {
    __shared__ int hist[256];
    __shared__ uint64_t sel[KTOP];
    __shared__ uint32_t red[2][8][2];
    __shared__ int s_digit, s_need, s_count;
    const int64_t q = blockIdx.x;
    if (gridDim.y > 1) {
        const int64_t per = (n_lists + gridDim.y - 1) / gridDim.y;
        const int64_t l0 = blockIdx.y * per;
        n_lists = l0 < n_lists ? (n_lists - l0 < per ? n_lists - l0 : per) : 0;
        lists += l0 * list_stride;
        out += static_cast<int64_t>(blockIdx.y) * gridDim.x * KTOP;
    }
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int total = static_cast<int>(n_lists) * KTOP;
    uint64_t v[MR];
    uint64_t a = ~0ull, o = 0ull;
#pragma unroll
    for (int r = 0; r < MR; r++) {
        const int i = r * 256 + tid;
        v[r] = i < total ? __ldg(lists + (i / KTOP) * list_stride + q * KTOP + (i % KTOP)) : 0ull;
        if (v[r] != 0ull) {
            a &= v[r];
            o |= v[r];
        }
    }
    // the bits every nonzero candidate shares
    uint32_t r0 = __reduce_and_sync(0xffffffffu, static_cast<uint32_t>(a)),
             r1 = __reduce_and_sync(0xffffffffu, static_cast<uint32_t>(a >> 32));
    uint32_t r2 = __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(o)),
             r3 = __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(o >> 32));
    if (lane == 0) {
        red[0][wid][0] = r0;
        red[0][wid][1] = r1;
        red[1][wid][0] = r2;
        red[1][wid][1] = r3;
    }
    int cnt = 0;
#pragma unroll
    for (int r = 0; r < MR; r++) cnt += v[r] != 0ull ? 1 : 0;
    cnt = __reduce_add_sync(0xffffffffu, cnt);
    if (tid == 0) s_count = 0;
    __syncthreads();
    if (lane == 0) atomicAdd(&s_count, cnt);
    uint64_t all = ~0ull, any = 0ull;
#pragma unroll
    for (int w = 0; w < 8; w++) {
        all &= (static_cast<uint64_t>(red[0][w][1]) << 32) | red[0][w][0];
        any |= (static_cast<uint64_t>(red[1][w][1]) << 32) | red[1][w][0];
    }
    __syncthreads();
    const int n_nonzero = s_count;
    __syncthreads();  // every thread has read the count before it is reused
    uint64_t T;
    if (n_nonzero <= KTOP) {
        T = 1ull;  // every nonzero candidate
    } else {
        const uint64_t diff = all ^ any;  // nonzero: the candidates are distinct
        const int top_byte = (63 - __clzll(static_cast<long long>(diff))) >> 3;
        uint64_t mask = top_byte == 7 ? 0ull : ~0ull << (8 * (top_byte + 1));
        uint64_t prefix = all & mask;
        int need = KTOP;
        for (int pass = top_byte; pass >= 0; --pass) {
            hist[tid] = 0;
            __syncthreads();
#pragma unroll
            for (int r = 0; r < MR; r++)
                if (v[r] != 0ull && (v[r] & mask) == prefix) atomicAdd(&hist[(v[r] >> (8 * pass)) & 0xff], 1);
            __syncthreads();
            if (wid == 0) {
                // lane l holds bins 255 - 8l .. 248 - 8l; counts at or above each bin, top down
                int c[8], s8 = 0;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    c[j] = hist[255 - 8 * lane - j];
                    s8 += c[j];
                }
                int incl = s8;  // inclusive prefix over lanes (higher bins first)
#pragma unroll
                for (int off = 1; off < 32; off <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, incl, off);
                    if (lane >= off) incl += t;
                }
                int acc = incl - s8;  // candidates in bins above this lane's
                int d = -1, left = 0;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (d < 0 && acc + c[j] >= need) {
                        d = 255 - 8 * lane - j;
                        left = need - acc;
                    }
                    acc += c[j];
                }
                const unsigned has = __ballot_sync(0xffffffffu, d >= 0);
                const int src = __ffs(has) - 1;  // the highest bin reaching `need` is in the first such lane
                if (lane == src) {
                    s_digit = d;
                    s_need = left;
                }
            }
            __syncthreads();
            prefix |= static_cast<uint64_t>(s_digit) << (8 * pass);
            mask |= 0xffull << (8 * pass);
            need = s_need;
            __syncthreads();
        }
        T = prefix;
    }
    if (tid == 0) s_count = 0;
    if (tid < KTOP) sel[tid] = 0ull;
    __syncthreads();
#pragma unroll
    for (int r = 0; r < MR; r++) {
        if (v[r] != 0ull && v[r] >= T) {
            const int p = atomicAdd(&s_count, 1);
            if (p < KTOP) sel[p] = v[r];
        }
    }
    __syncthreads();
    if (tid < KTOP) {
        const uint64_t x = sel[tid];
        int rank = 0;
        for (int j = 0; j < KTOP; j++) rank += sel[j] > x ? 1 : 0;
        if (x == 0ull) {
            int zeros_before = 0;
            for (int j = 0; j < tid; j++) zeros_before += sel[j] == 0ull ? 1 : 0;
            rank += zeros_before;
        }
        out[q * KTOP + rank] = x;
    }
}

// Keys -> (score, index).  DOT: q.k (EXACT divides out the query's 2^e);
// L2: |q|^2 - (2 q.k - |k|^2), clamped at 0.  Empty slots: (-inf | +inf, -1).
template <int MODE, int PREC>
__global__ void __launch_bounds__(128) k_knn_decode(const uint64_t *keys, const float *qs, int d, int k,
                                                    float *out_scores, int64_t *out_ids) {
    const int64_t q = blockIdx.x;
    __shared__ float s_qn, s_inv;
    if (threadIdx.x < 32) {
        const float *src = qs + q * d;
        float m = 0.0f, ss = 0.0f;
        for (int i = threadIdx.x; i < d; i += 32) {
            m = fmaxf(m, fabsf(src[i]));
            ss = fmaf(src[i], src[i], ss);
        }
        m = warp_max(m);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (threadIdx.x == 0) {
            const int e = PREC == PREC_EXACT ? query_exp(m) : 0;
            s_inv = MODE == MODE_DOT ? pow2f(-e) : pow2f(1 - e);
            s_qn = ss;
        }
    }
    __syncthreads();
    for (int r = threadIdx.x; r < k; r += blockDim.x) {
        const uint64_t key = keys[q * KTOP + r];
        float sc;
        int64_t id;
        if (key == 0ull) {
            sc = MODE == MODE_DOT ? -INFINITY : INFINITY;
            id = -1;
        } else {
            id = static_cast<int64_t>(0xffffffffu - static_cast<uint32_t>(key & 0xffffffffu));
            const float s = unord_f32(static_cast<uint32_t>(key >> 32));
            if (MODE == MODE_DOT) {
                sc = PREC == PREC_EXACT ? s * s_inv : s;
            } else {
                const float t = PREC == PREC_EXACT ? s * s_inv : s;
                sc = fmaxf(0.0f, s_qn - t);
            }
        }
        out_scores[q * k + r] = sc;
        out_ids[q * k + r] = id;
    }
}

// tile_of's 2-bit quantiser (knn.rs:190-221, quant_step :647-653), one thread
// per key, in the reference's f32 operation order: scale =
// max(0.9957 * sqrt(sum(x*x) / d), 1e-30); u = clamp(round(x/scale + 1.5), 0, 3)
// with round half away from zero; norm = sum of f16((u - 1.5) * scale)^2.
__global__ void k_knn_quantize(const float *keys, int64_t n, int d, uint8_t *codes, float *scales, float *norms) {
    for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < n;
         r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float *x = keys + r * d;
        float ss = 0.0f;
        for (int i = 0; i < d; i++) ss = __fadd_rn(ss, __fmul_rn(x[i], x[i]));
        float scale = __fmul_rn(0.9957f, __fsqrt_rn(__fdiv_rn(ss, static_cast<float>(d))));
        if (!(scale >= 1e-30f)) scale = 1e-30f;
        float nrm = 0.0f;
        uint8_t *row = codes + r * (d / 4);
        for (int i0 = 0; i0 < d; i0 += 4) {
            uint32_t byte = 0;
            for (int t = 0; t < 4; t++) {
                float u = roundf(__fadd_rn(__fdiv_rn(x[i0 + t], scale), 1.5f));
                u = fminf(fmaxf(u, 0.0f), 3.0f);
                byte |= static_cast<uint32_t>(u) << (2 * t);
                const float h = __half2float(__float2half_rn(__fmul_rn(__fsub_rn(u, 1.5f), scale)));
                nrm = __fadd_rn(nrm, __fmul_rn(h, h));
            }
            row[i0 / 4] = static_cast<uint8_t>(byte);
        }
        scales[r] = scale;
        if (norms) norms[r] = nrm;
    }
}

// Synthetic keys for the benchmark and tests: codes uniform over 0..3 and
// scale = |N(0,1)|, both from a counter-based hash of (seed, key), so any
// shard can make its keys without the others.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}
__global__ void k_knn_synth(uint8_t *codes, float *scales, int64_t n, int d, uint64_t seed, int64_t first) {
    const int words = d / 32;  // 8-byte words of codes per key
    for (int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; r < n;
         r += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint64_t key = static_cast<uint64_t>(first + r);
        const uint64_t base = mix64(seed ^ mix64(key));
        uint64_t *dst = reinterpret_cast<uint64_t *>(codes + r * (d / 4));
        for (int w = 0; w < words; w++) dst[w] = mix64(base + 1 + w);
        const uint64_t h = mix64(base ^ 0x5bd1e995ull);
        const float u1 = fmaxf(static_cast<float>((h >> 40) & 0xffffff) * (1.0f / 16777216.0f), 1e-9f);
        const float u2 = static_cast<float>((h >> 16) & 0xffffff) * (1.0f / 16777216.0f);
        scales[r] = fabsf(sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2));
    }
}

template <int MODE, int PREC, bool MASKED>
st_status launch_scan(st_handle *h, const ScanArgs &g, int grid) {
    auto kern = k_knn_scan<MODE, PREC, MASKED>;
    static bool attr_done = false;
    if (!attr_done) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, KNN_SMEM));
        attr_done = true;
    }
    kern<<<grid, KNN_THREADS, KNN_SMEM, h->stream>>>(g);
    return st_after_launch(h, "k_knn_scan");
}

template <int MODE, int PREC>
st_status launch_decode(st_handle *h, const uint64_t *keys, const float *q, int64_t nq, int d, int k, float *scores,
                        int64_t *ids) {
    k_knn_decode<MODE, PREC><<<static_cast<unsigned>(nq), 128, 0, h->stream>>>(keys, q, d, k, scores, ids);
    return st_after_launch(h, "k_knn_decode");
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

st_status check_common(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_keys, int32_t dim,
                       const float *queries, int64_t nq, int32_t mode, int32_t prec, int64_t index_base,
                       const char *who) {
    if (!codes || !scales || !queries) return h->fail(ST_INVALID_ARG, "%s: null buffer", who);
    if (dim < 64 || dim > KMAXD || dim % 64 != 0)
        return h->fail(ST_UNSUPPORTED_SHAPE, "%s: dim must be 64, 128, 192 or 256 (got %d)", who, dim);
    if (n_keys < 1 || nq < 1 || nq > (1 << 24)) return h->fail(ST_INVALID_ARG, "%s: bad n_keys / nq", who);
    if (index_base < 0 || index_base + n_keys >= 0xffffffffll)
        return h->fail(ST_UNSUPPORTED_SHAPE, "%s: key indices must stay below 2^32 - 1", who);
    if ((mode != 0 && mode != 1) || (prec != 0 && prec != 1)) return h->fail(ST_INVALID_ARG, "%s: bad mode/prec", who);
    if (!aligned16(codes) || !aligned16(queries))
        return h->fail(ST_INVALID_ARG, "%s: codes and queries must be 16-byte aligned", who);
    return ST_OK;
}

// ---- IVF building blocks (src/gpu_step/knn/ivf.rs) -------------------------

// out[r, j] = (u_j - 1.5) * scale_r: the 2-bit rows as f32 (k_dequant, knn.rs:630-643, without the f16 rounding).
__global__ void k_knn_dequant(const uint8_t *codes, const float *scales, int64_t n, int d, float *out) {
    const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;  // one code byte
    const int64_t nb = n * (d / 4);
    if (e >= nb) return;
    const int64_t r = e / (d / 4);
    const uint32_t byte = codes[e];
    const float sc = scales[r];
    float4 v;
    v.x = (static_cast<float>(byte & 3u) - 1.5f) * sc;
    v.y = (static_cast<float>((byte >> 2) & 3u) - 1.5f) * sc;
    v.z = (static_cast<float>((byte >> 4) & 3u) - 1.5f) * sc;
    v.w = (static_cast<float>((byte >> 6) & 3u) - 1.5f) * sc;
    reinterpret_cast<float4 *>(out)[e] = v;
}

// Nearest cell of each row from dots = rows . centroids^T: argmin over c of
// cnorm[c] - 2 dots[r, c], the lowest c among equals (k_argmin, ivf.rs:75-113).
// One warp per row.
__global__ void k_knn_nearest(const float *dots, const float *cnorm, int64_t n, int nl, int32_t *out) {
    const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= n) return;
    const float *row = dots + r * nl;
    float best = INFINITY;
    int bi = 0x7fffffff;
    for (int c = lane; c < nl; c += 32) {
        const float v = fmaf(-2.0f, row[c], cnorm[c]);
        if (v < best) {  // lanes visit their columns in increasing order: the first minimum is kept
            best = v;
            bi = c;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov < best || (ov == best && oi < bi)) {
            best = ov;
            bi = oi;
        }
    }
    if (lane == 0) out[r] = bi;
}

// Each query's nprobe nearest cells, nearest first, ties to the lower cell
// (k_probe, ivf.rs:126-165): nprobe rounds of a warp minimum over the entries
// after the last one taken in (distance, cell) order.
__global__ void k_knn_probe(const float *dots, const float *cnorm, int64_t nq, int nl, int nprobe, int32_t *out) {
    const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= nq) return;
    const float *row = dots + r * nl;
    float last = -INFINITY;
    int lasti = -1;
    for (int p = 0; p < nprobe; p++) {
        float best = INFINITY;
        int bi = 0x7fffffff;
        for (int c = lane; c < nl; c += 32) {
            const float v = fmaf(-2.0f, row[c], cnorm[c]);
            const bool after = v > last || (v == last && c > lasti);
            if (after && (v < best || (v == best && c < bi))) {
                best = v;
                bi = c;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov < best || (ov == best && oi < bi)) {
                best = ov;
                bi = oi;
            }
        }
        if (lane == 0) out[r * nprobe + p] = bi < nl ? bi : -1;
        last = best;
        lasti = bi;
    }
}

// (v, c) before (w, d) in (distance, cell) order.
__device__ __forceinline__ bool probe_less(float v, int c, float w, int d) { return v < w || (v == w && c < d); }

// k_knn_probe for nprobe <= PMAX in one pass over the row: each lane keeps
// its PMAX best (distance, cell) pairs sorted in registers, then nprobe
// rounds of a warp minimum over the lanes' heads take them in order.  Same
// results as k_knn_probe (the order is total: distance, then cell).
template <int PMAX>
__global__ void k_knn_probe_small(const float *dots, const float *cnorm, int64_t nq, int nl, int nprobe, int32_t *out) {
    const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= nq) return;
    const float *row = dots + r * nl;
    float lv[PMAX];
    int li[PMAX];
#pragma unroll
    for (int k = 0; k < PMAX; k++) lv[k] = INFINITY, li[k] = 0x7fffffff;
    for (int c = lane; c < nl; c += 32) {
        const float v = fmaf(-2.0f, row[c], cnorm[c]);
        if (probe_less(v, c, lv[PMAX - 1], li[PMAX - 1])) {
            lv[PMAX - 1] = v, li[PMAX - 1] = c;
#pragma unroll
            for (int k = PMAX - 1; k > 0; k--)
                if (probe_less(lv[k], li[k], lv[k - 1], li[k - 1])) {
                    const float tv = lv[k];
                    const int ti = li[k];
                    lv[k] = lv[k - 1], li[k] = li[k - 1], lv[k - 1] = tv, li[k - 1] = ti;
                }
        }
    }
    for (int p = 0; p < nprobe; p++) {
        float best = lv[0];
        int bi = li[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (probe_less(ov, oi, best, bi)) best = ov, bi = oi;
        }
        if (lane == 0) out[r * nprobe + p] = bi < nl ? bi : -1;
        if (li[0] == bi) {  // the lane holding the winner moves to its next
#pragma unroll
            for (int k = 0; k < PMAX - 1; k++) lv[k] = lv[k + 1], li[k] = li[k + 1];
            lv[PMAX - 1] = INFINITY, li[PMAX - 1] = 0x7fffffff;
        }
    }
}

// dst row i = src row perm[i]; rows of `words` 32-bit words.  A perm entry
// outside [0, n_src) yields a zero row and a DEV_BAD_ARG status.
__global__ void k_gather_rows(const uint32_t *src, int64_t n_src, uint32_t *dst, const int64_t *perm, int64_t n,
                              int words, int *status) {
    const int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (e >= n * words) return;
    const int64_t i = e / words;
    const int w = static_cast<int>(e % words);
    const int64_t j = perm[i];
    if (j < 0 || j >= n_src) {
        dst[e] = 0u;
        if (w == 0) st::set_status(status, st::DEV_BAD_ARG);
        return;
    }
    dst[e] = src[j * words + w];
}


// ---- the narrow scan: at most 32 queries per pass --------------------------
//
// With a handful of queries the scan above runs at its 128-query cost.  On the
// tensor core an M = 128 MMA costs at least ~50 cycles whatever N is (the A
// operand, 4 KB, is read for every instruction), so few queries only pay if
// each instruction does more work per key: k_knn_narrow puts 128 keys on the
// M side, in tensor memory, as one byte per dimension (u = 0..3), and runs
// kind::i8 (K = 32 per instruction, 8 instructions per 128-key tile) against
// the queries as NL signed-byte limbs of a fixed-point integer X_i =
// round(q_i 2^(e + 8 NL - 17)) (max |X| < 2^(8 NL - 2)), limb l of query q in
// B row l * NQP + q.  The products and sums are exact integers:
//   A_l = sum_i u_i limb_l,i     and     S = sum_l 2^8l (A_l - C_l) = sum_i (u_i - 1.5) X_i,
// with C_l = 1.5 sum_i limb_l,i, so the only rounding is the query's to 8 NL - 2
// bits (EXACT: NL = 4; F16REF: NL = 3, still finer than the reference's f16).
// Roles (576 threads, one CTA per SM, one key split per CTA):
//   warp 17 (one thread): bulk-copies each 128-key tile's codes (8 KB) and the
//     16-byte blocks holding its scales into a 12-stage shared-memory ring.
//   warps 8-15 (producers; warp w writes TMEM lanes 32 (w % 4) + 16 (w / 12)..):
//     spread the codes into bytes -- (word >> 2s) & 0x03030303 puts codes s,
//     s + 4, s + 8, s + 12 of a 16-code word into one 32-bit word -- and store
//     them with tcgen05.st (16x256b: a warp's 512 contiguous code bytes map onto
//     16 TMEM lanes without shuffles); the queries' K order follows that
//     permutation of the dimensions.
//   warp 16 (one thread): tcgen05.mma kind::i8, A = keys (u8, TMEM), B = limbs
//     (s8, shared memory), D = s32, N = NL * NQP columns; two accumulators.
//   warps 0-7 (epilogue; warp w reads TMEM lanes 32 (w % 4).. and the columns
//     of queries 16 (w / 4)..): thread = key.  A limb column plus 0x4B400000,
//     viewed as a float, is 1.5 2^23 + A_l exactly (|A_l| < 2^17); the accumulator
//     goes back to the MMA as soon as its last column is read; the two top limbs
//     bound S within +-R (R from the per-query sums of |limb|), and one FMA,
//     one FMA and a compare per (key, query) test the key against the query's
//     running 128th-best score with every term lowered -- never rejecting a
//     key whose exact score passes.  Keys that pass take the exact S from all
//     limbs and go into the candidate buffer of (warp, query), owned by lane q
//     of the warp.  The 128th-best scores are shared: each warp publishes its
//     own through a global atomicMax per query and filters against the best
//     any warp of any CTA has published (a key below another list's 128th
//     best cannot be in the final top 128), so after the first tiles keys
//     rarely reach the exact path.
// Scores come out in the wide scan's units, so k_knn_merge and k_knn_decode
// are shared.
constexpr int NQ = 32;                                  // queries per group (one accumulator's columns)
constexpr int NK = 128;                                 // keys per tile (MMA M, TMEM lanes)
constexpr int N_CODE_BYTES = NK * 64;                   // dim 256: 64 code bytes per key
constexpr int N_STAGE_BYTES = N_CODE_BYTES + NK * 4 + 16;  // scales from the 16-byte block of the first
constexpr int N_A = 2;                                  // TMEM A buffers, 64 columns each
constexpr int N_ACC = 3;                                // TMEM accumulators, 128 columns each
constexpr int N_ACC_COLS = 128;
constexpr int N_KF = 8;                                 // per-key factor slots (lifetime: see the producer)
constexpr int N_QUAD = 4;                               // TMEM lane quadrants: one candidate list per query each
constexpr int N_EPI = 8, N_PROD = 8;                    // epilogue warp w: quadrant w % 4, queries 16 (w / 4) ..
constexpr int EQ = NQ / 2;                              // queries per epilogue warp and group
constexpr int N_MMA_WARP = N_EPI + N_PROD;              // 16
constexpr int N_TMA_WARP = N_MMA_WARP + 1;              // 17
constexpr int N_THREADS = 32 * (N_TMA_WARP + 1);        // 576
constexpr int NQ_CHUNK = 128 * 128;                     // one K chunk of a group's B: 128 rows x 128 B, SW128
constexpr uint32_t N_TMEM_COLS = 512;
constexpr uint32_t N_ACC_COL = N_A * 64;                   // accumulators after the A buffers
constexpr int MAGIC_I = 0x4B400000;                        // float 1.5 * 2^23
constexpr float MAGIC_F = 12582912.0f;
static_assert(N_ACC_COL + N_ACC * N_ACC_COLS <= N_TMEM_COLS, "keys-on-M kNN scan TMEM budget");

// Shared-memory layout of the keys-on-M scan with NG groups of 32 queries
// resident per unit (the library launches NG = 1, the narrow pass).
template <int NG>
struct NarrowSmem {
    static constexpr int QB = NQ * NG;                       // queries per unit
    static constexpr int STAGES = NG == 1 ? 12 : 6;          // code / scale ring
    static constexpr int O_Q = 0;                            // NG x [2 K chunks][128 rows x 128 B]
    static constexpr int O_RING = O_Q + NG * 2 * NQ_CHUNK;
    static constexpr int O_KF = O_RING + STAGES * N_STAGE_BYTES;  // [N_KF][128] scale
    static constexpr int O_KN = O_KF + N_KF * NK * 4;             // [N_KF][128] |k|^2 (L2)
    static constexpr int O_QC = O_KN + N_KF * NK * 4;             // [2 units][8][QB] per-query constants
    static constexpr int O_THR = O_QC + 2 * 8 * QB * 4;           // [2][4 quadrants][QB] thresholds
    static constexpr int O_SLOT = O_THR + 2 * N_QUAD * QB * 4;    // [16 queries][256 threads] exact scores
    static constexpr int O_BAR = O_SLOT + EQ * N_EPI * 32 * 4;
    // rfull, rempty [STAGES]; afull, aempty [N_A]; accf, acce [N_ACC]; kfr [N_KF];
    // qready [2]; edone [2]; qfree; fin
    static constexpr int NBARS = 2 * STAGES + 2 * N_A + 2 * N_ACC + N_KF + 2 + 2 + 1 + 1;
    static constexpr int O_MISC = O_BAR + NBARS * 8;              // tmem slot, abort flag
    static constexpr int SMEM = O_MISC + 16 + 1024;
    static_assert(SMEM <= 232448, "keys-on-M kNN scan shared memory exceeds the sm_100 limit");
    static_assert(O_RING % 1024 == 0 && N_STAGE_BYTES % 16 == 0, "keys-on-M kNN scan alignment");
};

struct NarrowArgs {
    const uint8_t *codes;  // [n_keys, 64], 16-byte aligned
    const float *scales;   // [n_keys], 4-byte aligned
    const float *q;        // [nq, 256]
    int64_t n_keys;
    int nq, nqp;           // nqp: queries per limb block of a group's B (16 or 32)
    int nqb, units;        // query blocks of QB queries; units = nqb * splits, unit u = (split u / nqb, block u % nqb)
    int nq_pad;            // nqb * QB: rows of unit_out's lists and of gthr
    // split s scans 128-key tiles s * unit_step + i * tile_step, i < tiles_per_unit, below n_tiles
    int64_t n_tiles, unit_step, tile_step, tiles_per_unit;
    uint32_t index_base;
    uint64_t *cbuf;        // [gridDim.x][4 quadrants][QB queries][KCAP]
    uint64_t *unit_out;    // [splits * 4][nq_pad][KTOP]: list (split, quadrant) of every query
    uint32_t *gthr;        // [nq_pad] order-preserving bits of the best published 128th score (0: none)
    int exact;             // k_knn_tmem: 1 = exact scores (the full pass), 0 = lower bounds (a sample pass)
    // k_knn_tmem: the pass's (query block, sample) sequence, block-major, seg_len samples per block
    // (sample j = tile j * unit_step), flat_len = nqb * seg_len, cut into gridDim.x equal ranges;
    // nslot lists per (query, quadrant) in unit_out
    int64_t flat_len, seg_len;
    int nslot;
    int aligned;           // k_knn_tmem: 1 = CTA c takes part c / nqb of query block c % nqb (see tm_next)
    int *status;
};

// Dimension (0..255) held by byte k of the keys-on-M scan's A rows.
__device__ __forceinline__ int narrow_dim(int k) {
    const int col = k >> 2, p = k & 3;
    const int r = col >> 3, c = (col >> 1) & 3, b = col & 1;
    const int m = r >> 1, s = 2 * (r & 1) + b;
    return 16 * (4 * c + m) + 4 * p + s;
}

// x lowered by 2^-12 of its magnitude (-inf and +inf unchanged).
__device__ __forceinline__ float lowered(float x) { return x - fabsf(x) * 0.000244140625f; }

__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Stores 16 TMEM lanes x 64 columns (16x256b, 8 repetitions): repetition j,
// thread t: r[4j], r[4j+1] -> lane t/4, columns 8j + 2(t%4) + {0,1};
// r[4j+2], r[4j+3] -> lane 8 + t/4, the same columns.
__device__ __forceinline__ void tmem_st_16x256b_x8(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.16x256b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void umma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}


// kwait for the keys-on-M scan's hand-offs, which come every few hundred
// nanoseconds: try_wait without a sleep hint (the hardware parks the thread
// until the phase completes, so waiting warps take no issue slots from the
// working ones, and wakes it at once), still bounded by the time limit and
// the CTA's abort flag.
__device__ __forceinline__ bool nwait(uint64_t *bar, uint32_t parity, volatile int *abort_flag, int *status,
                                      int code) {
    if (st::mbar_try_wait(bar, parity)) return true;
    // the bound counts SM cycles (the SM's own counter, cheap to read):
    // 8e9 cycles is at least the 2 s limit at any clock up to 4 GHz
    const long long t0 = clock64();
    for (uint32_t i = 1;; ++i) {
        if (st::mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0) {
            if (*abort_flag) return false;
            if (clock64() - t0 > 8000000000ll) {
                *abort_flag = 1;
                st::set_status(status, code);
                return false;
            }
        }
    }
}


// Tile i of unit `unit`: its first key tb and key count nk; false past the unit's end.
__device__ __forceinline__ bool narrow_tile(const NarrowArgs &g, int unit, int64_t i, int64_t &tb, int &nk) {
    if (i >= g.tiles_per_unit) return false;
    const int64_t t = static_cast<int64_t>(unit / g.nqb) * g.unit_step + i * g.tile_step;
    if (t >= g.n_tiles) return false;
    tb = t * NK;
    nk = static_cast<int>(g.n_keys - tb < NK ? g.n_keys - tb : NK);
    return true;
}

// k_knn_tmem's work split.  With at most one query block per SM (g.aligned),
// the grid is nqb P CTAs and CTA c scans part c / nqb (of P equal parts) of
// query block c % nqb, writing its lists to slot c / nqb.  Otherwise CTA c
// takes the flat range [c L / G, (c + 1) L / G) of the pass's (query block,
// sample) sequence (L = g.flat_len, G = gridDim.x, block-major, g.seg_len
// samples per block), so every CTA has the same number of tiles and crosses at
// most a few block boundaries; a piece is the part of the range inside one
// query block, and the CTAs that cover block b write their lists to slots
// 0, 1, .. in range order (slot = c - the CTA holding b's first sample).
struct TPiece {
    int64_t pos, end;  // the CTA's remaining flat range
    int64_t j0, j1;    // the piece's samples of block qb
    int qb, slot;
};
__device__ __forceinline__ int64_t tm_seg_start(const NarrowArgs &g, int64_t c) {
    return c * g.flat_len / gridDim.x;
}
__device__ __forceinline__ void tm_begin(const NarrowArgs &g, TPiece &p) {
    p.pos = g.aligned ? 0 : tm_seg_start(g, blockIdx.x);
    p.end = g.aligned ? 1 : tm_seg_start(g, blockIdx.x + 1);
}
__device__ __forceinline__ bool tm_next(const NarrowArgs &g, TPiece &p) {
    if (p.pos >= p.end) return false;
    if (g.aligned) {
        // gridDim.x = nqb P: the CTAs of part k of every query block scan the same tiles
        // at the same time, so each tile comes from DRAM about once and from L2 for the
        // other blocks
        const int parts = gridDim.x / g.nqb, part = blockIdx.x / g.nqb;
        p.pos = 1;
        p.qb = blockIdx.x % g.nqb;
        p.j0 = part * g.seg_len / parts;
        p.j1 = (part + 1) * g.seg_len / parts;
        p.slot = part;
        return p.j1 > p.j0;
    }
    const int64_t qb = p.pos / g.seg_len;
    p.qb = static_cast<int>(qb);
    p.j0 = p.pos - qb * g.seg_len;
    p.j1 = min(g.seg_len, p.j0 + (p.end - p.pos));
    p.pos += p.j1 - p.j0;
    // the last CTA c0 with c0 L / G <= x (x = the block's first flat index): c0 = ceil((x + 1) G / L) - 1
    const int64_t x = qb * g.seg_len;
    const int64_t c0 = ((x + 1) * gridDim.x + g.flat_len - 1) / g.flat_len - 1;
    p.slot = static_cast<int>(blockIdx.x - c0);
    return true;
}
// Tile i of piece p: sample j0 + i is tile (j0 + i) * unit_step.
__device__ __forceinline__ bool tm_tile(const NarrowArgs &g, const TPiece &p, int64_t i, int64_t &tb, int &nk) {
    const int64_t j = p.j0 + i;
    if (j >= p.j1) return false;
    tb = j * g.unit_step * NK;
    nk = static_cast<int>(g.n_keys - tb < NK ? g.n_keys - tb : NK);
    return true;
}

// The keys-on-M 2-bit scan.  Unit u = (key split u / nqb, query block u % nqb)
// scans its split's 128-key tiles against the block's QB = 32 NG queries,
// which stay resident in shared memory as int8 limbs for the whole unit: each
// key tile is loaded and expanded into TMEM once and meets NG groups of 32
// queries, one accumulator each (8 MMAs of K = 32 per group).  The library
// launches NG = 1 (the narrow pass, <= 32 queries); a unit's thresholds start
// from the best 128th score any list of the query has published.
template <int MODE, int PREC, int NG>
__global__ void __launch_bounds__(N_THREADS, 1) k_knn_narrow(const NarrowArgs g) {
    using L = NarrowSmem<NG>;
    constexpr int QB = L::QB;
    constexpr int STAGES = L::STAGES;
    constexpr int NL = PREC == PREC_EXACT ? 4 : 3;   // query limbs
    constexpr int EB = 8 * NL - 17;                  // X = round(2^(e + EB) q)
    constexpr float SH = NL == 4 ? 1.52587890625e-05f : 0.00390625f;  // 2^-8 (NL - 2)
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *kf = reinterpret_cast<float *>(smem + L::O_KF);
    float *kn = reinterpret_cast<float *>(smem + L::O_KN);
    float *thr_s = reinterpret_cast<float *>(smem + L::O_THR);  // [4][QB] effective 128th-best score
    float *thr_l = thr_s + N_QUAD * QB;                         // [4][QB] the same / P * SH, lowered
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L::O_BAR);
    uint64_t *rfull = bars, *rempty = bars + STAGES, *afull = bars + 2 * STAGES, *aempty = afull + N_A;
    uint64_t *accf = aempty + N_A, *acce = accf + N_ACC, *kfr = acce + N_ACC, *qready = kfr + N_KF;
    uint64_t *edone = qready + 2, *qfree = edone + 2, *fin = qfree + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L::O_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + L::O_MISC + 4);
    // the per-query constants of the CTA's unit j live in buffer j % 2: [8][QB] floats
    float *qconst0 = reinterpret_cast<float *>(smem + L::O_QC);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nqp = g.nqp;
    if (threadIdx.x == 0) {
        // one arrival per warp: a warp's lanes meet at __syncwarp and lane 0 arrives
        for (int s = 0; s < STAGES; s++) {
            st::mbar_init(&rfull[s], 1);
            st::mbar_init(&rempty[s], N_PROD);
        }
        for (int b = 0; b < N_A; b++) {
            st::mbar_init(&afull[b], N_PROD);
            st::mbar_init(&aempty[b], 1);
        }
        for (int a = 0; a < N_ACC; a++) {
            st::mbar_init(&accf[a], 1);
            st::mbar_init(&acce[a], nqp > EQ ? N_EPI : N_EPI / 2);  // the warps that have queries
        }
        for (int k = 0; k < N_KF; k++) st::mbar_init(&kfr[k], N_PROD);
        for (int j = 0; j < 2; j++) {
            st::mbar_init(&qready[j], N_PROD);
            st::mbar_init(&edone[j], N_EPI);
        }
        st::mbar_init(qfree, 1);
        st::mbar_init(fin, 1);
        *abort_flag = 0;
        st::fence_mbar_init();
    }
    if (warp == N_MMA_WARP) {
        st::tmem_alloc(tmem_slot, N_TMEM_COLS);
        st::tmem_relinquish();
    }
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == N_TMA_WARP) {
        // ------------------------------------------------------------ code / scale loader
        if (lane == 0) {
            uint32_t gt = 0;
            bool ok = true;
            for (int unit = blockIdx.x; unit < g.units && ok; unit += gridDim.x) {
                int64_t tb;
                int nk;
                for (int64_t i = 0; narrow_tile(g, unit, i, tb, nk); ++i, ++gt) {
                    const uint32_t s = gt % STAGES;
                    if (gt >= STAGES &&
                        !nwait(&rempty[s], ((gt / STAGES) - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    // the scales go as the 16-byte blocks that hold them: a bulk copy
                    // starts and ends on 16-byte boundaries, and those blocks lie
                    // inside the scales' allocation
                    const uintptr_t s0 = reinterpret_cast<uintptr_t>(g.scales + tb) & ~uintptr_t(15);
                    const uintptr_t s1 = (reinterpret_cast<uintptr_t>(g.scales + tb + nk) + 15) & ~uintptr_t(15);
                    const uint32_t cb = static_cast<uint32_t>(nk) * 64u, sb = static_cast<uint32_t>(s1 - s0);
                    uint8_t *dst = smem + L::O_RING + s * N_STAGE_BYTES;
                    st::mbar_arrive_expect_tx(&rfull[s], cb + sb);
                    st::bulk_load(dst, g.codes + tb * 64, cb, &rfull[s]);
                    st::bulk_load(dst + N_CODE_BYTES, reinterpret_cast<const void *>(s0), sb, &rfull[s]);
                }
            }
            // copies still in flight land before the CTA's shared memory goes away
            const uint32_t first = gt > STAGES ? gt - STAGES : 0;
            for (uint32_t i = first; i < gt; i++)
                st::mbar_wait(&rfull[i % STAGES], (i / STAGES) & 1u, g.status, st::DEV_TIMEOUT_FULL);
        }
    } else if (warp >= N_EPI && warp < N_MMA_WARP) {
        // ------------------------------------------------------------ producers
        const int pw = warp - N_EPI;  // 0..7: TMEM lanes 32 (warp % 4) + 16 (pw / 4) ..
        const int quad = warp & 3, half = pw >> 2;
        uint32_t gt = 0, uj = 0;
        bool ok = true;
        for (int unit = blockIdx.x; unit < g.units && ok; unit += gridDim.x, ++uj) {
            // the unit's queries: the limbs overwrite the previous unit's, so the
            // MMAs of that unit must be done; the constants go to buffer uj % 2,
            // which the epilogue of unit uj - 2 must be done with
            if (uj >= 1 && !nwait(qfree, (uj - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_ACC)) break;
            if (uj >= 2 && !nwait(&edone[uj & 1u], ((uj - 2) >> 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_ACC))
                break;
            float *qc = qconst0 + (uj & 1u) * 8 * QB;
            float *qc_c = qc, *qc_ql = qc + QB, *qc_P = qc + 2 * QB, *qc_qf = qc + 3 * QB, *qc_C = qc + 4 * QB;
            const int qbase = (unit % g.nqb) * QB;
            // warp pw prepares queries pw, pw + 8, ..; lane l writes bytes
            // 8l .. 8l + 7 of every limb row (K chunk l / 16) of its group
            for (int r = pw; r < QB; r += N_PROD) {
                const int qg = qbase + r, grp = r / NQ, rr = r % NQ;
                const bool live = qg < g.nq;
                const float *qrow = g.q + static_cast<int64_t>(live ? qg : 0) * 256;
                float m = 0.0f;
                for (int i = lane; i < 256; i += 32) m = fmaxf(m, live ? fabsf(__ldg(qrow + i)) : 0.0f);
                m = warp_max(m);
                const int e = query_exp(m);
                const float sc = pow2f(e + EB);  // |X| < 2^(8 NL - 2)
                uint32_t lw[NL][2];
                int lsum[NL], labs[NL];
#pragma unroll
                for (int l = 0; l < NL; l++) {
                    lw[l][0] = lw[l][1] = 0u;
                    lsum[l] = labs[l] = 0;
                }
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int dim = narrow_dim(8 * lane + i);
                    int x = __float2int_rn((live ? __ldg(qrow + dim) : 0.0f) * sc);
#pragma unroll
                    for (int l = 0; l < NL; l++) {
                        int limb;
                        if (l < NL - 1) {
                            limb = ((x + 128) & 255) - 128;  // balanced digit in [-128, 127]
                            x = (x - limb) >> 8;
                        } else {
                            limb = x;  // |top limb| <= 64
                        }
                        lw[l][i >> 2] |= (static_cast<uint32_t>(limb) & 255u) << (8 * (i & 3));
                        lsum[l] += limb;
                        labs[l] += abs(limb);
                    }
                }
#pragma unroll
                for (int l = 0; l < NL; l++) {
                    lsum[l] = warp_sum(lsum[l]);
                    labs[l] = warp_sum(labs[l]);
                    if (rr < nqp) {
                        const int row = l * nqp + rr;
                        const uint32_t off = grp * 2 * NQ_CHUNK + (lane >> 4) * NQ_CHUNK +
                                             st::sw128_offset(row, (lane & 15) >> 1) + 8 * (lane & 1);
                        *reinterpret_cast<uint2 *>(smem + L::O_Q + off) = make_uint2(lw[l][0], lw[l][1]);
                    }
                }
                if (lane == 0) {
                    // S = sum_l 2^8l (A_l - C_l);  v = 2^8 (1.5 2^23 + A_top) + 1.5 2^23 + A_next
                    // (rounded by at most 128) and S <= 2^(8 (NL - 2)) (v - K) + R
                    float K = 257.0f * MAGIC_F, R = 0.0f;
                    for (int l = 0; l < NL; l++) {
                        const float C = 1.5f * static_cast<float>(lsum[l]);
                        qc_C[l * QB + r] = C;
                        if (l == NL - 1) K += 256.0f * C;
                        else if (l == NL - 2) K += C;
                        else R += 1.5f * static_cast<float>(labs[l]) * pow2f(8 * l);
                    }
                    float P, qf;
                    if (MODE == MODE_DOT) {
                        P = PREC == PREC_EXACT ? pow2f(-EB) : pow2f(-e - EB);
                        qf = 0.0f;
                    } else {
                        P = PREC == PREC_EXACT ? pow2f(-EB) : pow2f(1 - e - EB);
                        qf = PREC == PREC_EXACT ? pow2f(e - 1) : 1.0f;
                    }
                    // v and the filter's right-hand side round by at most 128 each, and
                    // K (about 3.2e9) by at most 256
                    qc_c[r] = live ? K - R * SH - 768.0f : INFINITY;
                    qc_ql[r] = lowered(qf / P * SH);
                    qc_P[r] = P;
                    qc_qf[r] = qf;
                }
            }
            st::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) st::mbar_arrive(&qready[uj & 1u]);

            int64_t tb;
            int nk;
            for (int64_t i = 0; narrow_tile(g, unit, i, tb, nk); ++i, ++gt) {
                const uint32_t s = gt % STAGES, b = gt % N_A, f = gt % N_KF;
                if (!nwait(&rfull[s], (gt / STAGES) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) {
                    ok = false;
                    break;
                }
                const uint8_t *stage = smem + L::O_RING + s * N_STAGE_BYTES;
                const int sofs = static_cast<int>((reinterpret_cast<uintptr_t>(g.scales + tb) & 15u) >> 2);
                uint4 cw[2];
                int key[2];
                float scl[2], nrm[2];
#pragma unroll
                for (int jj = 0; jj < 2; jj++) {
                    const int j = 2 * half + jj;
                    key[jj] = 32 * quad + 8 * j + (lane >> 2);
                    const bool in = key[jj] < nk;
                    cw[jj] = in ? *reinterpret_cast<const uint4 *>(stage + 2048 * quad + 512 * j + 16 * lane)
                                : make_uint4(0u, 0u, 0u, 0u);
                    scl[jj] = in ? reinterpret_cast<const float *>(stage + N_CODE_BYTES)[sofs + key[jj]] : 0.0f;
                    int c3 = 0;  // codes u in {0, 3}: the two bits are equal
                    if (MODE == MODE_L2) {
                        const uint32_t w[4] = {cw[jj].x, cw[jj].y, cw[jj].z, cw[jj].w};
#pragma unroll
                        for (int t = 0; t < 4; t++) c3 += __popc(~(w[t] ^ (w[t] >> 1)) & 0x55555555u);
                        c3 += __shfl_xor_sync(0xffffffffu, c3, 1);
                        c3 += __shfl_xor_sync(0xffffffffu, c3, 2);
                    }
                    if (PREC == PREC_EXACT) {
                        nrm[jj] = scl[jj] * scl[jj] * static_cast<float>(64 + 2 * c3);
                    } else {
                        const float h1 = __half2float(__float2half_rn(0.5f * scl[jj]));
                        const float h3 = __half2float(__float2half_rn(1.5f * scl[jj]));
                        nrm[jj] = static_cast<float>(256 - c3) * (h1 * h1) + static_cast<float>(c3) * (h3 * h3);
                    }
                }
                __syncwarp();
                if (lane == 0) st::mbar_arrive(&rempty[s]);  // the stage's bytes are in registers
                // A buffer b is free once the MMAs of tile gt - 2 are done.  Slot
                // f = gt % 8 is then free too: those MMAs started only after the
                // epilogue released the accumulator of step (gt - 2) NG + NG - 4,
                // so it is done with every tile up to gt - 5 (NG = 1) or gt - 3
                // (NG = 4), and slot f last held tile gt - 8.
                if (gt >= N_A &&
                    !nwait(&aempty[b], ((gt / N_A) - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_EMPTY)) {
                    ok = false;
                    break;
                }
                if ((lane & 3) == 0) {
#pragma unroll
                    for (int jj = 0; jj < 2; jj++) {
                        kf[f * NK + key[jj]] = scl[jj];
                        kn[f * NK + key[jj]] = nrm[jj];
                    }
                }
                __syncwarp();
                if (lane == 0) st::mbar_arrive(&kfr[f]);
                // codes -> bytes: register 4r + {0,1} belongs to key j = 2 half
                // (lane base + lane / 4), 4r + {2,3} to key j + 1 (lane base + 8 + lane / 4)
                uint32_t v[32];
#pragma unroll
                for (int jj = 0; jj < 2; jj++) {
                    const uint32_t w[4] = {cw[jj].x, cw[jj].y, cw[jj].z, cw[jj].w};
#pragma unroll
                    for (int m = 0; m < 4; m++)
#pragma unroll
                        for (int s2 = 0; s2 < 4; s2++)
                            v[4 * (2 * m + (s2 >> 1)) + 2 * jj + (s2 & 1)] = (w[m] >> (2 * s2)) & 0x03030303u;
                }
                const uint32_t taddr = tmem + (static_cast<uint32_t>(32 * quad + 16 * half) << 16) + b * 64u;
                tmem_st_16x256b_x8(taddr, v);
                st::tmem_st_wait();
                st::tc_fence_before();
                __syncwarp();
                if (lane == 0) st::mbar_arrive(&afull[b]);
            }
        }
    } else if (warp == N_MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            // kind::i8: D s32, A unsigned 8-bit, B signed 8-bit, M = 128
            const uint32_t idesc = (2u << 4) | (0u << 7) | (1u << 10) | (static_cast<uint32_t>(NL * nqp >> 3) << 17) |
                                   (static_cast<uint32_t>(NK >> 4) << 24);
            const uint32_t qbuf = st::smem_u32(smem + L::O_Q);
            uint32_t gt = 0, gs = 0, uj = 0;  // tiles, (tile, group) steps, units so far
            bool ok = true;
            for (int unit = blockIdx.x; unit < g.units && ok; unit += gridDim.x, ++uj) {
                if (!nwait(&qready[uj & 1u], (uj >> 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) break;
                st::tc_fence_after();
                int64_t tb;
                int nk;
                for (int64_t i = 0; narrow_tile(g, unit, i, tb, nk); ++i, ++gt) {
                    const uint32_t b = gt % N_A;
                    if (!nwait(&afull[b], (gt / N_A) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    st::tc_fence_after();
                    const uint32_t abuf = tmem + b * 64u;
#pragma unroll 1
                    for (int grp = 0; grp < NG; grp++, gs++) {
                        const uint32_t a = gs % N_ACC;
                        if (gs >= N_ACC &&
                            !nwait(&acce[a], ((gs / N_ACC) - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        st::tc_fence_after();
                        const uint32_t acc = tmem + N_ACC_COL + a * N_ACC_COLS;
                        const uint32_t gq = qbuf + grp * 2 * NQ_CHUNK;
#pragma unroll
                        for (int kk = 0; kk < 8; kk++)
                            umma_i8_ts(acc, abuf + 8 * kk,
                                       st::sdesc_sw128(gq + (kk >> 2) * NQ_CHUNK + (kk & 3) * 32, 16, 1024), idesc,
                                       kk > 0 ? 1u : 0u);
                        st::umma_commit(&accf[a]);
                    }
                    if (!ok) break;
                    st::umma_commit(&aempty[b]);
                }
                // the unit's MMAs are done with its queries once this arrives
                st::umma_commit(qfree);
            }
            // every MMA issued above completes before the TMEM is released
            st::umma_commit(fin);
            nwait(fin, 0, abort_flag, g.status, st::DEV_TIMEOUT_ACC);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        // Warp w reads TMEM lanes 32 (w % 4) .. (keys 32 (w % 4) + lane of every
        // tile) and, in every group, the columns of queries q0 = 16 (w / 4) ..
        // q0 + 15; lane l < 16 owns the candidate buffer, count and thresholds
        // of query 32 grp + q0 + l of its quadrant.
        const int quad = warp & 3, q0 = EQ * (warp >> 2);
        const unsigned lt = (1u << lane) - 1u;
        const uint32_t lane_addr = static_cast<uint32_t>(32 * quad) << 16;
        uint64_t *bufs = g.cbuf + (static_cast<int64_t>(blockIdx.x) * N_QUAD + quad) * QB * KCAP;
        float *slot = reinterpret_cast<float *>(smem + L::O_SLOT) + threadIdx.x;  // slot[i * 256]: query q0 + i
        float *wthr = thr_s + quad * QB, *wthrl = thr_l + quad * QB;
        const uint32_t acc0 = tmem + lane_addr + N_ACC_COL;
        const bool has_q = q0 < nqp;  // with 16 queries per limb block the second warp of each quadrant has none
        const int top = (NL - 1) * nqp + q0, next = (NL - 2) * nqp + q0;
        uint32_t gt = 0, gs = 0, uj = 0;
        bool ok = true;
        for (int unit = blockIdx.x; unit < g.units && ok; unit += gridDim.x, ++uj) {
            // every epilogue warp (even one without queries) waits for the unit's
            // queries, so no warp's edone arrival runs two units ahead
            if (!nwait(&qready[uj & 1u], (uj >> 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) break;
            const float *qc = qconst0 + (uj & 1u) * 8 * QB;
            const float *qc_c = qc, *qc_ql = qc + QB, *qc_P = qc + 2 * QB, *qc_qf = qc + 3 * QB, *qc_C = qc + 4 * QB;
            const int qbase = (unit % g.nqb) * QB;
            int cnt[NG];
            float thr[NG], eff[NG];          // this list's 128th best; the best 128th any list has published
            uint32_t pub[NG], pub_next[NG];  // published thresholds, read one tile ahead of use
            bool qlive[NG];
#pragma unroll
            for (int grp = 0; grp < NG; grp++) {
                const int qu = NQ * grp + q0 + lane;  // this lane's query in the unit
                qlive[grp] = has_q && lane < EQ && qbase + qu < g.nq;
                cnt[grp] = 0;
                thr[grp] = qlive[grp] ? -INFINITY : INFINITY;
                // a unit starts from the best 128th score any list of the query has
                // published (the sample passes' seeds, and earlier units'), not from -inf
                eff[grp] = qlive[grp] ? thr_of(__ldcg(g.gthr + qbase + qu)) : INFINITY;
                pub[grp] = pub_next[grp] = 0u;
                if (has_q && lane < EQ) {
                    wthr[qu] = eff[grp];
                    wthrl[qu] = qlive[grp] ? lowered(eff[grp] / qc_P[qu] * SH) : eff[grp];
                }
            }
            __syncwarp();
            int64_t tb;
            int nk;
            for (int64_t i = 0; has_q && narrow_tile(g, unit, i, tb, nk); ++i, ++gt) {
                const uint32_t f = gt % N_KF;
                if (!nwait(&kfr[f], (gt / N_KF) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_ACC)) {
                    ok = false;
                    break;
                }
                const int kk = 32 * quad + lane;
                const float scale = kf[f * NK + kk];
                const float nrm = kn[f * NK + kk];
                const bool klive = kk < nk;
                // a scale that is not a positive finite number turns the filter's
                // inequality around or into NaN: such a key takes the exact path for
                // every query
                const bool keep_all = !(scale > 0.0f && scale < INFINITY);
                const float inv_s = rcp_approx(scale);
                const uint32_t idx = g.index_base + static_cast<uint32_t>(tb) + static_cast<uint32_t>(kk);
#pragma unroll
                for (int grp = 0; grp < NG; grp++, gs++) {
                    const uint32_t a = gs % N_ACC;
                    const int qo = NQ * grp + q0;  // this warp's first query of the group, in the unit
                    uint64_t *gbuf = bufs + static_cast<int64_t>(qo) * KCAP;
                    uint64_t *my_buf = gbuf + static_cast<int64_t>(lane & (EQ - 1)) * KCAP;
                    // the published thresholds: read now, merged after the next tile (the
                    // read's latency stays off this tile's path)
                    pub[grp] = pub_next[grp];
                    pub_next[grp] = 0u;
                    if (qlive[grp] && (i & 15) == 15) pub_next[grp] = __ldcg(g.gthr + qbase + qo + lane);
                    if (!nwait(&accf[a], (gs / N_ACC) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_ACC)) {
                        ok = false;
                        break;
                    }
                    st::tc_fence_after();
                    const uint32_t acc = acc0 + a * N_ACC_COLS;
                    uint32_t rt[EQ], rn[EQ];
                    st::tmem_ld16(acc + top, rt);
                    st::tmem_ld16(acc + next, rn);
                    st::tmem_ld_wait();
                    bool any = false;
#pragma unroll
                    for (int q4 = 0; q4 < EQ; q4 += 4) {
                        const float4 cc = *reinterpret_cast<const float4 *>(qc_c + qo + q4);
                        const float4 th = *reinterpret_cast<const float4 *>(wthrl + qo + q4);
                        const float ca[4] = {cc.x, cc.y, cc.z, cc.w}, tha[4] = {th.x, th.y, th.z, th.w};
                        float qla[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                        if (MODE == MODE_L2) {
                            const float4 ql = *reinterpret_cast<const float4 *>(qc_ql + qo + q4);
                            qla[0] = ql.x; qla[1] = ql.y; qla[2] = ql.z; qla[3] = ql.w;
                        }
#pragma unroll
                        for (int i2 = 0; i2 < 4; i2++) {
                            const float v = fmaf(__uint_as_float(rt[q4 + i2] + MAGIC_I), 256.0f,
                                                 __uint_as_float(rn[q4 + i2] + MAGIC_I));
                            const float t = MODE == MODE_L2 ? fmaf(nrm, qla[i2], tha[i2]) : tha[i2];
                            any |= v >= fmaf(t, inv_s, ca[i2]);
                        }
                    }
                    any = klive && (any || keep_all);
                    const bool slow = __any_sync(0xffffffffu, any);
                    if (!slow) {  // nothing more to read: the accumulator goes back to the MMA now
                        st::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) st::mbar_arrive(&acce[a]);
                    }
                    if (slow) {
                        // the exact path: S = sum_l 2^8l (A_l - C_l) from every limb, top
                        // down, the partial sums kept in this thread's score slots
                        float *sl = slot;
                        if (any) {
#pragma unroll
                            for (int i2 = 0; i2 < EQ; i2++)
                                sl[i2 * (N_EPI * 32)] =
                                    fmaf(__uint_as_float(rt[i2] + MAGIC_I) - MAGIC_F - qc_C[(NL - 1) * QB + qo + i2],
                                         256.0f,
                                         __uint_as_float(rn[i2] + MAGIC_I) - MAGIC_F - qc_C[(NL - 2) * QB + qo + i2]);
                        }
#pragma unroll 1
                        for (int l = NL - 3; l >= 0; l--) {
                            st::tmem_ld16(acc + l * nqp + q0, rt);
                            st::tmem_ld_wait();
                            if (any) {
#pragma unroll
                                for (int i2 = 0; i2 < EQ; i2++)
                                    sl[i2 * (N_EPI * 32)] =
                                        fmaf(sl[i2 * (N_EPI * 32)], 256.0f,
                                             __uint_as_float(rt[i2] + MAGIC_I) - MAGIC_F - qc_C[l * QB + qo + i2]);
                            }
                        }
                        st::tc_fence_before();  // every limb is read: release the accumulator
                        __syncwarp();
                        if (lane == 0) st::mbar_arrive(&acce[a]);
                        uint32_t pass = 0;
                        if (any) {
#pragma unroll
                            for (int i2 = 0; i2 < EQ; i2++) {
                                float sc = sl[i2 * (N_EPI * 32)] * scale * qc_P[qo + i2];
                                if (MODE == MODE_L2) sc = fmaf(-nrm, qc_qf[qo + i2], sc);
                                sl[i2 * (N_EPI * 32)] = sc;
                                pass |= (sc >= wthr[qo + i2] ? 1u : 0u) << i2;
                            }
                        }
                        unsigned qm = __reduce_or_sync(0xffffffffu, pass);
                        while (qm) {
                            const int i2 = __ffs(qm) - 1;
                            qm &= qm - 1;
                            const bool p = (pass >> i2) & 1u;
                            const unsigned m = __ballot_sync(0xffffffffu, p);
                            const int base = __shfl_sync(0xffffffffu, cnt[grp], i2);
                            if (p)
                                gbuf[static_cast<int64_t>(i2) * KCAP + base + __popc(m & lt)] =
                                    make_key(slot[i2 * (N_EPI * 32)], idx);
                            if (lane == i2) cnt[grp] += __popc(m);
                        }
                    }
                    const unsigned need = __ballot_sync(0xffffffffu, cnt[grp] > KCAP - NK / 4);
                    if (need) {
                        const float before = thr[grp];
                        warp_compact(need, my_buf, cnt[grp], thr[grp], nullptr, false);
                        if (thr[grp] > before) atomicMax(g.gthr + qbase + qo + lane, ord_f32(thr[grp]));
                    }
                    const float ne = fmaxf(fmaxf(thr[grp], thr_of(pub[grp])), eff[grp]);
                    if (__any_sync(0xffffffffu, ne > eff[grp])) {
                        if (qlive[grp]) {
                            eff[grp] = ne;
                            wthr[qo + lane] = ne;
                            wthrl[qo + lane] = lowered(ne / qc_P[qo + lane] * SH);
                        }
                        __syncwarp();
                    }
                }
                if (!ok) break;
            }
            if (!ok) break;
            if (has_q) {
                const int split = unit / g.nqb;
#pragma unroll
                for (int grp = 0; grp < NG; grp++) {
                    const int qo = NQ * grp + q0;
                    uint64_t *my_buf = bufs + static_cast<int64_t>(qo + (lane & (EQ - 1))) * KCAP;
                    uint64_t *my_out = g.unit_out + ((static_cast<int64_t>(split) * N_QUAD + quad) * g.nq_pad +
                                                     qbase + qo + (lane & (EQ - 1))) * KTOP;
                    const unsigned need = __ballot_sync(0xffffffffu, qlive[grp]);
                    warp_compact(need, my_buf, cnt[grp], thr[grp], my_out, true);
                }
            }
            // this unit's constants may be overwritten now
            __syncwarp();
            if (lane == 0) st::mbar_arrive(&edone[uj & 1u]);
        }
    }

    st::tc_fence_before();
    __syncthreads();
    if (warp == N_MMA_WARP) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, N_TMEM_COLS);
    }
}

// gthr[q] = the score bits of the 128th best key of keys[q] (0 when the list
// holds fewer): a lower bound for query q's final 128th best, since the keys
// behind it are a subset of the keys scanned.
__global__ void k_knn_seed(const uint64_t *keys, int nq, uint32_t *gthr) {
    const int q = blockIdx.x * blockDim.x + threadIdx.x;
    if (q < nq) gthr[q] = static_cast<uint32_t>(keys[static_cast<int64_t>(q) * KTOP + KTOP - 1] >> 32);
}

// Best KTOP per query over n_lists lists (stride list_stride) into out, in two
// stages when the lists are many: G groups in parallel into tmp [G][nq][KTOP],
// then one merge of the G partial lists.
st_status merge_lists(st_handle *h, const uint64_t *lists, int64_t n_lists, int64_t list_stride, int64_t nq,
                      uint64_t *tmp, int groups, uint64_t *out) {
    constexpr int64_t REG_LISTS = 256 * MR / KTOP;  // lists one k_knn_merge_reg block holds
    if (n_lists > REG_LISTS && tmp && n_lists <= groups * REG_LISTS) {
        // groups of at most REG_LISTS lists, then one merge of the groups
        const int64_t gr = (n_lists + REG_LISTS - 1) / REG_LISTS;
        k_knn_merge_reg<<<dim3(static_cast<unsigned>(nq), static_cast<unsigned>(gr)), 256, 0, h->stream>>>(
            lists, n_lists, list_stride, tmp);
        st_status s = st_after_launch(h, "k_knn_merge_reg");
        if (s != ST_OK) return s;
        lists = tmp;
        n_lists = gr;
        list_stride = nq * KTOP;
    }
    if (n_lists <= REG_LISTS) {
        k_knn_merge_reg<<<static_cast<unsigned>(nq), 256, 0, h->stream>>>(lists, n_lists, list_stride, out);
        return st_after_launch(h, "k_knn_merge_reg");
    }
    if (n_lists > 2 * groups && tmp) {
        k_knn_merge<<<dim3(static_cast<unsigned>(nq), static_cast<unsigned>(groups)), 256, 0, h->stream>>>(
            lists, n_lists, list_stride, tmp);
        st_status s = st_after_launch(h, "k_knn_merge");
        if (s != ST_OK) return s;
        lists = tmp;
        n_lists = groups;
        list_stride = nq * KTOP;
    }
    k_knn_merge<<<static_cast<unsigned>(nq), 256, 0, h->stream>>>(lists, n_lists, list_stride, out);
    return st_after_launch(h, "k_knn_merge");
}

template <int MODE, int PREC, int NG>
st_status launch_narrow(st_handle *h, const NarrowArgs &g, int grid) {
    auto kern = k_knn_narrow<MODE, PREC, NG>;
    static bool attr_done = false;
    if (!attr_done) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              NarrowSmem<NG>::SMEM));
        attr_done = true;
    }
    kern<<<grid, N_THREADS, NarrowSmem<NG>::SMEM, h->stream>>>(g);
    return st_after_launch(h, "k_knn_narrow");
}


// ---- the wide scan with keys in tensor memory (k_knn_tmem) -----------------
//
// For more than 32 EXACT dot-product queries at dim 256.  A unit is (key
// split, block of TQ = 256 queries).  The block's queries stay in shared
// memory for the whole unit as hi = f16(q 2^e), 2^e chosen per query (max |q|
// 2^e in [2^14, 2^15), so hi neither overflows nor flushes).  Each 128-key
// tile is expanded once into TMEM -- code u of a key with scale s to the f16
// value v = f16((u - 1.5) s) -- where it is the A operand (M = 128 keys) of
// one tcgen05 kind::f16 pass per 128-query step (N = 128, K = 256 in 16
// MMAs): every expanded key meets all 256 queries, and shared memory carries
// only the queries' B tiles.
//
// A 17th MMA per step (both operands in shared memory, K = 16) adds each
// pair's filter terms: the key's filter row holds (1024, s16), the query's
// (w, +-E16), so the accumulator ends at acc' = sum hi v + 1024 w +- s16 E16.
//   s16 = |s| rounded up to f16.
//   E16 = E rounded up, E = (1.5 sum |q 2^e - hi| + 2^-9 sum |hi|) (1 + 2^-10)
//         + 2^-24: the query's rounding, the rounding of v (2^-11 relative) and
//         an f32 accumulation error of up to 2^-12 of the terms' magnitudes.
//   w   = -T' / 1024 rounded up to f16, T' = T - 2^-10 |T| - 2^-22 sum |hi|
//         - 2^-30 for the query's running 128th-best score T.
// A pair whose exact score s sum (u - 1.5) q 2^e reaches T then has acc' >=
// 0, so the full pass keeps only pairs whose accumulator is not negative -- a
// test of sign bits, by AND over 16 columns at a time.  Thresholds rise
// during the scan: the epilogue rewrites w in shared memory, and an MMA that
// still reads an older (smaller) threshold only keeps more pairs.  A key with
// |s| < 2^-13 is expanded as zeros with s16 = |s| 1024 rounded up (v would
// leave the normal f16 range; the bound then covers the whole dropped
// product); a key with |s| >= 2^14 or a non-finite scale as zeros with s16 =
// +inf, so that all its pairs are kept.
//
// A kept pair's exact score -- s sum (u_i - 1.5) q_i 2^e in f64 from the
// key's codes and the f32 query, rounded once, computed by the whole warp --
// decides its entry in the candidate buffer of (query, TMEM lane quadrant),
// as in k_knn_narrow.  The sample passes (every 1024th, then every 16th tile)
// stage w = 0 and -E16 instead: acc' is then a lower bound of the pair's
// exact score, and a pair whose acc' reaches its list's threshold enters the
// list as that bound lowered by 2^-12, so a list's 128th best bounds the
// final one from below and seeds the full pass.  Scores come out in the wide
// scan's units (q.k 2^e), so k_knn_merge and k_knn_decode are shared.
//
// Roles (448 threads, one CTA per SM, up to 128 registers a thread): warp 13
// bulk-copies each tile's codes and scales into a 6-stage ring; warps 8-11
// expand codes into TMEM (thread = key = TMEM lane, 32x32b stores; v through
// a byte permute of the key's four-entry table, eight values per code word
// from four shared selector computations) and write the keys' filter rows;
// warp 12 issues the MMAs (two A buffers, two 128-column accumulators); warps
// 0-7 filter (warp w: lane quadrant w % 4, columns 64 (w / 4) .. of each step).
constexpr int TQ = 256;                       // queries per unit: two 128-query steps
constexpr int T_EPI = 8;                      // filter warps: two per TMEM lane quadrant
constexpr int T_PROD = 4;                     // expanding warps: one per TMEM lane quadrant
constexpr int T_MMA_WARP = T_EPI + T_PROD;    // 12
constexpr int T_TMA_WARP = T_MMA_WARP + 1;    // 13
constexpr int T_THREADS = 32 * (T_TMA_WARP + 1);
constexpr int T_STAGES = 6;
constexpr int T_SN = 128;                     // queries per MMA step (N); 64 measured 1.41x slower
constexpr int T_NST = TQ / T_SN;              // steps per tile
constexpr int T_NACC = (512 - N_A * 128) / T_SN;  // accumulators: the TMEM the A buffers leave
constexpr int T_R = T_SN / 64;                // a filter lane's queries per step
constexpr int TO_Q = 0;                       // [2 query blocks of 128][4 K chunks][128 rows x 128 B] f16, SW128
constexpr int TO_X = TO_Q + 2 * 4 * 16384;    // filter rows [128 x 128 B] SW128, K slice j (dims 16 j ..):
                                              //   j = 0, 1 keys of A buffer j; j = 2, 3 queries of block j - 2
constexpr int TO_RING = TO_X + 16384;
constexpr int TO_KF = TO_RING + T_STAGES * N_STAGE_BYTES;   // [N_KF][128] scale
constexpr int TO_QC = TO_KF + N_KF * NK * 4;                // [2 units][4][TQ]: E, 2^e, live, sum |hi|
constexpr int TO_THR = TO_QC + 2 * 4 * TQ * 4;              // [4 quadrants][TQ] effective thresholds (stored units)
constexpr int TO_OTHR = TO_THR + N_QUAD * TQ * 4;           // [4 quadrants][TQ] lists' own 128th best
constexpr int TO_OCNT = TO_OTHR + N_QUAD * TQ * 4;          // [4 quadrants][TQ] lists' entry counts
constexpr int TO_BAR = TO_OCNT + N_QUAD * TQ * 4;
constexpr int T_NBARS = 2 * T_STAGES + 2 * N_A + 2 * T_NACC + N_KF + 2 + 2 + 1 + 1;
constexpr int TO_MISC = TO_BAR + T_NBARS * 8;
constexpr int TMEM_SMEM = TO_MISC + 16 + 1024;
static_assert(TMEM_SMEM <= 232448, "keys-in-TMEM kNN scan shared memory exceeds the sm_100 limit");
static_assert(N_A * 128 + T_NACC * T_SN <= 512 && T_NACC >= 2, "keys-in-TMEM kNN scan TMEM budget");
static_assert(T_SN == 64 || T_SN == 128, "keys-in-TMEM kNN scan step width");
static_assert(TO_X % 1024 == 0 && TO_RING % 16 == 0 && N_STAGE_BYTES % 16 == 0, "keys-in-TMEM kNN scan alignment");
constexpr float TM_SMALL = 1.220703125e-4f;   // 2^-13: smaller |s| expand as zeros (bound widened)
constexpr float TM_BIG = 16384.0f;            // 2^14: larger |s| expand as zeros (every pair kept)
constexpr uint32_t TM_H1024 = 0x6400u;        // f16 bit patterns: 1024, -inf, +inf
constexpr uint32_t TM_HNINF = 0xFC00u, TM_HPINF = 0x7C00u;
constexpr int TM_MAINT = 16;                  // tiles between the lists' compaction / threshold rounds
static_assert(KCAP - 32 * TM_MAINT >= KTOP && 32 * TM_MAINT <= KCAP - 32 * TM_MAINT,
              "a list must not overflow between two rounds");

// The 16 codes of word w (code i in bits 2i, 2i + 1) as eight pairs of f16
// values from the key's table {t1:t0} (bytes 2u, 2u + 1: the value for code
// u): out[p] holds codes 2p (lower half) and 2p + 1 (upper half).  The codes
// are spread one per byte (s_j: codes 4 i + j), bytes paired into (a + 256 b)
// per 16-bit half, and one multiply-add makes two permute selectors with
// nibbles (2a, 2a+1, 2b, 2b+1) = (a + 256 b) 34 + 0x1010.
__device__ __forceinline__ void tm_expand_word(uint32_t w, uint32_t t0, uint32_t t1, uint32_t *out) {
    const uint32_t s0 = w & 0x03030303u, s1 = (w >> 2) & 0x03030303u;
    const uint32_t s2 = (w >> 4) & 0x03030303u, s3 = (w >> 6) & 0x03030303u;
    const uint32_t q0 = __byte_perm(s0, s1, 0x5140) * 34u + 0x10101010u;  // pairs 0 | 2
    const uint32_t q1 = __byte_perm(s2, s3, 0x5140) * 34u + 0x10101010u;  // pairs 1 | 3
    const uint32_t q2 = __byte_perm(s0, s1, 0x7362) * 34u + 0x10101010u;  // pairs 4 | 6
    const uint32_t q3 = __byte_perm(s2, s3, 0x7362) * 34u + 0x10101010u;  // pairs 5 | 7
    out[0] = __byte_perm(t0, t1, q0 & 0xffffu);
    out[2] = __byte_perm(t0, t1, q0 >> 16);
    out[1] = __byte_perm(t0, t1, q1 & 0xffffu);
    out[3] = __byte_perm(t0, t1, q1 >> 16);
    out[4] = __byte_perm(t0, t1, q2 & 0xffffu);
    out[6] = __byte_perm(t0, t1, q2 >> 16);
    out[5] = __byte_perm(t0, t1, q3 & 0xffffu);
    out[7] = __byte_perm(t0, t1, q3 >> 16);
}

// The filter threshold w of a query (f16 bits): -T' / 1024 rounded up, T' =
// t - 2^-10 |t| - 2^-22 mag - 2^-30 (t = -inf: +inf, every pair kept).
__device__ __forceinline__ uint32_t tm_w_bits(float t, float mag) {
    const float tl = t - fabsf(t) * 0.0009765625f - mag * 2.384185791015625e-7f - 9.313225746154785e-10f;
    return __half_as_ushort(__float2half_ru(-tl * 0.0009765625f));
}

// The exact stored scores of up to TM_BATCH (key, query) pairs, computed by the
// whole warp (every lane calls it with the same arguments; n warp-uniform,
// entries from n on repeat pair 0 and are ignored): key codes `codes` (64
// bytes) and scale s, query row qrow (f32) with p2e = 2^e.  Lane l takes dims
// 8l .. 8l + 7 (its two code bytes, two float4 of the query); products and
// sums in f64, rounded once: s sum (u - 1.5) q 2^e.  The loads of all pairs
// are issued before any arithmetic and the shuffle reductions interleave, so
// the pairs' L2 latencies overlap.
constexpr int TM_BATCH = 2;  // kept pairs scored together (more spills the filter warps' registers)
__device__ __forceinline__ void tm_exact_warp_batch(int n, const uint8_t *const (&codes)[TM_BATCH], const float (&s)[TM_BATCH],
                                               const float *const (&qrow)[TM_BATCH], const float (&p2e)[TM_BATCH],
                                               float (&out)[TM_BATCH]) {
    const int lane = threadIdx.x & 31;
    uint32_t cb[TM_BATCH];
    float4 a[TM_BATCH], b[TM_BATCH];
#pragma unroll
    for (int j = 0; j < TM_BATCH; j++) {
        const uint8_t *cp = j < n ? codes[j] : codes[0];  // constant indices: no local-memory array
        const float *qp = j < n ? qrow[j] : qrow[0];
        cb[j] = __ldg(reinterpret_cast<const uint16_t *>(cp) + lane);
        a[j] = __ldg(reinterpret_cast<const float4 *>(qp) + 2 * lane);
        b[j] = __ldg(reinterpret_cast<const float4 *>(qp) + 2 * lane + 1);
    }
    double acc[TM_BATCH];
#pragma unroll
    for (int j = 0; j < TM_BATCH; j++) {
        const float q[8] = {a[j].x, a[j].y, a[j].z, a[j].w, b[j].x, b[j].y, b[j].z, b[j].w};
        double t = 0.0;
#pragma unroll
        for (int i = 0; i < 8; i++) t += (static_cast<double>((cb[j] >> (2 * i)) & 3u) - 1.5) * static_cast<double>(q[i]);
        acc[j] = t;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
        for (int j = 0; j < TM_BATCH; j++) acc[j] += __shfl_xor_sync(0xffffffffu, acc[j], o);
#pragma unroll
    for (int j = 0; j < TM_BATCH; j++) out[j] = static_cast<float>(acc[j] * static_cast<double>(s[j]) * static_cast<double>(p2e[j]));
}

// Slot sl (0..3) of filter lane `lane` in the warp of column half hw: the
// query it owns, T_R per step of T_SN queries.
__device__ __forceinline__ int tm_slot_query(int sl, int hw, int lane) {
    return (sl / T_R) * T_SN + (T_SN / 2) * hw + 32 * (sl % T_R) + lane;
}

// r[i] for a warp-uniform runtime i (a select chain: indexing the register
// array at run time would move it to local memory).
__device__ __forceinline__ uint32_t tm_pick16(const uint32_t (&r)[16], int i) {
    uint32_t v = r[0];
#pragma unroll
    for (int k = 1; k < 16; k++) v = i == k ? r[k] : v;
    return v;
}

template <bool EXACT>
__global__ void __launch_bounds__(T_THREADS, 1) k_knn_tmem(const NarrowArgs g) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float *kf = reinterpret_cast<float *>(smem + TO_KF);
    float *thr_s = reinterpret_cast<float *>(smem + TO_THR);  // [4][TQ] effective 128th best (stored units)
    float *thr_o = reinterpret_cast<float *>(smem + TO_OTHR);
    int *cnt_o = reinterpret_cast<int *>(smem + TO_OCNT);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + TO_BAR);
    uint64_t *rfull = bars, *rempty = bars + T_STAGES, *afull = bars + 2 * T_STAGES, *aempty = afull + N_A;
    uint64_t *accf = aempty + N_A, *acce = accf + T_NACC, *kfr = acce + T_NACC, *qready = kfr + N_KF;
    uint64_t *edone = qready + 2, *qfree = edone + 2, *fin = qfree + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + TO_MISC);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + TO_MISC + 4);
    // per-query constants of the CTA's unit j, buffer j % 2: E, 2^e, live (1 / 0), sum |hi|
    float *qconst0 = reinterpret_cast<float *>(smem + TO_QC);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the filter rows' unused dims stay zero
    for (int i = threadIdx.x; i < 16384 / 16; i += T_THREADS)
        reinterpret_cast<uint4 *>(smem + TO_X)[i] = make_uint4(0u, 0u, 0u, 0u);
    st::fence_proxy_async_smem();
    if (threadIdx.x == 0) {
        for (int s = 0; s < T_STAGES; s++) {
            st::mbar_init(&rfull[s], 1);
            st::mbar_init(&rempty[s], T_PROD);
        }
        for (int b = 0; b < N_A; b++) {
            st::mbar_init(&afull[b], T_PROD);
            st::mbar_init(&aempty[b], 1);
        }
        for (int a = 0; a < T_NACC; a++) {
            st::mbar_init(&accf[a], 1);
            st::mbar_init(&acce[a], T_EPI);
        }
        for (int k = 0; k < N_KF; k++) st::mbar_init(&kfr[k], T_PROD);
        for (int j = 0; j < 2; j++) {
            st::mbar_init(&qready[j], T_PROD);
            st::mbar_init(&edone[j], T_EPI);
        }
        st::mbar_init(qfree, 1);
        st::mbar_init(fin, 1);
        *abort_flag = 0;
        st::fence_mbar_init();
    }
    if (warp == T_MMA_WARP) {
        st::tmem_alloc(tmem_slot, N_TMEM_COLS);
        st::tmem_relinquish();
    }
    st::tc_fence_before();
    __syncthreads();
    st::tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    constexpr uint32_t ACC_COL = N_A * 128;  // accumulators after the two 128-column A buffers

    if (warp == T_TMA_WARP) {
        // ------------------------------------------------------------ code / scale loader
        if (lane == 0) {
            uint32_t gt = 0;
            bool ok = true;
            TPiece pc;
            tm_begin(g, pc);
            while (ok && tm_next(g, pc)) {
                int64_t tb;
                int nk;
                for (int64_t i = 0; tm_tile(g, pc, i, tb, nk); ++i, ++gt) {
                    const uint32_t s = gt % T_STAGES;
                    if (gt >= T_STAGES &&
                        !nwait(&rempty[s], ((gt / T_STAGES) - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_EMPTY)) {
                        ok = false;
                        break;
                    }
                    const uintptr_t s0 = reinterpret_cast<uintptr_t>(g.scales + tb) & ~uintptr_t(15);
                    const uintptr_t s1 = (reinterpret_cast<uintptr_t>(g.scales + tb + nk) + 15) & ~uintptr_t(15);
                    const uint32_t cb = static_cast<uint32_t>(nk) * 64u, sb = static_cast<uint32_t>(s1 - s0);
                    uint8_t *dst = smem + TO_RING + s * N_STAGE_BYTES;
                    st::mbar_arrive_expect_tx(&rfull[s], cb + sb);
                    st::bulk_load(dst, g.codes + tb * 64, cb, &rfull[s]);
                    st::bulk_load(dst + N_CODE_BYTES, reinterpret_cast<const void *>(s0), sb, &rfull[s]);
                }
            }
            const uint32_t first = gt > T_STAGES ? gt - T_STAGES : 0;
            for (uint32_t i = first; i < gt; i++)
                st::mbar_wait(&rfull[i % T_STAGES], (i / T_STAGES) & 1u, g.status, st::DEV_TIMEOUT_FULL);
        }
    } else if (warp >= T_EPI && warp < T_MMA_WARP) {
        // ------------------------------------------------------------ producers
        const int pw = warp - T_EPI;  // 0..3: TMEM lanes 32 pw .. (warp % 4 = pw)
        const int quad = warp & 3;
        uint32_t gt = 0, uj = 0;
        bool ok = true;
        TPiece pc;
        tm_begin(g, pc);
        for (; ok && tm_next(g, pc); ++uj) {
            // the query tiles and filter rows are rewritten once the MMAs and the
            // epilogue (which writes thresholds into the filter rows) are done with
            // the previous piece
            if (uj >= 1 && !nwait(qfree, (uj - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_ACC)) break;
            if (uj >= 1 &&
                !nwait(&edone[(uj - 1) & 1u], ((uj - 1) >> 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_ACC))
                break;
            float *qc = qconst0 + (uj & 1u) * 4 * TQ;
            const int qbase = pc.qb * TQ;
            // warp pw prepares queries pw, pw + 4, ..; lane l writes dims 8l .. 8l + 7 (one
            // 16-byte piece of the row's K chunk l / 8) as f16 of q 2^e
            for (int r = pw; r < TQ; r += T_PROD) {
                const int qg = qbase + r;
                const bool live = qg < g.nq;
                const float *qrow = g.q + static_cast<int64_t>(live ? qg : 0) * 256;
                float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
                if (live) {
                    a = __ldg(reinterpret_cast<const float4 *>(qrow) + 2 * lane);
                    b = __ldg(reinterpret_cast<const float4 *>(qrow) + 2 * lane + 1);
                }
                const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
                float mx = 0.0f;
#pragma unroll
                for (int i = 0; i < 8; i++) mx = fmaxf(mx, fabsf(v[i]));
                mx = warp_max(mx);
                const int e = query_exp(mx);
                const float p2e = pow2f(e);
                float err = 0.0f, mag = 0.0f;
                uint32_t hw[4];
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float x0 = v[2 * i] * p2e, x1 = v[2 * i + 1] * p2e;
                    const __half2 hh = __floats2half2_rn(x0, x1);
                    const float2 hf = __half22float2(hh);
                    err += fabsf(x0 - hf.x) + fabsf(x1 - hf.y);
                    mag += fabsf(hf.x) + fabsf(hf.y);
                    hw[i] = *reinterpret_cast<const uint32_t *>(&hh);
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    err += __shfl_xor_sync(0xffffffffu, err, o);
                    mag += __shfl_xor_sync(0xffffffffu, mag, o);
                }
                const int step = r >> 7, row = r & 127;
                *reinterpret_cast<uint4 *>(smem + TO_Q + step * 65536 + (lane >> 3) * 16384 +
                                           st::sw128_offset(row, lane & 7)) = make_uint4(hw[0], hw[1], hw[2], hw[3]);
                if (lane == 0) {
                    // the sums round up by far less than the 2^-10 slack
                    const float eb = live ? (1.5f * err + 0.001953125f * mag) * 1.0009765625f + 5.9604644775390625e-8f
                                          : 0.0f;
                    qc[r] = eb;
                    qc[TQ + r] = p2e;
                    qc[2 * TQ + r] = live ? 1.0f : 0.0f;
                    qc[3 * TQ + r] = mag;
                    // the query's filter row: (w, E16) in the full pass, (0, -E16) in a sample pass
                    uint32_t wb = TM_HNINF, ebits = 0u;
                    if (live) {
                        ebits = __half_as_ushort(__float2half_ru(eb));
                        if (EXACT) {
                            wb = tm_w_bits(thr_of(__ldcg(g.gthr + qg)), mag);
                        } else {
                            wb = 0u;
                            ebits ^= 0x8000u;
                        }
                    }
                    *reinterpret_cast<uint4 *>(smem + TO_X + st::sw128_offset(row, 2 * (2 + step))) =
                        make_uint4(wb | (ebits << 16), 0u, 0u, 0u);
                }
            }
            st::fence_proxy_async_smem();
            __syncwarp();
            if (lane == 0) st::mbar_arrive(&qready[uj & 1u]);

            int64_t tb;
            int nk;
            for (int64_t i = 0; tm_tile(g, pc, i, tb, nk); ++i, ++gt) {
                const uint32_t s = gt % T_STAGES, b = gt % N_A, f = gt % N_KF;
                if (!nwait(&rfull[s], (gt / T_STAGES) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) {
                    ok = false;
                    break;
                }
                const uint8_t *stage = smem + TO_RING + s * N_STAGE_BYTES;
                const int sofs = static_cast<int>((reinterpret_cast<uintptr_t>(g.scales + tb) & 15u) >> 2);
                const int key = 32 * quad + lane;  // this thread's key: TMEM lane 32 quad + lane
                const bool in = key < nk;
                const uint4 *src = reinterpret_cast<const uint4 *>(stage + 64 * key);
                uint4 cw[4];
#pragma unroll
                for (int w = 0; w < 4; w++) cw[w] = in ? src[w] : make_uint4(0u, 0u, 0u, 0u);
                const float scl = in ? reinterpret_cast<const float *>(stage + N_CODE_BYTES)[sofs + key] : 0.0f;
                // the key's table (u - 1.5) s and filter row (1024, s16)
                const float ab = fabsf(scl);
                const bool small = ab < TM_SMALL, normal = !small && ab < TM_BIG;  // NaN: neither
                const float sv = normal ? scl : 0.0f;
                const __half2 lo = __floats2half2_rn(-1.5f * sv, -0.5f * sv);
                const __half2 hi = __floats2half2_rn(0.5f * sv, 1.5f * sv);
                const uint32_t t0 = *reinterpret_cast<const uint32_t *>(&lo);
                const uint32_t t1 = *reinterpret_cast<const uint32_t *>(&hi);
                const uint32_t s16 = small    ? __half_as_ushort(__float2half_ru(ab * 1024.0f))
                                     : normal ? __half_as_ushort(__float2half_ru(ab))
                                              : TM_HPINF;
                __syncwarp();
                if (lane == 0) st::mbar_arrive(&rempty[s]);
                // A buffer b (and its filter rows) is free once the MMAs of tile gt - 2 are
                // done; they waited for the epilogue to release step 2 (gt - 2) - 1, so it
                // is done with tile gt - 3, and slot f last held tile gt - 8
                if (gt >= N_A &&
                    !nwait(&aempty[b], ((gt / N_A) - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_EMPTY)) {
                    ok = false;
                    break;
                }
                kf[f * NK + key] = scl;
                *reinterpret_cast<uint4 *>(smem + TO_X + st::sw128_offset(key, 2 * b)) =
                    make_uint4(TM_H1024 | (s16 << 16), 0u, 0u, 0u);
                __syncwarp();
                if (lane == 0) st::mbar_arrive(&kfr[f]);
                // column c of the key's A row holds dims 2c, 2c + 1: code word j (dims 16 j ..)
                // fills columns 8 j .. 8 j + 7, 32 columns (four words) per store
                const uint32_t trow = tmem + (static_cast<uint32_t>(32 * quad) << 16) + b * 128u;
#pragma unroll
                for (int h = 0; h < 4; h++) {
                    uint32_t v[32];
                    tm_expand_word(cw[h].x, t0, t1, v);
                    tm_expand_word(cw[h].y, t0, t1, v + 8);
                    tm_expand_word(cw[h].z, t0, t1, v + 16);
                    tm_expand_word(cw[h].w, t0, t1, v + 24);
                    st::tmem_st32(trow + 32u * h, v);
                }
                st::tmem_st_wait();
                st::fence_proxy_async_smem();  // the filter rows, for the MMA's shared-memory reads
                st::tc_fence_before();
                __syncwarp();
                if (lane == 0) st::mbar_arrive(&afull[b]);
            }
        }
    } else if (warp == T_MMA_WARP) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            constexpr uint32_t idesc = st::idesc_make(1, 0, false, false, 128, T_SN);  // f32 <- f16 x f16
            const uint32_t qbuf = st::smem_u32(smem + TO_Q), xbuf = st::smem_u32(smem + TO_X);
            uint32_t gt = 0, gs = 0, uj = 0;
            bool ok = true;
            TPiece pc;
            tm_begin(g, pc);
            for (; ok && tm_next(g, pc); ++uj) {
                if (!nwait(&qready[uj & 1u], (uj >> 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) break;
                st::tc_fence_after();
                int64_t tb;
                int nk;
                for (int64_t i = 0; tm_tile(g, pc, i, tb, nk); ++i, ++gt) {
                    const uint32_t b = gt % N_A;
                    if (!nwait(&afull[b], (gt / N_A) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) {
                        ok = false;
                        break;
                    }
                    st::tc_fence_after();
                    const uint32_t abuf = tmem + b * 128u;
#pragma unroll 1
                    for (int step = 0; step < T_NST; step++, gs++) {
                        const uint32_t a = gs % T_NACC;
                        if (gs >= T_NACC &&
                            !nwait(&acce[a], ((gs / T_NACC) - 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_EMPTY)) {
                            ok = false;
                            break;
                        }
                        st::tc_fence_after();
                        const uint32_t acc = tmem + ACC_COL + a * T_SN;
                        // queries T_SN step ..: 128-query block blk, from row rofs (8 KB per 64 rows,
                        // a whole number of swizzle atoms)
                        const uint32_t blk = (step * T_SN) >> 7, rofs = ((step * T_SN) & 127) * 128;
                        const uint32_t qs = qbuf + blk * 65536 + rofs;
#pragma unroll
                        for (int kk = 0; kk < 16; kk++)
                            st::umma_f16_ts(acc, abuf + 8 * kk,
                                            st::sdesc_sw128(qs + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024), idesc,
                                            kk > 0 ? 1u : 0u);
                        // the filter terms: K slice b of the keys' rows x slice 2 + blk of the queries'
                        st::umma_f16(acc, st::sdesc_sw128(xbuf + b * 32, 16, 1024),
                                     st::sdesc_sw128(xbuf + (2 + blk) * 32 + rofs, 16, 1024), idesc, 1u);
                        st::umma_commit(&accf[a]);
                    }
                    if (!ok) break;
                    st::umma_commit(&aempty[b]);
                }
                st::umma_commit(qfree);
            }
            st::umma_commit(fin);
            nwait(fin, 0, abort_flag, g.status, st::DEV_TIMEOUT_ACC);
        }
    } else {
        // ------------------------------------------------------------ epilogue
        // Warp w: TMEM lanes 32 (w % 4) .. (keys), accumulator columns T_SN / 2 (w / 4) ..
        // of each step (queries T_SN step + T_SN / 2 (w / 4) + c of the unit).  Lane l owns
        // the candidate buffers of the unit's queries tm_slot_query(s, w / 4, l), slots
        // s = 0..3 (four queries of each step of T_SN); the lists' counts, own 128th-best
        // scores and effective thresholds live in shared memory, so that the loops over
        // chunks and slots stay rolled (small code: the four roles share the SM's
        // instruction cache).
        const int quad = warp & 3, hw = warp >> 2;
        const unsigned lt = (1u << lane) - 1u;
        const uint32_t lane_addr = static_cast<uint32_t>(32 * quad) << 16;
        uint64_t *bufs = g.cbuf + static_cast<int64_t>(blockIdx.x * N_QUAD + quad) * TQ * KCAP;
        float *wthr = thr_s + quad * TQ;   // effective threshold (stored units)
        float *othr = thr_o + quad * TQ;   // the list's own 128th best
        int *ocnt = cnt_o + quad * TQ;     // the list's entries
        const uint32_t acc0 = tmem + lane_addr + ACC_COL;
        uint32_t gt = 0, gs = 0, uj = 0;
        bool ok = true;
        TPiece pc;
        tm_begin(g, pc);
        for (; ok && tm_next(g, pc); ++uj) {
            if (!nwait(&qready[uj & 1u], (uj >> 1) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_FULL)) break;
            const float *qc = qconst0 + (uj & 1u) * 4 * TQ;
            const float *qc_p = qc + TQ, *qc_mag = qc + 3 * TQ;
            const int qbase = pc.qb * TQ;
            const int nlive = g.nq - qbase;  // the unit's queries from nlive on are padding
#pragma unroll 1
            for (int sl = 0; sl < 4; sl++) {
                const int qu = tm_slot_query(sl, hw, lane);
                const bool live = qu < nlive;
                ocnt[qu] = 0;
                othr[qu] = live ? -INFINITY : INFINITY;
                const float e0 = live ? thr_of(__ldcg(g.gthr + qbase + qu)) : INFINITY;
                wthr[qu] = e0;
                if (EXACT && live)
                    *reinterpret_cast<uint16_t *>(smem + TO_X + st::sw128_offset(qu & 127, 2 * (2 + (qu >> 7)))) =
                        static_cast<uint16_t>(tm_w_bits(e0, qc_mag[qu]));
            }
            st::fence_proxy_async_smem();
            __syncwarp();
            int64_t tb;
            int nk;
            for (int64_t i = 0; tm_tile(g, pc, i, tb, nk); ++i, ++gt) {
                const uint32_t f = gt % N_KF;
                if (!nwait(&kfr[f], (gt / N_KF) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_ACC)) {
                    ok = false;
                    break;
                }
                const int kk = 32 * quad + lane;
                const float scale = kf[f * NK + kk];
                const bool klive = kk < nk;
                const uint32_t idx = g.index_base + static_cast<uint32_t>(tb) + static_cast<uint32_t>(kk);
#pragma unroll 1
                for (int step = 0; step < T_NST; step++, gs++) {
                    const uint32_t a = gs % T_NACC;
                    if (!nwait(&accf[a], (gs / T_NACC) & 1u, abort_flag, g.status, st::DEV_TIMEOUT_ACC)) {
                        ok = false;
                        break;
                    }
                    st::tc_fence_after();
                    const int qw = step * T_SN + (T_SN / 2) * hw;  // this warp's first query of the step
                    const uint32_t acc = acc0 + a * T_SN + (T_SN / 2) * hw;
                    const int lim0 = nlive - qw;
                    constexpr int NCH = T_SN / 32;  // this warp's 16-column chunks of a step
                    if (EXACT) {
                        // full pass: a pair is kept if its filtered accumulator is not negative
                        uint32_t pass[NCH];  // per 16-query chunk, bit i: the pair was kept
                        {
                            uint32_t r[NCH / 2][32];  // the warp's columns, one wait
#pragma unroll
                            for (int h2 = 0; h2 < NCH / 2; h2++) st::tmem_ld32(acc + 32 * h2, r[h2]);
                            st::tmem_ld_wait();
#pragma unroll
                            for (int hh = 0; hh < NCH; hh++) {
                                const uint32_t *rc = r[hh >> 1] + 16 * (hh & 1);
                                // all 16 negative <=> the AND of their sign bits is set
                                const uint32_t a0 = rc[0] & rc[1] & rc[2] & rc[3], a1 = rc[4] & rc[5] & rc[6] & rc[7];
                                const uint32_t a2 = rc[8] & rc[9] & rc[10] & rc[11];
                                const uint32_t a3 = rc[12] & rc[13] & rc[14] & rc[15];
                                uint32_t pm = 0u;
                                if (!((a0 & a1 & a2 & a3) >> 31)) {
#pragma unroll
                                    for (int j = 0; j < 16; j++) pm |= ((~rc[j]) >> 31) << j;
                                }
                                const int lim = lim0 - 16 * hh;
                                const uint32_t qmask = lim >= 16 ? 0xffffu : lim <= 0 ? 0u : (1u << lim) - 1u;
                                pass[hh] = klive ? pm & qmask : 0u;
                            }
                        }
                        // every column is read: the accumulator goes back to the MMA
                        st::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) st::mbar_arrive(&acce[a]);
                        // each kept pair's exact score, by the whole warp; inserted by the
                        // list's owner lane if it reaches the threshold
                        uint32_t pall = 0u;
#pragma unroll
                        for (int hh = 0; hh < NCH; hh++) pall |= pass[hh];
                        const unsigned any = __ballot_sync(0xffffffffu, pall != 0u);
                        if (any) {
                            // kept pairs in (chunk, key lane, query) order, scored TM_BATCH at a time;
                            // the owner lane of each query inserts in that order
                            int np = 0, pq[TM_BATCH], pk[TM_BATCH];
                            const uint8_t *pc_codes[TM_BATCH];
                            const float *pc_q[TM_BATCH];
                            float pc_s[TM_BATCH], pc_p[TM_BATCH], e4[TM_BATCH];
                            auto flush = [&]() {
                                tm_exact_warp_batch(np, pc_codes, pc_s, pc_q, pc_p, e4);
#pragma unroll
                                for (int j = 0; j < TM_BATCH; j++) {
                                    if (j >= np) break;
                                    const int qu = pq[j];
                                    if (lane == (qu & 31) && e4[j] >= wthr[qu]) {
                                        const int base = ocnt[qu];
                                        bufs[static_cast<int64_t>(qu) * KCAP + base] =
                                            make_key(e4[j], g.index_base + static_cast<uint32_t>(tb) +
                                                                static_cast<uint32_t>(pk[j]));
                                        ocnt[qu] = base + 1;
                                    }
                                }
                                np = 0;
                            };
#pragma unroll 1
                            for (int c = 0; c < NCH; c++) {
                                uint32_t pcm = pass[0];  // pass[c] (a select chain keeps it in registers)
#pragma unroll
                                for (int hh = 1; hh < NCH; hh++) pcm = c == hh ? pass[hh] : pcm;
                                unsigned lanes = __ballot_sync(0xffffffffu, pcm != 0u);
                                const int q0 = qw + 16 * c;
                                while (lanes) {
                                    const int L = __ffs(lanes) - 1;
                                    lanes &= lanes - 1;
                                    uint32_t bits = __shfl_sync(0xffffffffu, pcm, L);
                                    const float sL = __shfl_sync(0xffffffffu, scale, L);
                                    const int keyL = 32 * quad + L;
                                    const uint8_t *kcodes = g.codes + (tb + keyL) * 64;
                                    while (bits) {
                                        const int ib = __ffs(bits) - 1;
                                        bits &= bits - 1;
                                        const int qu = q0 + ib;
                                        const float *qrow = g.q + static_cast<int64_t>(qbase + qu) * 256;
                                        const float p2e = qc_p[qu];
#pragma unroll
                                        for (int j = 0; j < TM_BATCH; j++) {  // constant indices: registers
                                            if (j == np) {
                                                pq[j] = qu;
                                                pk[j] = keyL;
                                                pc_codes[j] = kcodes;
                                                pc_q[j] = qrow;
                                                pc_s[j] = sL;
                                                pc_p[j] = p2e;
                                            }
                                        }
                                        if (++np == TM_BATCH) flush();
                                    }
                                }
                            }
                            if (np) flush();
                        }
                    } else {
                        // sample pass: acc' is a lower bound of the pair's score; a pair enters
                        // its list, lowered by 2^-12, if the bound reaches the threshold
#pragma unroll 1
                        for (int c = 0; c < NCH; c++) {
                            uint32_t r[16];
                            st::tmem_ld16(acc + 16 * c, r);
                            st::tmem_ld_wait();
                            const int q0 = qw + 16 * c;
                            uint32_t pm = 0u;
#pragma unroll
                            for (int i4 = 0; i4 < 16; i4 += 4) {
                                const float4 tf = *reinterpret_cast<const float4 *>(wthr + q0 + i4);
                                pm |= (__uint_as_float(r[i4]) >= tf.x ? 1u : 0u) << i4;
                                pm |= (__uint_as_float(r[i4 + 1]) >= tf.y ? 1u : 0u) << (i4 + 1);
                                pm |= (__uint_as_float(r[i4 + 2]) >= tf.z ? 1u : 0u) << (i4 + 2);
                                pm |= (__uint_as_float(r[i4 + 3]) >= tf.w ? 1u : 0u) << (i4 + 3);
                            }
                            const int lim = lim0 - 16 * c;
                            const uint32_t qmask = lim >= 16 ? 0xffffu : lim <= 0 ? 0u : (1u << lim) - 1u;
                            pm = klive ? pm & qmask : 0u;
                            unsigned qm = __reduce_or_sync(0xffffffffu, pm);
                            while (qm) {
                                const int ib = __ffs(qm) - 1;
                                qm &= qm - 1;
                                const bool p = (pm >> ib) & 1u;
                                const unsigned mb = __ballot_sync(0xffffffffu, p);
                                const int qu = q0 + ib;
                                const int base = ocnt[qu];
                                if (p)
                                    bufs[static_cast<int64_t>(qu) * KCAP + base + __popc(mb & lt)] =
                                        make_key(lowered(__uint_as_float(tm_pick16(r, ib))), idx);
                                __syncwarp();  // every lane has read the count
                                if (lane == 16 * (c & 1) + ib) ocnt[qu] = base + __popc(mb);
                                __syncwarp();
                            }
                        }
                        st::tc_fence_before();
                        __syncwarp();
                        if (lane == 0) st::mbar_arrive(&acce[a]);
                    }
                    // every TM_MAINT tiles: compaction of lists that could overflow before the
                    // next round (a list gains at most 32 entries a tile); thresholds: own
                    // 128th best, published, and the best any list of the query has published
                    if (i % TM_MAINT != TM_MAINT - 1) continue;
#pragma unroll 1
                    for (int sh = 0; sh < T_R; sh++) {
                        const int qu = qw + 32 * sh + lane;
                        int cn = ocnt[qu];
                        float th = othr[qu];
                        const unsigned need = __ballot_sync(0xffffffffu, cn > KCAP - 32 * TM_MAINT);
                        if (need) {
                            const float before = th;
                            warp_compact(need, bufs + static_cast<int64_t>(qu) * KCAP, cn, th, nullptr, false);
                            ocnt[qu] = cn;
                            othr[qu] = th;
                            if (th > before) atomicMax(g.gthr + qbase + qu, ord_f32(th));
                        }
                        const float ef = wthr[qu];
                        float ne = fmaxf(th, ef);
                        if (qu < nlive) ne = fmaxf(ne, thr_of(__ldcg(g.gthr + qbase + qu)));
                        if (__any_sync(0xffffffffu, ne > ef)) {
                            if (ne > ef) {
                                wthr[qu] = ne;
                                if (EXACT)
                                    *reinterpret_cast<uint16_t *>(smem + TO_X +
                                                                  st::sw128_offset(qu & 127, 2 * (2 + (qu >> 7)))) =
                                        static_cast<uint16_t>(tm_w_bits(ne, qc_mag[qu]));
                            }
                            if (EXACT) st::fence_proxy_async_smem();
                            __syncwarp();
                        }
                    }
                }
                if (!ok) break;
            }
            if (!ok) break;
            if (pc.slot < 0 || pc.slot >= g.nslot) {  // the host sized nslot for every piece: not reached
                st::set_status(g.status, st::DEV_BAD_ARG);
                *abort_flag = 1;
                break;
            }
#pragma unroll 1
            for (int sl = 0; sl < 4; sl++) {
                const int qu = tm_slot_query(sl, hw, lane);
                int cn = ocnt[qu];
                float th = othr[qu];
                uint64_t *my_out =
                    g.unit_out + ((static_cast<int64_t>(pc.slot) * N_QUAD + quad) * g.nq_pad + qbase + qu) * KTOP;
                const unsigned need = __ballot_sync(0xffffffffu, qu < nlive);
                warp_compact(need, bufs + static_cast<int64_t>(qu) * KCAP, cn, th, my_out, true);
            }
            __syncwarp();
            if (lane == 0) st::mbar_arrive(&edone[uj & 1u]);
        }
    }

    st::tc_fence_before();
    __syncthreads();
    if (warp == T_MMA_WARP) {
        st::tc_fence_after();
        st::tmem_dealloc(tmem, N_TMEM_COLS);
    }
}

template <bool EXACT>
st_status launch_tmem_t(st_handle *h, const NarrowArgs &g, int grid) {
    static bool attr_done = false;
    if (!attr_done) {
        ST_CHECK_CUDA(h, cudaFuncSetAttribute(k_knn_tmem<EXACT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              TMEM_SMEM));
        attr_done = true;
    }
    k_knn_tmem<EXACT><<<grid, T_THREADS, TMEM_SMEM, h->stream>>>(g);
    return st_after_launch(h, "k_knn_tmem");
}

// The full pass (exact scores) or a sample pass (lower bounds), as g.exact says.
st_status launch_tmem(st_handle *h, const NarrowArgs &g, int grid) {
    return g.exact ? launch_tmem_t<true>(h, g, grid) : launch_tmem_t<false>(h, g, grid);
}

}  // namespace

bool st_knn_seeded_route(int32_t dim, int64_t nq, int32_t mode, int32_t prec) {
    // the keys-in-TMEM scan (> 32 EXACT dot-product queries) and the narrow scan (<= 32)
    return dim == 256 && ((nq > NQ && prec == 0 && mode == 0) || nq <= NQ);
}

static st_status topk_keys(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_keys, int32_t dim,
                           const float *queries, int64_t nq, int32_t mode, int32_t prec, int64_t index_base,
                           const int64_t *ranges, int64_t always, uint64_t *out_keys, const char *who) {
    if (!h) return ST_INVALID_ARG;
    st_status s = check_common(h, codes, scales, n_keys, dim, queries, nq, mode, prec, index_base, who);
    if (s != ST_OK) return s;
    if (!out_keys) return h->fail(ST_INVALID_ARG, "%s: null output", who);
    cudaSetDevice(h->device);
    if (!ranges && dim == 256 && nq > NQ && prec == 0 && mode == 0 && (reinterpret_cast<uintptr_t>(scales) & 3u) == 0) {
        // more than 32 EXACT dot-product queries at dim 256: keys in TMEM (k_knn_tmem).
        // Every pass cuts its (query block of 256, 128-key tile) sequence into one
        // equal range per CTA; the CTAs covering a block each leave one list per
        // (query, lane quadrant), in slots 0 .. nslot - 1 (unused slots stay zero).
        const int nqb = static_cast<int>((nq + TQ - 1) / TQ);
        const int64_t nq_pad = static_cast<int64_t>(nqb) * TQ;
        const int64_t tiles = (n_keys + NK - 1) / NK;
        if (static_cast<int64_t>(nqb) * tiles > (1LL << 50)) return h->fail(ST_UNSUPPORTED_SHAPE, "%s: too many queries", who);
        // a pass over `samples` tiles per block: its grid and the slots its pieces need
        auto plan = [&](int64_t samples, int &grid, int &nslot, int &aligned) {
            if (nqb <= h->num_sms) {
                // P aligned parts per query block, one per CTA
                const int parts = static_cast<int>(std::min<int64_t>(h->num_sms / nqb, samples));
                grid = nqb * parts;
                nslot = parts;
                aligned = 1;
                return;
            }
            const int64_t flat = static_cast<int64_t>(nqb) * samples;
            grid = static_cast<int>(std::min<int64_t>(flat, h->num_sms));
            const int64_t shortest = flat / grid;  // every CTA's range holds at least this many samples
            nslot = static_cast<int>((samples + shortest - 1) / shortest + 1);
            aligned = 0;
        };
        int grid_full, nslot_full, al;
        plan(tiles, grid_full, nslot_full, al);
        int nslot_max = nslot_full;
        for (int64_t stride : {int64_t(1024), int64_t(16)}) {
            const int64_t sample = (tiles + stride - 1) / stride;
            if (sample * nqb < 4 * h->num_sms || sample >= tiles) continue;
            int gr, ns;
            plan(sample, gr, ns, al);
            nslot_max = std::max(nslot_max, ns);
        }
        const int grid_cap = h->num_sms;
        uint64_t *cbuf = static_cast<uint64_t *>(
            st_scratch(h, SLOT_KNN_CAND, sizeof(uint64_t) * grid_cap * N_QUAD * TQ * KCAP));
        const size_t out_bytes = sizeof(uint64_t) * nslot_max * N_QUAD * nq_pad * KTOP;
        const size_t seed_bytes = sizeof(uint64_t) * nq_pad * KTOP;
        constexpr int MERGE_GROUPS = 16;
        const size_t tmp_bytes = sizeof(uint64_t) * MERGE_GROUPS * nq_pad * KTOP;
        uint8_t *part = static_cast<uint8_t *>(
            st_scratch(h, SLOT_KNN_PART, out_bytes + seed_bytes + tmp_bytes + sizeof(uint32_t) * nq_pad + 256));
        if (!cbuf || !part) return ST_NO_MEMORY;
        uint64_t *unit_out = reinterpret_cast<uint64_t *>(part);
        uint64_t *seed_keys = reinterpret_cast<uint64_t *>(part + out_bytes);
        uint64_t *merge_tmp = reinterpret_cast<uint64_t *>(part + out_bytes + seed_bytes);
        uint32_t *gthr = reinterpret_cast<uint32_t *>(part + out_bytes + seed_bytes + tmp_bytes);
        ST_CHECK_CUDA(h, cudaMemsetAsync(gthr, 0, nq_pad * sizeof(uint32_t), h->stream));
        NarrowArgs g{};
        g.codes = codes;
        g.scales = scales;
        g.q = queries;
        g.n_keys = n_keys;
        g.nq = static_cast<int>(nq);
        g.nqb = nqb;
        g.nq_pad = static_cast<int>(nq_pad);
        g.n_tiles = tiles;
        g.index_base = static_cast<uint32_t>(index_base);
        g.cbuf = cbuf;
        g.unit_out = unit_out;
        g.gthr = gthr;
        g.status = h->d_status;
        // one pass over every stride-th tile: lists zeroed, scan, merge into `dst`
        auto pass = [&](int64_t stride, int exact, uint64_t *dst) -> st_status {
            const int64_t samples = (tiles + stride - 1) / stride;
            int grid, nslot, aligned;
            plan(samples, grid, nslot, aligned);
            NarrowArgs a = g;
            a.aligned = aligned;
            a.exact = exact;
            a.unit_step = stride;
            a.seg_len = samples;
            a.flat_len = static_cast<int64_t>(nqb) * samples;
            a.nslot = nslot;
            ST_CHECK_CUDA(h, cudaMemsetAsync(unit_out, 0, sizeof(uint64_t) * nslot * N_QUAD * nq_pad * KTOP,
                                             h->stream));
            st_status r = launch_tmem(h, a, grid);
            if (r != ST_OK) return r;
            return merge_lists(h, unit_out, static_cast<int64_t>(nslot) * N_QUAD, nq_pad * KTOP, nq, merge_tmp,
                               MERGE_GROUPS, dst);
        };
        // two sample passes seed the thresholds (every 1024th, then every 16th tile):
        // a list's 128th best over a subset bounds the final 128th best from below
        // With h->seed_exchange set (a key-sharded search), every stage's lists are
        // merged with the other ranks' before seeding: the 128th best of the union of
        // the ranks' samples bounds the global 128th best from below, and only keys
        // reaching the global 128th best can be in the merged result.
        for (int64_t stride : {int64_t(1024), int64_t(16)}) {
            const int64_t sample = (tiles + stride - 1) / stride;
            const bool run_stage = sample * nqb >= 4 * h->num_sms && sample < tiles;
            if (run_stage) {
                s = pass(stride, 0, seed_keys);
                if (s != ST_OK) return s;
            }
            if (h->seed_exchange) {
                if (!run_stage) ST_CHECK_CUDA(h, cudaMemsetAsync(seed_keys, 0, seed_bytes, h->stream));
                s = h->seed_exchange(h, seed_keys, nq, h->seed_ctx);
                if (s != ST_OK) return s;
            }
            if (run_stage || h->seed_exchange) {
                k_knn_seed<<<static_cast<unsigned>((nq + 127) / 128), 128, 0, h->stream>>>(seed_keys,
                                                                                           static_cast<int>(nq), gthr);
                s = st_after_launch(h, "k_knn_seed");
                if (s != ST_OK) return s;
            }
        }
        return pass(1, 1, out_keys);
    }
    if (!ranges && dim == 256 && nq <= NQ && (reinterpret_cast<uintptr_t>(scales) & 3u) == 0) {
        // dim 256, up to 32 queries: the keys-on-M scan (keys as the kind::i8 A
        // operand in TMEM), one group of 32 queries per unit.  More queries run
        // k_knn_scan below: with 128 resident queries per unit (four groups per
        // key tile) the keys-on-M scan measured 0.96-1.0 s at 4096 x 2^27 against
        // k_knn_scan's 0.5 s -- its epilogue reads two limb columns per (key,
        // query) pair and every accumulator step passes through all eight
        // epilogue warps in turn (ncu: tensor pipe 10.6 %, issue 18.9 %) -- and
        // four int8 limbs cost the tensor core what k_knn_scan's f16 hi + lo
        // pair costs, so it could not win by much even with a faster epilogue.
        constexpr int qb_size = NQ;  // one query block: NG = 1
        const int nqb = 1;
        const int64_t nq_pad = qb_size;
        const int64_t tiles = (n_keys + NK - 1) / NK;
        int64_t splits = std::min<int64_t>(h->num_sms, tiles);  // one key split per SM
        const int64_t tps = (tiles + splits - 1) / splits;
        splits = (tiles + tps - 1) / tps;
        const int64_t units = splits * nqb;
        if (units > (1LL << 30)) return h->fail(ST_UNSUPPORTED_SHAPE, "%s: too many queries", who);
        const int grid = static_cast<int>(std::min<int64_t>(units, h->num_sms));
        const int64_t sample_splits = h->num_sms;  // the sample passes' key splits
        const int64_t max_splits = std::max(splits, sample_splits);
        // candidate buffers for the widest grid any pass launches (the sample passes have up to
        // sample_splits * nqb units)
        const int64_t grid_max = std::min<int64_t>(std::max(units, sample_splits * nqb), h->num_sms);
        uint64_t *cbuf = static_cast<uint64_t *>(
            st_scratch(h, SLOT_KNN_CAND, sizeof(uint64_t) * grid_max * N_QUAD * qb_size * KCAP));
        const size_t out_bytes = sizeof(uint64_t) * max_splits * N_QUAD * nq_pad * KTOP;
        const size_t seed_bytes = sizeof(uint64_t) * nq_pad * KTOP;
        constexpr int MERGE_GROUPS = 16;
        const size_t tmp_bytes = sizeof(uint64_t) * MERGE_GROUPS * nq_pad * KTOP;
        uint8_t *part = static_cast<uint8_t *>(
            st_scratch(h, SLOT_KNN_PART, out_bytes + seed_bytes + tmp_bytes + sizeof(uint32_t) * nq_pad + 256));
        if (!cbuf || !part) return ST_NO_MEMORY;
        uint64_t *unit_out = reinterpret_cast<uint64_t *>(part);
        uint64_t *seed_keys = reinterpret_cast<uint64_t *>(part + out_bytes);
        uint64_t *merge_tmp = reinterpret_cast<uint64_t *>(part + out_bytes + seed_bytes);
        uint32_t *gthr = reinterpret_cast<uint32_t *>(part + out_bytes + seed_bytes + tmp_bytes);
        ST_CHECK_CUDA(h, cudaMemsetAsync(gthr, 0, nq_pad * sizeof(uint32_t), h->stream));
        // queries per limb block: 16 or 32 (an epilogue warp takes 16; NL x 16 is a multiple of 16)
        const int nqp = nq <= EQ ? EQ : NQ;
        NarrowArgs g{};
        g.codes = codes;
        g.scales = scales;
        g.q = queries;
        g.n_keys = n_keys;
        g.nq = static_cast<int>(nq);
        g.nqp = nqp;
        g.nqb = nqb;
        g.nq_pad = static_cast<int>(nq_pad);
        g.n_tiles = tiles;
        g.index_base = static_cast<uint32_t>(index_base);
        g.cbuf = cbuf;
        g.unit_out = unit_out;
        g.gthr = gthr;
        g.status = h->d_status;
        auto run = [&](const NarrowArgs &a, int gr) {
            if (mode == 0 && prec == 0) return launch_narrow<MODE_DOT, PREC_EXACT, 1>(h, a, gr);
            if (mode == 0) return launch_narrow<MODE_DOT, PREC_F16REF, 1>(h, a, gr);
            if (prec == 0) return launch_narrow<MODE_L2, PREC_EXACT, 1>(h, a, gr);
            return launch_narrow<MODE_L2, PREC_F16REF, 1>(h, a, gr);
        };
        // Large scans first take a sample of the tiles: the best 128 of a sample
        // bound each query's final 128th best from below, and every list of the
        // next pass starts from it instead of from its own first keys.  Two
        // levels: every 1024th tile seeds a pass over every 16th, which seeds the
        // full scan.
        // (with h->seed_exchange set, each stage's lists are merged with the other
        // ranks' before seeding, as in the keys-in-TMEM scan above)
        for (int64_t stride : {int64_t(1024), int64_t(16)}) {
            const int64_t sample = (tiles + stride - 1) / stride;
            const bool run_stage = sample >= 2 * h->num_sms;
            if (run_stage) {
                NarrowArgs gs = g;
                const int64_t gsplits = std::min<int64_t>(sample_splits, sample);
                gs.units = static_cast<int>(gsplits * nqb);
                gs.unit_step = stride;
                gs.tile_step = stride * gsplits;
                gs.tiles_per_unit = (sample + gsplits - 1) / gsplits;
                s = run(gs, static_cast<int>(std::min<int64_t>(gs.units, h->num_sms)));
                if (s != ST_OK) return s;
                s = merge_lists(h, unit_out, gsplits * N_QUAD, nq_pad * KTOP, nq, merge_tmp, MERGE_GROUPS,
                                seed_keys);
                if (s != ST_OK) return s;
            }
            if (h->seed_exchange) {
                if (!run_stage) ST_CHECK_CUDA(h, cudaMemsetAsync(seed_keys, 0, seed_bytes, h->stream));
                s = h->seed_exchange(h, seed_keys, nq, h->seed_ctx);
                if (s != ST_OK) return s;
            }
            if (run_stage || h->seed_exchange) {
                k_knn_seed<<<static_cast<unsigned>((nq + 127) / 128), 128, 0, h->stream>>>(seed_keys,
                                                                                           static_cast<int>(nq), gthr);
                s = st_after_launch(h, "k_knn_seed");
                if (s != ST_OK) return s;
            }
        }
        g.units = static_cast<int>(units);
        g.unit_step = tps;
        g.tile_step = 1;
        g.tiles_per_unit = tps;
        s = run(g, grid);
        if (s != ST_OK) return s;
        return merge_lists(h, unit_out, splits * N_QUAD, nq_pad * KTOP, nq, merge_tmp, MERGE_GROUPS, out_keys);
    }
    const int nqb = static_cast<int>((nq + KQ - 1) / KQ);
    const int64_t tiles = (n_keys + KT - 1) / KT;
    // about eight units per SM, every split non-empty
    int64_t splits = std::max<int64_t>(1, (8LL * h->num_sms + nqb - 1) / nqb);
    splits = std::min(splits, tiles);
    const int64_t tps = (tiles + splits - 1) / splits;
    splits = (tiles + tps - 1) / tps;
    const int64_t units = splits * nqb;
    const int grid = static_cast<int>(std::min<int64_t>(units, h->num_sms));
    const int64_t nq_pad = static_cast<int64_t>(nqb) * KQ;

    uint64_t *cbuf = static_cast<uint64_t *>(st_scratch(h, SLOT_KNN_CAND, sizeof(uint64_t) * grid * NEPI * KCAP));
    const size_t part_bytes = sizeof(uint64_t) * 2 * splits * nq_pad * KTOP;
    uint64_t *unit_out = static_cast<uint64_t *>(st_scratch(h, SLOT_KNN_PART, part_bytes + sizeof(uint32_t) * nq_pad));
    if (!cbuf || !unit_out) return ST_NO_MEMORY;
    uint32_t *gthr = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(unit_out) + part_bytes);
    ST_CHECK_CUDA(h, cudaMemsetAsync(gthr, 0, sizeof(uint32_t) * nq_pad, h->stream));

    ScanArgs g{};
    g.codes = codes;
    g.scales = scales;
    g.q = queries;
    g.n_keys = n_keys;
    g.d = dim;
    g.nq = static_cast<int>(nq);
    g.nq_pad = static_cast<int>(nq_pad);
    g.nqb = nqb;
    g.splits = static_cast<int>(splits);
    g.tiles_per_split = tps;
    g.index_base = static_cast<uint32_t>(index_base);
    g.cbuf = cbuf;
    g.unit_out = unit_out;
    g.ranges = ranges;
    g.always = always;
    g.gthr = gthr;
    g.status = h->d_status;
    if (ranges) {
        if (mode == 0 && prec == 0) s = launch_scan<MODE_DOT, PREC_EXACT, true>(h, g, grid);
        else if (mode == 0) s = launch_scan<MODE_DOT, PREC_F16REF, true>(h, g, grid);
        else if (prec == 0) s = launch_scan<MODE_L2, PREC_EXACT, true>(h, g, grid);
        else s = launch_scan<MODE_L2, PREC_F16REF, true>(h, g, grid);
    } else {
        if (mode == 0 && prec == 0) s = launch_scan<MODE_DOT, PREC_EXACT, false>(h, g, grid);
        else if (mode == 0) s = launch_scan<MODE_DOT, PREC_F16REF, false>(h, g, grid);
        else if (prec == 0) s = launch_scan<MODE_L2, PREC_EXACT, false>(h, g, grid);
        else s = launch_scan<MODE_L2, PREC_F16REF, false>(h, g, grid);
    }
    if (s != ST_OK) return s;
    k_knn_merge<<<static_cast<unsigned>(nq), 256, 0, h->stream>>>(unit_out, 2 * splits, nq_pad * KTOP, out_keys);
    return st_after_launch(h, "k_knn_merge");
}

extern "C" st_status st_knn_scan_units(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_keys,
                                       int32_t dim, const float *queries, int64_t nq, int32_t mode, int32_t prec,
                                       int64_t index_base, int64_t n_units, const int32_t *unit_q,
                                       const int32_t *unit_list, const int64_t *unit_keys, int32_t n_lists,
                                       uint64_t *out_keys) {
    const char *who = "st_knn_scan_units";
    if (!h) return ST_INVALID_ARG;
    st_status s = check_common(h, codes, scales, n_keys, dim, queries, nq, mode, prec, index_base, who);
    if (s != ST_OK) return s;
    if (!out_keys || !unit_q || !unit_list || !unit_keys || n_units < 1 || n_units > (1LL << 30) || n_lists < 1 ||
        n_lists > 4096)
        return h->fail(ST_INVALID_ARG, "%s: bad unit tables", who);
    // the tables are host arrays: every row and range is checked here, before any device read depends on them
    for (int64_t u = 0; u < n_units; u++) {
        const int64_t k0 = unit_keys[2 * u], k1 = unit_keys[2 * u + 1];
        if (k0 < 0 || k1 < k0 || k1 > n_keys) return h->fail(ST_INVALID_ARG, "%s: unit %lld key range", who, (long long)u);
        for (int r = 0; r < KQ; r++) {
            const int32_t q = unit_q[u * KQ + r], l = unit_list[u * KQ + r];
            if (q < -1 || q >= nq || (q >= 0 && (l < 0 || l >= n_lists)))
                return h->fail(ST_INVALID_ARG, "%s: unit %lld row %d", who, (long long)u, r);
        }
    }
    cudaSetDevice(h->device);
    const int nqb = static_cast<int>((nq + KQ - 1) / KQ);
    const int64_t nq_pad = static_cast<int64_t>(nqb) * KQ;
    const int grid = static_cast<int>(std::min<int64_t>(n_units, h->num_sms));
    const size_t tab_bytes = sizeof(int32_t) * 2 * n_units * KQ + sizeof(int64_t) * 2 * n_units;
    uint8_t *tab = static_cast<uint8_t *>(st_scratch(h, SLOT_KNN_UNITS, tab_bytes));
    uint64_t *cbuf = static_cast<uint64_t *>(st_scratch(h, SLOT_KNN_CAND, sizeof(uint64_t) * grid * NEPI * KCAP));
    const size_t out_bytes = sizeof(uint64_t) * 2 * static_cast<size_t>(n_lists) * nq_pad * KTOP;
    uint64_t *unit_out = static_cast<uint64_t *>(st_scratch(h, SLOT_KNN_PART, out_bytes + sizeof(uint32_t) * nq_pad));
    if (!tab || !cbuf || !unit_out) return ST_NO_MEMORY;
    int64_t *d_keys = reinterpret_cast<int64_t *>(tab);
    int32_t *d_q = reinterpret_cast<int32_t *>(tab + sizeof(int64_t) * 2 * n_units);
    int32_t *d_list = d_q + n_units * KQ;
    ST_CHECK_CUDA(h, cudaMemcpyAsync(d_keys, unit_keys, sizeof(int64_t) * 2 * n_units, cudaMemcpyHostToDevice, h->stream));
    ST_CHECK_CUDA(h, cudaMemcpyAsync(d_q, unit_q, sizeof(int32_t) * n_units * KQ, cudaMemcpyHostToDevice, h->stream));
    ST_CHECK_CUDA(h, cudaMemcpyAsync(d_list, unit_list, sizeof(int32_t) * n_units * KQ, cudaMemcpyHostToDevice,
                                     h->stream));
    // lists no unit writes (a query with fewer probes than lists) read as
    // empty; the published thresholds behind them start at none
    ST_CHECK_CUDA(h, cudaMemsetAsync(unit_out, 0, out_bytes + sizeof(uint32_t) * nq_pad, h->stream));

    ScanArgs g{};
    g.codes = codes;
    g.scales = scales;
    g.q = queries;
    g.n_keys = n_keys;
    g.d = dim;
    g.nq = static_cast<int>(nq);
    g.nq_pad = static_cast<int>(nq_pad);
    g.nqb = nqb;
    g.splits = 1;
    g.tiles_per_split = 1;
    g.index_base = static_cast<uint32_t>(index_base);
    g.cbuf = cbuf;
    g.unit_out = unit_out;
    g.unit_q = d_q;
    g.unit_list = d_list;
    g.unit_keys = d_keys;
    g.n_units = static_cast<int>(n_units);
    g.gthr = reinterpret_cast<uint32_t *>(reinterpret_cast<uint8_t *>(unit_out) + out_bytes);
    g.status = h->d_status;
    if (mode == 0 && prec == 0) s = launch_scan<MODE_DOT, PREC_EXACT, false>(h, g, grid);
    else if (mode == 0) s = launch_scan<MODE_DOT, PREC_F16REF, false>(h, g, grid);
    else if (prec == 0) s = launch_scan<MODE_L2, PREC_EXACT, false>(h, g, grid);
    else s = launch_scan<MODE_L2, PREC_F16REF, false>(h, g, grid);
    if (s != ST_OK) return s;
    k_knn_merge<<<static_cast<unsigned>(nq), 256, 0, h->stream>>>(unit_out, 2 * n_lists, nq_pad * KTOP, out_keys);
    return st_after_launch(h, "k_knn_merge");
}

extern "C" st_status st_knn_ivf_units(const int32_t *probes, int64_t nq, int32_t nprobe, const int64_t *starts,
                                      int32_t nlist, int32_t n_sms, int64_t chunk, int32_t max_lists, int32_t *unit_q,
                                      int32_t *unit_list, int64_t *unit_keys, int64_t *n_units, int32_t *n_lists,
                                      int64_t *chunk_used) {
    if (!probes || !starts || nq < 1 || nprobe < 1 || nlist < 1 || !n_units || !n_lists || !chunk_used ||
        nq * nprobe > (1LL << 31))
        return ST_INVALID_ARG;
    for (int64_t i = 0; i < nq * nprobe; i++)
        if (probes[i] < 0 || probes[i] >= nlist) return ST_INVALID_ARG;
    for (int32_t c = 0; c < nlist; c++)
        if (starts[c + 1] < starts[c] || starts[c] < 0) return ST_INVALID_ARG;
    auto size_of = [&](int32_t c) { return starts[c + 1] - starts[c]; };
    auto nch_of = [&](int32_t c, int64_t ch) { return std::max<int64_t>(1, (size_of(c) + ch - 1) / ch); };
    auto lists_needed = [&](int64_t ch) {
        int64_t worst = 0;
        for (int64_t q = 0; q < nq; q++) {
            int64_t t = 0;
            for (int32_t p = 0; p < nprobe; p++) t += nch_of(probes[q * nprobe + p], ch);
            worst = std::max(worst, t);
        }
        return worst;
    };
    std::vector<int64_t> count(nlist, 0);  // queries probing each cell
    for (int64_t i = 0; i < nq * nprobe; i++) count[probes[i]]++;
    if (chunk <= 0) {
        // every probe is at least one list of its query, so fewer than nprobe
        // lists per query cannot be met by any chunk size
        if (max_lists < nprobe) return ST_INVALID_ARG;
        // about two units of work per SM: a cell's keys are scanned once per 128 queries probing it
        int64_t work = 0, largest = 1;
        for (int32_t c = 0; c < nlist; c++)
            if (count[c]) {
                work += size_of(c) * ((count[c] + KQ - 1) / KQ);
                largest = std::max(largest, size_of(c));
            }
        chunk = std::max<int64_t>(16384, (work + 2LL * std::max(1, n_sms) - 1) / (2LL * std::max(1, n_sms)));
        chunk = (chunk + 255) / 256 * 256;
        // once a chunk holds the largest probed cell each probe is one list
        // (nprobe <= max_lists), so the doubling stops there at the latest
        while (lists_needed(chunk) > max_lists && chunk < largest) chunk *= 2;
        if (lists_needed(chunk) > max_lists) return ST_UNSUPPORTED_SHAPE;
    }
    const int64_t nl = lists_needed(chunk);
    if (nl > 4096) return ST_UNSUPPORTED_SHAPE;
    // (cell, chunk) runs in cell order; each (query, probe, chunk) entry joins its run in query order
    std::vector<int64_t> run0(nlist + 1, 0);
    for (int32_t c = 0; c < nlist; c++) run0[c + 1] = run0[c] + (count[c] ? nch_of(c, chunk) : 0);
    const int64_t runs = run0[nlist];
    std::vector<int64_t> unit0(runs + 1, 0);  // first unit of each run
    for (int32_t c = 0; c < nlist; c++)
        for (int64_t j = 0; j < run0[c + 1] - run0[c]; j++)
            unit0[run0[c] + j + 1] = unit0[run0[c] + j] + (count[c] + KQ - 1) / KQ;
    const int64_t nu = unit0[runs];
    *n_units = nu;
    *n_lists = static_cast<int32_t>(nl);
    *chunk_used = chunk;
    if (!unit_q && !unit_list && !unit_keys) return ST_OK;
    if (!unit_q || !unit_list || !unit_keys) return ST_INVALID_ARG;
    // unit -> (cell, chunk) and its key range; then the longest-first order
    std::vector<int64_t> k0(nu), k1(nu);
    for (int32_t c = 0; c < nlist; c++)
        for (int64_t j = 0; j < run0[c + 1] - run0[c]; j++) {
            const int64_t a = starts[c] + j * chunk, b = std::min(starts[c + 1], a + chunk);
            for (int64_t u = unit0[run0[c] + j]; u < unit0[run0[c] + j + 1]; u++) k0[u] = a, k1[u] = b;
        }
    std::vector<int64_t> order(nu), pos(nu);
    for (int64_t u = 0; u < nu; u++) order[u] = u;
    std::stable_sort(order.begin(), order.end(), [&](int64_t x, int64_t y) { return k1[x] - k0[x] > k1[y] - k0[y]; });
    for (int64_t i = 0; i < nu; i++) {
        pos[order[i]] = i;
        unit_keys[2 * i] = k0[order[i]];
        unit_keys[2 * i + 1] = k1[order[i]];
    }
    std::fill(unit_q, unit_q + nu * KQ, -1);
    std::fill(unit_list, unit_list + nu * KQ, 0);
    std::vector<int64_t> fill(runs, 0);
    for (int64_t q = 0; q < nq; q++) {
        int64_t list = 0;
        for (int32_t p = 0; p < nprobe; p++) {
            const int32_t c = probes[q * nprobe + p];
            const int64_t nch = nch_of(c, chunk);
            for (int64_t j = 0; j < nch; j++, list++) {
                const int64_t r = run0[c] + j, k = fill[r]++;
                const int64_t u = pos[unit0[r] + k / KQ];
                unit_q[u * KQ + k % KQ] = static_cast<int32_t>(q);
                unit_list[u * KQ + k % KQ] = static_cast<int32_t>(list);
            }
        }
    }
    return ST_OK;
}

extern "C" st_status st_knn_topk_keys(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_keys,
                                      int32_t dim, const float *queries, int64_t nq, int32_t mode, int32_t prec,
                                      int64_t index_base, uint64_t *out_keys) {
    return topk_keys(h, codes, scales, n_keys, dim, queries, nq, mode, prec, index_base, nullptr, 0, out_keys,
                     "st_knn_topk_keys");
}

extern "C" st_status st_knn_merge_keys(st_handle *h, const uint64_t *lists, int64_t n_lists, int64_t list_stride,
                                       int64_t nq, uint64_t *out_keys) {
    if (!h) return ST_INVALID_ARG;
    if (!lists || !out_keys || n_lists < 1 || nq < 1 || list_stride < nq * KTOP)
        return h->fail(ST_INVALID_ARG, "st_knn_merge_keys: bad arguments");
    cudaSetDevice(h->device);
    k_knn_merge<<<static_cast<unsigned>(nq), 256, 0, h->stream>>>(lists, n_lists, list_stride, out_keys);
    return st_after_launch(h, "k_knn_merge");
}

extern "C" st_status st_knn_decode(st_handle *h, const uint64_t *keys, const float *queries, int64_t nq, int32_t dim,
                                   int32_t k, int32_t mode, int32_t prec, float *out_scores, int64_t *out_ids) {
    if (!h) return ST_INVALID_ARG;
    if (!keys || !queries || !out_scores || !out_ids || nq < 1 || dim < 1 || k < 1 || k > KTOP ||
        (mode != 0 && mode != 1) || (prec != 0 && prec != 1))
        return h->fail(ST_INVALID_ARG, "st_knn_decode: bad arguments (k must be 1..%d)", KTOP);
    cudaSetDevice(h->device);
    if (mode == 0 && prec == 0) return launch_decode<MODE_DOT, PREC_EXACT>(h, keys, queries, nq, dim, k, out_scores, out_ids);
    if (mode == 0) return launch_decode<MODE_DOT, PREC_F16REF>(h, keys, queries, nq, dim, k, out_scores, out_ids);
    if (prec == 0) return launch_decode<MODE_L2, PREC_EXACT>(h, keys, queries, nq, dim, k, out_scores, out_ids);
    return launch_decode<MODE_L2, PREC_F16REF>(h, keys, queries, nq, dim, k, out_scores, out_ids);
}

extern "C" st_status st_knn_search(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_keys,
                                   int32_t dim, const float *queries, int64_t nq, int32_t k, int32_t mode,
                                   int32_t prec, int64_t index_base, float *out_scores, int64_t *out_ids) {
    if (!h) return ST_INVALID_ARG;
    if (k < 1 || k > KTOP) return h->fail(ST_INVALID_ARG, "st_knn_search: k must be 1..%d", KTOP);
    if (!out_scores || !out_ids) return h->fail(ST_INVALID_ARG, "st_knn_search: null output");
    uint64_t *keys = static_cast<uint64_t *>(st_scratch(h, SLOT_KNN_MISC, sizeof(uint64_t) * std::max<int64_t>(nq, 1) * KTOP));
    if (!keys) return ST_NO_MEMORY;
    st_status s = st_knn_topk_keys(h, codes, scales, n_keys, dim, queries, nq, mode, prec, index_base, keys);
    if (s != ST_OK) return s;
    return st_knn_decode(h, keys, queries, nq, dim, k, mode, prec, out_scores, out_ids);
}

extern "C" st_status st_knn_quantize(st_handle *h, const float *keys, int64_t n, int32_t dim, uint8_t *codes,
                                     float *scales, float *norms) {
    if (!h) return ST_INVALID_ARG;
    if (!keys || !codes || !scales || n < 1 || dim < 4 || dim % 4 != 0)
        return h->fail(ST_INVALID_ARG, "st_knn_quantize: bad arguments");
    cudaSetDevice(h->device);
    const int blocks = static_cast<int>(std::min<int64_t>((n + 127) / 128, 65535));
    k_knn_quantize<<<blocks, 128, 0, h->stream>>>(keys, n, dim, codes, scales, norms);
    return st_after_launch(h, "k_knn_quantize");
}

extern "C" st_status st_knn_synth_keys(st_handle *h, uint8_t *codes, float *scales, int64_t n, int32_t dim,
                                       uint64_t seed, int64_t first_key) {
    if (!h) return ST_INVALID_ARG;
    if (!codes || !scales || n < 1 || dim < 32 || dim % 32 != 0 || !aligned16(codes))
        return h->fail(ST_INVALID_ARG, "st_knn_synth_keys: bad arguments");
    cudaSetDevice(h->device);
    const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 8 * 148 * 4));
    k_knn_synth<<<blocks, 256, 0, h->stream>>>(codes, scales, n, dim, seed, first_key);
    return st_after_launch(h, "k_knn_synth");
}

extern "C" st_status st_knn_search_masked(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_keys,
                                          int32_t dim, const float *queries, int64_t nq, int32_t k, int32_t mode,
                                          int32_t prec, int64_t index_base, const int64_t *ranges, int64_t always,
                                          float *out_scores, int64_t *out_ids) {
    if (!h) return ST_INVALID_ARG;
    if (k < 1 || k > KTOP) return h->fail(ST_INVALID_ARG, "st_knn_search_masked: k must be 1..%d", KTOP);
    if (!out_scores || !out_ids || !ranges || always < 0)
        return h->fail(ST_INVALID_ARG, "st_knn_search_masked: null output or ranges, or negative always");
    uint64_t *keys = static_cast<uint64_t *>(st_scratch(h, SLOT_KNN_MISC, sizeof(uint64_t) * std::max<int64_t>(nq, 1) * KTOP));
    if (!keys) return ST_NO_MEMORY;
    st_status s = topk_keys(h, codes, scales, n_keys, dim, queries, nq, mode, prec, index_base, ranges, always, keys,
                            "st_knn_search_masked");
    if (s != ST_OK) return s;
    return st_knn_decode(h, keys, queries, nq, dim, k, mode, prec, out_scores, out_ids);
}

// ---- IVF building blocks ---------------------------------------------------

extern "C" st_status st_knn_dequant(st_handle *h, const uint8_t *codes, const float *scales, int64_t n, int32_t dim,
                                    float *out) {
    if (!h) return ST_INVALID_ARG;
    if (!codes || !scales || !out || n < 1 || dim < 4 || dim % 4 != 0)
        return h->fail(ST_INVALID_ARG, "st_knn_dequant: bad arguments");
    cudaSetDevice(h->device);
    const int64_t nb = n * (dim / 4);
    k_knn_dequant<<<static_cast<unsigned>((nb + 255) / 256), 256, 0, h->stream>>>(codes, scales, n, dim, out);
    return st_after_launch(h, "k_knn_dequant");
}

extern "C" st_status st_knn_nearest(st_handle *h, const float *dots, const float *cnorm, int64_t n, int32_t nlist,
                                    int32_t *out) {
    if (!h) return ST_INVALID_ARG;
    if (!dots || !cnorm || !out || n < 1 || nlist < 1) return h->fail(ST_INVALID_ARG, "st_knn_nearest: bad arguments");
    cudaSetDevice(h->device);
    k_knn_nearest<<<static_cast<unsigned>((n + 7) / 8), 256, 0, h->stream>>>(dots, cnorm, n, nlist, out);
    return st_after_launch(h, "k_knn_nearest");
}

extern "C" st_status st_knn_probe(st_handle *h, const float *dots, const float *cnorm, int64_t nq, int32_t nlist,
                                  int32_t nprobe, int32_t *out) {
    if (!h) return ST_INVALID_ARG;
    if (!dots || !cnorm || !out || nq < 1 || nlist < 1 || nprobe < 1 || nprobe > nlist || nprobe > 64)
        return h->fail(ST_INVALID_ARG, "st_knn_probe: bad arguments (1 <= nprobe <= min(nlist, 64))");
    cudaSetDevice(h->device);
    if (nprobe <= 8) {
        k_knn_probe_small<8><<<static_cast<unsigned>((nq + 7) / 8), 256, 0, h->stream>>>(dots, cnorm, nq, nlist, nprobe,
                                                                                         out);
        return st_after_launch(h, "k_knn_probe_small");
    }
    k_knn_probe<<<static_cast<unsigned>((nq + 7) / 8), 256, 0, h->stream>>>(dots, cnorm, nq, nlist, nprobe, out);
    return st_after_launch(h, "k_knn_probe");
}

extern "C" st_status st_gather_rows(st_handle *h, const void *src, int64_t n_src, void *dst, const int64_t *perm,
                                    int64_t n, int64_t row_bytes) {
    if (!h) return ST_INVALID_ARG;
    if (!src || !dst || !perm || n < 1 || n_src < 1 || row_bytes < 4 || row_bytes % 4 != 0 || row_bytes > (1 << 20))
        return h->fail(ST_INVALID_ARG, "st_gather_rows: bad arguments");
    cudaSetDevice(h->device);
    const int words = static_cast<int>(row_bytes / 4);
    const int64_t total = n * words;
    k_gather_rows<<<static_cast<unsigned>((total + 255) / 256), 256, 0, h->stream>>>(
        static_cast<const uint32_t *>(src), n_src, static_cast<uint32_t *>(dst), perm, n, words, h->d_status);
    return st_after_launch(h, "k_gather_rows");
}
