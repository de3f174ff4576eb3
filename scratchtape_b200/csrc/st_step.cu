// st_step.cu -- the row and elementwise kernels of the byte-level transformer
// training step that surround its GEMMs and attention: token + position
// embedding, LayerNorm, cross-entropy, Adam.
//
// Reference (src/gpu_step): k_embed / k_embed_bwd_tok / k_embed_bwd_pos
// (tokens.rs:125-192), k_ln_fwd / k_ln_bwd_dx / k_ln_bwd_params
// (rows.rs:177-293, biased variance), k_ce_rows / k_ce_bwd (tokens.rs:194-253),
// and Adam (src/optim.rs:42-57; the reference runs it on the CPU).  As in the
// reference, every reduction has a fixed order (no float atomics), so a step
// is bit-reproducible.
//
// Layout: rows of d = 256 floats (one warp per row, lane owning columns lane,
// lane + 32, ... so that every load of the warp is one coalesced line), vocab 256.
#include <algorithm>

#include "st_internal.h"
#include "st_ptx.cuh"

namespace {

// Every kernel below is launched programmatically dependent on the previous
// kernel of the stream (st_launch_dependent) and begins with this: wait for
// that kernel's results, then let the next kernel's launch begin.
__device__ __forceinline__ void dep_enter() {
    st::grid_dep_wait();
    st::grid_dep_launch();
}

constexpr int MAXD = 1024;  // widest row the per-warp kernels take (32 lanes x 32)

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max_f(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// x[r, :] = tok[ids[r], :] + pos[r % t, :]
__global__ void k_embed_fwd(const int32_t *ids, const float *tok, const float *pos, float *x, int64_t rows, int t,
                            int d) {
    dep_enter();
    const int64_t n4 = rows * d / 4;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t e = i * 4;
        const int64_t r = e / d;
        const int c = static_cast<int>(e % d);
        const float4 a = *reinterpret_cast<const float4 *>(tok + static_cast<int64_t>(ids[r]) * d + c);
        const float4 b = *reinterpret_cast<const float4 *>(pos + static_cast<int64_t>(r % t) * d + c);
        *reinterpret_cast<float4 *>(x + e) = make_float4(a.x + b.x, a.y + b.y, a.z + b.z, a.w + b.w);
    }
}

// dtok[v, :] (+)= sum over rows r with ids[r] == v, in row order, of dx[r, :].
// One block per vocabulary row.  The block walks the ids in segments of
// EMB_SEG (every thread loads its EMB_SEG / EMB_THREADS ids of a segment
// before any test, so a segment costs one round trip), compacts the matching
// row numbers into shared memory in row order (warp ballots, warp offsets from
// a prefix over the warps), then every thread adds those rows for its
// columns, EMB_UNROLL loads in flight, the additions still in row order.
constexpr int EMB_THREADS = 256, EMB_SEG = 2048, EMB_UNROLL = 8;
__global__ void __launch_bounds__(EMB_THREADS) k_embed_bwd_tok(const int32_t *ids, const float *dx, float *dtok,
                                                               int64_t rows, int d, int vocab, int accumulate) {
    __shared__ int64_t list[EMB_SEG];
    __shared__ int warp_n[EMB_THREADS / 32];
    dep_enter();
    const int v = blockIdx.x;
    const int tid = threadIdx.x, warp = tid / 32, lane = tid & 31;
    constexpr int PER = MAXD / EMB_THREADS;
    float acc[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) acc[j] = 0.0f;
    for (int64_t s0 = 0; s0 < rows; s0 += EMB_SEG) {
        int32_t idv[EMB_SEG / EMB_THREADS];
#pragma unroll
        for (int i = 0; i < EMB_SEG / EMB_THREADS; i++) {
            const int64_t r = s0 + i * EMB_THREADS + tid;
            idv[i] = r < rows ? ids[r] : -1;  // ids are vocabulary rows, never negative
        }
        int n = 0;  // rows listed so far in this segment (the same in every thread)
#pragma unroll
        for (int i = 0; i < EMB_SEG; i += EMB_THREADS) {
            const int64_t r = s0 + i + tid;
            const bool hit = idv[i / EMB_THREADS] == v;
            const unsigned m = __ballot_sync(0xffffffffu, hit);
            if (lane == 0) warp_n[warp] = __popc(m);
            __syncthreads();
            int off = n, tot = 0;
#pragma unroll
            for (int w = 0; w < EMB_THREADS / 32; w++) {
                if (w < warp) off += warp_n[w];
                tot += warp_n[w];
            }
            if (hit) list[off + __popc(m & ((1u << lane) - 1u))] = r;
            n += tot;
            __syncthreads();
        }
        int e = 0;
        for (; e + EMB_UNROLL <= n; e += EMB_UNROLL) {
#pragma unroll
            for (int j = 0; j < PER; j++) {
                const int c = tid + j * EMB_THREADS;
                if (c < d) {
                    float x[EMB_UNROLL];
#pragma unroll
                    for (int u = 0; u < EMB_UNROLL; u++) x[u] = dx[list[e + u] * d + c];
#pragma unroll
                    for (int u = 0; u < EMB_UNROLL; u++) acc[j] += x[u];
                }
            }
        }
        for (; e < n; e++) {
#pragma unroll
            for (int j = 0; j < PER; j++) {
                const int c = tid + j * EMB_THREADS;
                if (c < d) acc[j] += dx[list[e] * d + c];
            }
        }
        __syncthreads();  // the list is rewritten by the next segment
    }
    float *out = dtok + static_cast<int64_t>(v) * d;
#pragma unroll
    for (int j = 0; j < PER; j++) {
        const int c = tid + j * EMB_THREADS;
        if (c < d) out[c] = accumulate ? out[c] + acc[j] : acc[j];
    }
}

// dpos[i, c] (+)= sum over b ascending of dx[b*t + i, c]
__global__ void k_embed_bwd_pos(const float *dx, float *dpos, int batch, int t, int d, int accumulate) {
    dep_enter();
    const int64_t n = static_cast<int64_t>(t) * d;
    for (int64_t e = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; e < n;
         e += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float s = 0.0f;
        for (int b = 0; b < batch; b++) s += dx[static_cast<int64_t>(b) * n + e];
        dpos[e] = accumulate ? dpos[e] + s : s;
    }
}

// y = (x - mean) * rstd * gamma + beta, rstd = 1 / sqrt(var + eps), biased var.
// One warp per row; lane owns columns lane, lane + 32, ... (coalesced).
__global__ void k_ln_fwd(const float *x, const float *gamma, const float *beta, float *y, float *mean, float *rstd,
                         int64_t rows, int d, float eps) {
    dep_enter();
    const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int per = d / 32;
    const float *xr = x + r * d + lane;
    float v[MAXD / 32];
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < MAXD / 32; j++)
        if (j < per) {
            v[j] = xr[32 * j];
            s += v[j];
        }
    const float mu = warp_sum_f(s) / static_cast<float>(d);
    float q = 0.0f;
#pragma unroll
    for (int j = 0; j < MAXD / 32; j++)
        if (j < per) {
            const float c = v[j] - mu;
            q += c * c;
        }
    const float var = warp_sum_f(q) / static_cast<float>(d);
    const float rs = 1.0f / sqrtf(var + eps);
    float *yr = y + r * d + lane;
#pragma unroll
    for (int j = 0; j < MAXD / 32; j++)
        if (j < per) yr[32 * j] = (v[j] - mu) * rs * gamma[lane + 32 * j] + beta[lane + 32 * j];
    if (lane == 0) {
        mean[r] = mu;
        rstd[r] = rs;
    }
}

// dx (+)= rstd * (g - mean(g) - xhat * mean(g * xhat)), g = dy * gamma.
// Each block takes LN_WARPS * RPW consecutive rows (warp w: rows w, w + 8,
// ..., RPW of them, RPW * PER <= 32 so a warp's rows fit its registers); a
// warp loads every row's dy, x (and dx) before any arithmetic, so its loads
// are in flight together.  The block also writes its partial parameter
// gradients -- per column, over its rows, sum of dy * xhat and of dy, rows
// in order within a warp, warps combined in warp order -- to
// part[block][2][d]; k_ln_params_sum adds the blocks in block order.
constexpr int LN_WARPS = 8, LN_MAXD = 512;  // LN_MAXD: widest row of the backward
template <int PER, int RPW>
__global__ void __launch_bounds__(LN_WARPS * 32) k_ln_bwd(const float *dy, const float *x, const float *gamma,
                                                          const float *mean, const float *rstd, float *dx, float *part,
                                                          int64_t rows, int accumulate) {
    constexpr int D = 32 * PER;
    __shared__ float sh[LN_WARPS][2][D];
    dep_enter();
    const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
    const int64_t row0 = blockIdx.x * static_cast<int64_t>(LN_WARPS * RPW);
    float dyv[RPW][PER], xv[RPW][PER], dxv[RPW][PER], mu[RPW], rs[RPW];
#pragma unroll
    for (int i = 0; i < RPW; i++) {
        const int64_t r = row0 + warp + static_cast<int64_t>(LN_WARPS) * i;
        const bool in = r < rows;
        mu[i] = in ? mean[r] : 0.0f;
        rs[i] = in ? rstd[r] : 0.0f;
#pragma unroll
        for (int j = 0; j < PER; j++) {
            const int64_t e = r * D + lane + 32 * j;
            dyv[i][j] = in ? dy[e] : 0.0f;
            xv[i][j] = in ? x[e] : 0.0f;
            dxv[i][j] = in && accumulate ? dx[e] : 0.0f;
        }
    }
    float gam[PER], pg[PER], pb[PER];
#pragma unroll
    for (int j = 0; j < PER; j++) {
        gam[j] = gamma[lane + 32 * j];
        pg[j] = pb[j] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < RPW; i++) {
        const int64_t r = row0 + warp + static_cast<int64_t>(LN_WARPS) * i;
        float gv[PER], xh[PER];
        float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
        for (int j = 0; j < PER; j++) {
            xh[j] = (xv[i][j] - mu[i]) * rs[i];
            gv[j] = dyv[i][j] * gam[j];
            s1 += gv[j];
            s2 += gv[j] * xh[j];
            pg[j] += dyv[i][j] * xh[j];  // rows beyond the end add dy = 0
            pb[j] += dyv[i][j];
        }
        const float m1 = warp_sum_f(s1) / static_cast<float>(D), m2 = warp_sum_f(s2) / static_cast<float>(D);
        if (r < rows) {
#pragma unroll
            for (int j = 0; j < PER; j++) {
                const int64_t e = r * D + lane + 32 * j;
                const float g = rs[i] * (gv[j] - m1 - xh[j] * m2);
                dx[e] = accumulate ? dxv[i][j] + g : g;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < PER; j++) {
        sh[warp][0][lane + 32 * j] = pg[j];
        sh[warp][1][lane + 32 * j] = pb[j];
    }
    __syncthreads();
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
        float sg = 0.0f, sb = 0.0f;
        for (int w = 0; w < LN_WARPS; w++) {
            sg += sh[w][0][c];
            sb += sh[w][1][c];
        }
        part[(static_cast<int64_t>(blockIdx.x) * 2) * D + c] = sg;
        part[(static_cast<int64_t>(blockIdx.x) * 2 + 1) * D + c] = sb;
    }
}

// dgamma[c] += sum of part[b][0][c], dbeta[c] += sum of part[b][1][c] over
// blocks b.  Block = 32 columns x 32 row groups: thread (g, c) adds blocks g,
// g + 32, ... in order with eight loads in flight (a warp's load is 32
// consecutive columns, one 128-byte line), so 256 blocks take one round trip;
// the 32 group sums are then added in a fixed tree (group g + w into g for
// w = 16, 8, 4, 2, 1).
constexpr int LNP_GROUPS = 32;
__global__ void __launch_bounds__(32 * LNP_GROUPS) k_ln_params_sum(const float *part, float *dgamma, float *dbeta,
                                                                   int d, int nblocks) {
    __shared__ float sg_s[LNP_GROUPS][32], sb_s[LNP_GROUPS][32];
    dep_enter();
    const int cl = threadIdx.x & 31, grp = threadIdx.x >> 5;
    const int c = blockIdx.x * 32 + cl;
    float sg = 0.0f, sb = 0.0f;
    if (c < d) {
        for (int b0 = grp; b0 < nblocks; b0 += 8 * LNP_GROUPS) {
            float vg[8], vb[8];
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int b = b0 + LNP_GROUPS * j;
                vg[j] = b < nblocks ? part[(static_cast<int64_t>(b) * 2) * d + c] : 0.0f;
                vb[j] = b < nblocks ? part[(static_cast<int64_t>(b) * 2 + 1) * d + c] : 0.0f;
            }
#pragma unroll
            for (int j = 0; j < 8; j++) {
                sg += vg[j];
                sb += vb[j];
            }
        }
    }
    sg_s[grp][cl] = sg;
    sb_s[grp][cl] = sb;
    __syncthreads();
#pragma unroll
    for (int w = LNP_GROUPS / 2; w > 0; w >>= 1) {
        if (grp < w) {
            sg_s[grp][cl] += sg_s[grp + w][cl];
            sb_s[grp][cl] += sb_s[grp + w][cl];
        }
        __syncthreads();
    }
    if (grp == 0 && c < d) {
        dgamma[c] += sg_s[0][cl];
        dbeta[c] += sb_s[0][cl];
    }
}

// Per row: loss_r = log(sum exp(x - max)) + max - x[y];
// dlogits = (softmax(x) - onehot(y)) * grad_scale.
__global__ void k_ce(const float *logits, const int32_t *targets, float *loss_rows, float *dlogits, int64_t rows,
                     int vocab, float grad_scale) {
    dep_enter();
    const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const int per = vocab / 32;
    const float *xr = logits + r * vocab + lane;
    float v[MAXD / 32];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < MAXD / 32; j++)
        if (j < per) {
            v[j] = xr[32 * j];
            m = fmaxf(m, v[j]);
        }
    m = warp_max_f(m);
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < MAXD / 32; j++)
        if (j < per) {
            v[j] = expf(v[j] - m);
            s += v[j];
        }
    s = warp_sum_f(s);
    const int y = targets[r];
    if (lane == 0) loss_rows[r] = logf(s) + m - logits[r * vocab + y];
    const float inv = 1.0f / s;
    if (dlogits) {
        float *dr = dlogits + r * vocab + lane;
#pragma unroll
        for (int j = 0; j < MAXD / 32; j++)
            if (j < per) dr[32 * j] = (v[j] * inv - (lane + 32 * j == y ? 1.0f : 0.0f)) * grad_scale;
    }
}

// out[0] = mean of x[0..n): per-thread strided sums, then a fixed tree.
__global__ void k_mean(const float *x, int64_t n, float *out) {
    __shared__ float sh[1024];
    dep_enter();
    float s = 0.0f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) s += x[i];
    sh[threadIdx.x] = s;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) sh[threadIdx.x] += sh[threadIdx.x + w];
        __syncthreads();
    }
    if (threadIdx.x == 0) out[0] = sh[0] / static_cast<float>(n);
}

// Adam (src/optim.rs:42-57) in the reference's f32 operation order:
// m = m*b1 + g*(1-b1); v = v*b2 + (g*g)*(1-b2); u = (m*i1 / (sqrt(v*i2) + eps)) * lr
__global__ void k_adam(float *p, const float *g, float *m, float *v, int64_t n, float lr, float b1, float b2, float eps,
                       float i1, float i2) {
    const float c1 = __fsub_rn(1.0f, b1), c2 = __fsub_rn(1.0f, b2);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float gi = g[i];
        const float mi = __fadd_rn(__fmul_rn(m[i], b1), __fmul_rn(gi, c1));
        const float vi = __fadd_rn(__fmul_rn(v[i], b2), __fmul_rn(__fmul_rn(gi, gi), c2));
        m[i] = mi;
        v[i] = vi;
        const float mh = __fmul_rn(mi, i1), vh = __fmul_rn(vi, i2);
        const float u = __fmul_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), eps)), lr);
        p[i] = __fsub_rn(p[i], u);
    }
}

// The step counter lives on the device, so a captured step replays correctly.
__global__ void k_step_inc(int32_t *step) {
    dep_enter();
    step[0] += 1;
}

__device__ __forceinline__ float powi_dev(float a, int b) {  // the host powi_f32, op for op
    float r = 1.0f;
    for (;;) {
        if (b & 1) r = __fmul_rn(r, a);
        b /= 2;
        if (b == 0) break;
        a = __fmul_rn(a, a);
    }
    return r;
}

// One Adam element in the reference's operation order (the same bits as k_adam).
struct AdamK {
    float b1, b2, c1, c2, i1, i2, lr, eps;
    __device__ __forceinline__ void operator()(float &p, float g, float &m, float &v) const {
        m = __fadd_rn(__fmul_rn(m, b1), __fmul_rn(g, c1));
        v = __fadd_rn(__fmul_rn(v, b2), __fmul_rn(__fmul_rn(g, g), c2));
        const float mh = __fmul_rn(m, i1), vh = __fmul_rn(v, i2);
        const float u = __fmul_rn(__fdiv_rn(mh, __fadd_rn(__fsqrt_rn(vh), eps)), lr);
        p = __fsub_rn(p, u);
    }
};

// VEC4: every pointer 16-byte aligned and n % 4 == 0, four elements per float4.
template <bool VEC4>
__global__ void k_adam_dev(float *p, const float *g, float *m, float *v, int64_t n, const int32_t *step, float lr,
                           float b1, float b2, float eps) {
    dep_enter();
    const int t = step[0];
    const AdamK a{b1, b2, __fsub_rn(1.0f, b1), __fsub_rn(1.0f, b2), __fdiv_rn(1.0f, __fsub_rn(1.0f, powi_dev(b1, t))),
                  __fdiv_rn(1.0f, __fsub_rn(1.0f, powi_dev(b2, t))), lr, eps};
    if (VEC4) {
        for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n / 4;
             i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
            float4 pi = reinterpret_cast<float4 *>(p)[i], mi = reinterpret_cast<float4 *>(m)[i];
            float4 vi = reinterpret_cast<float4 *>(v)[i];
            const float4 gi = reinterpret_cast<const float4 *>(g)[i];
            a(pi.x, gi.x, mi.x, vi.x);
            a(pi.y, gi.y, mi.y, vi.y);
            a(pi.z, gi.z, mi.z, vi.z);
            a(pi.w, gi.w, mi.w, vi.w);
            reinterpret_cast<float4 *>(m)[i] = mi;
            reinterpret_cast<float4 *>(v)[i] = vi;
            reinterpret_cast<float4 *>(p)[i] = pi;
        }
    } else {
        for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
             i += static_cast<int64_t>(gridDim.x) * blockDim.x)
            a(p[i], g[i], m[i], v[i]);
    }
}

int blocks_for(int64_t n, int threads) {
    return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, 148 * 16)));
}

float powi_f32(float a, int b) {  // square-and-multiply, as Rust's f32::powi lowers
    float r = 1.0f;
    for (;;) {
        if (b & 1) r *= a;
        b /= 2;
        if (b == 0) break;
        a *= a;
    }
    return r;
}

}  // namespace

extern "C" st_status st_embed_fwd(st_handle *h, const int32_t *ids, const float *tok, const float *pos, float *x,
                                  int64_t batch, int64_t t, int64_t d) {
    if (!h) return ST_INVALID_ARG;
    if (!ids || !tok || !pos || !x || batch < 1 || t < 1 || d < 4 || d % 4 != 0)
        return h->fail(ST_INVALID_ARG, "st_embed_fwd: bad arguments");
    cudaSetDevice(h->device);
    const int64_t rows = batch * t;
    ST_CHECK_CUDA(h, st_launch_dependent(h, k_embed_fwd, dim3(blocks_for(rows * d / 4, 256)), dim3(256), 0, ids, tok,
                                         pos, x, rows, static_cast<int>(t), static_cast<int>(d)));
    return st_after_launch(h, "k_embed_fwd");
}

extern "C" st_status st_embed_bwd(st_handle *h, const int32_t *ids, const float *dx, float *dtok, float *dpos,
                                  int64_t batch, int64_t t, int64_t d, int64_t vocab, int32_t accumulate) {
    if (!h) return ST_INVALID_ARG;
    if (!ids || !dx || !dtok || !dpos || batch < 1 || t < 1 || d < 32 || d % 32 != 0 || d > MAXD || vocab < 1 ||
        vocab > (1LL << 30))
        return h->fail(ST_INVALID_ARG, "st_embed_bwd: bad arguments");
    cudaSetDevice(h->device);
    ST_CHECK_CUDA(h, st_launch_dependent(h, k_embed_bwd_tok, dim3(static_cast<unsigned>(vocab)), dim3(EMB_THREADS), 0,
                                         ids, dx, dtok, batch * t, static_cast<int>(d), static_cast<int>(vocab),
                                         accumulate));
    st_status s = st_after_launch(h, "k_embed_bwd_tok");
    if (s != ST_OK) return s;
    ST_CHECK_CUDA(h, st_launch_dependent(h, k_embed_bwd_pos, dim3(blocks_for(t * d, 256)), dim3(256), 0, dx, dpos,
                                         static_cast<int>(batch), static_cast<int>(t), static_cast<int>(d),
                                         accumulate));
    return st_after_launch(h, "k_embed_bwd_pos");
}

extern "C" st_status st_layernorm_fwd(st_handle *h, const float *x, const float *gamma, const float *beta, float *y,
                                      float *mean, float *rstd, int64_t rows, int64_t d, float eps) {
    if (!h) return ST_INVALID_ARG;
    if (!x || !gamma || !beta || !y || !mean || !rstd || rows < 1 || d < 32 || d % 32 != 0 || d > MAXD)
        return h->fail(ST_INVALID_ARG, "st_layernorm_fwd: bad arguments (d a multiple of 32 up to %d)", MAXD);
    cudaSetDevice(h->device);
    const int wpb = 8;
    ST_CHECK_CUDA(h, st_launch_dependent(h, k_ln_fwd, dim3(static_cast<unsigned>((rows + wpb - 1) / wpb)),
                                         dim3(32 * wpb), 0, x, gamma, beta, y, mean, rstd, rows, static_cast<int>(d),
                                         eps));
    return st_after_launch(h, "k_ln_fwd");
}

extern "C" st_status st_layernorm_bwd(st_handle *h, const float *dy, const float *x, const float *gamma,
                                      const float *mean, const float *rstd, float *dx, float *dgamma, float *dbeta,
                                      int64_t rows, int64_t d, int32_t accumulate) {
    if (!h) return ST_INVALID_ARG;
    if (!dy || !x || !gamma || !mean || !rstd || !dx || !dgamma || !dbeta || rows < 1 || d < 32 || d % 32 != 0 ||
        d > LN_MAXD)
        return h->fail(ST_INVALID_ARG, "st_layernorm_bwd: bad arguments (d a multiple of 32 up to %d)", LN_MAXD);
    cudaSetDevice(h->device);
    // rows per warp: as many as fit 32 registers of each of dy, x, dx
    const int per = static_cast<int>(d / 32), rpw = std::max(1, 32 / per);
    const int64_t block_rows = static_cast<int64_t>(LN_WARPS) * rpw;
    const int64_t nblocks = (rows + block_rows - 1) / block_rows;
    if (nblocks > (1LL << 31) - 1) return h->fail(ST_UNSUPPORTED_SHAPE, "st_layernorm_bwd: too many rows");
    float *part = static_cast<float *>(st_scratch(h, SLOT_STEP, sizeof(float) * 2 * nblocks * d));
    if (!part) return ST_NO_MEMORY;
    const dim3 grid(static_cast<unsigned>(nblocks)), block(LN_WARPS * 32);
    switch (per) {
#define ST_LN_BWD(P)                                                                                     \
    case P:                                                                                              \
        ST_CHECK_CUDA(h, st_launch_dependent(h, k_ln_bwd<P, (32 / P > 1 ? 32 / P : 1)>, grid, block, 0, dy, x, \
                                             gamma, mean, rstd, dx, part, rows, accumulate));                 \
        break;
        ST_LN_BWD(1) ST_LN_BWD(2) ST_LN_BWD(3) ST_LN_BWD(4) ST_LN_BWD(5) ST_LN_BWD(6) ST_LN_BWD(7) ST_LN_BWD(8)
        ST_LN_BWD(9) ST_LN_BWD(10) ST_LN_BWD(11) ST_LN_BWD(12) ST_LN_BWD(13) ST_LN_BWD(14) ST_LN_BWD(15)
        ST_LN_BWD(16)
#undef ST_LN_BWD
        default:
            return h->fail(ST_INVALID_ARG, "st_layernorm_bwd: d = %lld", static_cast<long long>(d));
    }
    st_status s = st_after_launch(h, "k_ln_bwd");
    if (s != ST_OK) return s;
    ST_CHECK_CUDA(h, st_launch_dependent(h, k_ln_params_sum, dim3(static_cast<unsigned>((d + 31) / 32)),
                                         dim3(32 * LNP_GROUPS), 0, part, dgamma, dbeta, static_cast<int>(d),
                                         static_cast<int>(nblocks)));
    return st_after_launch(h, "k_ln_params_sum");
}

extern "C" st_status st_cross_entropy(st_handle *h, const float *logits, const int32_t *targets, float *loss,
                                      float *dlogits, int64_t rows, int64_t vocab) {
    if (!h) return ST_INVALID_ARG;
    if (!logits || !targets || !loss || rows < 1 || vocab < 32 || vocab % 32 != 0 || vocab > MAXD)
        return h->fail(ST_INVALID_ARG, "st_cross_entropy: bad arguments");
    cudaSetDevice(h->device);
    float *loss_rows = static_cast<float *>(st_scratch(h, SLOT_STEP_ROWS, sizeof(float) * rows));
    if (!loss_rows) return ST_NO_MEMORY;
    const int wpb = 8;
    ST_CHECK_CUDA(h, st_launch_dependent(h, k_ce, dim3(static_cast<unsigned>((rows + wpb - 1) / wpb)), dim3(32 * wpb),
                                         0, logits, targets, loss_rows, dlogits, rows, static_cast<int>(vocab),
                                         1.0f / static_cast<float>(rows)));
    st_status s = st_after_launch(h, "k_ce");
    if (s != ST_OK) return s;
    ST_CHECK_CUDA(h, st_launch_dependent(h, k_mean, dim3(1), dim3(1024), 0, loss_rows, rows, loss));
    return st_after_launch(h, "k_mean");
}

extern "C" st_status st_adam(st_handle *h, float *p, const float *g, float *m, float *v, int64_t n, int32_t step,
                             float lr, float beta1, float beta2, float eps) {
    if (!h) return ST_INVALID_ARG;
    if (!p || !g || !m || !v || n < 1 || step < 1) return h->fail(ST_INVALID_ARG, "st_adam: bad arguments");
    cudaSetDevice(h->device);
    const float bc1 = 1.0f - powi_f32(beta1, step), bc2 = 1.0f - powi_f32(beta2, step);
    k_adam<<<blocks_for(n, 256), 256, 0, h->stream>>>(p, g, m, v, n, lr, beta1, beta2, eps, 1.0f / bc1, 1.0f / bc2);
    return st_after_launch(h, "k_adam");
}

extern "C" st_status st_adam_dev(st_handle *h, float *p, const float *g, float *m, float *v, int64_t n, int32_t *step,
                                 float lr, float beta1, float beta2, float eps) {
    if (!h) return ST_INVALID_ARG;
    if (!p || !g || !m || !v || !step || n < 1) return h->fail(ST_INVALID_ARG, "st_adam_dev: bad arguments");
    cudaSetDevice(h->device);
    ST_CHECK_CUDA(h, st_launch_dependent(h, k_step_inc, dim3(1), dim3(1), 0, step));
    st_status s = st_after_launch(h, "k_step_inc");
    if (s != ST_OK) return s;
    const bool vec4 = n % 4 == 0 && ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
                                      reinterpret_cast<uintptr_t>(m) | reinterpret_cast<uintptr_t>(v)) & 15u) == 0;
    if (vec4)
        ST_CHECK_CUDA(h, st_launch_dependent(h, k_adam_dev<true>, dim3(blocks_for(n / 4, 256)), dim3(256), 0, p, g, m,
                                             v, n, step, lr, beta1, beta2, eps));
    else
        ST_CHECK_CUDA(h, st_launch_dependent(h, k_adam_dev<false>, dim3(blocks_for(n, 256)), dim3(256), 0, p, g, m, v,
                                             n, step, lr, beta1, beta2, eps));
    return st_after_launch(h, "k_adam_dev");
}
