// st_rows.cu -- row softmax forward / backward.
//
// Reference: rows::softmax / softmax_backward and k_softmax_fwd / k_softmax_bwd
// (src/gpu_step/rows.rs:106-123, :295-357): row r of scale*x, causal rows see
// columns 0..=r%t (the rest exactly 0), softmax1 shifts by max(row max, 0)
// and adds exp(-shift) to the denominator.  One warp per row; reductions are
// a fixed butterfly, so results are deterministic.
#include "st_internal.h"

namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__global__ void k_softmax_rows(const float *x, float *y, int64_t rows, int n, int t, float scale, int causal,
                               int one) {
    const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const float *xr = x + r * n;
    float *yr = y + r * n;
    const int limit = causal ? static_cast<int>(r % t) + 1 : n;
    float m = -INFINITY;
    for (int j = lane; j < limit; j += 32) m = fmaxf(m, scale * xr[j]);
    m = warp_max(m);
    if (one && m < 0.0f) m = 0.0f;
    float s = 0.0f;
    for (int j = lane; j < limit; j += 32) s += expf(scale * xr[j] - m);
    s = warp_sum(s);
    if (one) s += expf(-m);
    const float inv = 1.0f / s;
    for (int j = lane; j < n; j += 32) yr[j] = j < limit ? expf(scale * xr[j] - m) * inv : 0.0f;
}

__global__ void k_softmax_rows_bwd(const float *dy, const float *y, float *dx, int64_t rows, int n, float scale) {
    const int64_t r = blockIdx.x * static_cast<int64_t>(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x & 31;
    if (r >= rows) return;
    const float *dyr = dy + r * n, *yr = y + r * n;
    float *dxr = dx + r * n;
    float d = 0.0f;
    for (int j = lane; j < n; j += 32) d += dyr[j] * yr[j];
    d = warp_sum(d);
    for (int j = lane; j < n; j += 32) dxr[j] = scale * yr[j] * (dyr[j] - d);
}

}  // namespace

extern "C" st_status st_softmax_rows(st_handle *h, const float *x, float *y, int64_t rows, int64_t n, int64_t t,
                                     float scale, int32_t causal, int32_t one) {
    if (!h) return ST_INVALID_ARG;
    if (!x || !y || rows < 0 || n < 1 || (causal && t < 1) || n >= (1ll << 31))
        return h->fail(ST_INVALID_ARG, "st_softmax_rows: bad arguments");
    if (rows == 0) return ST_OK;
    cudaSetDevice(h->device);
    const int per_block = 8;
    const int64_t blocks = (rows + per_block - 1) / per_block;
    if (blocks > 0x7fffffff) return h->fail(ST_UNSUPPORTED_SHAPE, "st_softmax_rows: too many rows");
    k_softmax_rows<<<static_cast<unsigned>(blocks), per_block * 32, 0, h->stream>>>(x, y, rows, static_cast<int>(n),
                                                                                   static_cast<int>(causal ? t : 1),
                                                                                   scale, causal, one);
    return st_after_launch(h, "k_softmax_rows");
}

extern "C" st_status st_softmax_rows_bwd(st_handle *h, const float *dy, const float *y, float *dx, int64_t rows,
                                         int64_t n, float scale) {
    if (!h) return ST_INVALID_ARG;
    if (!dy || !y || !dx || rows < 0 || n < 1 || n >= (1ll << 31))
        return h->fail(ST_INVALID_ARG, "st_softmax_rows_bwd: bad arguments");
    if (rows == 0) return ST_OK;
    cudaSetDevice(h->device);
    const int per_block = 8;
    const int64_t blocks = (rows + per_block - 1) / per_block;
    k_softmax_rows_bwd<<<static_cast<unsigned>(blocks), per_block * 32, 0, h->stream>>>(dy, y, dx, rows,
                                                                                       static_cast<int>(n), scale);
    return st_after_launch(h, "k_softmax_rows_bwd");
}
