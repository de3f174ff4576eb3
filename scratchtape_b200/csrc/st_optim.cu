// st_optim.cu -- the device step's elementwise optimiser, model-average and
// dropout kernels.
//
// Reference (src/gpu_step): DeviceParams::sgd / momentum / decay
// (mod.rs:153-180, kernels k_sgd / k_momentum / k_decay :232-259), the
// in-device local-SGD average average_models / average_groups (mod.rs:182-195,
// k_average_models :261-275), and dropout / dropout_relu_backward with the
// lowbias32 mask hash (tape.rs:528-594).  Each element's arithmetic is the
// reference's f32 operation order with every multiply and add rounded on its
// own (__fmul_rn / __fadd_rn: never contracted into an FMA, as Rust never
// contracts), so results are bit-identical to a CPU restatement.
//
// All of these are HBM-bound streams: one pass over each operand, float4
// loads and stores when every pointer is 16-byte aligned, a grid of a few
// blocks per SM striding over the elements.
#include <algorithm>

#include "st_internal.h"

namespace {

constexpr int EW_THREADS = 256;

unsigned ew_blocks(const st_handle *h, int64_t n4) {
    const int64_t want = (n4 + EW_THREADS - 1) / EW_THREADS;
    return static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(want, 8LL * h->num_sms)));
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// p -= lr * g
__device__ __forceinline__ float sgd1(float p, float g, float lr) { return __fsub_rn(p, __fmul_rn(lr, g)); }

// p *= 1 - shrink * mask
__device__ __forceinline__ float decay1(float p, float mask, float shrink) {
    return __fmul_rn(p, __fsub_rn(1.0f, __fmul_rn(shrink, mask)));
}

template <bool VEC>
__global__ void k_sgd(float *p, const float *g, int64_t n, float lr) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (VEC) {
        for (; i < n / 4; i += stride) {
            float4 a = reinterpret_cast<float4 *>(p)[i];
            const float4 b = reinterpret_cast<const float4 *>(g)[i];
            a.x = sgd1(a.x, b.x, lr);
            a.y = sgd1(a.y, b.y, lr);
            a.z = sgd1(a.z, b.z, lr);
            a.w = sgd1(a.w, b.w, lr);
            reinterpret_cast<float4 *>(p)[i] = a;
        }
        i = n / 4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;  // the tail
        if (i < n) p[i] = sgd1(p[i], g[i], lr);
    } else {
        for (; i < n; i += stride) p[i] = sgd1(p[i], g[i], lr);
    }
}

// with decay: p *= 1 - shrink * mask first; then v = mu * v + g; p -= lr * v
__device__ __forceinline__ void momentum1(float &p, float g, float &v, float mask, float lr, float mu, float shrink,
                                          bool decay) {
    if (decay) p = decay1(p, mask, shrink);
    v = __fadd_rn(__fmul_rn(mu, v), g);
    p = __fsub_rn(p, __fmul_rn(lr, v));
}

template <bool VEC, bool DECAY>
__global__ void k_momentum(float *p, const float *g, float *v, const float *mask, int64_t n, float lr, float mu,
                           float shrink) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (VEC) {
        for (; i < n / 4; i += stride) {
            float4 a = reinterpret_cast<float4 *>(p)[i], vv = reinterpret_cast<float4 *>(v)[i];
            const float4 b = reinterpret_cast<const float4 *>(g)[i];
            const float4 mk = DECAY ? reinterpret_cast<const float4 *>(mask)[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            momentum1(a.x, b.x, vv.x, mk.x, lr, mu, shrink, DECAY);
            momentum1(a.y, b.y, vv.y, mk.y, lr, mu, shrink, DECAY);
            momentum1(a.z, b.z, vv.z, mk.z, lr, mu, shrink, DECAY);
            momentum1(a.w, b.w, vv.w, mk.w, lr, mu, shrink, DECAY);
            reinterpret_cast<float4 *>(p)[i] = a;
            reinterpret_cast<float4 *>(v)[i] = vv;
        }
        i = n / 4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
        if (i < n) momentum1(p[i], g[i], v[i], DECAY ? mask[i] : 0.0f, lr, mu, shrink, DECAY);
    } else {
        for (; i < n; i += stride) momentum1(p[i], g[i], v[i], DECAY ? mask[i] : 0.0f, lr, mu, shrink, DECAY);
    }
}

template <bool VEC>
__global__ void k_decay(float *p, const float *mask, int64_t n, float shrink) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (VEC) {
        for (; i < n / 4; i += stride) {
            float4 a = reinterpret_cast<float4 *>(p)[i];
            const float4 mk = reinterpret_cast<const float4 *>(mask)[i];
            a.x = decay1(a.x, mk.x, shrink);
            a.y = decay1(a.y, mk.y, shrink);
            a.z = decay1(a.z, mk.z, shrink);
            a.w = decay1(a.w, mk.w, shrink);
            reinterpret_cast<float4 *>(p)[i] = a;
        }
        i = n / 4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
        if (i < n) p[i] = decay1(p[i], mask[i], shrink);
    } else {
        for (; i < n; i += stride) p[i] = decay1(p[i], mask[i], shrink);
    }
}

// Models are `k` consecutive parameter vectors of `stride` floats; each group
// of `group` consecutive models gets its mean, summed in model order and
// divided (not multiplied by a reciprocal) by the group size.
__global__ void k_average_groups(float *p, int64_t stride, int k, int group) {
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    const float gf = static_cast<float>(group);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < stride; i += step) {
        for (int g = 0; g < k / group; g++) {
            float s = 0.0f;
            for (int m = 0; m < group; m++) s = __fadd_rn(s, p[static_cast<int64_t>(g * group + m) * stride + i]);
            const float mean = __fdiv_rn(s, gf);
            for (int m = 0; m < group; m++) p[static_cast<int64_t>(g * group + m) * stride + i] = mean;
        }
    }
}

// Every rank's parameters after an all-reduce sum: p = p / world.
__global__ void k_div(float *p, int64_t n, float by) {
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += step)
        p[i] = __fdiv_rn(p[i], by);
}

// lowbias32 (Wellons) of i + seed * golden ratio, in wrapping u32 arithmetic.
__device__ __forceinline__ uint32_t dropout_bits(uint32_t i, uint32_t seed) {
    uint32_t h = i + seed * 0x9e3779b9u;
    h ^= h >> 16;
    h *= 0x7feb352du;
    h ^= h >> 15;
    h *= 0x846ca68bu;
    return h ^ (h >> 16);
}

// y = x * scale where bits(seed, i) >= threshold, else 0.  With relu_y, also
// 0 where relu_y <= 0 (dropout's backward fused with ReLU's).
template <bool RELU>
__global__ void k_dropout(const float *x, const float *relu_y, float *y, int64_t n, uint32_t seed, uint32_t threshold,
                          float scale) {
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += step) {
        float v = 0.0f;
        bool keep = dropout_bits(static_cast<uint32_t>(i), seed) >= threshold;
        if (RELU) keep = keep && relu_y[i] > 0.0f;
        if (keep) v = __fmul_rn(x[i], scale);
        y[i] = v;
    }
}

// The same with 4 elements per thread (16-byte aligned pointers).
template <bool RELU>
__global__ void k_dropout4(const float *x, const float *relu_y, float *y, int64_t n, uint32_t seed,
                           uint32_t threshold, float scale) {
    const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t j = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; j < n / 4; j += step) {
        const float4 a = reinterpret_cast<const float4 *>(x)[j];
        const float4 r = RELU ? reinterpret_cast<const float4 *>(relu_y)[j] : make_float4(1.f, 1.f, 1.f, 1.f);
        const float av[4] = {a.x, a.y, a.z, a.w}, rv[4] = {r.x, r.y, r.z, r.w};
        float o[4];
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const bool keep = dropout_bits(static_cast<uint32_t>(4 * j + c), seed) >= threshold && rv[c] > 0.0f;
            o[c] = keep ? __fmul_rn(av[c], scale) : 0.0f;
        }
        reinterpret_cast<float4 *>(y)[j] = make_float4(o[0], o[1], o[2], o[3]);
    }
    const int64_t i = n / 4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i < n) {
        const bool keep = dropout_bits(static_cast<uint32_t>(i), seed) >= threshold && (!RELU || relu_y[i] > 0.0f);
        y[i] = keep ? __fmul_rn(x[i], scale) : 0.0f;
    }
}

// The reference's host-side constants: threshold = (rate as f64 * 2^32) as u32
// (Rust's cast saturates at both ends; NaN gives 0), scale = 1 / (1 - rate) in f32.
uint32_t dropout_threshold(float rate) {
    const double t = static_cast<double>(rate) * 4294967296.0;
    if (!(t > 0.0)) return 0u;
    if (t >= 4294967295.0) return 0xffffffffu;
    return static_cast<uint32_t>(t);
}

}  // namespace

extern "C" st_status st_sgd(st_handle *h, float *p, const float *g, int64_t n, float lr) {
    if (!h) return ST_INVALID_ARG;
    if (!p || !g || n < 1) return h->fail(ST_INVALID_ARG, "st_sgd: null pointer or n < 1");
    cudaSetDevice(h->device);
    if (aligned16(p) && aligned16(g))
        k_sgd<true><<<ew_blocks(h, (n + 3) / 4), EW_THREADS, 0, h->stream>>>(p, g, n, lr);
    else
        k_sgd<false><<<ew_blocks(h, n), EW_THREADS, 0, h->stream>>>(p, g, n, lr);
    return st_after_launch(h, "k_sgd");
}

extern "C" st_status st_momentum(st_handle *h, float *p, const float *g, float *v, const float *mask, int64_t n,
                                 float lr, float mu, float shrink) {
    if (!h) return ST_INVALID_ARG;
    if (!p || !g || !v || n < 1) return h->fail(ST_INVALID_ARG, "st_momentum: null pointer or n < 1");
    cudaSetDevice(h->device);
    const bool vec = aligned16(p) && aligned16(g) && aligned16(v) && (!mask || aligned16(mask));
    const unsigned blocks = ew_blocks(h, vec ? (n + 3) / 4 : n);
    if (vec && mask)
        k_momentum<true, true><<<blocks, EW_THREADS, 0, h->stream>>>(p, g, v, mask, n, lr, mu, shrink);
    else if (vec)
        k_momentum<true, false><<<blocks, EW_THREADS, 0, h->stream>>>(p, g, v, mask, n, lr, mu, shrink);
    else if (mask)
        k_momentum<false, true><<<blocks, EW_THREADS, 0, h->stream>>>(p, g, v, mask, n, lr, mu, shrink);
    else
        k_momentum<false, false><<<blocks, EW_THREADS, 0, h->stream>>>(p, g, v, mask, n, lr, mu, shrink);
    return st_after_launch(h, "k_momentum");
}

extern "C" st_status st_decay(st_handle *h, float *p, const float *mask, int64_t n, float shrink) {
    if (!h) return ST_INVALID_ARG;
    if (!p || !mask || n < 1) return h->fail(ST_INVALID_ARG, "st_decay: null pointer or n < 1");
    cudaSetDevice(h->device);
    if (aligned16(p) && aligned16(mask))
        k_decay<true><<<ew_blocks(h, (n + 3) / 4), EW_THREADS, 0, h->stream>>>(p, mask, n, shrink);
    else
        k_decay<false><<<ew_blocks(h, n), EW_THREADS, 0, h->stream>>>(p, mask, n, shrink);
    return st_after_launch(h, "k_decay");
}

extern "C" st_status st_average_models(st_handle *h, float *p, int64_t stride, int32_t models, int32_t group) {
    if (!h) return ST_INVALID_ARG;
    if (!p || stride < 1 || models < 1 || group < 1 || models % group != 0)
        return h->fail(ST_INVALID_ARG, "st_average_models: %d models do not split into groups of %d", models, group);
    cudaSetDevice(h->device);
    k_average_groups<<<ew_blocks(h, stride), EW_THREADS, 0, h->stream>>>(p, stride, models, group);
    return st_after_launch(h, "k_average_groups");
}

extern "C" st_status st_dropout(st_handle *h, const float *x, float *y, int64_t n, float rate, uint32_t seed) {
    if (!h) return ST_INVALID_ARG;
    if (!x || !y || n < 1 || n > 0xffffffffLL || !(rate >= 0.0f && rate < 1.0f))
        return h->fail(ST_INVALID_ARG, "st_dropout: null pointer, n outside [1, 2^32) or rate outside [0, 1)");
    cudaSetDevice(h->device);
    const uint32_t thr = dropout_threshold(rate);
    const float scale = 1.0f / (1.0f - rate);
    if (aligned16(x) && aligned16(y))
        k_dropout4<false><<<ew_blocks(h, (n + 3) / 4), EW_THREADS, 0, h->stream>>>(x, nullptr, y, n, seed, thr, scale);
    else
        k_dropout<false><<<ew_blocks(h, n), EW_THREADS, 0, h->stream>>>(x, nullptr, y, n, seed, thr, scale);
    return st_after_launch(h, "k_dropout");
}

extern "C" st_status st_dropout_relu_bwd(st_handle *h, const float *dy, const float *relu_y, float *dx, int64_t n,
                                         float rate, uint32_t seed) {
    if (!h) return ST_INVALID_ARG;
    if (!dy || !relu_y || !dx || n < 1 || n > 0xffffffffLL || !(rate >= 0.0f && rate < 1.0f))
        return h->fail(ST_INVALID_ARG,
                       "st_dropout_relu_bwd: null pointer, n outside [1, 2^32) or rate outside [0, 1)");
    cudaSetDevice(h->device);
    const uint32_t thr = dropout_threshold(rate);
    const float scale = 1.0f / (1.0f - rate);
    if (aligned16(dy) && aligned16(relu_y) && aligned16(dx))
        k_dropout4<true><<<ew_blocks(h, (n + 3) / 4), EW_THREADS, 0, h->stream>>>(dy, relu_y, dx, n, seed, thr, scale);
    else
        k_dropout<true><<<ew_blocks(h, n), EW_THREADS, 0, h->stream>>>(dy, relu_y, dx, n, seed, thr, scale);
    return st_after_launch(h, "k_dropout_relu_bwd");
}

// Used by the collectives (st_comm.cu): p = p / world after an all-reduce sum.
st_status st_divide_by(st_handle *h, float *p, int64_t n, float by) {
    k_div<<<ew_blocks(h, n), EW_THREADS, 0, h->stream>>>(p, n, by);
    return st_after_launch(h, "k_div");
}
