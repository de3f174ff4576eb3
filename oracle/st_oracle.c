/*
 * st_oracle.c -- CPU restatement of scratchtape's hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle and the timed CPU
 * baseline ("port" kind).  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * (libst_b200.so and the scratchtape_b200 package) never links or calls it.
 *
 * Parity is pinned: the forward pass of the plain batched transformer block
 * restated here reproduces the reference's golden fixture
 * src/testdata/batched_heads_reference.bin bit for bit (array 0), and the
 * f64 backward reproduces its parameter gradients and dx (arrays 1-2) within
 * the reference test's own 1e-4 relative bound (src/nn.rs:1076-1152).
 *
 * Build flags mirror .cargo/config.toml:1-7 of the reference (+avx2,+fma, not
 * -march=native) plus -ffp-contract=off: Rust never fuses a*b+c into an FMA,
 * so neither may this restatement if products are to match bit for bit.
 *
 * Every function cites the reference line range it restates.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

#define EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* Rng: xorshift64 + Box-Muller (src/nn.rs:8-36)                             */
/* ------------------------------------------------------------------------ */

/* next_f32: x ^= x<<13; x ^= x>>7; x ^= x<<17; (x as f64 / u64::MAX as f64) as f32 */
EXPORT float orc_rng_next_f32(uint64_t *state) {
    uint64_t x = *state;
    x ^= x << 13;
    x ^= x >> 7;
    x ^= x << 17;
    *state = x;
    return (float)((double)x / (double)UINT64_MAX);
}

/* next_gaussian: u1 = max(next_f32, 1e-9); u2 = next_f32;
 * sqrt(-2 ln u1) * cos(2 pi u2), all in f32 (src/nn.rs:30-34). */
EXPORT float orc_rng_next_gaussian(uint64_t *state) {
    float u1 = orc_rng_next_f32(state);
    if (!(u1 >= 1e-9f)) u1 = 1e-9f; /* f32::max(1e-9): NaN-free input, max */
    float u2 = orc_rng_next_f32(state);
    float two_pi = 2.0f * 3.14159265358979323846264338327950288f;
    return sqrtf(-2.0f * logf(u1)) * cosf(two_pi * u2);
}

/* (next_f32() * 2 - 1) * scale for n draws: Linear/Embedding init and the
 * uniform[-1,1) inputs of benches/gpu_matmul.rs (src/gpu.rs:191). */
EXPORT void orc_rng_uniform(uint64_t *state, float *out, int64_t n, float scale) {
    for (int64_t i = 0; i < n; i++) out[i] = (orc_rng_next_f32(state) * 2.0f - 1.0f) * scale;
}

EXPORT void orc_rng_gaussian(uint64_t *state, float *out, int64_t n) {
    for (int64_t i = 0; i < n; i++) out[i] = orc_rng_next_gaussian(state);
}

/* ------------------------------------------------------------------------ */
/* NdArray::matmul / transpose (src/tensor.rs:241-288)                      */
/* ------------------------------------------------------------------------ */

/* matmul_inner: out zero-filled, i and p blocked by 64, j full width;
 * out[i*n+j] += a[i*k+p] * b[p*n+j] with p ascending for every element
 * (src/tensor.rs:248-276).  rows [i_lo, i_hi) only (for the row-parallel
 * variant; per-element arithmetic is unchanged by the split). */
static void matmul_rows(const float *a, const float *b, float *out, int64_t m, int64_t k, int64_t n,
                        int64_t i_lo, int64_t i_hi) {
    const int64_t BLOCK = 64;
    (void)m;
    for (int64_t i = i_lo; i < i_hi; i++)
        for (int64_t j = 0; j < n; j++) out[i * n + j] = 0.0f;
    for (int64_t i0 = i_lo; i0 < i_hi; i0 += BLOCK) {
        int64_t i_max = i0 + BLOCK < i_hi ? i0 + BLOCK : i_hi;
        for (int64_t p0 = 0; p0 < k; p0 += BLOCK) {
            int64_t p_max = p0 + BLOCK < k ? p0 + BLOCK : k;
            for (int64_t i = i0; i < i_max; i++) {
                for (int64_t p = p0; p < p_max; p++) {
                    float a_ip = a[i * k + p];
                    const float *brow = b + p * n;
                    float *orow = out + i * n;
                    for (int64_t j = 0; j < n; j++) orow[j] += a_ip * brow[j];
                }
            }
        }
    }
}

EXPORT void orc_matmul(const float *a, const float *b, float *out, int64_t m, int64_t k, int64_t n) {
    matmul_rows(a, b, out, m, k, n, 0, m);
}

/* transpose: out[j*m+i] = a[i*n+j] (src/tensor.rs:278-288) */
EXPORT void orc_transpose(const float *a, float *out, int64_t m, int64_t n) {
    for (int64_t i = 0; i < m; i++)
        for (int64_t j = 0; j < n; j++) out[j * m + i] = a[i * n + j];
}

/* The tape's layouts (src/tape.rs:505-510): NT = dC . B^T and TN = A^T . dC,
 * each as an explicit transposed copy followed by NN.  ta: a is stored
 * [k, m]; tb: b is stored [n, k]. */
EXPORT void orc_matmul_layout(const float *a, const float *b, float *out, int64_t m, int64_t k, int64_t n,
                              int ta, int tb) {
    float *at = NULL, *bt = NULL;
    if (ta) {
        at = (float *)malloc(sizeof(float) * m * k);
        orc_transpose(a, at, k, m);
        a = at;
    }
    if (tb) {
        bt = (float *)malloc(sizeof(float) * k * n);
        orc_transpose(b, bt, n, k);
        b = bt;
    }
    orc_matmul(a, b, out, m, k, n);
    free(at);
    free(bt);
}

/* Row-parallel variant for the CPU baseline's multi-thread line (labelled as
 * not the reference, which is single threaded).  Same bits as orc_matmul. */
struct mm_job {
    const float *a, *b;
    float *out;
    int64_t m, k, n, lo, hi;
};
static void *mm_worker(void *p) {
    struct mm_job *j = (struct mm_job *)p;
    matmul_rows(j->a, j->b, j->out, j->m, j->k, j->n, j->lo, j->hi);
    return NULL;
}
EXPORT void orc_matmul_threads(const float *a, const float *b, float *out, int64_t m, int64_t k, int64_t n,
                               int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t tid[256];
    struct mm_job jobs[256];
    int64_t per = (m + threads - 1) / threads;
    per = (per + 63) / 64 * 64;
    int used = 0;
    for (int t = 0; t < threads; t++) {
        int64_t lo = t * per, hi = lo + per < m ? lo + per : m;
        if (lo >= hi) break;
        jobs[t] = (struct mm_job){a, b, out, m, k, n, lo, hi};
        pthread_create(&tid[t], NULL, mm_worker, &jobs[t]);
        used++;
    }
    for (int t = 0; t < used; t++) pthread_join(tid[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* Batched matmul (src/tape.rs:52-112) and head permutations (:119-150)     */
/* ------------------------------------------------------------------------ */

/* batched_matmul_forward: per chunk i, a_chunk . b_chunk or
 * a_chunk . transpose(b_chunk), chunks being contiguous row ranges. */
EXPORT void orc_batched_matmul_fwd(const float *a, const float *b, float *out, int64_t batch, int64_t a_rows,
                                   int64_t a_cols, int64_t b_rows, int64_t b_cols, int transpose_b) {
    int64_t ar = a_rows / batch, br = b_rows / batch;
    int64_t out_cols = transpose_b ? br : b_cols;
    float *bt = (float *)malloc(sizeof(float) * br * b_cols);
    for (int64_t z = 0; z < batch; z++) {
        const float *ac = a + z * ar * a_cols;
        const float *bc = b + z * br * b_cols;
        if (transpose_b) {
            orc_transpose(bc, bt, br, b_cols);
            orc_matmul(ac, bt, out + z * ar * out_cols, ar, a_cols, br);
        } else {
            orc_matmul(ac, bc, out + z * ar * out_cols, ar, a_cols, b_cols);
        }
    }
    free(bt);
}

/* batched_matmul_backward: transpose_b: dA = dC.B, dB = dC^T.A;
 * else dA = dC.B^T, dB = A^T.dC (src/tape.rs:90-112). */
EXPORT void orc_batched_matmul_bwd(const float *a, const float *b, const float *grad, float *grad_a, float *grad_b,
                                   int64_t batch, int64_t a_rows, int64_t a_cols, int64_t b_rows, int64_t b_cols,
                                   int transpose_b) {
    int64_t ar = a_rows / batch, br = b_rows / batch;
    int64_t gc = transpose_b ? br : b_cols;
    for (int64_t z = 0; z < batch; z++) {
        const float *ac = a + z * ar * a_cols;
        const float *bc = b + z * br * b_cols;
        const float *g = grad + z * ar * gc;
        float *da = grad_a + z * ar * a_cols;
        float *db = grad_b + z * br * b_cols;
        if (transpose_b) {
            orc_matmul(g, bc, da, ar, gc, b_cols);
            orc_matmul_layout(g, ac, db, br, ar, a_cols, 1, 0);
        } else {
            orc_matmul_layout(g, bc, da, ar, gc, br, 0, 1);
            orc_matmul_layout(ac, g, db, a_cols, ar, gc, 1, 0);
        }
    }
}

/* split_heads_forward (src/tape.rs:119-133) */
EXPORT void orc_split_heads(const float *a, float *out, int64_t rows, int64_t cols, int64_t col0, int64_t n_heads,
                            int64_t width, int64_t batch) {
    int64_t t_len = rows / batch;
    for (int64_t b = 0; b < batch; b++)
        for (int64_t h = 0; h < n_heads; h++)
            for (int64_t t = 0; t < t_len; t++)
                memcpy(out + ((b * n_heads + h) * t_len + t) * width, a + (b * t_len + t) * cols + col0 + h * width,
                       sizeof(float) * width);
}

/* merge_heads_forward (src/tape.rs:136-150) */
EXPORT void orc_merge_heads(const float *a, float *out, int64_t rows, int64_t width, int64_t n_heads, int64_t batch) {
    int64_t t_len = rows / (batch * n_heads);
    int64_t cols = n_heads * width;
    for (int64_t b = 0; b < batch; b++)
        for (int64_t h = 0; h < n_heads; h++)
            for (int64_t t = 0; t < t_len; t++)
                memcpy(out + (b * t_len + t) * cols + h * width, a + ((b * n_heads + h) * t_len + t) * width,
                       sizeof(float) * width);
}

/* ------------------------------------------------------------------------ */
/* Composed softmax (src/tape.rs:385-392, src/tensor.rs:97-124)             */
/* ------------------------------------------------------------------------ */

/* softmax over rows of x [rows, n], in place: max fold from -inf (f32::max),
 * shifted = x - max, e = exp(shifted), s = fold-sum from 0, e / s.
 * softmax1 adds the phantom exp(-max) term to the denominator the way
 * Tape::softmax1 does it (src/tape.rs:418-431): weights = e / (s + exp(-max)). */
EXPORT void orc_softmax_rows(float *x, int64_t rows, int64_t n, int one) {
    for (int64_t r = 0; r < rows; r++) {
        float *row = x + r * n;
        float mx = -INFINITY;
        for (int64_t j = 0; j < n; j++) mx = fmaxf(mx, row[j]);
        if (one) mx = fmaxf(mx, 0.0f); /* Tape::softmax1 shifts by max(row max, 0) (src/tape.rs:418-431) */
        float s = 0.0f;
        for (int64_t j = 0; j < n; j++) {
            row[j] = expf(row[j] - mx);
        }
        for (int64_t j = 0; j < n; j++) s += row[j];
        if (one) s = s + expf(-mx);
        for (int64_t j = 0; j < n; j++) row[j] = row[j] / s;
    }
}

/* ------------------------------------------------------------------------ */
/* Batched causal attention (src/nn.rs:396-407, :646-671)                   */
/* ------------------------------------------------------------------------ */

/* Forward for bh independent heads of [t, d] rows (q, k, v contiguous per
 * head, head z at z*t*d): scores = q . k^T (per chunk, via transpose),
 * scaled = scores * scale, masked = scaled + mask (-inf above the diagonal
 * when causal), softmax, out = weights . v.  probs (nullable) receives the
 * weights [bh*t, t]. */
EXPORT void orc_attention_fwd(const float *q, const float *k, const float *v, float *out, float *probs, int64_t bh,
                              int64_t t, int64_t d, float scale, int causal, int one) {
    float *w = (float *)malloc(sizeof(float) * bh * t * t);
    orc_batched_matmul_fwd(q, k, w, bh, bh * t, d, bh * t, d, 1);
    for (int64_t i = 0; i < bh * t * t; i++) {
        float sc = w[i] * scale;
        int64_t row = (i / t) % t, col = i % t;
        float mask = (causal && col > row) ? -INFINITY : 0.0f;
        w[i] = sc + mask;
    }
    orc_softmax_rows(w, bh * t, t, one);
    orc_batched_matmul_fwd(w, v, out, bh, bh * t, t, bh * t, d, 0);
    if (probs) memcpy(probs, w, sizeof(float) * bh * t * t);
    free(w);
}

/* Analytic backward of the forward above, in f64 (the chain rule the tape
 * applies op by op, src/tape.rs:479-640, collapsed):
 *   dV = P^T dO;  dP = dO V^T;  dS = P * (dP - rowsum(dP * P)) * scale;
 *   dQ = dS K;    dK = dS^T Q.
 * (For softmax1 the row term is the same expression; P rows sum to < 1.) */
EXPORT void orc_attention_bwd(const float *q, const float *k, const float *v, const float *dout, float *dq, float *dk,
                              float *dv, int64_t bh, int64_t t, int64_t d, float scale, int causal, int one) {
    double *p = (double *)malloc(sizeof(double) * t * t);
    double *dp = (double *)malloc(sizeof(double) * t * t);
    for (int64_t z = 0; z < bh; z++) {
        const float *qz = q + z * t * d, *kz = k + z * t * d, *vz = v + z * t * d, *doz = dout + z * t * d;
        float *dqz = dq + z * t * d, *dkz = dk + z * t * d, *dvz = dv + z * t * d;
        for (int64_t i = 0; i < t; i++) {
            double mx = -INFINITY;
            for (int64_t j = 0; j < t; j++) {
                double s = 0;
                for (int64_t c = 0; c < d; c++) s += (double)qz[i * d + c] * kz[j * d + c];
                s *= scale;
                if (causal && j > i) s = -INFINITY;
                p[i * t + j] = s;
                if (s > mx) mx = s;
            }
            double sum = one ? exp(-mx) : 0.0;
            for (int64_t j = 0; j < t; j++) {
                p[i * t + j] = exp(p[i * t + j] - mx);
                sum += p[i * t + j];
            }
            for (int64_t j = 0; j < t; j++) p[i * t + j] /= sum;
        }
        for (int64_t i = 0; i < t; i++)
            for (int64_t j = 0; j < t; j++) {
                double s = 0;
                for (int64_t c = 0; c < d; c++) s += (double)doz[i * d + c] * vz[j * d + c];
                dp[i * t + j] = s;
            }
        for (int64_t j = 0; j < t; j++)
            for (int64_t c = 0; c < d; c++) {
                double s = 0;
                for (int64_t i = 0; i < t; i++) s += p[i * t + j] * doz[i * d + c];
                dvz[j * d + c] = (float)s;
            }
        for (int64_t i = 0; i < t; i++) {
            double rs = 0;
            for (int64_t j = 0; j < t; j++) rs += dp[i * t + j] * p[i * t + j];
            for (int64_t j = 0; j < t; j++) dp[i * t + j] = p[i * t + j] * (dp[i * t + j] - rs) * scale;
        }
        for (int64_t i = 0; i < t; i++)
            for (int64_t c = 0; c < d; c++) {
                double s = 0;
                for (int64_t j = 0; j < t; j++) s += dp[i * t + j] * kz[j * d + c];
                dqz[i * d + c] = (float)s;
            }
        for (int64_t j = 0; j < t; j++)
            for (int64_t c = 0; c < d; c++) {
                double s = 0;
                for (int64_t i = 0; i < t; i++) s += dp[i * t + j] * qz[i * d + c];
                dkz[j * d + c] = (float)s;
            }
    }
    free(p);
    free(dp);
}

/* Row softmax as the device kernel computes it (src/gpu_step/rows.rs:106-123,
 * :295-357), in f64: row r of rows x n, causal limit r % t + 1, masked
 * entries exactly 0, optional softmax1.  y may alias x. */
EXPORT void orc_rows_softmax(const float *x, float *y, int64_t rows, int64_t n, int64_t t, float scale, int causal,
                             int one) {
    for (int64_t r = 0; r < rows; r++) {
        int64_t lim = causal ? (r % t) + 1 : n;
        double mx = one ? 0.0 : -INFINITY;
        for (int64_t j = 0; j < lim; j++) {
            double s = (double)x[r * n + j] * scale;
            if (s > mx) mx = s;
        }
        double sum = one ? exp(-mx) : 0.0;
        for (int64_t j = 0; j < lim; j++) sum += exp((double)x[r * n + j] * scale - mx);
        for (int64_t j = 0; j < n; j++)
            y[r * n + j] = j < lim ? (float)(exp((double)x[r * n + j] * scale - mx) / sum) : 0.0f;
    }
}

/* Backward of the above: dx = scale * y * (dy - sum(dy * y)) (rows.rs:117). */
EXPORT void orc_rows_softmax_bwd(const float *y, const float *dy, float *dx, int64_t rows, int64_t n, float scale) {
    for (int64_t r = 0; r < rows; r++) {
        double s = 0;
        for (int64_t j = 0; j < n; j++) s += (double)dy[r * n + j] * y[r * n + j];
        for (int64_t j = 0; j < n; j++) dx[r * n + j] = (float)(scale * (double)y[r * n + j] * ((double)dy[r * n + j] - s));
    }
}

/* ------------------------------------------------------------------------ */
/* LayerNorm (src/nn.rs:290-322) composed from tape ops, and the block       */
/* ------------------------------------------------------------------------ */

/* Forward, bitwise: mean = sum*(1/d); c = x-mean; var = sum(c*c)*(1/d);
 * std = sqrt(var+eps); y = (c/std)*gamma + beta. */
EXPORT void orc_layernorm_fwd(const float *x, const float *gamma, const float *beta, float *y, int64_t rows,
                              int64_t d) {
    float invd = 1.0f / (float)d;
    float *c = (float *)malloc(sizeof(float) * d);
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * d;
        float s = 0.0f;
        for (int64_t j = 0; j < d; j++) s += xr[j];
        float mean = s * invd;
        float ss = 0.0f;
        for (int64_t j = 0; j < d; j++) {
            c[j] = xr[j] - mean;
        }
        for (int64_t j = 0; j < d; j++) ss += c[j] * c[j];
        float var = ss * invd;
        float sd = sqrtf(var + 1e-5f);
        for (int64_t j = 0; j < d; j++) y[r * d + j] = (c[j] / sd) * gamma[j] + beta[j];
    }
    free(c);
}

/* f64 analytic LayerNorm backward; accumulates into dgamma/dbeta, writes dx. */
static void ln_bwd64(const float *x, const float *gamma, const double *dy, double *dx, double *dgamma, double *dbeta,
                     int64_t rows, int64_t d) {
    for (int64_t r = 0; r < rows; r++) {
        const float *xr = x + r * d;
        double mean = 0, var = 0;
        for (int64_t j = 0; j < d; j++) mean += xr[j];
        mean /= d;
        for (int64_t j = 0; j < d; j++) var += (xr[j] - mean) * (xr[j] - mean);
        var /= d;
        double rstd = 1.0 / sqrt(var + (double)1e-5f);
        double sg = 0, sgx = 0;
        for (int64_t j = 0; j < d; j++) {
            double xh = (xr[j] - mean) * rstd;
            double g = dy[r * d + j] * gamma[j];
            dgamma[j] += dy[r * d + j] * xh;
            dbeta[j] += dy[r * d + j];
            sg += g;
            sgx += g * xh;
        }
        for (int64_t j = 0; j < d; j++) {
            double xh = (xr[j] - mean) * rstd;
            double g = dy[r * d + j] * gamma[j];
            dx[r * d + j] = rstd * (g - sg / d - xh * sgx / d);
        }
    }
}

/* y = x.W + b (Linear::forward_shared, src/nn.rs:110-114) */
static void linear_fwd(const float *x, const float *w, const float *b, float *y, int64_t rows, int64_t in,
                       int64_t out) {
    orc_matmul(x, w, y, rows, in, out);
    for (int64_t r = 0; r < rows; r++)
        for (int64_t j = 0; j < out; j++) y[r * out + j] = y[r * out + j] + b[j];
}

/* Parameter layout of a plain block in to_flat order (src/nn.rs:738-760). */
struct blk_off {
    int64_t ln1g, ln1b, qkvw, qkvb, ow, ob, ln2g, ln2b, f1w, f1b, f2w, f2b, total;
};
static struct blk_off blk_layout(int64_t d, int64_t dff) {
    struct blk_off o;
    int64_t p = 0;
    o.ln1g = p; p += d;
    o.ln1b = p; p += d;
    o.qkvw = p; p += d * 3 * d;
    o.qkvb = p; p += 3 * d;
    o.ow = p; p += d * d;
    o.ob = p; p += d;
    o.ln2g = p; p += d;
    o.ln2b = p; p += d;
    o.f1w = p; p += d * dff;
    o.f1b = p; p += dff;
    o.f2w = p; p += dff * d;
    o.f2b = p; p += d;
    o.total = p;
    return o;
}

EXPORT int64_t orc_block_param_count(int64_t d, int64_t dff) { return blk_layout(d, dff).total; }

/* TransformerBlock::new (src/nn.rs:436-452): 3H Linear(d, d_k) heads (Q heads,
 * then K, then V, fused column-wise), out_proj, ffn1, ffn2; LayerNorms 1/0. */
EXPORT void orc_block_init(uint64_t *state, float *params, int64_t d, int64_t n_heads, int64_t dff) {
    struct blk_off o = blk_layout(d, dff);
    int64_t dk = d / n_heads;
    memset(params, 0, sizeof(float) * o.total);
    for (int64_t j = 0; j < d; j++) {
        params[o.ln1g + j] = 1.0f;
        params[o.ln2g + j] = 1.0f;
    }
    float *tmp = (float *)malloc(sizeof(float) * d * (dff > d ? dff : d));
    float lim = sqrtf(6.0f / (float)d);
    for (int64_t hh = 0; hh < 3 * n_heads; hh++) {
        orc_rng_uniform(state, tmp, d * dk, lim);
        for (int64_t r = 0; r < d; r++)
            for (int64_t j = 0; j < dk; j++) params[o.qkvw + r * 3 * d + hh * dk + j] = tmp[r * dk + j];
    }
    orc_rng_uniform(state, params + o.ow, d * d, lim);
    orc_rng_uniform(state, params + o.f1w, d * dff, lim);
    orc_rng_uniform(state, params + o.f2w, dff * d, sqrtf(6.0f / (float)dff));
    free(tmp);
}

/* forward_full of a plain block (softmax, no extras), bitwise
 * (src/nn.rs:627-712).  x [batch*t, d] -> y. */
EXPORT void orc_block_forward(const float *params, const float *x, float *y, int64_t batch, int64_t t, int64_t d,
                              int64_t n_heads, int64_t dff) {
    struct blk_off o = blk_layout(d, dff);
    int64_t rows = batch * t, dk = d / n_heads, heads = batch * n_heads;
    float *ln1 = malloc(sizeof(float) * rows * d), *qkv = malloc(sizeof(float) * rows * 3 * d);
    float *qh = malloc(sizeof(float) * rows * d), *kh = malloc(sizeof(float) * rows * d),
          *vh = malloc(sizeof(float) * rows * d);
    float *ho = malloc(sizeof(float) * rows * d), *merged = malloc(sizeof(float) * rows * d);
    float *x1 = malloc(sizeof(float) * rows * d), *ln2 = malloc(sizeof(float) * rows * d);
    float *hid = malloc(sizeof(float) * rows * dff), *f2 = malloc(sizeof(float) * rows * d);
    orc_layernorm_fwd(x, params + o.ln1g, params + o.ln1b, ln1, rows, d);
    linear_fwd(ln1, params + o.qkvw, params + o.qkvb, qkv, rows, d, 3 * d);
    orc_split_heads(qkv, qh, rows, 3 * d, 0, n_heads, dk, batch);
    orc_split_heads(qkv, kh, rows, 3 * d, d, n_heads, dk, batch);
    orc_split_heads(qkv, vh, rows, 3 * d, 2 * d, n_heads, dk, batch);
    float scale = 1.0f / sqrtf((float)dk);
    orc_attention_fwd(qh, kh, vh, ho, NULL, heads, t, dk, scale, 1, 0);
    orc_merge_heads(ho, merged, rows * n_heads, dk, n_heads, batch);
    linear_fwd(merged, params + o.ow, params + o.ob, x1, rows, d, d);
    for (int64_t i = 0; i < rows * d; i++) x1[i] = x[i] + x1[i];
    orc_layernorm_fwd(x1, params + o.ln2g, params + o.ln2b, ln2, rows, d);
    linear_fwd(ln2, params + o.f1w, params + o.f1b, hid, rows, d, dff);
    for (int64_t i = 0; i < rows * dff; i++) hid[i] = hid[i] > 0.0f ? hid[i] : 0.0f;
    linear_fwd(hid, params + o.f2w, params + o.f2b, f2, rows, dff, d);
    for (int64_t i = 0; i < rows * d; i++) y[i] = x1[i] + f2[i];
    free(ln1); free(qkv); free(qh); free(kh); free(vh); free(ho); free(merged);
    free(x1); free(ln2); free(hid); free(f2);
}

/* f64 helpers for the block backward */
static void mm64_nt(const double *g, const float *w, double *dx, int64_t rows, int64_t in, int64_t out) {
    /* dx[r, i] = sum_j g[r, j] * w[i, j] */
    for (int64_t r = 0; r < rows; r++)
        for (int64_t i = 0; i < in; i++) {
            double s = 0;
            for (int64_t j = 0; j < out; j++) s += g[r * out + j] * w[i * out + j];
            dx[r * in + i] = s;
        }
}
static void mm64_tn(const float *x, const double *g, double *dw, double *db, int64_t rows, int64_t in, int64_t out) {
    for (int64_t i = 0; i < in; i++)
        for (int64_t j = 0; j < out; j++) {
            double s = 0;
            for (int64_t r = 0; r < rows; r++) s += (double)x[r * in + i] * g[r * out + j];
            dw[i * out + j] = s;
        }
    for (int64_t j = 0; j < out; j++) {
        double s = 0;
        for (int64_t r = 0; r < rows; r++) s += g[r * out + j];
        db[j] = s;
    }
}

/* Backward of the plain block under upstream gradient dy, in f64: parameter
 * gradients in to_flat order and dx (what batched_heads_match_per_head_reference
 * reads back, src/nn.rs:1131-1151). */
EXPORT void orc_block_backward(const float *params, const float *x, const float *dy, float *dparams, float *dx,
                               int64_t batch, int64_t t, int64_t d, int64_t n_heads, int64_t dff) {
    struct blk_off o = blk_layout(d, dff);
    int64_t rows = batch * t, dk = d / n_heads, heads = batch * n_heads;
    /* recompute forward intermediates (f32, bitwise as the forward) */
    float *ln1 = malloc(sizeof(float) * rows * d), *qkv = malloc(sizeof(float) * rows * 3 * d);
    float *qh = malloc(sizeof(float) * rows * d), *kh = malloc(sizeof(float) * rows * d),
          *vh = malloc(sizeof(float) * rows * d);
    float *ho = malloc(sizeof(float) * rows * d), *merged = malloc(sizeof(float) * rows * d);
    float *x1 = malloc(sizeof(float) * rows * d), *ln2 = malloc(sizeof(float) * rows * d);
    float *pre = malloc(sizeof(float) * rows * dff), *hid = malloc(sizeof(float) * rows * dff);
    orc_layernorm_fwd(x, params + o.ln1g, params + o.ln1b, ln1, rows, d);
    linear_fwd(ln1, params + o.qkvw, params + o.qkvb, qkv, rows, d, 3 * d);
    orc_split_heads(qkv, qh, rows, 3 * d, 0, n_heads, dk, batch);
    orc_split_heads(qkv, kh, rows, 3 * d, d, n_heads, dk, batch);
    orc_split_heads(qkv, vh, rows, 3 * d, 2 * d, n_heads, dk, batch);
    float scale = 1.0f / sqrtf((float)dk);
    orc_attention_fwd(qh, kh, vh, ho, NULL, heads, t, dk, scale, 1, 0);
    orc_merge_heads(ho, merged, rows * n_heads, dk, n_heads, batch);
    linear_fwd(merged, params + o.ow, params + o.ob, x1, rows, d, d);
    for (int64_t i = 0; i < rows * d; i++) x1[i] = x[i] + x1[i];
    orc_layernorm_fwd(x1, params + o.ln2g, params + o.ln2b, ln2, rows, d);
    linear_fwd(ln2, params + o.f1w, params + o.f1b, pre, rows, d, dff);
    for (int64_t i = 0; i < rows * dff; i++) hid[i] = pre[i] > 0.0f ? pre[i] : 0.0f;

    double *g = calloc(o.total, sizeof(double));
    double *dy64 = malloc(sizeof(double) * rows * d), *dx1 = malloc(sizeof(double) * rows * d);
    double *dhid = malloc(sizeof(double) * rows * dff), *dln2 = malloc(sizeof(double) * rows * d);
    double *dmerged = malloc(sizeof(double) * rows * d), *dqkv = calloc(rows * 3 * d, sizeof(double));
    double *dln1 = malloc(sizeof(double) * rows * d), *dx64 = malloc(sizeof(double) * rows * d);
    for (int64_t i = 0; i < rows * d; i++) dy64[i] = dy[i];
    /* y = x1 + ffn2(relu(ffn1(ln2(x1)))) */
    mm64_tn(hid, dy64, g + o.f2w, g + o.f2b, rows, dff, d);
    mm64_nt(dy64, params + o.f2w, dhid, rows, dff, d);
    for (int64_t i = 0; i < rows * dff; i++) dhid[i] = pre[i] > 0.0f ? dhid[i] : 0.0;
    mm64_tn(ln2, dhid, g + o.f1w, g + o.f1b, rows, d, dff);
    mm64_nt(dhid, params + o.f1w, dln2, rows, d, dff);
    ln_bwd64(x1, params + o.ln2g, dln2, dx1, g + o.ln2g, g + o.ln2b, rows, d);
    for (int64_t i = 0; i < rows * d; i++) dx1[i] += dy64[i];
    /* x1 = x + out_proj(merge(attn(split(qkv(ln1(x)))))) */
    mm64_tn(merged, dx1, g + o.ow, g + o.ob, rows, d, d);
    mm64_nt(dx1, params + o.ow, dmerged, rows, d, d);
    {
        float *dho = malloc(sizeof(float) * rows * d), *dmf = malloc(sizeof(float) * rows * d);
        float *dq = malloc(sizeof(float) * rows * d), *dk_ = malloc(sizeof(float) * rows * d),
              *dv = malloc(sizeof(float) * rows * d);
        /* split(dmerged) -> per-head dO; kept f64-exact by an f64 attention
         * backward on f32 inputs; the f32 round trip of dO costs < 1e-7 rel. */
        for (int64_t i = 0; i < rows * d; i++) dmf[i] = (float)dmerged[i];
        orc_split_heads(dmf, dho, rows, d, 0, n_heads, dk, batch);
        orc_attention_bwd(qh, kh, vh, dho, dq, dk_, dv, heads, t, dk, scale, 1, 0);
        for (int64_t b = 0; b < batch; b++)
            for (int64_t h = 0; h < n_heads; h++)
                for (int64_t tt = 0; tt < t; tt++)
                    for (int64_t j = 0; j < dk; j++) {
                        int64_t src = ((b * n_heads + h) * t + tt) * dk + j;
                        int64_t dst = (b * t + tt) * 3 * d + h * dk + j;
                        dqkv[dst] = dq[src];
                        dqkv[dst + d] = dk_[src];
                        dqkv[dst + 2 * d] = dv[src];
                    }
        free(dho); free(dmf); free(dq); free(dk_); free(dv);
    }
    mm64_tn(ln1, dqkv, g + o.qkvw, g + o.qkvb, rows, d, 3 * d);
    mm64_nt(dqkv, params + o.qkvw, dln1, rows, d, 3 * d);
    ln_bwd64(x, params + o.ln1g, dln1, dx64, g + o.ln1g, g + o.ln1b, rows, d);
    for (int64_t i = 0; i < rows * d; i++) dx[i] = (float)(dx64[i] + dx1[i]);
    for (int64_t i = 0; i < o.total; i++) dparams[i] = (float)g[i];
    free(ln1); free(qkv); free(qh); free(kh); free(vh); free(ho); free(merged); free(x1); free(ln2);
    free(pre); free(hid); free(g); free(dy64); free(dx1); free(dhid); free(dln2); free(dmerged);
    free(dqkv); free(dln1); free(dx64);
}

/* ------------------------------------------------------------------------ */
/* Adam (src/optim.rs:42-57) and the local-SGD mean (src/gpu_step/mod.rs:261-275) */
/* ------------------------------------------------------------------------ */

/* f32::powi as LLVM lowers it (repeated squaring, compiler-rt __powisf2). */
EXPORT float orc_powi(float a, int b) {
    int recip = b < 0;
    float r = 1.0f;
    if (recip) b = -b;
    for (;;) {
        if (b & 1) r *= a;
        b /= 2;
        if (b == 0) break;
        a *= a;
    }
    return recip ? 1.0f / r : r;
}

/* One Adam step on n parameters with step counter t (already incremented):
 * m = m*b1 + g*(1-b1); v = v*b2 + (g*g)*(1-b2); m_hat = m*(1/bc1);
 * v_hat = v*(1/bc2); p -= (m_hat / (sqrt(v_hat) + eps)) * lr. */
EXPORT void orc_adam(float *p, const float *g, float *m, float *v, int64_t n, int t, float lr, float b1, float b2,
                     float eps) {
    float bc1 = 1.0f - orc_powi(b1, t), bc2 = 1.0f - orc_powi(b2, t);
    float i1 = 1.0f / bc1, i2 = 1.0f / bc2, c1 = 1.0f - b1, c2 = 1.0f - b2;
    for (int64_t i = 0; i < n; i++) {
        m[i] = m[i] * b1 + g[i] * c1;
        v[i] = v[i] * b2 + (g[i] * g[i]) * c2;
        float mh = m[i] * i1, vh = v[i] * i2;
        float u = (mh / (sqrtf(vh) + eps)) * lr;
        p[i] -= u;
    }
}

/* Mean of `models` parameter vectors of length n (model m at m*n), written
 * back to every model: sequential sum in model order, then / models. */
EXPORT void orc_average_models(float *p, int64_t n, int64_t models) {
    for (int64_t i = 0; i < n; i++) {
        float s = 0.0f;
        for (int64_t mm = 0; mm < models; mm++) s += p[mm * n + i];
        float mean = s / (float)models;
        for (int64_t mm = 0; mm < models; mm++) p[mm * n + i] = mean;
    }
}

/* ------------------------------------------------------------------------ */
/* Device optimiser steps, in-device model average and dropout              */
/* (src/gpu_step/mod.rs:232-275, src/gpu_step/tape.rs:526-582)              */
/* ------------------------------------------------------------------------ */

/* k_sgd (mod.rs:232-238): p -= lr * g */
EXPORT void orc_sgd(float *p, const float *g, int64_t n, float lr) {
    for (int64_t i = 0; i < n; i++) p[i] -= lr * g[i];
}

/* k_momentum (mod.rs:240-251): [p *= 1 - shrink * mask]; v = mu * v + g; p -= lr * v */
EXPORT void orc_momentum(float *p, const float *g, float *v, const float *mask, int64_t n, float lr, float mu,
                         float shrink) {
    for (int64_t i = 0; i < n; i++) {
        if (mask) p[i] *= 1.0f - shrink * mask[i];
        v[i] = mu * v[i] + g[i];
        p[i] -= lr * v[i];
    }
}

/* k_decay (mod.rs:253-259): p *= 1 - shrink * mask */
EXPORT void orc_decay(float *p, const float *mask, int64_t n, float shrink) {
    for (int64_t i = 0; i < n; i++) p[i] *= 1.0f - shrink * mask[i];
}

/* k_average_models (mod.rs:261-275): models k of `stride` floats, each group
 * of `group` consecutive models gets its mean (sequential sum / group). */
EXPORT void orc_average_groups(float *p, int64_t stride, int64_t k, int64_t group) {
    for (int64_t i = 0; i < stride; i++)
        for (int64_t g = 0; g < k / group; g++) {
            float s = 0.0f;
            for (int64_t m = 0; m < group; m++) s += p[(g * group + m) * stride + i];
            float mean = s / (float)group;
            for (int64_t m = 0; m < group; m++) p[(g * group + m) * stride + i] = mean;
        }
}

/* dropout_bits (tape.rs:545-555): lowbias32 of i + seed * 0x9e3779b9, wrapping u32. */
EXPORT uint32_t orc_dropout_bits(uint32_t i, uint32_t seed) {
    uint32_t h = i + seed * 0x9e3779b9u;
    h ^= h >> 16;
    h *= 0x7feb352du;
    h ^= h >> 15;
    h *= 0x846ca68bu;
    return h ^ (h >> 16);
}

/* dropout / dropout_relu_backward (tape.rs:526-543, k_dropout :557-568,
 * k_dropout_relu_bwd :570-582): threshold = (rate as f64 * 2^32) as u32
 * (saturating), scale = 1 / (1 - rate); relu_y may be NULL. */
EXPORT void orc_dropout(const float *x, const float *relu_y, float *y, int64_t n, float rate, uint32_t seed) {
    double t = (double)rate * 4294967296.0;
    uint32_t thr = !(t > 0.0) ? 0u : (t >= 4294967295.0 ? 0xffffffffu : (uint32_t)t);
    float scale = 1.0f / (1.0f - rate);
    for (int64_t i = 0; i < n; i++) {
        float v = 0.0f;
        int keep = orc_dropout_bits((uint32_t)i, seed) >= thr;
        if (relu_y) keep = keep && relu_y[i] > 0.0f;
        if (keep) v = x[i] * scale;
        y[i] = v;
    }
}
