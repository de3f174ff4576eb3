/*
 * st_oracle_knn.c -- CPU restatement of the kNN memory's 2-bit key path.
 *
 * TEST INFRASTRUCTURE ONLY (see st_oracle.c): the parity oracle and the
 * timed CPU baseline for the 2-bit scan.  The product never links it.
 *
 * Reference: src/gpu_step/knn.rs of scratchtape.
 *   - quantiser: tile_of (knn.rs:190-221) and quant_step (knn.rs:647-653);
 *   - dequant: k_dequant (knn.rs:630-643), value = (u - half) * scale;
 *   - L2 ranking: dist = |k|^2 - 2 q.k (+ |q|^2 on the host, clamped >= 0)
 *     (knn.rs:5, :522-532, :855); brute force as the tests do (knn.rs:893-906).
 * Exact mode computes q.k in f64 from the stored codes and scales; f16 mode
 * restates the reference's f16 matrix-core numerics (queries and dequantised
 * keys rounded to f16 before the product, knn.rs:403-411, :630-643) with the
 * products summed in f64.
 *
 * Parity for 2-bit scores is pinned only by this definition: the reference's
 * own quantised-key test tolerates any 2-bit error (ivf.rs:746-780).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

#define EXPORT __attribute__((visibility("default")))

/* quant_step (knn.rs:647-653) */
static float quant_step(int bits) { return bits == 2 ? 0.9957f : bits == 4 ? 0.3352f : 0.031f; }

/* IEEE binary16 round-to-nearest-even of a float, returned as float
 * (half::f16::from_f32(x).to_f32()). */
EXPORT float orc_round_f16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    uint32_t sign = u & 0x80000000u;
    uint32_t ax = u & 0x7fffffffu;
    float r;
    if (ax >= 0x7f800000u) return x; /* inf / nan */
    float a;
    memcpy(&a, &ax, 4);
    if (a >= 65520.0f) {
        r = INFINITY;
    } else if (a < 6.103515625e-05f) {
        /* subnormal half: quantum 2^-24 */
        double q = ldexp(1.0, -24);
        double v = (double)a / q;
        double fl = floor(v);
        double frac = v - fl;
        double n = fl;
        if (frac > 0.5 || (frac == 0.5 && fmod(fl, 2.0) != 0.0)) n = fl + 1.0;
        r = (float)(n * q);
    } else {
        int e;
        frexp(a, &e); /* a = f * 2^e, f in [0.5,1) */
        double q = ldexp(1.0, e - 11);
        double v = (double)a / q;
        double fl = floor(v);
        double frac = v - fl;
        double n = fl;
        if (frac > 0.5 || (frac == 0.5 && fmod(fl, 2.0) != 0.0)) n = fl + 1.0;
        r = (float)(n * q);
    }
    uint32_t ru;
    memcpy(&ru, &r, 4);
    ru |= sign;
    memcpy(&r, &ru, 4);
    return r;
}

/* tile_of's quantiser for `bits` in {2,4,8} (knn.rs:199-220): per row,
 * scale = max(step * sqrt(sum(x*x) / d), 1e-30); u = clamp(round(x/scale + half), 0, top)
 * (round half away from zero, f32::round); codes packed low bits first;
 * norm = sum over i of f16((u - half) * scale)^2 (f32, sequential). */
EXPORT void orc_quantize_rows(const float *keys, int64_t n, int64_t d, int bits, uint8_t *codes, float *scales,
                              float *norms) {
    float half = (float)((1u << bits) - 1) / 2.0f, top = (float)((1u << bits) - 1);
    float step = quant_step(bits);
    int64_t kb = d * bits / 8;
    int *v = (int *)malloc(sizeof(int) * d);
    for (int64_t r = 0; r < n; r++) {
        const float *k = keys + r * d;
        float ss = 0.0f;
        for (int64_t i = 0; i < d; i++) ss += k[i] * k[i];
        float scale = step * sqrtf(ss / (float)d);
        if (!(scale >= 1e-30f)) scale = 1e-30f;
        for (int64_t i = 0; i < d; i++) {
            float u = roundf(k[i] / scale + half);
            if (u < 0.0f) u = 0.0f;
            if (u > top) u = top;
            v[i] = (int)u;
        }
        uint8_t *row = codes + r * kb;
        memset(row, 0, kb);
        for (int64_t i = 0; i < d; i++) {
            int64_t at = i * bits;
            row[at / 8] |= (uint8_t)((v[i] & ((1 << bits) - 1)) << (at % 8));
        }
        scales[r] = scale;
        float nrm = 0.0f;
        for (int64_t i = 0; i < d; i++) {
            float h = orc_round_f16(((float)v[i] - half) * scale);
            nrm += h * h;
        }
        if (norms) norms[r] = nrm;
    }
    free(v);
}

/* k_dequant (knn.rs:630-643): rows [n, d] of (u - half) * scale; as f16 when
 * to_f16 (the reference's matmul operand), else exact f32. */
EXPORT void orc_dequant_rows(const uint8_t *codes, const float *scales, int64_t n, int64_t d, int bits, int to_f16,
                             float *out) {
    int64_t kb = d * bits / 8;
    float half = (float)((1u << bits) - 1) * 0.5f;
    for (int64_t r = 0; r < n; r++)
        for (int64_t i = 0; i < d; i++) {
            int64_t at = i * bits;
            int u = (codes[r * kb + at / 8] >> (at % 8)) & ((1 << bits) - 1);
            float v = ((float)u - half) * scales[r];
            out[r * d + i] = to_f16 ? orc_round_f16(v) : v;
        }
}

/* ------------------------------------------------------------------------ */
/* Brute-force top-k over 2-bit keys                                         */
/* ------------------------------------------------------------------------ */

/* Modes: 0 = DOT (score = q.k, largest first), 1 = L2 (dist = |k|^2 - 2 q.k
 * + |q|^2 clamped >= 0, smallest first; knn.rs:522-532).  prec: 0 = exact
 * (f64 from codes and scales), 1 = f16 reference numerics.  Ties are broken
 * by the lower key index.  mask (nullable): key j is allowed for query r iff
 * j < always or lo[r] <= j < hi[r] (search_masked, knn.rs:280-291).
 * Fewer than k allowed keys pad with (+-inf, -1). */
struct knn_job {
    const uint8_t *codes;
    const float *scales;
    int64_t n, d;
    const float *q;
    int64_t q_lo, q_hi, k;
    int mode, prec;
    const int64_t *lo, *hi;
    int64_t always;
    float *out_s;
    int64_t *out_i;
    double *out_s64;
};

static int better(int mode, double a, int64_t ia, double b, int64_t ib) {
    if (a != b) return mode == 0 ? a > b : a < b;
    return ia < ib;
}

/* sift-down in a heap whose root is the WORST kept entry */
static void heap_down(double *hs, int64_t *hi, int64_t k, int64_t i, int mode) {
    for (;;) {
        int64_t l = 2 * i + 1, r = l + 1, w = i;
        if (l < k && better(mode, hs[w], hi[w], hs[l], hi[l])) w = l;
        if (r < k && better(mode, hs[w], hi[w], hs[r], hi[r])) w = r;
        if (w == i) return;
        double ts = hs[i]; hs[i] = hs[w]; hs[w] = ts;
        int64_t ti = hi[i]; hi[i] = hi[w]; hi[w] = ti;
        i = w;
    }
}

static void *knn_worker(void *p) {
    struct knn_job *J = (struct knn_job *)p;
    int64_t d = J->d, kb = d / 4, k = J->k;
    double *qv = (double *)malloc(sizeof(double) * d);
    double *hs = (double *)malloc(sizeof(double) * k);
    int64_t *hix = (int64_t *)malloc(sizeof(int64_t) * k);
    double lut[4] = {-1.5, -0.5, 0.5, 1.5};
    for (int64_t r = J->q_lo; r < J->q_hi; r++) {
        const float *q = J->q + r * d;
        double qn = 0;
        for (int64_t i = 0; i < d; i++) {
            float qq = J->prec ? orc_round_f16(q[i]) : q[i];
            qv[i] = qq;
        }
        {
            float qf = 0.0f; /* |q|^2 as the host adds it: f32 sequential over the raw query */
            for (int64_t i = 0; i < d; i++) qf += q[i] * q[i];
            qn = qf;
        }
        int64_t cnt = 0;
        for (int64_t j = 0; j < J->n; j++) {
            if (J->lo && !(j < J->always || (j >= J->lo[r] && j < J->hi[r]))) continue;
            const uint8_t *c = J->codes + j * kb;
            double s = J->scales[j];
            double dot = 0, nrm = 0;
            if (J->prec == 0) {
                for (int64_t w = 0; w < kb; w++) {
                    uint8_t b = c[w];
                    dot += lut[b & 3] * qv[4 * w] + lut[(b >> 2) & 3] * qv[4 * w + 1] + lut[(b >> 4) & 3] * qv[4 * w + 2] +
                           lut[(b >> 6) & 3] * qv[4 * w + 3];
                    nrm += lut[b & 3] * lut[b & 3] + lut[(b >> 2) & 3] * lut[(b >> 2) & 3] +
                           lut[(b >> 4) & 3] * lut[(b >> 4) & 3] + lut[(b >> 6) & 3] * lut[(b >> 6) & 3];
                }
                dot *= s;
                nrm *= s * s;
            } else {
                float fs = J->scales[j];
                for (int64_t i = 0; i < d; i++) {
                    int u = (c[i / 4] >> (2 * (i % 4))) & 3;
                    double kv = orc_round_f16(((float)u - 1.5f) * fs);
                    dot += kv * qv[i];
                    nrm += kv * kv;
                }
            }
            double score = J->mode == 0 ? dot : nrm - 2.0 * dot + qn;
            if (J->mode == 1 && score < 0) score = 0;
            if (cnt < k) {
                hs[cnt] = score;
                hix[cnt] = j;
                cnt++;
                if (cnt == k)
                    for (int64_t i = k / 2 - 1; i >= 0; i--) heap_down(hs, hix, k, i, J->mode);
            } else if (better(J->mode, score, j, hs[0], hix[0])) {
                hs[0] = score;
                hix[0] = j;
                heap_down(hs, hix, k, 0, J->mode);
            }
        }
        /* sort kept entries best first (insertion sort; k is small) */
        for (int64_t a = 1; a < cnt; a++) {
            double ts = hs[a];
            int64_t ti = hix[a];
            int64_t b = a - 1;
            while (b >= 0 && better(J->mode, ts, ti, hs[b], hix[b])) {
                hs[b + 1] = hs[b];
                hix[b + 1] = hix[b];
                b--;
            }
            hs[b + 1] = ts;
            hix[b + 1] = ti;
        }
        for (int64_t a = 0; a < k; a++) {
            double sc = a < cnt ? hs[a] : (J->mode == 0 ? -INFINITY : INFINITY);
            if (J->out_s) J->out_s[r * k + a] = (float)sc;
            if (J->out_s64) J->out_s64[r * k + a] = sc;
            J->out_i[r * k + a] = a < cnt ? hix[a] : -1;
        }
    }
    free(qv);
    free(hs);
    free(hix);
    return NULL;
}

EXPORT void orc_knn_topk(const uint8_t *codes, const float *scales, int64_t n, int64_t d, const float *queries,
                         int64_t nq, int64_t k, int mode, int prec, const int64_t *lo, const int64_t *hi,
                         int64_t always, float *out_scores, double *out_scores64, int64_t *out_ids, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (threads > nq) threads = (int)(nq > 0 ? nq : 1);
    pthread_t tid[256];
    struct knn_job jobs[256];
    int64_t per = (nq + threads - 1) / threads;
    int used = 0;
    for (int t = 0; t < threads; t++) {
        int64_t a = t * per, b = a + per < nq ? a + per : nq;
        if (a >= b) break;
        jobs[t] = (struct knn_job){codes, scales, n, d, queries, a, b, k, mode, prec, lo, hi, always,
                                   out_scores, out_ids, out_scores64};
        pthread_create(&tid[t], NULL, knn_worker, &jobs[t]);
        used++;
    }
    for (int t = 0; t < used; t++) pthread_join(tid[t], NULL);
}

/* Exact f64 dot products q.k for given (query, key) pairs: the error check
 * of a returned list.  out[i] = q[qi[i]] . dequant(key kj[i]). */
EXPORT void orc_knn_pair_dots(const uint8_t *codes, const float *scales, int64_t d, const float *queries,
                              const int64_t *qi, const int64_t *kj, int64_t pairs, double *out) {
    int64_t kb = d / 4;
    double lut[4] = {-1.5, -0.5, 0.5, 1.5};
    for (int64_t p = 0; p < pairs; p++) {
        const uint8_t *c = codes + kj[p] * kb;
        const float *q = queries + qi[p] * d;
        double dot = 0;
        for (int64_t i = 0; i < d; i++) dot += lut[(c[i / 4] >> (2 * (i % 4))) & 3] * (double)q[i];
        out[p] = dot * (double)scales[kj[p]];
    }
}

/* ------------------------------------------------------------------------ */
/* Brute force over the benchmark's synthetic keys, regenerated on the fly   */
/* ------------------------------------------------------------------------ */

/* The synthetic keys' code bytes (no reference counterpart: the library's
 * st_knn_synth_keys, which makes the benchmark's 2^27 keys): the 64-bit
 * words of key `key` are mix64(base + 1 + w), base = mix64(seed ^ mix64(key)),
 * mix64 being SplitMix64's finaliser.  Integer arithmetic only, so the codes
 * regenerate bit for bit; the scales (which use logf/cosf) are taken from the
 * device instead. */
static uint64_t mix64(uint64_t z) {
    z += 0x9e3779b97f4a7c15ull;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

EXPORT void orc_synth_codes(uint64_t seed, int64_t first, int64_t n, int64_t d, uint8_t *codes) {
    int64_t words = d / 32;
    for (int64_t r = 0; r < n; r++) {
        uint64_t base = mix64(seed ^ mix64((uint64_t)(first + r)));
        for (int64_t w = 0; w < words; w++) {
            uint64_t v = mix64(base + 1 + (uint64_t)w);
            memcpy(codes + r * (d / 4) + 8 * w, &v, 8);
        }
    }
}

struct synth_job {
    uint64_t seed;
    int64_t first, a, b, d, nq, k;
    const float *scales; /* [n], indexed by row */
    const double *tab;   /* [nq][d/4][256] byte tables */
    double *best_s;      /* [nq][k] this thread's best, descending */
    int64_t *best_i;
};

/* insert (s, i) into a descending list of k (ties: lower index first) */
static void put_best(double *bs, int64_t *bi, int64_t k, double s, int64_t i) {
    if (!(s > bs[k - 1] || (s == bs[k - 1] && i < bi[k - 1]))) return;
    int64_t p = k - 1;
    while (p > 0 && (s > bs[p - 1] || (s == bs[p - 1] && i < bi[p - 1]))) {
        bs[p] = bs[p - 1];
        bi[p] = bi[p - 1];
        p--;
    }
    bs[p] = s;
    bi[p] = i;
}

static void *synth_worker(void *arg) {
    struct synth_job *j = (struct synth_job *)arg;
    int64_t kb = j->d / 4;
    uint8_t codes[64];
    for (int64_t q = 0; q < j->nq * j->k; q++) {
        j->best_s[q] = -INFINITY;
        j->best_i[q] = -1;
    }
    for (int64_t r = j->a; r < j->b; r++) {
        orc_synth_codes(j->seed, j->first + r, 1, j->d, codes);
        double sc = (double)j->scales[r];
        for (int64_t q = 0; q < j->nq; q++) {
            const double *t = j->tab + q * kb * 256;
            double dot = 0;
            for (int64_t c = 0; c < kb; c++) dot += t[c * 256 + codes[c]];
            put_best(j->best_s + q * j->k, j->best_i + q * j->k, j->k, dot * sc, j->first + r);
        }
    }
    return NULL;
}

/* DOT-mode top-k of nq queries over the n synthetic keys first..first+n-1
 * (scales from the device), exact in f64: q.k = scale * sum_i (u_i - 1.5) q_i,
 * the per-byte partial sums of four dimensions tabulated per query.  Scores
 * descending, ties to the lower index; out_scores64 [nq, k], out_ids [nq, k]. */
EXPORT void orc_knn_topk_synth(uint64_t seed, int64_t first, int64_t n, int64_t d, const float *scales,
                               const float *queries, int64_t nq, int64_t k, double *out_scores64, int64_t *out_ids,
                               int threads) {
    int64_t kb = d / 4;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    double *tab = (double *)malloc(sizeof(double) * nq * kb * 256);
    static const double lut[4] = {-1.5, -0.5, 0.5, 1.5};
    for (int64_t q = 0; q < nq; q++)
        for (int64_t c = 0; c < kb; c++)
            for (int v = 0; v < 256; v++) {
                double s = 0;
                for (int p = 0; p < 4; p++) s += lut[(v >> (2 * p)) & 3] * (double)queries[q * d + 4 * c + p];
                tab[(q * kb + c) * 256 + v] = s;
            }
    pthread_t tid[256];
    struct synth_job jobs[256];
    int64_t per = (n + threads - 1) / threads;
    int used = 0;
    for (int t = 0; t < threads; t++) {
        int64_t a = t * per, b = a + per < n ? a + per : n;
        if (a >= b) break;
        jobs[t] = (struct synth_job){seed, first, a, b, d, nq, k, scales, tab,
                                     (double *)malloc(sizeof(double) * nq * k),
                                     (int64_t *)malloc(sizeof(int64_t) * nq * k)};
        pthread_create(&tid[t], NULL, synth_worker, &jobs[t]);
        used++;
    }
    for (int t = 0; t < used; t++) pthread_join(tid[t], NULL);
    for (int64_t q = 0; q < nq; q++) {
        double *bs = out_scores64 + q * k;
        int64_t *bi = out_ids + q * k;
        for (int64_t i = 0; i < k; i++) {
            bs[i] = -INFINITY;
            bi[i] = -1;
        }
        for (int t = 0; t < used; t++)
            for (int64_t i = 0; i < k; i++)
                if (jobs[t].best_i[q * k + i] >= 0)
                    put_best(bs, bi, k, jobs[t].best_s[q * k + i], jobs[t].best_i[q * k + i]);
    }
    for (int t = 0; t < used; t++) {
        free(jobs[t].best_s);
        free(jobs[t].best_i);
    }
    free(tab);
}

/* Exact f64 q.k for given (query, synthetic key) pairs (scales indexed by
 * key - first). */
EXPORT void orc_knn_pair_dots_synth(uint64_t seed, int64_t first, int64_t d, const float *scales,
                                    const float *queries, const int64_t *qi, const int64_t *kj, int64_t pairs,
                                    double *out) {
    static const double lut[4] = {-1.5, -0.5, 0.5, 1.5};
    uint8_t codes[64];
    for (int64_t p = 0; p < pairs; p++) {
        orc_synth_codes(seed, kj[p], 1, d, codes);
        const float *q = queries + qi[p] * d;
        double dot = 0;
        for (int64_t i = 0; i < d; i++) dot += lut[(codes[i / 4] >> (2 * (i % 4))) & 3] * (double)q[i];
        out[p] = dot * (double)scales[kj[p] - first];
    }
}
