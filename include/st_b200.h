/*
 * st_b200.h -- C ABI of scratchtape-b200, the B200 (sm_100a) implementation
 * of scratchtape's matmul family, batched causal attention and 2-bit kNN
 * scoring.
 *
 * Conventions
 *  - Every call enqueues on the handle's CUDA stream and returns at once; no
 *    call aborts across the FFI: failures come back as st_status, with text
 *    from st_last_error().  Device-side waits are bounded; a wait that runs
 *    out sets a device status word that st_sync() reports as ST_TIMEOUT.
 *  - Pointers marked "device" are caller-owned device memory.  The library
 *    owns only its scratch pool (grown on demand, reused afterwards, so a
 *    call repeated with the same shapes allocates nothing).
 *  - One handle per host thread; handles are not internally locked.
 *  - Results are deterministic: no float atomics; split-k partial sums are
 *    added in a fixed order.
 *
 * Each entry point names the reference interface it replaces (paths inside
 * the scratchtape crate).
 */
#ifndef ST_B200_H
#define ST_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define ST_API __attribute__((visibility("default")))
#else
#define ST_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    ST_OK = 0,
    ST_INVALID_ARG = 1,
    ST_UNSUPPORTED_SHAPE = 2,
    ST_CUDA_ERROR = 3,
    ST_NCCL_ERROR = 4,
    ST_TIMEOUT = 5,
    ST_NO_MEMORY = 6,
    ST_NOT_FOUND = 7
} st_status;

typedef enum { ST_F32 = 0, ST_F16 = 1, ST_BF16 = 2 } st_dtype;

/* Arithmetic of st_gemm.
 * F32_EXACT: SIMT, each output a k-ascending sequence of f32 multiply then
 *            add from 0 -- bit-identical to NdArray::matmul (src/tensor.rs:248-276).
 * TF32:      tcgen05 kind::tf32 tensor cores, f32 accumulate in TMEM.
 * F16:       a and b in f16 (ST_F16) or bf16 (ST_BF16), both the same; tcgen05
 *            kind::f16, f32 accumulate and an f32 out -- the reference's f16 x
 *            f16 -> f32 matrix-core path (k_matmul_cmma, src/gpu_step/matmul.rs:632-880).
 *            No col_sum; operands must be TMA-describable (16-byte aligned
 *            starts and row strides).
 * TF32X3:    f32 operands, each split into a TF32 high part and a TF32 rest;
 *            three TF32 tensor-core products (hi.hi + hi.lo + lo.hi) over
 *            operands concatenated along k (scratch: 3x each operand), error
 *            about 2^-21 of |a| |b| per product -- f32 accuracy at tensor-core
 *            speed, for what matmul_f32 (src/gpu_step/matmul.rs:93) keeps in f32. */
typedef enum { ST_PREC_F32_EXACT = 0, ST_PREC_TF32 = 1, ST_PREC_F16 = 2, ST_PREC_TF32X3 = 3 } st_precision;

typedef struct st_handle st_handle;

/* A matrix inside a device buffer -- mirrors MatRef (src/gpu_step/matmul.rs:31-60).
 * Matrix z starts at element off + (z / group) * stride + (z % group) * inner
 * of ptr; its stored rows are ld elements apart (0: packed).  trans: a
 * logical [r, c] operand stored as [c, r].  stride 0 reuses one matrix for
 * every batch.  group 0 is read as 1. */
typedef struct {
    void *ptr;
    int64_t off;
    int64_t stride;
    int64_t inner;
    int64_t ld;
    int32_t group;
    int32_t trans;
    int32_t dtype; /* st_dtype; st_gemm takes ST_F32 */
    int32_t reserved;
} st_mat;

/* Per-element epilogue in this order -- mirrors Epilogue
 * (src/gpu_step/matmul.rs:66-79): + bias[bias_off + z*bias_stride + col],
 * ReLU, zero where mask (out's layout, at mask_off) is not positive,
 * + residual (out's layout, at residual_off), + the value already in out.
 * col_sum: also add the column sums of b[z] over k into
 * col_sum[col_sum_off + z*col_sum_stride + col] (always +=).
 * Every pointer may be NULL. */
typedef struct {
    const float *bias;
    int64_t bias_off;
    int64_t bias_stride;
    const float *mask;
    int64_t mask_off;
    const float *residual;
    int64_t residual_off;
    float *col_sum;
    int64_t col_sum_off;
    int64_t col_sum_stride;
    int32_t relu;
    int32_t accumulate;
} st_epilogue;

/* ---- handle -------------------------------------------------------------- */

/* Creates a handle on CUDA device `device` that enqueues on `stream`
 * (a cudaStream_t; NULL = the legacy default stream).  Replaces the
 * cubecl client setup of src/gpu_step/mod.rs:78-97. */
ST_API st_status st_create(int device, void *stream, st_handle **out);
ST_API st_status st_destroy(st_handle *h);
ST_API st_status st_set_stream(st_handle *h, void *stream);
/* Text of the last failure on this handle (valid until the next call). */
ST_API const char *st_last_error(const st_handle *h);
/* Waits for the handle's stream, then reports a device-side status
 * (ST_TIMEOUT if a bounded wait ran out) and clears it. */
ST_API st_status st_sync(st_handle *h);
/* Kernels this library has launched on the handle since creation. */
ST_API int64_t st_launch_count(const st_handle *h);
/* Name of the last kernel this handle launched ("" before the first). */
ST_API const char *st_last_kernel(const st_handle *h);
/* Bytes currently held by the handle's scratch pool. */
ST_API int64_t st_scratch_bytes(const st_handle *h);

/* ---- matmul family --------------------------------------------------------- */

/* out[z] (+)= epilogue(a[z] . b[z]) for z < batch, a[z] logically [m, k],
 * b[z] [k, n], out[z] row-major [m, n] (out->trans must be 0).  NN, NT and
 * TN come from the operands' trans flags (transpose by descriptor, no
 * copy).  Replaces gpu_step::matmul::{matmul, matmul_f32, matmul_with}
 * (src/gpu_step/matmul.rs:86-192) and, with batch > 1, Tape::batched_matmul
 * (src/tape.rs:73-112).  TF32 needs 16-byte aligned rows (ld*4 % 16 == 0,
 * 16-byte aligned matrix starts); other layouts run the F32_EXACT kernel. */
ST_API st_status st_gemm(st_handle *h, const st_mat *a, const st_mat *b, const st_mat *out, int64_t batch, int64_t m,
                  int64_t k, int64_t n, const st_epilogue *epi, st_precision prec);

/* One GEMM of a group: out (+)= epilogue(a . b), batch 1, TF32.  after: bit j
 * set when this GEMM reads the output of the group's GEMM j (j < its index). */
typedef struct {
    st_mat a, b, out;
    int64_t m, k, n;
    const st_epilogue *epi; /* NULL, or an epilogue without col_sum */
    uint32_t after;
    int32_t reserved;
} st_group_gemm;

/* Up to 8 dependent TF32 GEMMs in one persistent launch: the sequence of
 * matmul calls that Tape::backward's MatMul arm and the layer forward issue
 * one by one (src/tape.rs:505-510, src/gpu_step/matmul.rs:106-192), with the
 * same results as calling st_gemm on each in order.  A tile of GEMM i starts
 * as soon as every GEMM named in its `after` mask has finished.  Needs
 * 16-byte aligned rows and n % 4 == 0 for every output; returns
 * ST_UNSUPPORTED_SHAPE otherwise (call st_gemm per GEMM then). */
ST_API st_status st_gemm_group(st_handle *h, const st_group_gemm *gemms, int32_t count);

/* st_gemm with ST_PREC_TF32 for callers that cannot let this library call
 * cudaMalloc: a host program that has already divided the GPU's memory among
 * its own pools and lends none to plug-ins, or a latency-critical loop where
 * a cudaMalloc / cudaFree (which may synchronise the whole device) would
 * stall it.  Split-k partial sums go to one 8 MiB array compiled into the
 * library (every GPU that loads the library holds it until the process
 * exits) instead of the handle's growable scratch pool, so the call calls no
 * cudaMalloc / cudaFree and no allocating library routine.
 * Limits: batch * m * n <= 1,048,576 output elements, k >= 1, f32 operands
 * that TMA can describe (16-byte aligned starts and rows); beyond them the
 * call returns ST_UNSUPPORTED_SHAPE (bad arguments: ST_INVALID_ARG) and
 * launches nothing.  Argument and shape refusals come back as the return
 * value only (st_last_error keeps its old text); a launch that fails returns
 * ST_CUDA_ERROR and also sets st_last_error; a device-side wait that runs out
 * is reported later, by st_sync (ST_TIMEOUT).  The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress); make that first call before
 * any stream capture.  All calls share the one array and it keeps the last
 * call's contents: calls that overlap on the GPU (other streams, other host
 * threads) race on it.
 * This entry point has no counterpart in the reference. */
ST_API st_status st_gemm_tf32_fixed_scratch(st_handle *h, const st_mat *a, const st_mat *b, const st_mat *out,
                                            int64_t batch, int64_t m, int64_t k, int64_t n, const st_epilogue *epi);

/* One Linear -> ReLU -> Linear layer without bias, forward and backward --
 * the six GEMMs Tape::backward's MatMul and Relu arms issue for it
 * (src/tape.rs:505-510, :530-534): h = relu(x w1), y = h w2,
 * dh = (dy w2^T) * (h > 0), dw2 = h^T dy, dx = dh w1^T, dw1 = x^T dh, on the
 * TF32 tensor cores in one fused cooperative kernel (h and dh never make a
 * round trip through global memory; each 128 x 128 block makes its own) that
 * also adds up the per-block partial products in a fixed order, so results
 * are deterministic.  Row-major device f32: x, dy, y, dx [m, d]; w1, dw1
 * [d, f]; w2, dw2 [f, d]; h, dh [m, f] (outputs; either may be null to skip
 * writing it).  Needs d == 128, m and f multiples of 128, (m/128)*(f/128) no
 * more than the GPU's SMs, 16-byte aligned buffers; returns
 * ST_UNSUPPORTED_SHAPE otherwise (use st_gemm per product then).  Calls on
 * one handle must not overlap on the GPU (they share its scratch and its
 * block counters).  The CTAs wait for each other with bounded waits; a wait
 * that runs out sets ST_TIMEOUT on the handle and leaves its counters
 * unusable: destroy that handle and create a new one. */
ST_API st_status st_mlp_step_tf32(st_handle *h, const float *x, const float *w1, const float *w2, const float *dy,
                                  float *hout, float *y, float *dhout, float *dx, float *dw1, float *dw2, int64_t m,
                                  int64_t d, int64_t f);

/* NdArray::matmul with host buffers (src/tensor.rs:241 and the drop-in
 * gpu_matmul, src/gpu.rs:98-169): out[m, n] = op(a) . op(b), row-major host
 * f32, ta: a stored [k, m], tb: b stored [n, k].  Copies in, computes,
 * copies out, and waits.  Device buffers come from the scratch pool. */
ST_API st_status st_matmul_host(st_handle *h, const float *a, const float *b, float *out, int64_t m, int64_t k, int64_t n,
                         int32_t ta, int32_t tb, st_precision prec);

/* ---- rows ------------------------------------------------------------------ */

/* Row softmax of scale*x over x [rows, n] (device f32); causal: row r sees
 * columns 0..=r%t and the rest are exactly 0; one: softmax1 with a phantom
 * 0 logit, shifted by max(row max, 0).  y may alias x.  Replaces
 * rows::softmax (src/gpu_step/rows.rs:106-112). */
ST_API st_status st_softmax_rows(st_handle *h, const float *x, float *y, int64_t rows, int64_t n, int64_t t, float scale,
                          int32_t causal, int32_t one);
/* dx = scale * y * (dy - sum(dy*y)) per row (rows.rs:117-123). */
ST_API st_status st_softmax_rows_bwd(st_handle *h, const float *dy, const float *y, float *dx, int64_t rows, int64_t n,
                              float scale);

/* ---- fused causal attention ----------------------------------------------- */

/* Fused attention over bh independent heads, f16 storage with f32
 * accumulation on tcgen05 (kind::f16): per head S = scale * Q K^T, causal
 * mask (column j visible to row i iff j <= i), P = softmax(S), O = P V.
 * one: softmax1 instead -- a phantom zero logit in every row's denominator,
 * shifted by max(row max, 0) (DeviceTape::causal_softmax(x, scale, one),
 * src/gpu_step/tape.rs:225; Config.softmax1 :400).
 * q, k, v, o: device f16 [bh, t, d], head z at z*t*d (16-byte aligned);
 * lse: device f32 [bh, t], the natural-log sum of exp of each scaled, masked
 * row, the phantom term included (for the backward).  t <= 256 (the
 * reference's MAX_SEQ), d = 64.  Replaces the chain
 * batched_matmul(q, k, transpose_b) -> scale -> + mask -> softmax ->
 * batched_matmul(w, v) of TransformerBlock::forward_full (src/nn.rs:646-671)
 * and of DeviceTape::block_forward (src/gpu_step/tape.rs:481-484). */
ST_API st_status st_attn_fwd(st_handle *h, const void *q, const void *k, const void *v, void *o, float *lse, int64_t bh,
                             int64_t t, int64_t d, float scale, int32_t causal, int32_t one);
/* Backward: dq, dk, dv (device f16 [bh, t, d]) from q, k, v, o, dout (f16)
 * and lse (f32) of st_attn_fwd (softmax or softmax1: lse carries it).  Replaces batched_matmul_backward
 * (src/tape.rs:90-112) and the softmax backward (src/gpu_step/rows.rs:117-123,
 * src/gpu_step/tape.rs:363-375). */
ST_API st_status st_attn_bwd(st_handle *h, const void *q, const void *k, const void *v, const void *o, const void *dout,
                             const float *lse, void *dq, void *dk, void *dv, int64_t bh, int64_t t, int64_t d, float scale,
                             int32_t causal);

/* st_attn_fwd on the transformer step's packed f32 layouts, as DeviceTape
 * addresses them through head views (MatRef::heads, src/gpu_step/matmul.rs:51-53;
 * src/gpu_step/tape.rs:196-212, :481-484): qkv [batch*t, 3*heads*d] (Q, K, V
 * column blocks of the fused QKV projection), o [batch*t, heads*d] (heads
 * merged), lse [batch*heads, t].  Operands are rounded to f16 as they are
 * staged (f32 accumulation); no split/merge copies. */
ST_API st_status st_attn_fwd_packed(st_handle *h, const float *qkv, float *o, float *lse, int64_t batch, int64_t heads,
                                    int64_t t, int64_t d, float scale, int32_t causal, int32_t one);
/* Backward on the same layouts: dqkv [batch*t, 3*heads*d] from qkv, o, dout
 * [batch*t, heads*d] and lse. */
ST_API st_status st_attn_bwd_packed(st_handle *h, const float *qkv, const float *o, const float *dout, const float *lse,
                                    float *dqkv, int64_t batch, int64_t heads, int64_t t, int64_t d, float scale,
                                    int32_t causal);

/* ---- transformer step: embedding, LayerNorm, cross-entropy, Adam ---------- */

/* x[r, :] = tok[ids[r], :] + pos[r % t, :] for r < batch*t (device f32 rows of d,
 * ids int32).  Replaces tokens::embed / k_embed (src/gpu_step/tokens.rs:22-67, :125-135). */
ST_API st_status st_embed_fwd(st_handle *h, const int32_t *ids, const float *tok, const float *pos, float *x,
                              int64_t batch, int64_t t, int64_t d);
/* dtok[v] (+)= sum of dx rows whose id is v, in row order; dpos[i] (+)= sum over
 * the batch of dx[b*t + i], in batch order (no atomics).  Replaces k_embed_bwd_tok /
 * k_embed_bwd_pos (src/gpu_step/tokens.rs:137-192).  d a multiple of 32, <= 1024. */
ST_API st_status st_embed_bwd(st_handle *h, const int32_t *ids, const float *dx, float *dtok, float *dpos,
                              int64_t batch, int64_t t, int64_t d, int64_t vocab, int32_t accumulate);
/* y = (x - mean) / sqrt(var + eps) * gamma + beta per row (biased variance);
 * saves mean and rstd per row.  Replaces rows::layer_norm (src/gpu_step/rows.rs:65-99). */
ST_API st_status st_layernorm_fwd(st_handle *h, const float *x, const float *gamma, const float *beta, float *y,
                                  float *mean, float *rstd, int64_t rows, int64_t d, float eps);
/* dx (+)= the input gradient; dgamma, dbeta += the parameter gradients (fixed
 * order).  d a multiple of 32, at most 512.  Replaces rows::layer_norm_backward
 * (src/gpu_step/rows.rs:100-293). */
ST_API st_status st_layernorm_bwd(st_handle *h, const float *dy, const float *x, const float *gamma,
                                  const float *mean, const float *rstd, float *dx, float *dgamma, float *dbeta,
                                  int64_t rows, int64_t d, int32_t accumulate);
/* loss[0] = mean over rows of -log softmax(logits)[target]; dlogits (may be
 * NULL) = (softmax - onehot) / rows.  Replaces tokens::cross_entropy and its
 * backward (src/gpu_step/tokens.rs:84-123, :194-253), without distillation. */
ST_API st_status st_cross_entropy(st_handle *h, const float *logits, const int32_t *targets, float *loss,
                                  float *dlogits, int64_t rows, int64_t vocab);
/* One Adam step over n parameters (step = the 1-based step count), in the
 * f32 operation order of Adam::step (src/optim.rs:42-57). */
ST_API st_status st_adam(st_handle *h, float *p, const float *g, float *m, float *v, int64_t n, int32_t step, float lr,
                         float beta1, float beta2, float eps);
/* st_adam with the step count in device memory: increments *step (device
 * int32), then updates with it -- the form a captured CUDA graph replays. */
ST_API st_status st_adam_dev(st_handle *h, float *p, const float *g, float *m, float *v, int64_t n, int32_t *step,
                             float lr, float beta1, float beta2, float eps);

/* ---- device optimiser, model average, dropout ---------------------------- */

/* p -= lr * g over n parameters (device f32).  Replaces DeviceParams::sgd
 * (src/gpu_step/mod.rs:153-157, k_sgd :232-238); same f32 operations. */
ST_API st_status st_sgd(st_handle *h, float *p, const float *g, int64_t n, float lr);
/* Heavy-ball momentum: with mask (may be NULL) first p *= 1 - shrink * mask,
 * then v = mu * v + g; p -= lr * v (v: device f32 [n], zero at the start).
 * Replaces DeviceParams::momentum (mod.rs:159-166, k_momentum :240-251). */
ST_API st_status st_momentum(st_handle *h, float *p, const float *g, float *v, const float *mask, int64_t n, float lr,
                             float mu, float shrink);
/* p *= 1 - shrink * mask (mask 0 or 1 per parameter).  Replaces
 * DeviceParams::decay (mod.rs:168-174, k_decay :253-259). */
ST_API st_status st_decay(st_handle *h, float *p, const float *mask, int64_t n, float shrink);
/* models consecutive parameter vectors of stride floats on one device, split
 * into consecutive groups of `group`: every model becomes its group's mean
 * (summed in model order, divided by group).  Replaces
 * DeviceParams::average_models / average_groups (mod.rs:182-195,
 * k_average_models :261-275). */
ST_API st_status st_average_models(st_handle *h, float *p, int64_t stride, int32_t models, int32_t group);
/* y = x / (1 - rate) where lowbias32(i + seed * 0x9e3779b9) >= rate * 2^32,
 * else 0 (n < 2^32, 0 <= rate < 1).  The same call on dy with the same seed is
 * dropout's backward.  Replaces gpu_step::tape::dropout
 * (src/gpu_step/tape.rs:526-534, k_dropout :557-568); bit-identical mask. */
ST_API st_status st_dropout(st_handle *h, const float *x, float *y, int64_t n, float rate, uint32_t seed);
/* dx = dropout(dy) where relu_y > 0, else 0: dropout's backward fused with
 * ReLU's (tape.rs:536-543, k_dropout_relu_bwd :570-582). */
ST_API st_status st_dropout_relu_bwd(st_handle *h, const float *dy, const float *relu_y, float *dx, int64_t n,
                                     float rate, uint32_t seed);

/* ---- across GPUs: NCCL over NVLink ------------------------------------------ */
/* NCCL is loaded at run time (libnccl.so.2, the process's own copy when one
 * is loaded); without it these return ST_NCCL_ERROR.  `comm` is an
 * ncclComm_t -- the host's own, or one from st_nccl_comm_init. */

/* 128 bytes of an ncclUniqueId, made on one rank and sent to the others by
 * the host's own channel. */
ST_API st_status st_nccl_unique_id(uint8_t *out);
/* ncclCommInitRank on `device` (made current): every rank calls it with the
 * same id; it returns once all nranks have joined. */
ST_API st_status st_nccl_comm_init(int32_t nranks, int32_t rank, const uint8_t *unique_id, int32_t device,
                                   void **comm_out);
ST_API st_status st_nccl_comm_destroy(void *comm);
/* Local-SGD model average across ranks: p (device f32 [n], the flat
 * parameters) becomes the mean over the communicator's ranks -- an in-place
 * sum all-reduce on the handle's stream, then p / world.  Replaces
 * DeviceParams::average_models (src/gpu_step/mod.rs:182-195) across GPUs, as
 * the training driver calls it every sync_every steps
 * (examples/tiny_lm/fused_models_check.rs:394). */
ST_API st_status st_avg_params(st_handle *h, float *p, int64_t n, void *comm);
/* st_knn_search over a key set split by rows across the communicator's
 * ranks: this rank holds rows index_base .. index_base + n_local - 1 (codes,
 * scales as st_knn_search; n_local may be 0) and every rank passes the same
 * queries.  Each rank scans its shard, the per-query best-128 lists are
 * all-gathered over NCCL and merged, and every rank gets the global best k
 * (out_scores / out_ids as st_knn_search, ids global).  Where the scan
 * seeds its thresholds from samples of the keys (dim 256: up to 32 queries,
 * or more than 32 EXACT dot-product queries), each sampling stage's lists
 * are also all-gathered and merged, so every rank filters against the best
 * 128 of all ranks' samples.  Every rank must call it with the same nq, dim,
 * mode and prec (the collectives are the same on every rank).  Replaces
 * k_sort_lists + k_merge_parts (src/gpu_step/knn.rs:661-715) across GPUs. */
ST_API st_status st_knn_search_sharded(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_local,
                                       int32_t dim, const float *queries, int64_t nq, int32_t k, int32_t mode,
                                       int32_t prec, int64_t index_base, void *comm, float *out_scores,
                                       int64_t *out_ids);

/* ---- kNN memory: 2-bit key scan fused with top-k ------------------------- */

/* Ranking modes (src/gpu_step/knn.rs:5, :522-532, :855).
 * DOT: q.k, largest first.  L2: |k|^2 - 2 q.k + |q|^2 clamped at 0,
 * smallest first.  Ties go to the lower key index. */
typedef enum { ST_KNN_DOT = 0, ST_KNN_L2 = 1 } st_knn_mode;
/* Arithmetic.  EXACT: every returned score within about 2^-22 of
 * sum_i |q_i k_i| of the exact score -- more than 32 dot-product queries at
 * dim 256 are filtered on the tensor cores and rescored exactly in f64 (one
 * rounding); up to 32 queries at dim 256 use a 30-bit fixed-point query with
 * exact integer products; other shapes split the query into two f16 parts
 * with f32 accumulation.  F16REF: the reference's numerics --
 * query and dequantised key (u - 1.5) * scale rounded to f16 before the
 * product (knn.rs:403-411, :630-643). */
typedef enum { ST_KNN_EXACT = 0, ST_KNN_F16REF = 1 } st_knn_prec;

/* The best k (1..128) keys per query.  codes: device [n_keys, dim/4] bytes,
 * 2-bit codes packed low bits first (16-byte aligned); scales: device f32
 * [n_keys]; queries: device f32 [nq, dim] (16-byte aligned); dim in {64, 128,
 * 192, 256}.  out_scores: device f32 [nq, k] (DOT: q.k; L2: distance);
 * out_ids: device int64 [nq, k] = index_base + key row, best first; missing
 * entries (fewer than k keys) are (-inf or +inf, -1).  index_base + n_keys
 * must stay below 2^32 - 1.  Replaces KnnStore::search / search_tagged and
 * the search_from / search_block path (src/gpu_step/knn.rs:264-331,
 * :401-535), with indices returned instead of values. */
ST_API st_status st_knn_search(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_keys, int32_t dim,
                               const float *queries, int64_t nq, int32_t k, int32_t mode, int32_t prec,
                               int64_t index_base, float *out_scores, int64_t *out_ids);
/* st_knn_search restricted per query: key j (global index) is visible to
 * query q iff j < always or ranges[2q] <= j < ranges[2q+1] (ranges: device
 * int64 [nq, 2]).  Replaces KnnStore::search_masked / search_tagged with a
 * mask (src/gpu_step/knn.rs:280-299). */
ST_API st_status st_knn_search_masked(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_keys,
                                      int32_t dim, const float *queries, int64_t nq, int32_t k, int32_t mode,
                                      int32_t prec, int64_t index_base, const int64_t *ranges, int64_t always,
                                      float *out_scores, int64_t *out_ids);
/* The same scan, stopping before decoding: out_keys, device u64 [nq, 128],
 * holds each query's best 128 as sortable 64-bit keys (score bits << 32 |
 * 0xFFFFFFFF - index), best first, 0 = empty.  Keys of different shards (each
 * with its own index_base) merge with st_knn_merge_keys -- the multi-GPU path
 * gathers them over NCCL first.  Replaces k_sort_lists + k_merge_parts
 * (src/gpu_step/knn.rs:661-715) across shards. */
ST_API st_status st_knn_topk_keys(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_keys,
                                  int32_t dim, const float *queries, int64_t nq, int32_t mode, int32_t prec,
                                  int64_t index_base, uint64_t *out_keys);
/* out_keys[q] = best 128 of lists[l * list_stride + q * 128 + r] over
 * l < n_lists (device u64), best first. */
ST_API st_status st_knn_merge_keys(st_handle *h, const uint64_t *lists, int64_t n_lists, int64_t list_stride,
                                   int64_t nq, uint64_t *out_keys);
/* Keys [nq, 128] -> out_scores [nq, k], out_ids [nq, k] as st_knn_search
 * returns them (queries as given to the scan). */
ST_API st_status st_knn_decode(st_handle *h, const uint64_t *keys, const float *queries, int64_t nq, int32_t dim,
                               int32_t k, int32_t mode, int32_t prec, float *out_scores, int64_t *out_ids);
/* The 2-bit quantiser of KnnStore::add (tile_of, src/gpu_step/knn.rs:190-221,
 * quant_step :647-653) on the device, bit-identical to the reference's f32
 * arithmetic: keys device f32 [n, dim] -> codes [n, dim/4], scales [n],
 * norms [n] (sum of f16-rounded squares; may be NULL). */
ST_API st_status st_knn_quantize(st_handle *h, const float *keys, int64_t n, int32_t dim, uint8_t *codes,
                                 float *scales, float *norms);
/* The fused scan over a table of work units -- the IVF search of
 * src/gpu_step/knn/ivf.rs:466-690 (search_ivf / scan_group): unit u scans
 * store rows unit_keys[2u] .. unit_keys[2u + 1] (a cell) for the queries
 * unit_q[u * 128 + r] (-1: an empty row), and row r's best 128 become list
 * unit_list[u * 128 + r] (< n_lists) of that query; out_keys [nq, 128]
 * (device u64, as st_knn_topk_keys) is each query's best 128 over its lists.
 * The three tables are HOST arrays, checked before anything is launched. */
ST_API st_status st_knn_scan_units(st_handle *h, const uint8_t *codes, const float *scales, int64_t n_keys,
                                   int32_t dim, const float *queries, int64_t nq, int32_t mode, int32_t prec,
                                   int64_t index_base, int64_t n_units, const int32_t *unit_q,
                                   const int32_t *unit_list, const int64_t *unit_keys, int32_t n_lists,
                                   uint64_t *out_keys);
/* Host-side planning of that scan for an IVF search (the cell loop of
 * search_ivf, src/gpu_step/knn/ivf.rs:466-526): probes [nq, nprobe] (host
 * int32, each query's probed cells), starts [nlist + 1] (host, cell c holds
 * store rows starts[c] .. starts[c + 1]).  A cell longer than `chunk` keys is
 * scanned as several chunks, each its own unit and its own list of the
 * query; chunk <= 0 picks one that gives about two units of work per SM
 * (n_sms) and at most max_lists lists per query.  Units are (cell chunk, up
 * to 128 of the queries probing it), longest first.  Call it first with
 * NULL tables to learn *n_units (and *n_lists, *chunk_used), then with
 * tables of that many units (unit_q, unit_list [n_units, 128],
 * unit_keys [n_units, 2]) for st_knn_scan_units.  Needs no handle and no GPU. */
ST_API st_status st_knn_ivf_units(const int32_t *probes, int64_t nq, int32_t nprobe, const int64_t *starts,
                                  int32_t nlist, int32_t n_sms, int64_t chunk, int32_t max_lists, int32_t *unit_q,
                                  int32_t *unit_list, int64_t *unit_keys, int64_t *n_units, int32_t *n_lists,
                                  int64_t *chunk_used);
/* out [n, dim] f32 = (u - 1.5) * scale of 2-bit rows (k_dequant, knn.rs:630-643, kept in f32). */
ST_API st_status st_knn_dequant(st_handle *h, const uint8_t *codes, const float *scales, int64_t n, int32_t dim,
                                float *out);
/* out[r] = the nearest centroid of row r from dots = rows . centroids^T [n, nlist]
 * and cnorm = |centroid|^2 (argmin of cnorm - 2 dot, lowest index on ties;
 * k_argmin, ivf.rs:75-113). */
ST_API st_status st_knn_nearest(st_handle *h, const float *dots, const float *cnorm, int64_t n, int32_t nlist,
                                int32_t *out);
/* out [nq, nprobe] = each query's nprobe nearest centroids, nearest first
 * (k_probe, ivf.rs:126-165); nprobe <= min(nlist, 64). */
ST_API st_status st_knn_probe(st_handle *h, const float *dots, const float *cnorm, int64_t nq, int32_t nlist,
                              int32_t nprobe, int32_t *out);
/* dst row i = src row perm[i] (device i64) for i < n, rows of row_bytes (a
 * multiple of 4): the cell-order reordering of build_ivf (ivf.rs:395-425) on
 * the device.  An entry outside [0, n_src) gives a zero row and ST_INVALID_ARG
 * at the next st_sync. */
ST_API st_status st_gather_rows(st_handle *h, const void *src, int64_t n_src, void *dst, const int64_t *perm,
                                int64_t n, int64_t row_bytes);

/* Synthetic keys (benchmark and tests): codes uniform on 0..3 and scale =
 * |N(0,1)|, from a counter-based hash of (seed, first_key + row), so each
 * shard makes its own rows independently.  No reference counterpart (the
 * reference builds keys from trained hidden states). */
ST_API st_status st_knn_synth_keys(st_handle *h, uint8_t *codes, float *scales, int64_t n, int32_t dim, uint64_t seed,
                                   int64_t first_key);

#ifdef __cplusplus
}
#endif

#endif /* ST_B200_H */
