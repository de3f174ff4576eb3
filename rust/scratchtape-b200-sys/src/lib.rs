//! Raw declarations of libst_b200.so, the B200 (sm_100a) kernels for
//! scratchtape's matmul family, batched causal attention and 2-bit kNN
//! scoring.  Every item mirrors `include/st_b200.h` of scratchtape-b200 one
//! to one (`tests/test_rust_ffi.py` checks the two against each other); the
//! header documents each entry point and the reference interface it
//! replaces.  Enumerations (`st_precision`, the kNN mode and precision) are
//! passed as `c_int`.  A communicator argument is an `ncclComm_t`.
#![allow(non_camel_case_types)]
use std::os::raw::{c_char, c_int, c_void};

/// Opaque library handle: one CUDA device and stream, its scratch pool and
/// its error text.  Not internally locked: one per host thread.
#[repr(C)]
pub struct st_handle {
    _p: [u8; 0],
}

/// Status of every call: `ST_OK` or the reason it refused or failed.
pub type st_status = c_int;
pub const ST_OK: st_status = 0;
pub const ST_INVALID_ARG: st_status = 1;
pub const ST_UNSUPPORTED_SHAPE: st_status = 2;
pub const ST_CUDA_ERROR: st_status = 3;
pub const ST_NCCL_ERROR: st_status = 4;
pub const ST_TIMEOUT: st_status = 5;
pub const ST_NO_MEMORY: st_status = 6;
pub const ST_NOT_FOUND: st_status = 7;

pub const ST_F32: i32 = 0;
pub const ST_F16: i32 = 1;
pub const ST_BF16: i32 = 2;
pub const ST_PREC_F32_EXACT: c_int = 0;
pub const ST_PREC_TF32: c_int = 1;
pub const ST_PREC_F16: c_int = 2;
pub const ST_PREC_TF32X3: c_int = 3;
pub const ST_KNN_DOT: i32 = 0;
pub const ST_KNN_L2: i32 = 1;
pub const ST_KNN_EXACT: i32 = 0;
pub const ST_KNN_F16REF: i32 = 1;

/// A matrix inside a device buffer: `MatRef` (src/gpu_step/matmul.rs) field for field.
#[repr(C)]
#[derive(Clone, Copy)]
pub struct st_mat {
    pub ptr: *mut c_void,
    pub off: i64,
    pub stride: i64,
    pub inner: i64,
    pub ld: i64,
    pub group: i32,
    pub trans: i32,
    pub dtype: i32,
    pub reserved: i32,
}

/// The per-element epilogue: `Epilogue` (src/gpu_step/matmul.rs) field for field.
#[repr(C)]
#[derive(Clone, Copy)]
pub struct st_epilogue {
    pub bias: *const f32,
    pub bias_off: i64,
    pub bias_stride: i64,
    pub mask: *const f32,
    pub mask_off: i64,
    pub residual: *const f32,
    pub residual_off: i64,
    pub col_sum: *mut f32,
    pub col_sum_off: i64,
    pub col_sum_stride: i64,
    pub relu: i32,
    pub accumulate: i32,
}

/// One GEMM of an `st_gemm_group` launch.
#[repr(C)]
#[derive(Clone, Copy)]
pub struct st_group_gemm {
    pub a: st_mat,
    pub b: st_mat,
    pub out: st_mat,
    pub m: i64,
    pub k: i64,
    pub n: i64,
    pub epi: *const st_epilogue,
    pub after: u32,
    pub reserved: i32,
}

extern "C" {
    pub fn st_create(device: c_int, stream: *mut c_void, out: *mut *mut st_handle) -> st_status;
    pub fn st_destroy(h: *mut st_handle) -> st_status;
    pub fn st_set_stream(h: *mut st_handle, stream: *mut c_void) -> st_status;
    pub fn st_last_error(h: *const st_handle) -> *const c_char;
    pub fn st_sync(h: *mut st_handle) -> st_status;
    pub fn st_launch_count(h: *const st_handle) -> i64;
    pub fn st_last_kernel(h: *const st_handle) -> *const c_char;
    pub fn st_scratch_bytes(h: *const st_handle) -> i64;
    pub fn st_gemm(h: *mut st_handle, a: *const st_mat, b: *const st_mat, out: *const st_mat, batch: i64, m: i64,
                   k: i64, n: i64, epi: *const st_epilogue, prec: c_int) -> st_status;
    pub fn st_gemm_group(h: *mut st_handle, gemms: *const st_group_gemm, count: i32) -> st_status;
    pub fn st_gemm_tf32_fixed_scratch(h: *mut st_handle, a: *const st_mat, b: *const st_mat, out: *const st_mat,
                                      batch: i64, m: i64, k: i64, n: i64, epi: *const st_epilogue) -> st_status;
    pub fn st_mlp_step_tf32(h: *mut st_handle, x: *const f32, w1: *const f32, w2: *const f32, dy: *const f32,
                            hout: *mut f32, y: *mut f32, dhout: *mut f32, dx: *mut f32, dw1: *mut f32, dw2: *mut f32,
                            m: i64, d: i64, f: i64) -> st_status;
    pub fn st_matmul_host(h: *mut st_handle, a: *const f32, b: *const f32, out: *mut f32, m: i64, k: i64, n: i64,
                          ta: i32, tb: i32, prec: c_int) -> st_status;
    pub fn st_softmax_rows(h: *mut st_handle, x: *const f32, y: *mut f32, rows: i64, n: i64, t: i64, scale: f32,
                           causal: i32, one: i32) -> st_status;
    pub fn st_softmax_rows_bwd(h: *mut st_handle, dy: *const f32, y: *const f32, dx: *mut f32, rows: i64, n: i64,
                               scale: f32) -> st_status;
    pub fn st_attn_fwd(h: *mut st_handle, q: *const c_void, k: *const c_void, v: *const c_void, o: *mut c_void,
                       lse: *mut f32, bh: i64, t: i64, d: i64, scale: f32, causal: i32, one: i32) -> st_status;
    pub fn st_attn_bwd(h: *mut st_handle, q: *const c_void, k: *const c_void, v: *const c_void, o: *const c_void,
                       dout: *const c_void, lse: *const f32, dq: *mut c_void, dk: *mut c_void, dv: *mut c_void,
                       bh: i64, t: i64, d: i64, scale: f32, causal: i32) -> st_status;
    pub fn st_attn_fwd_packed(h: *mut st_handle, qkv: *const f32, o: *mut f32, lse: *mut f32, batch: i64, heads: i64,
                              t: i64, d: i64, scale: f32, causal: i32, one: i32) -> st_status;
    pub fn st_attn_bwd_packed(h: *mut st_handle, qkv: *const f32, o: *const f32, dout: *const f32, lse: *const f32,
                              dqkv: *mut f32, batch: i64, heads: i64, t: i64, d: i64, scale: f32,
                              causal: i32) -> st_status;
    pub fn st_embed_fwd(h: *mut st_handle, ids: *const i32, tok: *const f32, pos: *const f32, x: *mut f32, batch: i64,
                        t: i64, d: i64) -> st_status;
    pub fn st_embed_bwd(h: *mut st_handle, ids: *const i32, dx: *const f32, dtok: *mut f32, dpos: *mut f32,
                        batch: i64, t: i64, d: i64, vocab: i64, accumulate: i32) -> st_status;
    pub fn st_layernorm_fwd(h: *mut st_handle, x: *const f32, gamma: *const f32, beta: *const f32, y: *mut f32,
                            mean: *mut f32, rstd: *mut f32, rows: i64, d: i64, eps: f32) -> st_status;
    pub fn st_layernorm_bwd(h: *mut st_handle, dy: *const f32, x: *const f32, gamma: *const f32, mean: *const f32,
                            rstd: *const f32, dx: *mut f32, dgamma: *mut f32, dbeta: *mut f32, rows: i64, d: i64,
                            accumulate: i32) -> st_status;
    pub fn st_cross_entropy(h: *mut st_handle, logits: *const f32, targets: *const i32, loss: *mut f32,
                            dlogits: *mut f32, rows: i64, vocab: i64) -> st_status;
    pub fn st_adam(h: *mut st_handle, p: *mut f32, g: *const f32, m: *mut f32, v: *mut f32, n: i64, step: i32,
                   lr: f32, beta1: f32, beta2: f32, eps: f32) -> st_status;
    pub fn st_adam_dev(h: *mut st_handle, p: *mut f32, g: *const f32, m: *mut f32, v: *mut f32, n: i64,
                       step: *mut i32, lr: f32, beta1: f32, beta2: f32, eps: f32) -> st_status;
    pub fn st_sgd(h: *mut st_handle, p: *mut f32, g: *const f32, n: i64, lr: f32) -> st_status;
    pub fn st_momentum(h: *mut st_handle, p: *mut f32, g: *const f32, v: *mut f32, mask: *const f32, n: i64, lr: f32,
                       mu: f32, shrink: f32) -> st_status;
    pub fn st_decay(h: *mut st_handle, p: *mut f32, mask: *const f32, n: i64, shrink: f32) -> st_status;
    pub fn st_average_models(h: *mut st_handle, p: *mut f32, stride: i64, models: i32, group: i32) -> st_status;
    pub fn st_dropout(h: *mut st_handle, x: *const f32, y: *mut f32, n: i64, rate: f32, seed: u32) -> st_status;
    pub fn st_dropout_relu_bwd(h: *mut st_handle, dy: *const f32, relu_y: *const f32, dx: *mut f32, n: i64, rate: f32,
                               seed: u32) -> st_status;
    pub fn st_nccl_unique_id(out: *mut u8) -> st_status;
    pub fn st_nccl_comm_init(nranks: i32, rank: i32, unique_id: *const u8, device: i32,
                             comm_out: *mut *mut c_void) -> st_status;
    pub fn st_nccl_comm_destroy(comm: *mut c_void) -> st_status;
    pub fn st_avg_params(h: *mut st_handle, p: *mut f32, n: i64, comm: *mut c_void) -> st_status;
    pub fn st_knn_search_sharded(h: *mut st_handle, codes: *const u8, scales: *const f32, n_local: i64, dim: i32,
                                 queries: *const f32, nq: i64, k: i32, mode: i32, prec: i32, index_base: i64,
                                 comm: *mut c_void, out_scores: *mut f32, out_ids: *mut i64) -> st_status;
    pub fn st_knn_search(h: *mut st_handle, codes: *const u8, scales: *const f32, n_keys: i64, dim: i32,
                         queries: *const f32, nq: i64, k: i32, mode: i32, prec: i32, index_base: i64,
                         out_scores: *mut f32, out_ids: *mut i64) -> st_status;
    pub fn st_knn_search_masked(h: *mut st_handle, codes: *const u8, scales: *const f32, n_keys: i64, dim: i32,
                                queries: *const f32, nq: i64, k: i32, mode: i32, prec: i32, index_base: i64,
                                ranges: *const i64, always: i64, out_scores: *mut f32,
                                out_ids: *mut i64) -> st_status;
    pub fn st_knn_topk_keys(h: *mut st_handle, codes: *const u8, scales: *const f32, n_keys: i64, dim: i32,
                            queries: *const f32, nq: i64, mode: i32, prec: i32, index_base: i64,
                            out_keys: *mut u64) -> st_status;
    pub fn st_knn_merge_keys(h: *mut st_handle, lists: *const u64, n_lists: i64, list_stride: i64, nq: i64,
                             out_keys: *mut u64) -> st_status;
    pub fn st_knn_decode(h: *mut st_handle, keys: *const u64, queries: *const f32, nq: i64, dim: i32, k: i32,
                         mode: i32, prec: i32, out_scores: *mut f32, out_ids: *mut i64) -> st_status;
    pub fn st_knn_quantize(h: *mut st_handle, keys: *const f32, n: i64, dim: i32, codes: *mut u8, scales: *mut f32,
                           norms: *mut f32) -> st_status;
    pub fn st_knn_scan_units(h: *mut st_handle, codes: *const u8, scales: *const f32, n_keys: i64, dim: i32,
                             queries: *const f32, nq: i64, mode: i32, prec: i32, index_base: i64, n_units: i64,
                             unit_q: *const i32, unit_list: *const i32, unit_keys: *const i64, n_lists: i32,
                             out_keys: *mut u64) -> st_status;
    pub fn st_knn_ivf_units(probes: *const i32, nq: i64, nprobe: i32, starts: *const i64, nlist: i32, n_sms: i32,
                            chunk: i64, max_lists: i32, unit_q: *mut i32, unit_list: *mut i32, unit_keys: *mut i64,
                            n_units: *mut i64, n_lists: *mut i32, chunk_used: *mut i64) -> st_status;
    pub fn st_knn_dequant(h: *mut st_handle, codes: *const u8, scales: *const f32, n: i64, dim: i32,
                          out: *mut f32) -> st_status;
    pub fn st_knn_nearest(h: *mut st_handle, dots: *const f32, cnorm: *const f32, n: i64, nlist: i32,
                          out: *mut i32) -> st_status;
    pub fn st_knn_probe(h: *mut st_handle, dots: *const f32, cnorm: *const f32, nq: i64, nlist: i32, nprobe: i32,
                        out: *mut i32) -> st_status;
    pub fn st_gather_rows(h: *mut st_handle, src: *const c_void, n_src: i64, dst: *mut c_void, perm: *const i64,
                          n: i64, row_bytes: i64) -> st_status;
    pub fn st_knn_synth_keys(h: *mut st_handle, codes: *mut u8, scales: *mut f32, n: i64, dim: i32, seed: u64,
                             first_key: i64) -> st_status;
}

/// A status and the handle's error text, as the reference's callers want a
/// `Result` (or, where they `expect`, a panic message) instead of a code.
#[derive(Debug, Clone)]
pub struct StError {
    pub status: st_status,
    pub text: String,
}

/// `Ok(())` for `ST_OK`, else the status with `st_last_error(h)`'s text.
///
/// # Safety
/// `h` is null or a live handle from `st_create`.
pub unsafe fn check(h: *const st_handle, status: st_status) -> Result<(), StError> {
    if status == ST_OK {
        return Ok(());
    }
    let text = if h.is_null() {
        String::new()
    } else {
        std::ffi::CStr::from_ptr(st_last_error(h)).to_string_lossy().into_owned()
    };
    Err(StError { status, text })
}
