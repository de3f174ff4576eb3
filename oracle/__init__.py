"""CPU oracle for scratchtape's hot path -- TEST INFRASTRUCTURE ONLY.

ctypes bindings to ``liboracle_st.so`` (built from ``st_oracle.c`` and
``st_oracle_knn.c`` by ``oracle/Makefile``).  Only ``tests/``,
``__graft_entry__.smoke()`` and the CPU-baseline legs of ``bench.py`` import
this package; the product library never does.
"""
import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle_st.so")
_lib = None

_f32p = ctypes.POINTER(ctypes.c_float)
_f64p = ctypes.POINTER(ctypes.c_double)
_i64p = ctypes.POINTER(ctypes.c_int64)
_u8p = ctypes.POINTER(ctypes.c_uint8)
_u64p = ctypes.POINTER(ctypes.c_uint64)
_i64 = ctypes.c_int64
_int = ctypes.c_int
_f32 = ctypes.c_float


def build(force=False):
    """Compile liboracle_st.so with the Makefile beside this file."""
    srcs = [os.path.join(_HERE, f) for f in ("st_oracle.c", "st_oracle_knn.c", "Makefile")]
    if not force and os.path.exists(_LIB_PATH):
        if os.path.getmtime(_LIB_PATH) >= max(os.path.getmtime(s) for s in srcs):
            return _LIB_PATH
    subprocess.check_call(["make", "-s", "-B", "liboracle_st.so"], cwd=_HERE)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = ctypes.CDLL(_LIB_PATH)
        sig = {
            "orc_rng_next_f32": (_f32, [_u64p]),
            "orc_rng_next_gaussian": (_f32, [_u64p]),
            "orc_rng_uniform": (None, [_u64p, _f32p, _i64, _f32]),
            "orc_rng_gaussian": (None, [_u64p, _f32p, _i64]),
            "orc_matmul": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64]),
            "orc_transpose": (None, [_f32p, _f32p, _i64, _i64]),
            "orc_matmul_layout": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64, _int, _int]),
            "orc_matmul_threads": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64, _int]),
            "orc_batched_matmul_fwd": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64, _int]),
            "orc_batched_matmul_bwd": (None, [_f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64, _int]),
            "orc_split_heads": (None, [_f32p, _f32p, _i64, _i64, _i64, _i64, _i64, _i64]),
            "orc_merge_heads": (None, [_f32p, _f32p, _i64, _i64, _i64, _i64]),
            "orc_softmax_rows": (None, [_f32p, _i64, _i64, _int]),
            "orc_attention_fwd": (None, [_f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _f32, _int, _int]),
            "orc_attention_bwd": (None, [_f32p] * 7 + [_i64, _i64, _i64, _f32, _int, _int]),
            "orc_rows_softmax": (None, [_f32p, _f32p, _i64, _i64, _i64, _f32, _int, _int]),
            "orc_rows_softmax_bwd": (None, [_f32p, _f32p, _f32p, _i64, _i64, _f32]),
            "orc_layernorm_fwd": (None, [_f32p, _f32p, _f32p, _f32p, _i64, _i64]),
            "orc_block_param_count": (_i64, [_i64, _i64]),
            "orc_block_init": (None, [_u64p, _f32p, _i64, _i64, _i64]),
            "orc_block_forward": (None, [_f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64]),
            "orc_block_backward": (None, [_f32p, _f32p, _f32p, _f32p, _f32p, _i64, _i64, _i64, _i64, _i64]),
            "orc_powi": (_f32, [_f32, _int]),
            "orc_adam": (None, [_f32p, _f32p, _f32p, _f32p, _i64, _int, _f32, _f32, _f32, _f32]),
            "orc_average_models": (None, [_f32p, _i64, _i64]),
            "orc_sgd": (None, [_f32p, _f32p, _i64, _f32]),
            "orc_momentum": (None, [_f32p, _f32p, _f32p, _f32p, _i64, _f32, _f32, _f32]),
            "orc_decay": (None, [_f32p, _f32p, _i64, _f32]),
            "orc_average_groups": (None, [_f32p, _i64, _i64, _i64]),
            "orc_dropout_bits": (ctypes.c_uint32, [ctypes.c_uint32, ctypes.c_uint32]),
            "orc_dropout": (None, [_f32p, _f32p, _f32p, _i64, _f32, ctypes.c_uint32]),
            "orc_round_f16": (_f32, [_f32]),
            "orc_quantize_rows": (None, [_f32p, _i64, _i64, _int, _u8p, _f32p, _f32p]),
            "orc_dequant_rows": (None, [_u8p, _f32p, _i64, _i64, _int, _int, _f32p]),
            "orc_knn_topk": (None, [_u8p, _f32p, _i64, _i64, _f32p, _i64, _i64, _int, _int, _i64p, _i64p, _i64,
                                    _f32p, _f64p, _i64p, _int]),
            "orc_knn_pair_dots": (None, [_u8p, _f32p, _i64, _f32p, _i64p, _i64p, _i64, _f64p]),
            "orc_synth_codes": (None, [ctypes.c_uint64, _i64, _i64, _i64, _u8p]),
            "orc_knn_topk_synth": (None, [ctypes.c_uint64, _i64, _i64, _i64, _f32p, _f32p, _i64, _i64, _f64p, _i64p,
                                          _int]),
            "orc_knn_pair_dots_synth": (None, [ctypes.c_uint64, _i64, _i64, _f32p, _f32p, _i64p, _i64p, _i64,
                                               _f64p]),
        }
        for name, (res, args) in sig.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def _p(a, ty):
    if a is None:
        return None
    return a.ctypes.data_as(ty)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


class Rng:
    """The reference's xorshift64 generator (src/nn.rs:8-36)."""

    def __init__(self, seed):
        self.state = ctypes.c_uint64(seed)

    def next_f32(self):
        return lib().orc_rng_next_f32(ctypes.byref(self.state))

    def uniform(self, n, scale=1.0):
        out = np.empty(n, np.float32)
        lib().orc_rng_uniform(ctypes.byref(self.state), _p(out, _f32p), n, scale)
        return out

    def gaussian(self, n):
        out = np.empty(n, np.float32)
        lib().orc_rng_gaussian(ctypes.byref(self.state), _p(out, _f32p), n)
        return out


def matmul(a, b):
    """NdArray::matmul, bitwise (src/tensor.rs:248-276)."""
    a, b = _c(a, np.float32), _c(b, np.float32)
    m, k = a.shape
    n = b.shape[1]
    out = np.empty((m, n), np.float32)
    lib().orc_matmul(_p(a, _f32p), _p(b, _f32p), _p(out, _f32p), m, k, n)
    return out


def matmul_layout(a, b, ta=False, tb=False, threads=1):
    """out = op(a) . op(b) with the tape's explicit transposes (src/tape.rs:505-510)."""
    a, b = _c(a, np.float32), _c(b, np.float32)
    m, k = (a.shape[1], a.shape[0]) if ta else a.shape
    n = b.shape[0] if tb else b.shape[1]
    out = np.empty((m, n), np.float32)
    if threads > 1 and not ta and not tb:
        lib().orc_matmul_threads(_p(a, _f32p), _p(b, _f32p), _p(out, _f32p), m, k, n, threads)
    else:
        lib().orc_matmul_layout(_p(a, _f32p), _p(b, _f32p), _p(out, _f32p), m, k, n, int(ta), int(tb))
    return out


def transpose(a):
    a = _c(a, np.float32)
    out = np.empty((a.shape[1], a.shape[0]), np.float32)
    lib().orc_transpose(_p(a, _f32p), _p(out, _f32p), a.shape[0], a.shape[1])
    return out


def batched_matmul_fwd(a, b, batch, transpose_b):
    a, b = _c(a, np.float32), _c(b, np.float32)
    out_cols = b.shape[0] // batch if transpose_b else b.shape[1]
    out = np.empty((a.shape[0], out_cols), np.float32)
    lib().orc_batched_matmul_fwd(_p(a, _f32p), _p(b, _f32p), _p(out, _f32p), batch, a.shape[0], a.shape[1],
                                 b.shape[0], b.shape[1], int(transpose_b))
    return out


def batched_matmul_bwd(a, b, grad, batch, transpose_b):
    a, b, grad = _c(a, np.float32), _c(b, np.float32), _c(grad, np.float32)
    ga, gb = np.empty_like(a), np.empty_like(b)
    lib().orc_batched_matmul_bwd(_p(a, _f32p), _p(b, _f32p), _p(grad, _f32p), _p(ga, _f32p), _p(gb, _f32p), batch,
                                 a.shape[0], a.shape[1], b.shape[0], b.shape[1], int(transpose_b))
    return ga, gb


def attention_fwd(q, k, v, scale, causal=True, one=False, want_probs=False):
    """Batched causal attention as the CPU block composes it (src/nn.rs:646-671).
    q, k, v: [BH, T, D] float32."""
    q, k, v = _c(q, np.float32), _c(k, np.float32), _c(v, np.float32)
    bh, t, d = q.shape
    out = np.empty_like(q)
    probs = np.empty((bh, t, t), np.float32) if want_probs else None
    lib().orc_attention_fwd(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), _p(out, _f32p), _p(probs, _f32p), bh, t, d,
                            scale, int(causal), int(one))
    return (out, probs) if want_probs else out


def attention_bwd(q, k, v, dout, scale, causal=True, one=False):
    q, k, v, dout = (_c(x, np.float32) for x in (q, k, v, dout))
    bh, t, d = q.shape
    dq, dk, dv = np.empty_like(q), np.empty_like(q), np.empty_like(q)
    lib().orc_attention_bwd(_p(q, _f32p), _p(k, _f32p), _p(v, _f32p), _p(dout, _f32p), _p(dq, _f32p), _p(dk, _f32p),
                            _p(dv, _f32p), bh, t, d, scale, int(causal), int(one))
    return dq, dk, dv


def rows_softmax(x, t, scale, causal=True, one=False):
    x = _c(x, np.float32)
    rows, n = x.shape
    y = np.empty_like(x)
    lib().orc_rows_softmax(_p(x, _f32p), _p(y, _f32p), rows, n, t, scale, int(causal), int(one))
    return y


def rows_softmax_bwd(y, dy, scale):
    y, dy = _c(y, np.float32), _c(dy, np.float32)
    dx = np.empty_like(y)
    lib().orc_rows_softmax_bwd(_p(y, _f32p), _p(dy, _f32p), _p(dx, _f32p), y.shape[0], y.shape[1], scale)
    return dx


def layernorm_fwd(x, gamma, beta):
    x, gamma, beta = _c(x, np.float32), _c(gamma, np.float32), _c(beta, np.float32)
    y = np.empty_like(x)
    lib().orc_layernorm_fwd(_p(x, _f32p), _p(gamma, _f32p), _p(beta, _f32p), _p(y, _f32p), x.shape[0], x.shape[1])
    return y


def block_init(rng, d, n_heads, dff):
    n = lib().orc_block_param_count(d, dff)
    p = np.empty(n, np.float32)
    lib().orc_block_init(ctypes.byref(rng.state), _p(p, _f32p), d, n_heads, dff)
    return p


def block_forward(params, x, batch, t, d, n_heads, dff):
    params, x = _c(params, np.float32), _c(x, np.float32)
    y = np.empty_like(x)
    lib().orc_block_forward(_p(params, _f32p), _p(x, _f32p), _p(y, _f32p), batch, t, d, n_heads, dff)
    return y


def block_backward(params, x, dy, batch, t, d, n_heads, dff):
    params, x, dy = _c(params, np.float32), _c(x, np.float32), _c(dy, np.float32)
    dp, dx = np.empty_like(params), np.empty_like(x)
    lib().orc_block_backward(_p(params, _f32p), _p(x, _f32p), _p(dy, _f32p), _p(dp, _f32p), _p(dx, _f32p), batch, t,
                             d, n_heads, dff)
    return dp, dx


def adam(p, g, m, v, t, lr, b1=0.9, b2=0.999, eps=1e-8):
    """In place on float32 arrays (src/optim.rs:42-57)."""
    lib().orc_adam(_p(p, _f32p), _p(_c(g, np.float32), _f32p), _p(m, _f32p), _p(v, _f32p), p.size, t, lr, b1, b2,
                   eps)


def average_models(p, models):
    lib().orc_average_models(_p(p, _f32p), p.size // models, models)


def sgd(p, g, lr):
    """In place (src/gpu_step/mod.rs:232-238)."""
    lib().orc_sgd(_p(p, _f32p), _p(_c(g, np.float32), _f32p), p.size, lr)


def momentum(p, g, v, lr, mu, mask=None, shrink=0.0):
    """In place on p and v (src/gpu_step/mod.rs:240-251)."""
    lib().orc_momentum(_p(p, _f32p), _p(_c(g, np.float32), _f32p), _p(v, _f32p),
                       None if mask is None else _p(_c(mask, np.float32), _f32p), p.size, lr, mu, shrink)


def decay(p, mask, shrink):
    """In place (src/gpu_step/mod.rs:253-259)."""
    lib().orc_decay(_p(p, _f32p), _p(_c(mask, np.float32), _f32p), p.size, shrink)


def average_groups(p, models, group):
    """In place: p holds `models` vectors (src/gpu_step/mod.rs:261-275)."""
    lib().orc_average_groups(_p(p, _f32p), p.size // models, models, group)


def dropout(x, rate, seed, relu_y=None):
    """(src/gpu_step/tape.rs:526-582)"""
    x = _c(x, np.float32)
    y = np.empty_like(x)
    lib().orc_dropout(_p(x, _f32p), None if relu_y is None else _p(_c(relu_y, np.float32), _f32p), _p(y, _f32p),
                      x.size, rate, seed)
    return y


def round_f16(x):
    return lib().orc_round_f16(x)


def quantize_rows(keys, bits=2):
    keys = _c(keys, np.float32)
    n, d = keys.shape
    codes = np.zeros((n, d * bits // 8), np.uint8)
    scales = np.empty(n, np.float32)
    norms = np.empty(n, np.float32)
    lib().orc_quantize_rows(_p(keys, _f32p), n, d, bits, _p(codes, _u8p), _p(scales, _f32p), _p(norms, _f32p))
    return codes, scales, norms


def dequant_rows(codes, scales, d, bits=2, to_f16=False):
    codes, scales = _c(codes, np.uint8), _c(scales, np.float32)
    n = scales.shape[0]
    out = np.empty((n, d), np.float32)
    lib().orc_dequant_rows(_p(codes, _u8p), _p(scales, _f32p), n, d, bits, int(to_f16), _p(out, _f32p))
    return out


def knn_topk(codes, scales, queries, k, mode="dot", prec="exact", ranges=None, always=0, threads=None):
    """Brute-force top-k over 2-bit keys; returns (scores f64 [nq,k], ids int64 [nq,k])."""
    codes, scales, queries = _c(codes, np.uint8), _c(scales, np.float32), _c(queries, np.float32)
    n = scales.shape[0]
    nq, d = queries.shape
    lo = hi = None
    if ranges is not None:
        ranges = np.asarray(ranges, np.int64)
        lo, hi = _c(ranges[:, 0], np.int64), _c(ranges[:, 1], np.int64)
    s64 = np.empty((nq, k), np.float64)
    ids = np.empty((nq, k), np.int64)
    if threads is None:
        threads = os.cpu_count() or 1
    lib().orc_knn_topk(_p(codes, _u8p), _p(scales, _f32p), n, d, _p(queries, _f32p), nq, k,
                       0 if mode == "dot" else 1, 0 if prec == "exact" else 1, _p(lo, _i64p), _p(hi, _i64p), always,
                       None, _p(s64, _f64p), _p(ids, _i64p), threads)
    return s64, ids


def knn_pair_dots(codes, scales, queries, qi, kj):
    codes, scales, queries = _c(codes, np.uint8), _c(scales, np.float32), _c(queries, np.float32)
    qi, kj = _c(qi, np.int64), _c(kj, np.int64)
    out = np.empty(qi.shape[0], np.float64)
    lib().orc_knn_pair_dots(_p(codes, _u8p), _p(scales, _f32p), queries.shape[1], _p(queries, _f32p), _p(qi, _i64p),
                            _p(kj, _i64p), qi.shape[0], _p(out, _f64p))
    return out


def pack_keys(scores, ids):
    """A best-k list in the scan's exchange format: order-preserving f32
    score bits << 32 | 0xFFFFFFFF - index (the higher key ranks first), 0
    for an empty entry (id < 0).  DOT scores (the higher the better)."""
    u = np.asarray(scores, np.float32).view(np.uint32).astype(np.uint64)
    o = np.where(u & 0x80000000, ~u & 0xFFFFFFFF, u | 0x80000000)
    keys = (o << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - np.asarray(ids, np.int64).astype(np.uint64))
    return np.where(np.asarray(ids) >= 0, keys, 0).astype(np.uint64)


def merge_keys(lists, k=128):
    """k_merge_parts (src/gpu_step/knn.rs:661-702) on exchange-format lists
    [n_lists, nq, width] (u64): each query's best k over all lists, best
    first (keys are unique per key index, so the order is total)."""
    lists = np.asarray(lists, np.uint64)
    allk = np.concatenate(list(lists), axis=1)
    return np.sort(allk, axis=1)[:, ::-1][:, :k].copy()


def synth_codes(seed, first, n, d):
    """The code bytes st_knn_synth_keys makes for keys first..first+n-1."""
    out = np.empty((n, d // 4), np.uint8)
    lib().orc_synth_codes(seed, first, n, d, _p(out, _u8p))
    return out


def knn_topk_synth(seed, first, n, d, scales, queries, k, threads=None):
    """Exact f64 DOT top-k over the synthetic keys first..first+n-1 (codes
    regenerated from the seed, scales as given, [n]): (scores f64, ids)."""
    q = _c(queries, np.float32)
    sc = _c(scales, np.float32)
    nq = q.shape[0]
    s = np.empty((nq, k), np.float64)
    i = np.empty((nq, k), np.int64)
    lib().orc_knn_topk_synth(seed, first, n, d, _p(sc, _f32p), _p(q, _f32p), nq, k, _p(s, _f64p), _p(i, _i64p),
                             threads or (os.cpu_count() or 1))
    return s, i


def knn_pair_dots_synth(seed, first, d, scales, queries, qi, kj):
    """Exact f64 q.k of (query qi[p], synthetic key kj[p]) pairs; scales [n] from key `first`."""
    q = _c(queries, np.float32)
    qi = _c(qi, np.int64)
    kj = _c(kj, np.int64)
    out = np.empty(qi.size, np.float64)
    lib().orc_knn_pair_dots_synth(seed, first, d, _p(_c(scales, np.float32), _f32p), _p(q, _f32p), _p(qi, _i64p),
                                  _p(kj, _i64p), qi.size, _p(out, _f64p))
    return out
