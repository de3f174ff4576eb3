"""ctypes binding of libst_b200.so (declared in include/st_b200.h).

The library is required: importing this module without the built .so raises
ImportError with the build command, and there is no fallback path.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libst_b200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError("scratchtape_b200: native library %s is missing; build it with "
                      "`python -c 'import __graft_entry__ as g; g.build()'` or `python scratchtape_b200/build.py`"
                      % LIB_PATH)

lib = ctypes.CDLL(LIB_PATH)

ST_OK, ST_INVALID_ARG, ST_UNSUPPORTED_SHAPE, ST_CUDA_ERROR, ST_NCCL_ERROR, ST_TIMEOUT, ST_NO_MEMORY, ST_NOT_FOUND = \
    range(8)
STATUS_NAMES = ["OK", "INVALID_ARG", "UNSUPPORTED_SHAPE", "CUDA_ERROR", "NCCL_ERROR", "TIMEOUT", "NO_MEMORY",
                "NOT_FOUND"]
ST_F32, ST_F16, ST_BF16 = 0, 1, 2
PREC_F32_EXACT, PREC_TF32, PREC_F16, PREC_TF32X3 = 0, 1, 2, 3
KNN_DOT, KNN_L2 = 0, 1
KNN_EXACT, KNN_F16REF = 0, 1
KNN_KMAX = 128


class StMat(ctypes.Structure):
    _fields_ = [("ptr", ctypes.c_void_p), ("off", ctypes.c_int64), ("stride", ctypes.c_int64),
                ("inner", ctypes.c_int64), ("ld", ctypes.c_int64), ("group", ctypes.c_int32),
                ("trans", ctypes.c_int32), ("dtype", ctypes.c_int32), ("reserved", ctypes.c_int32)]


class StEpilogue(ctypes.Structure):
    _fields_ = [("bias", ctypes.c_void_p), ("bias_off", ctypes.c_int64), ("bias_stride", ctypes.c_int64),
                ("mask", ctypes.c_void_p), ("mask_off", ctypes.c_int64), ("residual", ctypes.c_void_p),
                ("residual_off", ctypes.c_int64), ("col_sum", ctypes.c_void_p), ("col_sum_off", ctypes.c_int64),
                ("col_sum_stride", ctypes.c_int64), ("relu", ctypes.c_int32), ("accumulate", ctypes.c_int32)]


class StGroupGemm(ctypes.Structure):
    _fields_ = [("a", StMat), ("b", StMat), ("out", StMat), ("m", ctypes.c_int64), ("k", ctypes.c_int64),
                ("n", ctypes.c_int64), ("epi", ctypes.POINTER(StEpilogue)), ("after", ctypes.c_uint32),
                ("reserved", ctypes.c_int32)]


_h = ctypes.c_void_p
_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float
_st = ctypes.c_int

# name -> (restype, argtypes); every name here is declared in include/st_b200.h
SIGNATURES = {
    "st_create": (_st, [ctypes.c_int, _vp, ctypes.POINTER(_h)]),
    "st_destroy": (_st, [_h]),
    "st_set_stream": (_st, [_h, _vp]),
    "st_last_error": (ctypes.c_char_p, [_h]),
    "st_sync": (_st, [_h]),
    "st_launch_count": (_i64, [_h]),
    "st_scratch_bytes": (_i64, [_h]),
    "st_last_kernel": (ctypes.c_char_p, [_h]),
    "st_gemm": (_st, [_h, ctypes.POINTER(StMat), ctypes.POINTER(StMat), ctypes.POINTER(StMat), _i64, _i64, _i64, _i64,
                      ctypes.POINTER(StEpilogue), ctypes.c_int]),
    "st_gemm_group": (_st, [_h, ctypes.POINTER(StGroupGemm), _i32]),
    "st_gemm_tf32_fixed_scratch": (_st, [_h, ctypes.POINTER(StMat), ctypes.POINTER(StMat), ctypes.POINTER(StMat), _i64,
                                         _i64, _i64, _i64, ctypes.POINTER(StEpilogue)]),
    "st_matmul_host": (_st, [_h, _vp, _vp, _vp, _i64, _i64, _i64, _i32, _i32, ctypes.c_int]),
    "st_knn_ivf_units": (_st, [_vp, _i64, _i32, _vp, _i32, _i32, _i64, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "st_mlp_step_tf32": (_st, [_h, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64]),
    "st_softmax_rows": (_st, [_h, _vp, _vp, _i64, _i64, _i64, _f32, _i32, _i32]),
    "st_softmax_rows_bwd": (_st, [_h, _vp, _vp, _vp, _i64, _i64, _f32]),
    "st_attn_fwd": (_st, [_h, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _f32, _i32, _i32]),
    "st_attn_bwd": (_st, [_h, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _f32, _i32]),
    "st_attn_fwd_packed": (_st, [_h, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _i32, _i32]),
    "st_attn_bwd_packed": (_st, [_h, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _f32, _i32]),
    "st_embed_fwd": (_st, [_h, _vp, _vp, _vp, _vp, _i64, _i64, _i64]),
    "st_embed_bwd": (_st, [_h, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i32]),
    "st_layernorm_fwd": (_st, [_h, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _f32]),
    "st_layernorm_bwd": (_st, [_h, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i32]),
    "st_cross_entropy": (_st, [_h, _vp, _vp, _vp, _vp, _i64, _i64]),
    "st_adam": (_st, [_h, _vp, _vp, _vp, _vp, _i64, _i32, _f32, _f32, _f32, _f32]),
    "st_adam_dev": (_st, [_h, _vp, _vp, _vp, _vp, _i64, _vp, _f32, _f32, _f32, _f32]),
    "st_knn_search": (_st, [_h, _vp, _vp, _i64, _i32, _vp, _i64, _i32, _i32, _i32, _i64, _vp, _vp]),
    "st_knn_search_masked": (_st, [_h, _vp, _vp, _i64, _i32, _vp, _i64, _i32, _i32, _i32, _i64, _vp, _i64, _vp, _vp]),
    "st_knn_topk_keys": (_st, [_h, _vp, _vp, _i64, _i32, _vp, _i64, _i32, _i32, _i64, _vp]),
    "st_knn_merge_keys": (_st, [_h, _vp, _i64, _i64, _i64, _vp]),
    "st_knn_decode": (_st, [_h, _vp, _vp, _i64, _i32, _i32, _i32, _i32, _vp, _vp]),
    "st_knn_quantize": (_st, [_h, _vp, _i64, _i32, _vp, _vp, _vp]),
    "st_knn_scan_units": (_st, [_h, _vp, _vp, _i64, _i32, _vp, _i64, _i32, _i32, _i64, _i64, _vp, _vp, _vp, _i32,
                                _vp]),
    "st_knn_dequant": (_st, [_h, _vp, _vp, _i64, _i32, _vp]),
    "st_knn_nearest": (_st, [_h, _vp, _vp, _i64, _i32, _vp]),
    "st_knn_probe": (_st, [_h, _vp, _vp, _i64, _i32, _i32, _vp]),
    "st_gather_rows": (_st, [_h, _vp, _i64, _vp, _vp, _i64, _i64]),
    "st_knn_synth_keys": (_st, [_h, _vp, _vp, _i64, _i32, ctypes.c_uint64, _i64]),
    "st_sgd": (_st, [_h, _vp, _vp, _i64, _f32]),
    "st_momentum": (_st, [_h, _vp, _vp, _vp, _vp, _i64, _f32, _f32, _f32]),
    "st_decay": (_st, [_h, _vp, _vp, _i64, _f32]),
    "st_average_models": (_st, [_h, _vp, _i64, _i32, _i32]),
    "st_dropout": (_st, [_h, _vp, _vp, _i64, _f32, ctypes.c_uint32]),
    "st_dropout_relu_bwd": (_st, [_h, _vp, _vp, _vp, _i64, _f32, ctypes.c_uint32]),
    "st_nccl_unique_id": (_st, [_vp]),
    "st_nccl_comm_init": (_st, [_i32, _i32, _vp, _i32, ctypes.POINTER(_vp)]),
    "st_nccl_comm_destroy": (_st, [_vp]),
    "st_avg_params": (_st, [_h, _vp, _i64, _vp]),
    "st_knn_search_sharded": (_st, [_h, _vp, _vp, _i64, _i32, _vp, _i64, _i32, _i32, _i32, _i64, _vp, _vp, _vp]),
}

for _name, (_res, _args) in SIGNATURES.items():
    _fn = getattr(lib, _name)
    _fn.restype = _res
    _fn.argtypes = _args


class StError(RuntimeError):
    def __init__(self, status, text):
        self.status = status
        name = STATUS_NAMES[status] if 0 <= status < len(STATUS_NAMES) else str(status)
        super().__init__("ST_%s: %s" % (name, text))


def check(handle_ptr, status):
    if status != ST_OK:
        txt = lib.st_last_error(handle_ptr)
        raise StError(status, txt.decode() if txt else "")
    return status
