"""The matmul family on the device: NN / NT / TN, batched, head views, epilogue.

Host-side mirror of gpu_step::matmul (src/gpu_step/matmul.rs:31-192) over
torch CUDA tensors: ``MatRef`` and ``Epilogue`` keep the reference's field
names and meaning, ``matmul`` / ``matmul_f32`` keep its argument order
``(a, b, out, batch, m, k, n, epi)``.  ``gpu_matmul`` is the host-array
drop-in of src/gpu.rs:98 and ``NdArray::matmul``; ``batched_matmul`` is
Tape::batched_matmul's forward (src/tape.rs:73-85).

Precision: ``matmul`` runs on the tcgen05 TF32 tensor cores (the role the
reference's default f16 matrix-core path plays); ``matmul_f32`` runs the
SIMT kernel whose every output is bit-identical to NdArray::matmul; with
float16 or bfloat16 operand buffers and ``precision=F16`` the product runs on
the kind::f16 tensor cores into an f32 out (the reference's f16 x f16 -> f32
k_matmul_cmma, src/gpu_step/matmul.rs:632-880).
"""
import ctypes
from dataclasses import dataclass
from typing import Optional, Tuple

import numpy as np
import torch

from . import _native as N
from .device import handle

TF32 = N.PREC_TF32
F32_EXACT = N.PREC_F32_EXACT
F16 = N.PREC_F16
TF32X3 = N.PREC_TF32X3  # three TF32 products per f32 product: f32 accuracy on the tensor cores
_DTYPES = {torch.float32: N.ST_F32, torch.float16: N.ST_F16, torch.bfloat16: N.ST_BF16}


@dataclass
class MatRef:
    """A matrix inside a device buffer (src/gpu_step/matmul.rs:31-60): matrix z
    starts at element off + (z // group) * stride + (z % group) * inner; stored
    rows are ``ld`` apart (0 = packed); ``trans``: stored transposed."""
    h: torch.Tensor
    off: int = 0
    stride: int = 0
    trans: bool = False
    ld: int = 0
    group: int = 1
    inner: int = 0

    @staticmethod
    def heads(h, col0, cols, t, heads, width):
        """Attention heads in place (matmul.rs:49-53): matrix z = b*heads + hd is
        rows b*t .. b*t+t, columns col0 + hd*width .. + width of [B*t, cols]."""
        return MatRef(h, off=col0, stride=t * cols, ld=cols, group=heads, inner=width)

    def _c(self):
        if self.h.dtype not in _DTYPES or not self.h.is_cuda:
            raise TypeError("MatRef buffers are CUDA float32, float16 or bfloat16 tensors")
        return N.StMat(self.h.data_ptr(), self.off, self.stride, self.inner, self.ld, max(self.group, 1),
                       int(self.trans), _DTYPES[self.h.dtype], 0)


@dataclass
class Epilogue:
    """Per-element epilogue (src/gpu_step/matmul.rs:66-79), applied in order:
    + bias[bias_off + z*bias_stride + col], ReLU, zero where mask <= 0,
    + residual, + the value already in out.  ``bias``/``mask``/``residual`` are
    (tensor, element offset) pairs; mask and residual share out's layout.
    ``col_sum``: (offset, stride) into out's buffer, or (tensor, offset, stride):
    adds the column sums of b[z] over k (a bias gradient)."""
    bias: Optional[Tuple[torch.Tensor, int]] = None
    bias_stride: int = 0
    relu: bool = False
    mask: Optional[Tuple[torch.Tensor, int]] = None
    residual: Optional[Tuple[torch.Tensor, int]] = None
    accumulate: bool = False
    col_sum: Optional[tuple] = None

    def _c(self, out_buf):
        e = N.StEpilogue()
        if self.bias is not None:
            e.bias, e.bias_off = self.bias[0].data_ptr(), self.bias[1]
        e.bias_stride = self.bias_stride
        if self.mask is not None:
            e.mask, e.mask_off = self.mask[0].data_ptr(), self.mask[1]
        if self.residual is not None:
            e.residual, e.residual_off = self.residual[0].data_ptr(), self.residual[1]
        if self.col_sum is not None:
            if len(self.col_sum) == 3:
                e.col_sum, e.col_sum_off, e.col_sum_stride = self.col_sum[0].data_ptr(), self.col_sum[1], self.col_sum[2]
            else:
                e.col_sum, e.col_sum_off, e.col_sum_stride = out_buf.data_ptr(), self.col_sum[0], self.col_sum[1]
        e.relu = int(self.relu)
        e.accumulate = int(self.accumulate)
        return e


def matmul_with(a: MatRef, b: MatRef, out: MatRef, batch, m, k, n, epi: Optional[Epilogue] = None, precision=TF32,
                h=None):
    """out[z] (+)= epi(a[z] @ b[z]) for z < batch; one or two launches, enqueued
    on torch's current stream (matmul.rs:106-192).  ``h``: the handle to use
    (default: the device's); GEMMs running concurrently need distinct handles."""
    if h is None:
        h = handle(out.h.device)
    ca, cb, co = a._c(), b._c(), out._c()
    ce = epi._c(out.h) if epi is not None else None
    h.call("st_gemm", ctypes.byref(ca), ctypes.byref(cb), ctypes.byref(co), batch, m, k, n,
           ctypes.byref(ce) if ce is not None else None, precision)
    return out


def matmul(a, b, out, batch, m, k, n, epi=None):
    """gpu_step::matmul (matmul.rs:86-88) on the TF32 tensor cores."""
    return matmul_with(a, b, out, batch, m, k, n, epi, TF32)


def matmul_f32(a, b, out, batch, m, k, n, epi=None):
    """gpu_step::matmul_f32 (matmul.rs:90-95): exact f32, bit-identical to
    NdArray::matmul for each output element."""
    return matmul_with(a, b, out, batch, m, k, n, epi, F32_EXACT)


def mm(a: torch.Tensor, b: torch.Tensor, ta=False, tb=False, precision=None, out=None):
    """op(a) @ op(b) for 2-D CUDA tensors (ta: a holds A^T; tb: b holds B^T):
    float32 operands on TF32 (default) or F32_EXACT, float16 / bfloat16 on F16;
    the out is float32."""
    if precision is None:
        precision = TF32 if a.dtype == torch.float32 else F16
    m, k = (a.shape[1], a.shape[0]) if ta else a.shape
    n = b.shape[0] if tb else b.shape[1]
    if out is None:
        out = torch.empty((m, n), dtype=torch.float32, device=a.device)
    matmul_with(MatRef(a.contiguous(), trans=ta), MatRef(b.contiguous(), trans=tb), MatRef(out), 1, m, k, n, None,
                precision)
    return out


def batched_matmul(a: torch.Tensor, b: torch.Tensor, batch: int, transpose_b: bool, precision=TF32):
    """Tape::batched_matmul forward (src/tape.rs:73-85): row chunk z of a times
    row chunk z of b (or its transpose)."""
    ar, br = a.shape[0] // batch, b.shape[0] // batch
    k = a.shape[1]
    n = br if transpose_b else b.shape[1]
    out = torch.empty((a.shape[0], n), dtype=torch.float32, device=a.device)
    matmul_with(MatRef(a, stride=ar * k), MatRef(b, stride=br * b.shape[1], trans=transpose_b),
                MatRef(out, stride=ar * n), batch, ar, k, n, None, precision)
    return out


def gpu_matmul(a: np.ndarray, b: np.ndarray, precision=TF32, ta=False, tb=False, device=None):
    """NdArray::matmul / gpu_matmul with host arrays (src/gpu.rs:98-169,
    src/tensor.rs:241): copies in, multiplies on the device, copies out."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = (a.shape[1], a.shape[0]) if ta else a.shape
    n = b.shape[0] if tb else b.shape[1]
    kb = b.shape[1] if tb else b.shape[0]
    if kb != k:
        raise ValueError("matmul inner dims must match: %s vs %s" % (a.shape, b.shape))
    out = np.empty((m, n), np.float32)
    h = handle(device)
    h.call("st_matmul_host", a.ctypes.data_as(ctypes.c_void_p), b.ctypes.data_as(ctypes.c_void_p),
           out.ctypes.data_as(ctypes.c_void_p), m, k, n, int(ta), int(tb), precision)
    return out


def matmul_group(gemms, h=None):
    """Several dependent TF32 GEMMs in one persistent launch (st_gemm_group).

    ``gemms``: up to 8 tuples (a, b, out, m, k, n, epi, after) of MatRefs,
    shape, Epilogue (or None, no col_sum) and the indices of earlier GEMMs
    whose outputs this one reads.  Results equal matmul_with on each in order;
    raises StError(ST_UNSUPPORTED_SHAPE) for layouts the grouped kernel does
    not take (unaligned rows, n % 4 != 0)."""
    if not gemms:
        return
    dev = gemms[0][2].h.device
    if h is None:
        h = handle(dev)
    arr = (N.StGroupGemm * len(gemms))()
    keep = []
    for i, (a, b, out, m, k, n, epi, after) in enumerate(gemms):
        g = arr[i]
        g.a, g.b, g.out = a._c(), b._c(), out._c()
        g.m, g.k, g.n = m, k, n
        if epi is not None:
            ce = epi._c(out.h)
            keep.append(ce)
            g.epi = ctypes.pointer(ce)
        mask = 0
        for j in after:
            if not 0 <= j < i:
                raise ValueError("GEMM %d may only follow earlier GEMMs" % i)
            mask |= 1 << j
        g.after = mask
    h.call("st_gemm_group", arr, len(gemms))
