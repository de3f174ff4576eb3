"""scratchtape_b200: B200 (sm_100a) kernels for scratchtape's hot path.

The package is a thin host layer over ``libst_b200.so`` (C ABI in
``include/st_b200.h``): the matmul family, row softmax, fused causal
attention and 2-bit kNN scoring.  Importing it without the built library
fails; there is no CPU fallback.
"""
from . import _native  # noqa: F401  (fails loudly when the library is missing)
from .device import handle, Handle  # noqa: F401
from .matmul import (MatRef, Epilogue, matmul, matmul_f32, matmul_with, mm, batched_matmul,  # noqa: F401
                     gpu_matmul, TF32, F32_EXACT, F16, TF32X3)
from .rows import softmax, softmax_backward  # noqa: F401

__version__ = "0.1.0"
