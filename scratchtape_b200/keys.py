"""The kNN key build path on the device: whitening / rotation GEMM, then the
2-bit quantiser, with no host round trip of the hidden states.

Reference (examples/tiny_lm/tier_eval.rs): ``whiten_device`` (:1202-1222)
computes keys = (x - mu) W^T on the device as ``matmul_f32(x, W^T)`` with the
bias c = -W mu in the epilogue, c summed on the host in f32; ``random_rotation``
(:1282-1297) is Gram-Schmidt (two passes) on Gaussian rows of the reference's
``Rng`` (src/nn.rs:8-36), in f64; ``fit_whitener`` (:1319-1324) folds the
rotation into W (R W, f64, then f32).  The keys then go through KnnStore's
quantiser (src/gpu_step/knn.rs:190-221), here ``st_knn_quantize``.

The whitening GEMM runs on ``st_gemm``: ``F32_EXACT`` gives the bits of the
reference's CPU matmul order, ``TF32`` the tensor cores.
"""
import numpy as np
import torch

from .matmul import F32_EXACT, Epilogue, MatRef, matmul_with


class Rng:
    """The reference's generator (src/nn.rs:8-36): xorshift64, uniforms as
    (x / u64::MAX) rounded to f32, Box-Muller in f32."""
    MASK = (1 << 64) - 1

    def __init__(self, seed: int):
        self.s = seed & self.MASK

    def next_f32(self) -> np.float32:
        s = self.s
        s ^= (s << 13) & self.MASK
        s ^= s >> 7
        s ^= (s << 17) & self.MASK
        self.s = s
        return np.float32(s / float(self.MASK))

    def next_gaussian(self) -> np.float32:
        u1 = max(self.next_f32(), np.float32(1e-9))
        u2 = self.next_f32()
        two, pi = np.float32(2.0), np.float32(np.pi)
        return np.float32(np.sqrt(np.float32(-two * np.log(u1))) * np.cos(np.float32(two * pi * u2)))


def random_rotation(d: int, seed: int) -> np.ndarray:
    """A random orthogonal [d, d] matrix (row-major, f64): Gram-Schmidt, two
    passes, on Gaussian rows from ``Rng(seed)`` (tier_eval.rs:1282-1297)."""
    rng = Rng(seed)
    r = np.zeros((d, d), dtype=np.float64)
    for i in range(d):
        v = np.array([rng.next_gaussian() for _ in range(d)], dtype=np.float64)
        for _ in range(2):
            for j in range(i):
                v -= np.dot(v, r[j]) * r[j]
        r[i] = v / np.sqrt(np.dot(v, v))
    return r


def rotate_whitener(w: np.ndarray, r: np.ndarray) -> np.ndarray:
    """R W in f64, rounded to f32 (tier_eval.rs:1319-1324): rotating keys and
    queries alike keeps every distance and makes the coordinates closer to
    Gaussian with equal variance, which the 2-bit quantiser assumes."""
    return (r @ np.asarray(w, dtype=np.float64)).astype(np.float32)


class Whitener:
    """keys = (x - mu) W^T for hidden states x [rows, d]; W [kd, d].  W and the
    bias c = -W mu (each c_j summed in f32, in order, as tier_eval.rs:1210)
    go to the device once."""

    def __init__(self, mu: np.ndarray, w: np.ndarray, device=None):
        mu = np.asarray(mu, dtype=np.float32).reshape(-1)
        w = np.asarray(w, dtype=np.float32)
        if w.ndim != 2 or w.shape[1] != mu.shape[0]:
            raise ValueError("W is [kd, d] with d = len(mu)")
        prods = w * mu[None, :]
        c = -np.cumsum(prods, axis=1, dtype=np.float32)[:, -1]  # sequential f32 sums
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.w = torch.from_numpy(np.ascontiguousarray(w)).to(dev)
        self.c = torch.from_numpy(c.astype(np.float32)).to(dev)
        self.kd, self.d = w.shape

    def apply(self, x: torch.Tensor, precision=F32_EXACT, out=None):
        """(x - mu) W^T on the device: one st_gemm, W read transposed by
        descriptor, c added in the epilogue."""
        x = x.contiguous()
        rows = x.shape[0]
        if out is None:
            out = torch.empty((rows, self.kd), dtype=torch.float32, device=x.device)
        matmul_with(MatRef(x), MatRef(self.w, trans=True), MatRef(out), 1, rows, self.d, self.kd,
                    Epilogue(bias=(self.c, 0)), precision)
        return out


def build_keys(x: torch.Tensor, whitener: Whitener, precision=F32_EXACT):
    """Hidden states (device f32 [rows, d]) -> 2-bit keys: whitening GEMM,
    then the quantiser.  Returns (codes u8 [rows, kd/4], scales, norms)."""
    from .knn import quantize
    return quantize(whitener.apply(x, precision))
