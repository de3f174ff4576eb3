"""One MLP layer forward + backward on the device: the six GEMMs the tape emits.

Forward  H = ReLU(X W1) (NN), Y = H W2 (NN); backward dH = (dY W2^T) masked by
H > 0 (NT, ReLU's backward as a GEMM epilogue), dW2 = H^T dY (TN),
dX = dH W1^T (NT), dW1 = X^T dH (TN) -- the layouts Tape::backward's MatMul
arm produces (src/tape.rs:505-510) for Linear layers without bias
(src/nn.rs:110-114), with ReLU's mask as in the Relu arm (src/tape.rs:530-534).
"""
from dataclasses import dataclass

import numpy as np
import torch

from .matmul import MatRef, Epilogue, matmul_group, matmul_with, TF32
from .pipeline import HostPipeline


@dataclass
class MlpBuffers:
    """Device tensors of one layer: inputs x, w1, w2, dy; outputs h, y, dh, dx, dw1, dw2."""
    x: torch.Tensor
    w1: torch.Tensor
    w2: torch.Tensor
    dy: torch.Tensor
    h: torch.Tensor
    y: torch.Tensor
    dh: torch.Tensor
    dx: torch.Tensor
    dw1: torch.Tensor
    dw2: torch.Tensor

    @staticmethod
    def allocate(m, d, dff, device):
        f = lambda *s: torch.empty(s, dtype=torch.float32, device=device)
        return MlpBuffers(f(m, d), f(d, dff), f(dff, d), f(m, d), f(m, dff), f(m, d), f(m, dff), f(m, d), f(d, dff),
                          f(dff, d))


def gemm_list(b: MlpBuffers):
    """The six (a, b, out, m, k, n, epilogue) GEMMs of the step, in order."""
    m, d = b.x.shape
    dff = b.w1.shape[1]
    return [
        (MatRef(b.x), MatRef(b.w1), MatRef(b.h), m, d, dff, Epilogue(relu=True)),                # H = relu(X W1)
        (MatRef(b.h), MatRef(b.w2), MatRef(b.y), m, dff, d, None),                               # Y = H W2
        (MatRef(b.dy), MatRef(b.w2, trans=True), MatRef(b.dh), m, d, dff, Epilogue(mask=(b.h, 0))),  # dH
        (MatRef(b.h, trans=True), MatRef(b.dy), MatRef(b.dw2), dff, m, d, None),                 # dW2 = H^T dY
        (MatRef(b.dh), MatRef(b.w1, trans=True), MatRef(b.dx), m, dff, d, None),                 # dX = dH W1^T
        (MatRef(b.x, trans=True), MatRef(b.dh), MatRef(b.dw1), d, m, dff, None),                 # dW1 = X^T dH
    ]


# which GEMMs of gemm_list each one reads the output of
GEMM_AFTER = [(), (0,), (0,), (0,), (2,), (2,)]


def forward_backward_grouped(b: MlpBuffers):
    """The six GEMMs as one persistent grouped launch (matmul_group), on torch's
    current stream: H first, then Y, dH and dW2 as soon as H is complete,
    then dX and dW1 once dH is."""
    g = gemm_list(b)
    matmul_group([(a_, b_, o_, m, k, n, epi, after) for (a_, b_, o_, m, k, n, epi), after in zip(g, GEMM_AFTER)])
    return b


def fused_fits(m, d, dff, device=None) -> bool:
    """Shapes the fused step (forward_backward_fused) takes: d == 128, m and
    dff multiples of 128, and no more 128 x 128 blocks than the GPU has SMs
    (they all run at once)."""
    if not (d == 128 and m % 128 == 0 and dff % 128 == 0):
        return False
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    return (m // 128) * (dff // 128) <= torch.cuda.get_device_properties(dev).multi_processor_count


def forward_backward_fused(b: MlpBuffers, write_h: bool = True):
    """The six GEMMs in one fused tcgen05 kernel (st_mlp_step_tf32) plus a
    fixed-order reduction, on torch's current stream: each 128-token block
    makes its own slice of H and dH and uses it at once from TMEM and shared
    memory.  Shapes: ``fused_fits``.  ``write_h`` False leaves b.h and b.dh
    unwritten."""
    from .device import handle, ptr
    m, d = b.x.shape
    dff = b.w1.shape[1]
    for t in (b.x, b.w1, b.w2, b.dy, b.h, b.y, b.dh, b.dx, b.dw1, b.dw2):
        if not (t.is_contiguous() and t.dtype == torch.float32):
            raise ValueError("forward_backward_fused needs contiguous f32 buffers")
    hh = ptr(b.h) if write_h else None
    dh = ptr(b.dh) if write_h else None
    handle(b.x.device).call("st_mlp_step_tf32", ptr(b.x), ptr(b.w1), ptr(b.w2), ptr(b.dy), hh, ptr(b.y), dh,
                            ptr(b.dx), ptr(b.dw1), ptr(b.dw2), m, d, dff)
    return b


def gemm_bytes(m, d, dff):
    """Algorithmic f32 bytes each GEMM must move (read A, B, mask; write C)."""
    x, w, hh = m * d * 4, d * dff * 4, m * dff * 4
    return [x + w + hh, hh + w + x, x + w + hh + hh, hh + x + w, hh + w + x, x + hh + w]


class StepStreams:
    """Two side streams (with their own library handles) so the step's
    independent GEMMs overlap: after H, {Y, dH, dW2} run concurrently; after
    dH, {dX, dW1}."""

    def __init__(self, device):
        from .device import handle_for_stream
        self.s1 = torch.cuda.Stream(device)
        self.s2 = torch.cuda.Stream(device)
        self.h1 = handle_for_stream(self.s1)
        self.h2 = handle_for_stream(self.s2)


def forward_backward(b: MlpBuffers, precision=TF32, streams: StepStreams = None):
    """Enqueues the six GEMMs on torch's current stream (and, with `streams`,
    overlaps the independent ones on two side streams)."""
    g = gemm_list(b)
    if streams is None:
        for a_, b_, o_, m, k, n, epi in g:
            matmul_with(a_, b_, o_, 1, m, k, n, epi, precision)
        return b
    main = torch.cuda.current_stream()
    run = lambda i, h=None: matmul_with(*g[i][:3], 1, *g[i][3:6], g[i][6], precision, h)
    run(0)                                   # H = relu(X W1)
    e_h = torch.cuda.Event()
    e_h.record(main)
    for s in (streams.s1, streams.s2):
        s.wait_event(e_h)
    with torch.cuda.stream(streams.s1):
        run(1, streams.h1)                   # Y = H W2
    with torch.cuda.stream(streams.s2):
        run(3, streams.h2)                   # dW2 = H^T dY
    run(2)                                   # dH
    e_dh = torch.cuda.Event()
    e_dh.record(main)
    streams.s1.wait_event(e_dh)
    with torch.cuda.stream(streams.s1):
        run(5, streams.h1)                   # dW1 = X^T dH
    run(4)                                   # dX = dH W1^T
    for s in (streams.s1, streams.s2):
        e = torch.cuda.Event()
        e.record(s)
        main.wait_event(e)
    return b


def forward_backward_host(x: np.ndarray, w1: np.ndarray, w2: np.ndarray, dy: np.ndarray, bufs: MlpBuffers = None,
                          outs=None, precision=TF32, streams: StepStreams = None, fused: bool = False):
    """Host arrays in, host gradients out: copies x, w1, w2, dy to the device,
    runs the layer forward and backward, and reads back (y, dx, dw1, dw2).
    ``outs`` may hold preallocated (pinned) host tensors for the results.
    ``fused``: the one-kernel step where the shape allows it (TF32 only)."""
    m, d = x.shape
    dff = w1.shape[1]
    dev = torch.device("cuda", torch.cuda.current_device())
    if bufs is None:
        bufs = MlpBuffers.allocate(m, d, dff, dev)
    for dst, src in ((bufs.x, x), (bufs.w1, w1), (bufs.w2, w2), (bufs.dy, dy)):
        dst.copy_(torch.as_tensor(src), non_blocking=True)
    if fused and precision == TF32 and fused_fits(m, d, dff):
        forward_backward_fused(bufs)
    else:
        forward_backward(bufs, precision, streams)
    if outs is None:
        outs = tuple(torch.empty(t.shape, dtype=torch.float32, pin_memory=True) for t in (bufs.y, bufs.dx, bufs.dw1,
                                                                                          bufs.dw2))
    for dst, src in zip(outs, (bufs.y, bufs.dx, bufs.dw1, bufs.dw2)):
        dst.copy_(src, non_blocking=True)
    torch.cuda.current_stream().synchronize()
    return outs


class HostStream(HostPipeline):
    """MLP layer steps from host arrays, pipelined (``HostPipeline``):
    ``submit((x, w1, w2, dy), (y, dx, dw1, dw2))`` with pinned host tensors."""

    def __init__(self, m, d, dff, device=None, depth=3, precision=TF32, fused: bool = False):
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        self.bufs = [MlpBuffers.allocate(m, d, dff, dev) for _ in range(depth)]
        self.sides = StepStreams(dev)
        sets = [([b.x, b.w1, b.w2, b.dy], [b.y, b.dx, b.dw1, b.dw2]) for b in self.bufs]
        if fused and precision == TF32 and fused_fits(m, d, dff):
            step = lambda j: forward_backward_fused(self.bufs[j])
        else:
            step = lambda j: forward_backward(self.bufs[j], precision, self.sides)
        super().__init__(sets, step, dev)
