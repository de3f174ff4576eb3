"""Row softmax on the device (src/gpu_step/rows.rs:100-123)."""
import torch

from .device import handle, ptr


def softmax(x: torch.Tensor, rows: int, n: int, t: int, scale: float, causal: bool, one: bool, out=None):
    """rows::softmax (rows.rs:106-112): softmax of scale*x per row of [rows, n];
    causal rows r see columns 0..=r%t; one: softmax1."""
    y = torch.empty_like(x) if out is None else out
    handle(x.device).call("st_softmax_rows", ptr(x), ptr(y), rows, n, t, scale, int(causal), int(one))
    return y


def softmax_backward(dy: torch.Tensor, y: torch.Tensor, rows: int, n: int, scale: float):
    """rows::softmax_backward (rows.rs:117-123): scale * y * (dy - sum(dy*y))."""
    dx = torch.empty_like(y)
    handle(y.device).call("st_softmax_rows_bwd", ptr(dy), ptr(y), ptr(dx), rows, n, scale)
    return dx
