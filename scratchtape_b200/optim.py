"""The device step's optimiser, model average and dropout (src/gpu_step/mod.rs:153-195,
src/gpu_step/tape.rs:526-543), on flat f32 device tensors.

Names follow the reference: ``sgd``, ``momentum`` and ``decay`` are
DeviceParams' methods, ``average_models`` / ``average_groups`` its local-SGD
sync across the K models held on one device, ``dropout`` and
``dropout_relu_backward`` the tape's functions.  Every one is a single
launch of libst_b200.so, bit-identical to the reference's f32 arithmetic.
"""
import torch

from .device import handle, ptr


def _flat(t: torch.Tensor, name: str):
    if t.dtype != torch.float32 or not t.is_contiguous() or not t.is_cuda:
        raise ValueError("%s must be a contiguous float32 CUDA tensor" % name)
    return t


def sgd(params: torch.Tensor, grads: torch.Tensor, lr: float):
    """DeviceParams::sgd (mod.rs:153-157): p -= lr * g."""
    _flat(params, "params"), _flat(grads, "grads")
    handle(params.device).call("st_sgd", ptr(params), ptr(grads), params.numel(), lr)


def momentum(params: torch.Tensor, grads: torch.Tensor, velocity: torch.Tensor, lr: float, mu: float,
             decay=None):
    """DeviceParams::momentum (mod.rs:159-166): with decay = (shrink, mask),
    p *= 1 - shrink * mask first; then v = mu v + g, p -= lr v."""
    _flat(params, "params"), _flat(grads, "grads"), _flat(velocity, "velocity")
    shrink, mask = decay if decay is not None else (0.0, None)
    handle(params.device).call("st_momentum", ptr(params), ptr(grads), ptr(velocity), ptr(mask), params.numel(), lr,
                               mu, shrink)


def decay(params: torch.Tensor, shrink: float, mask: torch.Tensor):
    """DeviceParams::decay (mod.rs:168-174): p *= 1 - shrink * mask."""
    _flat(params, "params"), _flat(mask, "mask")
    handle(params.device).call("st_decay", ptr(params), ptr(mask), params.numel(), shrink)


def average_groups(params: torch.Tensor, models: int, group: int):
    """DeviceParams::average_groups (mod.rs:188-195): params holds `models`
    consecutive models; each group of `group` consecutive models gets its mean."""
    _flat(params, "params")
    if params.numel() % models:
        raise ValueError("%d parameters do not split into %d models" % (params.numel(), models))
    handle(params.device).call("st_average_models", ptr(params), params.numel() // models, models, group)


def average_models(params: torch.Tensor, models: int):
    """DeviceParams::average_models (mod.rs:182-186): every model becomes the mean of all."""
    average_groups(params, models, models)


def dropout(x: torch.Tensor, rate: float, seed: int, out=None):
    """gpu_step::tape::dropout (tape.rs:526-534): x / (1 - rate) where the
    element's lowbias32 hash clears rate * 2^32, else 0."""
    _flat(x, "x")
    y = torch.empty_like(x) if out is None else out
    handle(x.device).call("st_dropout", ptr(x), ptr(y), x.numel(), rate, seed & 0xffffffff)
    return y


def dropout_relu_backward(dy: torch.Tensor, relu_y: torch.Tensor, rate: float, seed: int, out=None):
    """gpu_step::tape::dropout_relu_backward (tape.rs:536-543): dropout(dy)
    where relu_y > 0, else 0."""
    _flat(dy, "dy"), _flat(relu_y, "relu_y")
    dx = torch.empty_like(dy) if out is None else out
    handle(dy.device).call("st_dropout_relu_bwd", ptr(dy), ptr(relu_y), ptr(dx), dy.numel(), rate,
                           seed & 0xffffffff)
    return dx
