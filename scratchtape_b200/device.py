"""Per-device handles on the native library, bound to torch's current stream.

Mirrors the reference's process-wide device client (src/gpu_step/mod.rs:42-97):
one handle per CUDA device, created on first use.  Every call re-binds the
handle to torch's current stream, so the library's kernels order with torch
work on that stream.
"""
import ctypes
import threading

import torch

from . import _native as N

_lock = threading.Lock()
_handles = {}


class Handle:
    def __init__(self, device):
        self.device = device
        h = ctypes.c_void_p()
        with torch.cuda.device(device):
            stream = torch.cuda.current_stream(device).cuda_stream
            N.check(None, N.lib.st_create(device, ctypes.c_void_p(stream), ctypes.byref(h)))
        self.ptr = h

    def bind(self, stream=None):
        """Points the handle at `stream` (default: torch's current stream)."""
        if stream is None:
            stream = torch.cuda.current_stream(self.device)
        N.lib.st_set_stream(self.ptr, ctypes.c_void_p(stream.cuda_stream))
        return self.ptr

    def call(self, name, *args):
        fn = getattr(N.lib, name)
        return N.check(self.ptr, fn(self.bind(), *args))

    def sync(self):
        return N.check(self.ptr, N.lib.st_sync(self.bind()))

    @property
    def launches(self):
        return N.lib.st_launch_count(self.ptr)

    @property
    def last_kernel(self):
        return N.lib.st_last_kernel(self.ptr).decode()

    @property
    def scratch_bytes(self):
        return N.lib.st_scratch_bytes(self.ptr)


def handle(device=None):
    """The handle of `device` (default: torch's current CUDA device)."""
    if not torch.cuda.is_available():
        raise RuntimeError("scratchtape_b200 needs a CUDA device (sm_100a); none is visible")
    if device is None:
        device = torch.cuda.current_device()
    if isinstance(device, torch.device):
        device = device.index if device.index is not None else torch.cuda.current_device()
    with _lock:
        h = _handles.get(device)
        if h is None:
            h = Handle(device)
            _handles[device] = h
        return h


_stream_handles = {}


def handle_for_stream(stream):
    """A handle of its own for `stream` (own scratch pool), for GEMMs that run
    concurrently with others on side streams."""
    key = (stream.device.index, stream.cuda_stream)
    with _lock:
        h = _stream_handles.get(key)
        if h is None:
            with torch.cuda.stream(stream):
                h = Handle(stream.device.index)
            _stream_handles[key] = h
        return h


def ptr(t):
    """Raw data pointer of a tensor (None -> NULL)."""
    return None if t is None else ctypes.c_void_p(t.data_ptr())
