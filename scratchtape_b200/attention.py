"""Fused causal attention on the device (f16 storage, f32 accumulation).

Mirrors the attention of TransformerBlock::forward_full (src/nn.rs:646-671)
and DeviceTape (src/gpu_step/tape.rs:481-484, :349-375): per head,
O = softmax(scale * Q K^T + causal mask) V -- or softmax1 (a phantom zero
logit, DeviceTape::causal_softmax(x, scale, one), tape.rs:225) -- and its
backward, for sequences up to 256 (the reference's MAX_SEQ).  One kernel
launch per direction for all heads (st_attn_fwd / st_attn_bwd); there is no
CPU path.
"""
import torch

from .device import handle, ptr


def attention_fwd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float, causal: bool = True, out=None,
                  one: bool = False):
    """q, k, v: f16 [bh, t, d] (d = 64, t <= 256) -> (o f16 [bh, t, d], lse f32 [bh, t]).
    ``one``: softmax1.  The backward needs no flag: lse carries it."""
    q, k, v = (x.contiguous() for x in (q, k, v))
    bh, t, d = q.shape
    if out is None:
        out = (torch.empty_like(q), torch.empty((bh, t), dtype=torch.float32, device=q.device))
    handle(q.device).call("st_attn_fwd", ptr(q), ptr(k), ptr(v), ptr(out[0]), ptr(out[1]), bh, t, d, float(scale),
                          int(causal), int(one))
    return out


def attention_bwd(q, k, v, o, dout, lse, scale: float, causal: bool = True, out=None):
    """-> (dq, dk, dv), f16 [bh, t, d]."""
    q, k, v, o, dout = (x.contiguous() for x in (q, k, v, o, dout))
    bh, t, d = q.shape
    if out is None:
        out = (torch.empty_like(q), torch.empty_like(q), torch.empty_like(q))
    handle(q.device).call("st_attn_bwd", ptr(q), ptr(k), ptr(v), ptr(o), ptr(dout), ptr(lse), ptr(out[0]),
                          ptr(out[1]), ptr(out[2]), bh, t, d, float(scale), int(causal))
    return out


def attention_fwd_packed(qkv: torch.Tensor, batch: int, heads: int, t: int, scale: float, causal: bool = True,
                         out=None, one: bool = False):
    """Fused attention on the packed f32 layout of the transformer step:
    qkv [batch*t, 3*heads*64] -> (o [batch*t, heads*64] f32, lse [batch*heads, t])."""
    d = 64
    if out is None:
        out = (torch.empty((batch * t, heads * d), dtype=torch.float32, device=qkv.device),
               torch.empty((batch * heads, t), dtype=torch.float32, device=qkv.device))
    handle(qkv.device).call("st_attn_fwd_packed", ptr(qkv), ptr(out[0]), ptr(out[1]), batch, heads, t, d,
                            float(scale), int(causal), int(one))
    return out


def attention_bwd_packed(qkv, o, dout, lse, batch: int, heads: int, t: int, scale: float, causal: bool = True,
                         out=None):
    """-> dqkv [batch*t, 3*heads*64] f32."""
    d = 64
    if out is None:
        out = torch.empty_like(qkv)
    handle(qkv.device).call("st_attn_bwd_packed", ptr(qkv), ptr(o), ptr(dout), ptr(lse), ptr(out), batch, heads, t,
                            d, float(scale), int(causal))
    return out


class HostStream:
    """Attention steps (forward + backward of every head) from host arrays,
    pipelined: ``submit((q, k, v, dout), (o, dq, dk, dv))`` with pinned f16
    host tensors [bh, t, 64]; uploads, the two kernels and downloads overlap
    across consecutive steps (``pipeline.HostPipeline``)."""

    def __init__(self, bh, t, scale, causal=True, device=None, depth=3):
        from .pipeline import HostPipeline
        dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
        f = lambda: torch.empty((bh, t, 64), dtype=torch.float16, device=dev)
        self.sets = []
        for _ in range(depth):
            q, k, v, dout, o, dq, dk, dv = (f() for _ in range(8))
            lse = torch.empty((bh, t), dtype=torch.float32, device=dev)
            self.sets.append(((q, k, v, dout), (o, dq, dk, dv), lse))

        def run(j):
            (q, k, v, dout), (o, dq, dk, dv), lse = self.sets[j]
            attention_fwd(q, k, v, scale, causal, out=(o, lse))
            attention_bwd(q, k, v, o, dout, lse, scale, causal, out=(dq, dk, dv))

        self.pipe = HostPipeline([(list(i), list(o)) for i, o, _ in self.sets], run, dev)

    def submit(self, host_inputs, host_outputs):
        return self.pipe.submit(host_inputs, host_outputs)

    def wait(self, ticket):
        self.pipe.wait(ticket)

    def close(self):
        self.pipe.close()
