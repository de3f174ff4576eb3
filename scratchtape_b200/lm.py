"""The byte-level transformer training step on the device.

Model (the reference's device step, src/gpu_step/tape.rs:393-506, with
BASELINE's choices): token + learned position embeddings, ``layers`` pre-LN
blocks (LN -> fused QKV projection -> causal attention over ``heads`` heads of
64 -> output projection + residual; LN -> d_ff ReLU MLP + residual), a final
LN, an output head tied to the token embedding (BASELINE; the reference's
head is untied, tape.rs:431-437), mean cross-entropy, Adam.  Data parallel:
one model per GPU on its own batch, parameters averaged over the ranks every
``sync_every`` steps (local SGD, fused_models_check.rs:16-33 / mod.rs:182-195).

Every piece runs in libst_b200.so: the TF32 tcgen05 GEMMs carry the linear
layers with bias / ReLU / residual / bias-gradient epilogues, the fused
attention reads Q, K, V straight out of the QKV projection's output (head
views, no split/merge copies), and the row kernels do embedding, LayerNorm,
cross-entropy and Adam.  torch supplies device memory and the stream only.
"""
from dataclasses import dataclass

import torch

from . import shard
from .attention import attention_bwd_packed, attention_fwd_packed
from .device import handle, ptr
from .matmul import TF32, Epilogue, MatRef, matmul_with


@dataclass
class LmConfig:
    vocab: int = 256
    d: int = 256
    layers: int = 4
    heads: int = 4
    dff: int = 1024
    t: int = 128
    batch: int = 64
    ln_eps: float = 1e-5
    lr: float = 1e-3
    beta1: float = 0.9
    beta2: float = 0.999
    adam_eps: float = 1e-8
    sync_every: int = 8
    softmax1: bool = False  # the device tape's Config.softmax1 (src/gpu_step/tape.rs:400)
    gemm_prec: int = TF32   # the linear layers' arithmetic: TF32, or TF32X3 (three TF32 products, f32 accuracy)

    def flops_per_step(self):
        """GEMM flops of one forward + backward (attention over causal pairs)."""
        rows = self.batch * self.t
        lin = 2 * rows * (self.d * 3 * self.d + self.d * self.d + 2 * self.d * self.dff)
        head = 2 * rows * self.d * self.vocab
        attn = 4 * self.batch * self.heads * (self.t * (self.t + 1) // 2) * (self.d // self.heads)
        fwd = self.layers * (lin + attn) + head
        return 3 * fwd


def _layout(c: LmConfig):
    """(name, shape) of every parameter, in flat order."""
    out = [("tok", (c.vocab, c.d)), ("pos", (c.t, c.d))]
    for i in range(c.layers):
        p = "l%d." % i
        out += [(p + "ln1_g", (c.d,)), (p + "ln1_b", (c.d,)), (p + "wqkv", (c.d, 3 * c.d)), (p + "bqkv", (3 * c.d,)),
                (p + "wo", (c.d, c.d)), (p + "bo", (c.d,)), (p + "ln2_g", (c.d,)), (p + "ln2_b", (c.d,)),
                (p + "w1", (c.d, c.dff)), (p + "b1", (c.dff,)), (p + "w2", (c.dff, c.d)), (p + "b2", (c.d,))]
    out += [("lnf_g", (c.d,)), ("lnf_b", (c.d,))]
    return out


class TinyLM:
    def __init__(self, cfg: LmConfig, device, seed: int = 0):
        self.c = cfg
        self.device = torch.device(device)
        self.layout = _layout(cfg)
        self.offsets = {}
        n = 0
        for name, shape in self.layout:
            size = 1
            for s in shape:
                size *= s
            self.offsets[name] = (n, shape)
            n += size
        self.n_params = n
        mk = lambda: torch.zeros(n, dtype=torch.float32, device=self.device)
        self.params, self.grads, self.m, self.v = mk(), mk(), mk(), mk()
        self.p = self._views(self.params)
        self.g = self._views(self.grads)
        self.step_count = 0
        self.step_dev = torch.zeros(1, dtype=torch.int32, device=self.device)  # Adam's t, on the device
        self._init(seed)
        self._alloc()

    def _views(self, flat):
        return {name: flat[o:o + int(torch.Size(shape).numel())].view(shape) for name, (o, shape) in self.offsets.items()}

    def _init(self, seed):
        # Linear: He-uniform weights, zero bias (src/nn.rs:74-79); Embedding
        # U(-0.02, 0.02) (src/nn.rs:215-219); LayerNorm gamma 1, beta 0.
        # BASELINE's seed s maps to generator seed s + 1, as for the reference's Rng.
        g = torch.Generator(device=self.device)
        g.manual_seed(seed + 1)
        for name, (o, shape) in self.offsets.items():
            t = self.p[name]
            base = name.split(".")[-1]
            if name in ("tok", "pos"):
                t.copy_((torch.rand(shape, generator=g, device=self.device) * 2 - 1) * 0.02)
            elif base.startswith("w"):
                lim = (6.0 / shape[0]) ** 0.5
                t.copy_((torch.rand(shape, generator=g, device=self.device) * 2 - 1) * lim)
            elif base.endswith("_g"):
                t.fill_(1.0)
            else:
                t.zero_()

    def _alloc(self):
        c, dev = self.c, self.device
        rows = c.batch * c.t
        f = lambda *s: torch.empty(s, dtype=torch.float32, device=dev)
        self.x = [f(rows, c.d) for _ in range(c.layers + 1)]        # block inputs, and the final one
        self.xm = [f(rows, c.d) for _ in range(c.layers)]           # after the attention residual
        self.a = [f(rows, c.d) for _ in range(c.layers)]            # LN1 out
        self.bn = [f(rows, c.d) for _ in range(c.layers)]           # LN2 out
        self.qkv = [f(rows, 3 * c.d) for _ in range(c.layers)]
        self.o = [f(rows, c.d) for _ in range(c.layers)]
        self.lse = [f(c.batch * c.heads, c.t) for _ in range(c.layers)]
        self.hid = [f(rows, c.dff) for _ in range(c.layers)]
        self.ln_stats = [[(f(rows), f(rows)), (f(rows), f(rows))] for _ in range(c.layers)]
        self.xf, self.lnf_stats = f(rows, c.d), (f(rows), f(rows))
        self.logits, self.dlogits = f(rows, c.vocab), f(rows, c.vocab)
        self.loss = f(1)
        self.dx, self.dxm, self.dtmp = f(rows, c.d), f(rows, c.d), f(rows, c.d)
        self.dqkv, self.dhid = f(rows, 3 * c.d), f(rows, c.dff)
        # the weight-gradient GEMMs (off the backward's critical path) run on a
        # side stream with a handle (and scratch) of their own
        from .device import handle_for_stream
        self.side = torch.cuda.Stream(dev)
        self.side_h = handle_for_stream(self.side)

    # -- pieces -------------------------------------------------------------
    def _gemm(self, a, b, out, m, k, n, ta=False, tb=False, epi=None, h=None):
        matmul_with(MatRef(a, trans=ta), MatRef(b, trans=tb), MatRef(out), 1, m, k, n, epi, self.c.gemm_prec, h)

    def _mark(self):
        """An event on the current stream, now."""
        ev = torch.cuda.Event()
        ev.record()
        return ev

    def _side_gemm(self, after, *args, **kw):
        """A weight-gradient GEMM on the side stream once `after` has happened;
        returns the event of its completion."""
        self.side.wait_event(after)
        with torch.cuda.stream(self.side):
            self._gemm(*args, h=self.side_h, **kw)
        ev = torch.cuda.Event()
        ev.record(self.side)
        return ev

    def _ln(self, x, gname, bname, y, stats):
        handle(self.device).call("st_layernorm_fwd", ptr(x), ptr(self.p[gname]), ptr(self.p[bname]), ptr(y),
                                 ptr(stats[0]), ptr(stats[1]), x.shape[0], x.shape[1], self.c.ln_eps)

    def _ln_bwd(self, dy, x, gname, bname, stats, dx, accumulate):
        handle(self.device).call("st_layernorm_bwd", ptr(dy), ptr(x), ptr(self.p[gname]), ptr(stats[0]),
                                 ptr(stats[1]), ptr(dx), ptr(self.g[gname]), ptr(self.g[bname]), x.shape[0],
                                 x.shape[1], int(accumulate))

    # -- step ---------------------------------------------------------------
    def forward(self, ids: torch.Tensor, targets: torch.Tensor, with_grad=True):
        """Loss (device scalar) of one batch; ids/targets int32 [batch*t].
        With ``with_grad`` the logits gradient is kept for backward()."""
        c, h = self.c, handle(self.device)
        rows = c.batch * c.t
        scale = 1.0 / (c.d // c.heads) ** 0.5
        h.call("st_embed_fwd", ptr(ids), ptr(self.p["tok"]), ptr(self.p["pos"]), ptr(self.x[0]), c.batch, c.t, c.d)
        for i in range(c.layers):
            p = "l%d." % i
            self._ln(self.x[i], p + "ln1_g", p + "ln1_b", self.a[i], self.ln_stats[i][0])
            self._gemm(self.a[i], self.p[p + "wqkv"], self.qkv[i], rows, c.d, 3 * c.d,
                       epi=Epilogue(bias=(self.p[p + "bqkv"], 0)))
            attention_fwd_packed(self.qkv[i], c.batch, c.heads, c.t, scale, True, out=(self.o[i], self.lse[i]),
                                 one=c.softmax1)
            self._gemm(self.o[i], self.p[p + "wo"], self.xm[i], rows, c.d, c.d,
                       epi=Epilogue(bias=(self.p[p + "bo"], 0), residual=(self.x[i], 0)))
            self._ln(self.xm[i], p + "ln2_g", p + "ln2_b", self.bn[i], self.ln_stats[i][1])
            self._gemm(self.bn[i], self.p[p + "w1"], self.hid[i], rows, c.d, c.dff,
                       epi=Epilogue(bias=(self.p[p + "b1"], 0), relu=True))
            self._gemm(self.hid[i], self.p[p + "w2"], self.x[i + 1], rows, c.dff, c.d,
                       epi=Epilogue(bias=(self.p[p + "b2"], 0), residual=(self.xm[i], 0)))
        self._ln(self.x[c.layers], "lnf_g", "lnf_b", self.xf, self.lnf_stats)
        # tied head: logits = xf . tok^T
        self._gemm(self.xf, self.p["tok"], self.logits, rows, c.d, c.vocab, tb=True)
        h.call("st_cross_entropy", ptr(self.logits), ptr(targets), ptr(self.loss),
               ptr(self.dlogits) if with_grad else None, rows, c.vocab)
        return self.loss

    def backward(self, ids: torch.Tensor):
        """Gradients of the last forward() into self.grads (overwritten).

        The chain dlogits -> dx -> ... -> embedding runs on the current stream;
        each weight gradient (a TN GEMM over all rows, with its bias gradient
        as a column-sum epilogue) runs on the side stream as soon as its
        inputs exist.  Before the chain overwrites a buffer that a pending
        side GEMM reads (dx, dxm, dhid, dqkv), it waits for that GEMM; at the
        end it waits for the side stream, so Adam sees every gradient."""
        c = self.c
        rows = c.batch * c.t
        scale = 1.0 / (c.d // c.heads) ** 0.5
        main = torch.cuda.current_stream(self.device)
        self.grads.zero_()
        # head: dxf = dlogits . tok (chain); dtok = dlogits^T . xf (side)
        last = self._side_gemm(self._mark(), self.dlogits, self.xf, self.g["tok"], c.vocab, rows, c.d, ta=True)
        tok_done = last
        self._gemm(self.dlogits, self.p["tok"], self.dtmp, rows, c.vocab, c.d)
        self._ln_bwd(self.dtmp, self.x[c.layers], "lnf_g", "lnf_b", self.lnf_stats, self.dx, False)
        reads = {}  # buffer -> completion event of the last side GEMM reading it
        for i in reversed(range(c.layers)):
            p = "l%d." % i
            # MLP: x[i+1] = xm + relu(bn W1 + b1) W2 + b2
            w2_done = self._side_gemm(self._mark(), self.hid[i], self.dx, self.g[p + "w2"], c.dff, rows, c.d,
                                      ta=True, epi=Epilogue(col_sum=(self.g[p + "b2"], 0, 0)))
            if "dhid" in reads:
                main.wait_event(reads["dhid"])
            self._gemm(self.dx, self.p[p + "w2"], self.dhid, rows, c.d, c.dff, tb=True,
                       epi=Epilogue(mask=(self.hid[i], 0)))
            reads["dhid"] = self._side_gemm(self._mark(), self.bn[i], self.dhid, self.g[p + "w1"], c.d, rows, c.dff,
                                            ta=True, epi=Epilogue(col_sum=(self.g[p + "b1"], 0, 0)))
            self._gemm(self.dhid, self.p[p + "w1"], self.dtmp, rows, c.dff, c.d, tb=True)
            if "dxm" in reads:
                main.wait_event(reads["dxm"])
            self.dxm.copy_(self.dx)
            self._ln_bwd(self.dtmp, self.xm[i], p + "ln2_g", p + "ln2_b", self.ln_stats[i][1], self.dxm, True)
            # attention: xm = x + attn(qkv(LN1 x)) Wo + bo
            reads["dxm"] = self._side_gemm(self._mark(), self.o[i], self.dxm, self.g[p + "wo"], c.d, rows, c.d,
                                           ta=True, epi=Epilogue(col_sum=(self.g[p + "bo"], 0, 0)))
            self._gemm(self.dxm, self.p[p + "wo"], self.dtmp, rows, c.d, c.d, tb=True)
            if "dqkv" in reads:
                main.wait_event(reads["dqkv"])
            attention_bwd_packed(self.qkv[i], self.o[i], self.dtmp, self.lse[i], c.batch, c.heads, c.t, scale, True,
                                 out=self.dqkv)
            last = reads["dqkv"] = self._side_gemm(self._mark(), self.a[i], self.dqkv, self.g[p + "wqkv"], c.d, rows,
                                                   3 * c.d, ta=True,
                                                   epi=Epilogue(col_sum=(self.g[p + "bqkv"], 0, 0)))
            self._gemm(self.dqkv, self.p[p + "wqkv"], self.dtmp, rows, 3 * c.d, c.d, tb=True)
            main.wait_event(w2_done)
            self.dx.copy_(self.dxm)
            self._ln_bwd(self.dtmp, self.x[i], p + "ln1_g", p + "ln1_b", self.ln_stats[i][0], self.dx, True)
        main.wait_event(tok_done)
        handle(self.device).call("st_embed_bwd", ptr(ids), ptr(self.dx), ptr(self.g["tok"]), ptr(self.g["pos"]),
                                 c.batch, c.t, c.d, c.vocab, 1)
        main.wait_event(last)

    def adam_step(self):
        c = self.c
        self.step_count += 1
        handle(self.device).call("st_adam_dev", ptr(self.params), ptr(self.grads), ptr(self.m), ptr(self.v),
                                 self.n_params, ptr(self.step_dev), c.lr, c.beta1, c.beta2, c.adam_eps)

    def capture_step(self, ids_buf: torch.Tensor, tg_buf: torch.Tensor):
        """A CUDA graph of forward + backward + Adam reading the static buffers
        ids_buf / tg_buf; each replay() is one optimiser step (the model
        average of local SGD stays outside, between replays).  Runs one eager
        step first, which sizes every scratch buffer."""
        s = torch.cuda.Stream(self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.train_step(ids_buf, tg_buf)
        torch.cuda.current_stream(self.device).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            self.forward(ids_buf, tg_buf)
            self.backward(ids_buf)
            self.adam_step()
        return graph

    def train_step(self, ids, targets, group=None):
        """forward + backward + Adam; every sync_every steps (distributed) the
        parameters are averaged over the ranks."""
        loss = self.forward(ids, targets)
        self.backward(ids)
        self.adam_step()
        if group is not None and self.step_count % self.c.sync_every == 0:
            shard.average_params(self.params, group)
        return loss
