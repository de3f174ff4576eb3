"""kNN memory over 2-bit keys on the device: the host mirror of KnnStore
(src/gpu_step/knn.rs:114-331).

Keys are held as the reference holds 2-bit keys (set_key_bits(2),
knn.rs:142-145): per key d/4 bytes of codes u (low bits first) and one f32
scale, dequantised as (u - 1.5) * scale.  Quantisation (tile_of,
knn.rs:190-221) runs on the device with the reference's f32 arithmetic.  A
search is one call of the fused scan + top-k kernel; results come back best
first as (score, key index) -- and, when values were stored, the values.

There is no CPU path: every method calls libst_b200.so.
"""
from typing import Optional

import numpy as np
import torch

from . import _native as N
from .device import handle, ptr

MODES = {"dot": N.KNN_DOT, "l2": N.KNN_L2}
DOC = 256  # value tag of keys added with add_doc (src/gpu_step/knn.rs:19)
PRECS = {"exact": N.KNN_EXACT, "f16": N.KNN_F16REF}
KMAX = N.KNN_KMAX


def _dev(device):
    if device is None:
        return torch.device("cuda", torch.cuda.current_device())
    return torch.device(device)


def quantize(keys: torch.Tensor):
    """tile_of's 2-bit quantiser on the device: keys f32 [n, d] ->
    (codes u8 [n, d/4], scales f32 [n], norms f32 [n])."""
    keys = keys.contiguous().float()
    n, d = keys.shape
    codes = torch.empty((n, d // 4), dtype=torch.uint8, device=keys.device)
    scales = torch.empty(n, dtype=torch.float32, device=keys.device)
    norms = torch.empty(n, dtype=torch.float32, device=keys.device)
    handle(keys.device).call("st_knn_quantize", ptr(keys), n, d, ptr(codes), ptr(scales), ptr(norms))
    return codes, scales, norms


def synth_keys(n: int, d: int, seed: int, first_key: int = 0, device=None):
    """Synthetic 2-bit keys: codes uniform on 0..3, scales |N(0,1)|, from a
    counter hash of (seed, first_key + row)."""
    device = _dev(device)
    codes = torch.empty((n, d // 4), dtype=torch.uint8, device=device)
    scales = torch.empty(n, dtype=torch.float32, device=device)
    handle(device).call("st_knn_synth_keys", ptr(codes), ptr(scales), n, d, seed, first_key)
    return codes, scales


def search(codes: torch.Tensor, scales: torch.Tensor, queries: torch.Tensor, k: int = KMAX, mode: str = "l2",
           prec: str = "exact", index_base: int = 0, out=None):
    """The fused scan: best k keys per query.  Returns (scores f32 [nq, k],
    ids int64 [nq, k]) on the device, best first (DOT: q.k; L2: distance)."""
    queries = queries.contiguous().float()
    nq, d = queries.shape
    assert codes.shape[1] * 4 == d, "codes hold d/4 bytes per key"
    if out is None:
        out = (torch.empty((nq, k), dtype=torch.float32, device=queries.device),
               torch.empty((nq, k), dtype=torch.int64, device=queries.device))
    handle(queries.device).call("st_knn_search", ptr(codes), ptr(scales), codes.shape[0], d, ptr(queries), nq, k,
                                MODES[mode], PRECS[prec], index_base, ptr(out[0]), ptr(out[1]))
    return out


def search_masked(codes: torch.Tensor, scales: torch.Tensor, queries: torch.Tensor, ranges: torch.Tensor,
                  always: int = 0, k: int = KMAX, mode: str = "l2", prec: str = "exact", index_base: int = 0):
    """search() where query q sees only keys j < always or ranges[q, 0] <= j < ranges[q, 1]
    (KnnStore::search_masked, src/gpu_step/knn.rs:287-291)."""
    queries = queries.contiguous().float()
    nq, d = queries.shape
    ranges = ranges.to(device=queries.device, dtype=torch.int64).contiguous()
    out = (torch.empty((nq, k), dtype=torch.float32, device=queries.device),
           torch.empty((nq, k), dtype=torch.int64, device=queries.device))
    handle(queries.device).call("st_knn_search_masked", ptr(codes), ptr(scales), codes.shape[0], d, ptr(queries), nq, k,
                                MODES[mode], PRECS[prec], index_base, ptr(ranges), always, ptr(out[0]), ptr(out[1]))
    return out


def topk_keys(codes, scales, queries, mode="l2", prec="exact", index_base=0, out=None):
    """The scan without decoding: sortable u64 keys [nq, 128] (as int64)."""
    queries = queries.contiguous().float()
    nq, d = queries.shape
    if out is None:
        out = torch.empty((nq, KMAX), dtype=torch.int64, device=queries.device)
    handle(queries.device).call("st_knn_topk_keys", ptr(codes), ptr(scales), codes.shape[0], d, ptr(queries), nq,
                                MODES[mode], PRECS[prec], index_base, ptr(out))
    return out


def merge_keys(lists: torch.Tensor, nq: int, out=None):
    """Best 128 per query over lists [L, nq, 128] of sortable keys."""
    lists = lists.contiguous()
    n_lists = lists.shape[0]
    if out is None:
        out = torch.empty((nq, KMAX), dtype=torch.int64, device=lists.device)
    handle(lists.device).call("st_knn_merge_keys", ptr(lists), n_lists, nq * KMAX, nq, ptr(out))
    return out


def decode(keys, queries, k=KMAX, mode="l2", prec="exact", out=None):
    queries = queries.contiguous().float()
    nq, d = queries.shape
    if out is None:
        out = (torch.empty((nq, k), dtype=torch.float32, device=queries.device),
               torch.empty((nq, k), dtype=torch.int64, device=queries.device))
    handle(queries.device).call("st_knn_decode", ptr(keys), ptr(queries), nq, d, k, MODES[mode], PRECS[prec],
                                ptr(out[0]), ptr(out[1]))
    return out


class KnnStore:
    """KnnStore (src/gpu_step/knn.rs:114-331) for 2-bit keys.

    ``add(keys, vals)`` appends keys (row-major [n, d]) and their byte values;
    ``add_doc`` marks them in-document (value ``DOC + byte``, knn.rs:157-160);
    ``finish()`` quantises pending keys on the device; ``search(queries, rows)``
    returns, per query, the 128 nearest keys as (distance, value) sorted
    ascending, like the reference (L2 with |q|^2 added, clamped at 0), the
    value with its tag stripped; ``search_tagged`` keeps the tag;
    ``search_tail`` scans only the keys from ``from_key`` on.  ``search_ids``
    returns key indices instead, and ``mode="dot"`` ranks by the dot product.
    """

    def __init__(self, d: int, tile: int = 16384, device=None):
        if d % 64 != 0 or not 64 <= d <= 256:
            raise ValueError("2-bit key scan supports d in {64, 128, 192, 256}")
        self.d, self.tile = d, tile
        self.device = _dev(device)
        self.kbits = 2
        self.codes = torch.empty((0, d // 4), dtype=torch.uint8, device=self.device)
        self.scales = torch.empty(0, dtype=torch.float32, device=self.device)
        self.norms = torch.empty(0, dtype=torch.float32, device=self.device)
        self.vals = torch.empty(0, dtype=torch.int32, device=self.device)
        self.first = 0  # global index of the first key (a loaded shard)
        self._pending = []
        self._pending_vals = []

    def set_key_bits(self, bits: int):
        """Only 2-bit keys run on the fused scan (knn.rs:142-145)."""
        if bits != 2 or len(self) != 0:
            raise ValueError("this store holds 2-bit keys; set_key_bits(2) before the first add")
        self.kbits = bits

    def __len__(self):
        return int(self.scales.shape[0]) + sum(int(p.shape[0]) for p in self._pending)

    def add(self, keys, vals=None):
        self._add_tagged(keys, vals, 0)

    def add_doc(self, keys, vals=None):
        """``add``, but search_tagged returns DOC + byte for these keys (knn.rs:157-160)."""
        self._add_tagged(keys, vals, DOC)

    def _add_tagged(self, keys, vals, tag):
        keys = torch.as_tensor(keys, dtype=torch.float32).reshape(-1, self.d)
        self._pending.append(keys)
        v = torch.zeros(keys.shape[0], dtype=torch.int32) if vals is None else torch.as_tensor(
            np.asarray(vals), dtype=torch.int32).reshape(-1)
        if v.shape[0] != keys.shape[0]:
            raise ValueError("one value per key")
        self._pending_vals.append(v + tag)

    def add_codes(self, codes: torch.Tensor, scales: torch.Tensor, vals=None):
        """Appends already-quantised keys (codes [n, d/4], scales [n])."""
        self.finish()
        n = codes.shape[0]
        norms = torch.zeros(n, dtype=torch.float32, device=self.device)
        self.codes = torch.cat([self.codes, codes.to(self.device)])
        self.scales = torch.cat([self.scales, scales.to(self.device)])
        self.norms = torch.cat([self.norms, norms])
        v = torch.zeros(n, dtype=torch.int32) if vals is None else torch.as_tensor(np.asarray(vals), dtype=torch.int32)
        self.vals = torch.cat([self.vals, v.to(self.device)])

    def add_states(self, x: torch.Tensor, vals=None, whitener=None, precision=None):
        """Appends keys built on the device from hidden states x (device f32
        [n, d]): the whitening / rotation GEMM of ``whitener`` (a
        keys.Whitener; None: x already is the key), then the quantiser -- the
        reference's whiten_device + KnnStore::add (tier_eval.rs:1202-1222,
        knn.rs:153-221) without the host round trip."""
        from .keys import build_keys
        from .matmul import F32_EXACT
        self.finish()
        if whitener is not None:
            codes, scales, norms = build_keys(x, whitener, F32_EXACT if precision is None else precision)
        else:
            codes, scales, norms = quantize(x)
        if codes.shape[1] * 4 != self.d:
            raise ValueError("keys are %d wide, the store holds %d" % (codes.shape[1] * 4, self.d))
        n = codes.shape[0]
        self.codes = torch.cat([self.codes, codes])
        self.scales = torch.cat([self.scales, scales])
        self.norms = torch.cat([self.norms, norms])
        v = torch.zeros(n, dtype=torch.int32) if vals is None else torch.as_tensor(np.asarray(vals), dtype=torch.int32)
        self.vals = torch.cat([self.vals, v.to(self.device)])

    def save(self, path, key: str, extra: int = 0):
        """KnnStore::save (src/gpu_step/knn/cache.rs:33-79): the store's keys
        in tiles of ``tile`` keys, tagged with ``key``; see memfile."""
        from .memfile import write_mem
        self.finish()
        write_mem(path, key, extra, self.d, self.tile, self.codes.cpu().numpy(), self.scales.cpu().numpy(),
                  self.norms.cpu().numpy(), self.vals.cpu().numpy().astype(np.float32))

    @staticmethod
    def load(path, key: str, device=None, rows=None):
        """KnnStore::load (cache.rs:81-135): (store, extra), or None when there
        is no file or it was saved under another key.  ``rows = (lo, hi)``
        loads only keys lo..hi -- one rank's shard; the store then reports
        global key indices (its scans run with index_base = lo).  Tiles stream
        from a reader thread into pinned buffers and up on a side stream."""
        from .memfile import read_mem
        dev = _dev(device)
        parts = []
        stream = torch.cuda.Stream(dev)
        inflight = []

        def on_tile(first, codes, scales, norms, vals):
            host = [torch.from_numpy(np.ascontiguousarray(a)).pin_memory() for a in (codes, scales, norms, vals)]
            with torch.cuda.stream(stream):
                devs = [t.to(dev, non_blocking=True) for t in host]
            ev = torch.cuda.Event()
            ev.record(stream)
            inflight.append((ev, host))
            while len(inflight) > 4:  # bound the pinned memory held by copies in flight
                inflight.pop(0)[0].synchronize()
            parts.append((first, devs))

        meta = read_mem(path, key, rows=rows, on_tile=on_tile)
        if meta is None:
            return None
        stream.synchronize()
        store = KnnStore(meta["d"], tile=meta["tile"], device=dev)
        store.kbits = 2
        if parts:
            store.codes = torch.cat([p[1][0] for p in parts])
            store.scales = torch.cat([p[1][1] for p in parts])
            store.norms = torch.cat([p[1][2] for p in parts])
            store.vals = torch.cat([p[1][3] for p in parts]).to(torch.int32)
        store.first = meta["first"]
        store.ivf_raw = meta["ivf"]  # kept for a later IVF search; flat scans ignore it
        return store, meta["extra"]

    def finish(self):
        if not self._pending:
            return
        keys = torch.cat(self._pending).to(self.device)
        codes, scales, norms = quantize(keys)
        self.codes = torch.cat([self.codes, codes])
        self.scales = torch.cat([self.scales, scales])
        self.norms = torch.cat([self.norms, norms])
        self.vals = torch.cat([self.vals, torch.cat(self._pending_vals).to(self.device)])
        self._pending, self._pending_vals = [], []

    def search_ids(self, queries, rows: Optional[int] = None, k: int = KMAX, mode: str = "l2", prec: str = "exact"):
        self.finish()
        return search(self.codes, self.scales, self._queries(queries, rows), k=k, mode=mode, prec=prec,
                      index_base=self.first)

    def _values(self, ids):
        """Stored values of key indices; -1 where a list ran out of keys."""
        return torch.where(ids >= 0, self.vals[(ids - self.first).clamp(min=0)],
                           torch.full_like(ids, -1, dtype=torch.int32))

    def _queries(self, queries, rows):
        q = torch.as_tensor(queries, dtype=torch.float32).reshape(-1, self.d).to(self.device)
        return q if rows is None else q[:rows]

    def search_tagged(self, queries, rows: Optional[int] = None, mask=None, mode: str = "l2", prec: str = "exact"):
        """(distance or score, value) with DOC + byte for add_doc keys
        (knn.rs:291-294); mask = (ranges [rows, 2], always) or None."""
        self.finish()
        q = self._queries(queries, rows)
        if mask is None:
            scores, ids = search(self.codes, self.scales, q, k=KMAX, mode=mode, prec=prec, index_base=self.first)
        else:
            ranges, always = mask
            scores, ids = search_masked(self.codes, self.scales, q, torch.as_tensor(np.asarray(ranges)), always,
                                        mode=mode, prec=prec, index_base=self.first)
        return scores, self._values(ids)

    def search_masked(self, queries, rows: Optional[int] = None, mask=None, mode: str = "l2", prec: str = "exact"):
        """search() with mask = (ranges [rows, 2], always) as in knn.rs:287-289:
        query r sees key j iff j < always or ranges[r, 0] <= j < ranges[r, 1];
        mask None searches every key.  Values come back without their tag."""
        scores, vals = self.search_tagged(queries, rows, mask, mode, prec)
        return scores, torch.where(vals >= 0, vals % DOC, vals)

    def search(self, queries, rows: Optional[int] = None, mode: str = "l2", prec: str = "exact"):
        """(distance or score, value) pairs, [rows, 128] each, best first."""
        return self.search_masked(queries, rows, None, mode, prec)

    def search_tail(self, queries, rows: Optional[int], ranges, from_key: int, mode: str = "l2",
                    prec: str = "exact"):
        """The 128 best among keys j with ranges[r, 0] <= j < ranges[r, 1], every
        ranges[r, 0] >= from_key (knn.rs:296-301): only keys from_key.. are
        scanned, with their global indices.  Values keep their tag."""
        self.finish()
        ranges = np.asarray(ranges, dtype=np.int64).reshape(-1, 2)
        loc = from_key - self.first  # row of key from_key in this store
        if (ranges[:, 0] < from_key).any() or not 0 <= loc < len(self):
            raise ValueError("search_tail: every range must start at or after from_key")
        q = self._queries(queries, rows)
        scores, ids = search_masked(self.codes[loc:], self.scales[loc:], q, torch.from_numpy(ranges), 0,
                                    mode=mode, prec=prec, index_base=from_key)
        return scores, self._values(ids)
