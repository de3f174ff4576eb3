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
import ctypes
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


def dequant(codes: torch.Tensor, scales: torch.Tensor):
    """2-bit rows -> f32 [n, d]: (u - 1.5) * scale."""
    n = codes.shape[0]
    out = torch.empty((n, codes.shape[1] * 4), dtype=torch.float32, device=codes.device)
    handle(codes.device).call("st_knn_dequant", ptr(codes), ptr(scales), n, codes.shape[1] * 4, ptr(out))
    return out


def gather_rows(src: torch.Tensor, perm: torch.Tensor):
    """src[perm] on the device (st_gather_rows); rows of 4-byte multiples."""
    src = src.contiguous()
    perm = perm.to(device=src.device, dtype=torch.int64).contiguous()
    out = torch.empty((perm.shape[0],) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device)
    row_bytes = src[0].numel() * src.element_size()
    handle(src.device).call("st_gather_rows", ptr(src), src.shape[0], ptr(out), ptr(perm), perm.shape[0], row_bytes)
    return out


def _centroid_dots(x: torch.Tensor, cent: torch.Tensor, out=None):
    """x . cent^T [n, nlist] on the TF32 tensor cores."""
    from .matmul import TF32, MatRef, matmul_with
    n, nl = x.shape[0], cent.shape[0]
    if out is None:
        out = torch.empty((n, nl), dtype=torch.float32, device=x.device)
    matmul_with(MatRef(x), MatRef(cent, trans=True), MatRef(out), 1, n, x.shape[1], nl, None, TF32)
    return out


def nearest_cells(x: torch.Tensor, cent: torch.Tensor, cnorm: torch.Tensor, chunk_bytes: int = 1 << 30):
    """Each row's nearest centroid (argmin |c|^2 - 2 x.c), int32 [n], in chunks
    whose distance block stays under chunk_bytes."""
    n, nl = x.shape[0], cent.shape[0]
    out = torch.empty(n, dtype=torch.int32, device=x.device)
    rows = max(1024, chunk_bytes // (4 * nl))
    buf = torch.empty((min(rows, n), nl), dtype=torch.float32, device=x.device)
    h = handle(x.device)
    for a in range(0, n, rows):
        b = min(n, a + rows)
        dots = _centroid_dots(x[a:b], cent, out=buf[:b - a])
        h.call("st_knn_nearest", ptr(dots), ptr(cnorm), b - a, nl, ptr(out[a:]))
    return out


def probe_cells(q: torch.Tensor, cent: torch.Tensor, cnorm: torch.Tensor, nprobe: int):
    """Each query's nprobe nearest centroids, nearest first: int32 [nq, nprobe]."""
    dots = _centroid_dots(q, cent)
    out = torch.empty((q.shape[0], nprobe), dtype=torch.int32, device=q.device)
    handle(q.device).call("st_knn_probe", ptr(dots), ptr(cnorm), q.shape[0], cent.shape[0], nprobe, ptr(out))
    return out


def ivf_units_native(probes: np.ndarray, starts: np.ndarray, chunk: Optional[int] = None, n_sms: int = 148,
                     max_lists: int = 64, reuse: Optional[dict] = None):
    """The scan's unit tables for queries probing cells, from the library's
    native planner (st_knn_ivf_units): one unit per (cell chunk, up to 128 of
    the queries probing the cell), longest first.  A cell longer than
    ``chunk`` keys is scanned as several chunks, each its own unit and its own
    list of the query, so one crowded cell does not leave a single CTA
    scanning it while the others idle; chunk None picks one giving about two
    units of work per SM (n_sms) and at most max_lists lists per query.  Row r
    of a unit is (query, list).  Returns (unit_q int32 [u, 128], unit_list
    int32 [u, 128], unit_keys int64 [u, 2], n_lists).  ``reuse``: a dict whose
    arrays are kept and refilled by later calls (the returned tables are views
    of them)."""
    probes = np.ascontiguousarray(probes, np.int32)
    starts = np.ascontiguousarray(starts, np.int64)
    nq, nprobe = probes.shape
    nu, nl, ch = ctypes.c_int64(), ctypes.c_int32(), ctypes.c_int64()
    args = (probes.ctypes.data_as(ctypes.c_void_p), nq, nprobe, starts.ctypes.data_as(ctypes.c_void_p),
            len(starts) - 1, n_sms, 0 if chunk is None else int(chunk), max_lists)
    def planned(status):
        if status != N.ST_OK:
            raise N.StError(status, "st_knn_ivf_units: probes must name cells < len(starts) - 1, starts must not "
                                    "decrease, and a query may need at most 4096 lists")

    planned(N.lib.st_knn_ivf_units(*args, None, None, None, ctypes.byref(nu), ctypes.byref(nl), ctypes.byref(ch)))
    n = nu.value
    if reuse is None:
        reuse = {}
    if reuse.get("cap", -1) < n:
        reuse["cap"] = max(n, int(reuse.get("cap", 0) * 1.25))
        reuse["q"] = np.empty((reuse["cap"], KQ_ROWS), np.int32)
        reuse["l"] = np.empty((reuse["cap"], KQ_ROWS), np.int32)
        reuse["k"] = np.empty((reuse["cap"], 2), np.int64)
    uq, ul, uk = reuse["q"][:n], reuse["l"][:n], reuse["k"][:n]
    planned(N.lib.st_knn_ivf_units(*args, uq.ctypes.data_as(ctypes.c_void_p), ul.ctypes.data_as(ctypes.c_void_p),
                                   uk.ctypes.data_as(ctypes.c_void_p), ctypes.byref(nu), ctypes.byref(nl),
                                   ctypes.byref(ch)))
    return uq, ul, uk, int(nl.value)


def scan_units(codes, scales, queries, unit_q, unit_list, unit_keys, n_lists, mode="l2", prec="exact",
               index_base=0, out=None):
    """The fused scan over unit tables (host numpy arrays): sortable keys [nq, 128]."""
    queries = queries.contiguous().float()
    nq, d = queries.shape
    if out is None:
        out = torch.empty((nq, KMAX), dtype=torch.int64, device=queries.device)
    uq, ul, uk = (np.ascontiguousarray(a) for a in (unit_q, unit_list, unit_keys))
    handle(queries.device).call("st_knn_scan_units", ptr(codes), ptr(scales), codes.shape[0], d, ptr(queries), nq,
                                MODES[mode], PRECS[prec], index_base, uq.shape[0], uq.ctypes.data_as(ctypes.c_void_p),
                                ul.ctypes.data_as(ctypes.c_void_p), uk.ctypes.data_as(ctypes.c_void_p), n_lists,
                                ptr(out))
    return out


KQ_ROWS = 128  # queries per scan unit (the MMA tile's M)


def _num_sms(device) -> int:
    return torch.cuda.get_device_properties(device).multi_processor_count


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
        self.f16 = 1    # the .mem header's f16 flag: kept from a loaded file, written back by save
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
                  self.norms.cpu().numpy(), self.vals.cpu().numpy().astype(np.float32), ivf=self._ivf_section(),
                  f16=self.f16)

    def _ivf_section(self):
        """The IVF part of a .mem file (cache.rs:54-70): centroids as f16
        rows padded to a multiple of 16, their squared norms, and each cell
        as pieces (tile, a, b, g0) -- rows a..b of tile ``tile``, which are
        store rows g0.. (ivf.rs:37-43, 451-460).  None without an IVF."""
        iv = getattr(self, "ivf", None)
        if iv is None or self.first != 0:
            return None
        nl = iv["nlist"]
        cent = iv["cent"].cpu().numpy().astype(np.float16)
        pad = np.zeros(((nl + 15) // 16 * 16, self.d), np.float16)
        pad[:nl] = cent
        cells = []
        for c in range(nl):
            a, b = int(iv["starts"][c]), int(iv["starts"][c + 1])
            pieces = []
            for t in range(a // self.tile, (b + self.tile - 1) // self.tile):
                lo, hi = max(a, t * self.tile), min(b, (t + 1) * self.tile)
                if lo < hi:
                    pieces.append((t, lo - t * self.tile, hi - t * self.tile, lo))
            cells.append(pieces)
        return {"nlist": nl, "n": int(iv["starts"][-1]), "keys": pad.tobytes(), "norm": iv["cnorm"].cpu().numpy(),
                "cells": cells}

    def _restore_ivf(self, raw):
        """Rebuilds the device IVF from a file's IVF section when its cells are
        consecutive store ranges in cell order (what build_ivf writes, and the
        reference's build_ivf too, ivf.rs:385-447); otherwise leaves it out."""
        nl, d = int(raw["nlist"]), self.d
        starts = np.zeros(nl + 1, np.int64)
        pos = 0
        for c, cell in enumerate(raw["cells"]):
            for (t, a, b, g0) in cell:
                if g0 != pos or t * self.tile + a != g0 or b < a:
                    return
                pos += b - a
            starts[c + 1] = pos
        if pos != raw["n"] or pos > len(self) or len(raw["keys"]) < nl * d * 2 or len(raw["norm"]) < nl:
            return
        cent = np.frombuffer(raw["keys"], np.float16)[:nl * d].reshape(nl, d).astype(np.float32)
        self.ivf = {"cent": torch.from_numpy(cent).to(self.device),
                    "cnorm": torch.from_numpy(np.asarray(raw["norm"][:nl], np.float32).copy()).to(self.device),
                    "starts": starts, "nlist": nl}

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
            host = [torch.from_numpy(np.require(a, requirements=["C", "W"])).pin_memory()
                    for a in (codes, scales, norms, vals)]
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
        store.f16 = int(meta["f16"])
        store.ivf_raw = meta["ivf"]
        if meta["ivf"] is not None and rows is None:
            store._restore_ivf(meta["ivf"])  # a shard keeps only the raw section
        return store, meta["extra"]

    def build_ivf(self, nlist: int, iters: int = 10, sample: Optional[int] = None):
        """KnnStore::build_ivf (src/gpu_step/knn/ivf.rs:337-449): Lloyd's
        k-means on an evenly spaced sample of the keys (starting from evenly
        spaced sample keys; an empty cell restarts at another sample key, as
        the reference does), then every key's nearest cell, then the keys,
        scales, norms and values reordered cell by cell on the device.  The
        distance GEMMs run on the TF32 tensor cores and the assignments in
        st_knn_nearest; the centroid sums are taken on the host in f64 over
        the sample (the reference sums on the host too).  ``self.ivf_order``
        maps the new key positions to the old ones."""
        self.finish()
        n, d = len(self), self.d
        if not 1 <= nlist <= n:
            raise ValueError("build_ivf: 1 <= nlist <= keys")
        ns = min(n, sample if sample is not None else max(8 * nlist, min(n, 32 * nlist)))
        idx = (torch.arange(ns, dtype=torch.int64, device=self.device) * n) // ns
        xs = dequant(gather_rows(self.codes, idx), gather_rows(self.scales.view(-1, 1), idx).view(-1))
        xs_h = xs.cpu().numpy().astype(np.float64)
        cent = xs_h[(np.arange(nlist) * ns) // nlist].copy()
        for it in range(iters):
            c_dev = torch.from_numpy(cent.astype(np.float32)).to(self.device)
            cnorm = torch.from_numpy(np.square(cent).sum(1).astype(np.float32)).to(self.device)
            a = nearest_cells(xs, c_dev, cnorm).cpu().numpy().astype(np.int64)
            order = np.argsort(a, kind="stable")
            counts = np.bincount(a, minlength=nlist)
            sums = np.zeros((nlist, d))
            nz = np.flatnonzero(counts)
            sums[nz] = np.add.reduceat(xs_h[order], np.r_[0, np.cumsum(counts)[:-1]][nz], axis=0)
            for c in range(nlist):
                if counts[c] > 0:
                    cent[c] = sums[c] / counts[c]
                else:
                    cent[c] = xs_h[(c * 7919 + it * 104729) % ns]
        # the final centroids are rounded to f16, as the reference keeps them
        # (ivf.rs:433-434), so a store saved and loaded probes the same cells
        cent = cent.astype(np.float16).astype(np.float64)
        c_dev = torch.from_numpy(cent.astype(np.float32)).to(self.device)
        cnorm = torch.from_numpy(np.square(cent).sum(1).astype(np.float32)).to(self.device)
        cell = torch.empty(n, dtype=torch.int32, device=self.device)
        chunk = 1 << 16
        for a0 in range(0, n, chunk):
            b0 = min(n, a0 + chunk)
            cell[a0:b0] = nearest_cells(dequant(self.codes[a0:b0], self.scales[a0:b0]), c_dev, cnorm)
        cell_h = cell.cpu().numpy().astype(np.int64)
        order = np.argsort(cell_h, kind="stable")
        starts = np.r_[0, np.cumsum(np.bincount(cell_h, minlength=nlist))].astype(np.int64)
        perm = torch.from_numpy(order).to(self.device)
        self.codes = gather_rows(self.codes, perm)
        self.scales = gather_rows(self.scales.view(-1, 1), perm).view(-1)
        self.norms = gather_rows(self.norms.view(-1, 1), perm).view(-1)
        self.vals = gather_rows(self.vals.view(-1, 1), perm).view(-1)
        self.ivf_order = order
        self.ivf = {"cent": c_dev, "cnorm": cnorm, "starts": starts, "nlist": nlist}

    def search_ivf(self, queries, rows: Optional[int] = None, nprobe: int = 8, mode: str = "l2",
                   prec: str = "exact", with_ids: bool = False):
        """KnnStore::search_ivf (ivf.rs:466-526): for each query, the 128 best
        among the keys of its nprobe nearest cells.  One scan launch over a
        table of (cell chunk, up to 128 queries probing it) units -- crowded
        cells split so the SMs share them -- then one merge of each query's
        lists.  Returns (scores, values), or (scores, key indices) with
        ``with_ids``."""
        if getattr(self, "ivf", None) is None:
            raise RuntimeError("search_ivf needs build_ivf")
        q = self._queries(queries, rows)
        iv = self.ivf
        probes = probe_cells(q, iv["cent"], iv["cnorm"], nprobe).cpu().numpy()
        uq, ul, uk, n_lists = ivf_units_native(probes, iv["starts"], n_sms=_num_sms(q.device),
                                               reuse=iv.setdefault("plan", {}))
        keys = scan_units(self.codes, self.scales, q, uq, ul, uk, n_lists, mode=mode, prec=prec,
                          index_base=self.first)
        scores, ids = decode(keys, q, KMAX, mode=mode, prec=prec)
        return (scores, ids) if with_ids else (scores, self._values(ids))

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
