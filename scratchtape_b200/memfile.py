"""The on-disk kNN memory (`.mem`) of the reference: KnnStore::save / load
(src/gpu_step/knn/cache.rs:9-136), for 2-bit stores.

Layout, every integer a little-endian u64, every byte string length-prefixed
(u64 length, then the bytes):
  MAGIC, key string, extra, d, tile, f16, kbits, ntiles,
  per tile: len, codes (rows padded to a multiple of 16, d*kbits/8 bytes per
            row, low bits first), scales (f32, padded alike), norms (f32 [len]),
            values (f32 [len]: byte + DOC tag),
  the key sample (an empty byte string), the IVF flag (0 / 1) and, when 1:
  nlist, n, centroid bytes, centroid norms (f32), then per cell its piece
  count and (tile, a, b, g0) per piece.
A file saved under another key reads as absent (load returns None), as in the
reference.  Reading streams tile by tile: a reader thread stays ahead of the
device uploads, which go from pinned staging buffers on a side stream, so the
file reads overlap the host-to-device copies (cache.rs:86-109 does the same
with a channel); with ``rows = (lo, hi)`` only the tiles holding keys lo..hi
are read and uploaded -- one rank's shard of a memory split over GPUs.
"""
import os
import queue
import struct
import threading

import numpy as np

MAGIC = 0x5343_5254_4b4e_4e02


def _put(f, x):
    f.write(struct.pack("<Q", int(x)))


def _put_bytes(f, b):
    b = bytes(b)
    _put(f, len(b))
    f.write(b)


def _get(f):
    b = f.read(8)
    if len(b) != 8:
        raise EOFError("truncated .mem file")
    return struct.unpack("<Q", b)[0]


def _get_bytes(f):
    n = _get(f)
    b = f.read(n)
    if len(b) != n:
        raise EOFError("truncated .mem file")
    return b


def write_mem(path, key: str, extra: int, d: int, tile: int, codes: np.ndarray, scales: np.ndarray,
              norms: np.ndarray, vals: np.ndarray, kbits: int = 2, ivf=None, f16: int = 1):
    """Writes a 2-bit store (host arrays: codes u8 [n, d*kbits/8], scales /
    norms / vals [n]) in tiles of `tile` keys, through a temporary file so a
    crash never leaves a half-written cache (cache.rs:35-78).  ``f16`` is the
    header's f16 flag, written as given (a store read from a file passes the
    flag it was read with, so a re-save keeps it).  The temporary file is the
    path with its extension replaced by ``.part``, as the reference's
    ``path.with_extension("part")`` names it."""
    n = int(codes.shape[0])
    kb = d * kbits // 8
    codes = np.ascontiguousarray(codes, dtype=np.uint8).reshape(n, kb)
    scales = np.asarray(scales, dtype=np.float32).reshape(n)
    norms = np.asarray(norms, dtype=np.float32).reshape(n)
    vals = np.asarray(vals, dtype=np.float32).reshape(n)
    ntiles = (n + tile - 1) // tile
    tmp = os.path.splitext(os.fspath(path))[0] + ".part"
    with open(tmp, "wb") as f:
        _put(f, MAGIC)
        _put_bytes(f, key.encode())
        for x in (extra, d, tile, int(f16), kbits, ntiles):
            _put(f, x)
        for t in range(ntiles):
            a, b = t * tile, min(n, (t + 1) * tile)
            rows = b - a
            rp = (rows + 15) // 16 * 16
            cp = np.zeros((rp, kb), np.uint8)
            cp[:rows] = codes[a:b]
            sp = np.zeros(rp, np.float32)
            sp[:rows] = scales[a:b]
            _put(f, rows)
            _put_bytes(f, cp.tobytes())
            _put_bytes(f, sp.tobytes())
            _put_bytes(f, norms[a:b].tobytes())
            _put_bytes(f, vals[a:b].tobytes())
        _put_bytes(f, b"")  # the key sample: older files carry one, it is derived from the tiles now
        if ivf is None:
            _put(f, 0)
        else:
            _put(f, 1)
            _put(f, ivf["nlist"])
            _put(f, ivf["n"])
            _put_bytes(f, ivf["keys"])
            _put_bytes(f, np.asarray(ivf["norm"], np.float32).tobytes())
            for cell in ivf["cells"]:
                _put(f, len(cell))
                for piece in cell:
                    for x in piece:
                        _put(f, x)
    os.replace(tmp, path)


def read_header(f, key: str):
    """(extra, d, tile, f16, kbits, ntiles), or None when the file was saved under another key."""
    if _get(f) != MAGIC or _get_bytes(f) != key.encode():
        return None
    return tuple(_get(f) for _ in range(6))


def read_mem(path, key: str, rows=None, on_tile=None):
    """Reads a 2-bit .mem file.  Returns None if absent or saved under another
    key, else a dict with extra, d, tile, kbits, n (all keys in the file),
    first (index of the first key returned) and the IVF section (host).
    Each tile overlapping ``rows = (lo, hi)`` (default: all) is passed as
    (first_key, codes, scales, norms, vals) numpy arrays to ``on_tile`` --
    from the calling thread, in order, while a reader thread fetches the
    next tiles."""
    if not os.path.exists(path):
        return None
    f = open(path, "rb", buffering=1 << 24)
    try:
        hdr = read_header(f, key)
        if hdr is None:
            return None
        extra, d, tile, f16, kbits, ntiles = hdr
        if kbits != 2:
            raise ValueError(".mem holds %d-bit keys; this library scans 2-bit keys" % kbits)
        kb = d * kbits // 8
        lo, hi = rows if rows is not None else (0, 1 << 62)
        q = queue.Queue(maxsize=8)
        err = []

        def reader():
            try:
                first = 0
                for _ in range(ntiles):
                    n = _get(f)
                    cb, sb, nb, vb = _get_bytes(f), _get_bytes(f), _get_bytes(f), _get_bytes(f)
                    if first + n > lo and first < hi:
                        q.put((first, n, cb, sb, nb, vb))
                    first += n
                q.put(first)
            except Exception as e:  # handed to the caller
                err.append(e)
                q.put(None)

        th = threading.Thread(target=reader, daemon=True)
        th.start()
        total = None
        while True:
            item = q.get()
            if item is None:
                th.join()
                raise err[0]
            if isinstance(item, int):
                total = item
                break
            first, n, cb, sb, nb, vb = item
            codes = np.frombuffer(cb, np.uint8).reshape(-1, kb)[:n]
            scales = np.frombuffer(sb, np.float32)[:n]
            a, b = max(lo, first) - first, min(hi, first + n) - first
            if on_tile is not None:
                on_tile(first + a, codes[a:b], scales[a:b], np.frombuffer(nb, np.float32)[a:b],
                        np.frombuffer(vb, np.float32)[a:b])
        th.join()
        _get_bytes(f)  # key sample
        ivf = None
        if _get(f) == 1:
            nlist, n_ivf = _get(f), _get(f)
            ivf = {"nlist": nlist, "n": n_ivf, "keys": _get_bytes(f),
                   "norm": np.frombuffer(_get_bytes(f), np.float32).copy(), "cells": []}
            for _ in range(nlist):
                ivf["cells"].append([tuple(_get(f) for _ in range(4)) for _ in range(_get(f))])
        return {"extra": extra, "d": d, "tile": tile, "f16": f16, "kbits": kbits, "n": total,
                "first": min(lo, total), "ivf": ivf}
    finally:
        f.close()
