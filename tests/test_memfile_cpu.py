"""The .mem format (src/gpu_step/knn/cache.rs:9-136) on the host: a file
written field by field in the reference's order (restated here with struct,
independently of memfile) reads back exactly, sharded reads return the right
rows, a wrong key reads as absent, and write -> read round-trips an IVF
section."""
import struct

import numpy as np

MAGIC = 0x5343_5254_4b4e_4e02


def _u64(x):
    return struct.pack("<Q", x)


def _bytes(b):
    return _u64(len(b)) + bytes(b)


def _reference_layout(key, extra, d, tile, codes, scales, norms, vals):
    """KnnStore::save's byte order for a 2-bit store without IVF."""
    n = codes.shape[0]
    out = _u64(MAGIC) + _bytes(key.encode())
    ntiles = (n + tile - 1) // tile
    for x in (extra, d, tile, 1, 2, ntiles):
        out += _u64(x)
    for t in range(ntiles):
        a, b = t * tile, min(n, (t + 1) * tile)
        rp = (b - a + 15) // 16 * 16
        cp = np.zeros((rp, d // 4), np.uint8)
        cp[:b - a] = codes[a:b]
        sp = np.zeros(rp, np.float32)
        sp[:b - a] = scales[a:b]
        out += _u64(b - a) + _bytes(cp.tobytes()) + _bytes(sp.tobytes()) + _bytes(norms[a:b].tobytes()) + \
            _bytes(vals[a:b].tobytes())
    return out + _bytes(b"") + _u64(0)


def _data(n, d, seed=0):
    rng = np.random.default_rng(seed)
    return (rng.integers(0, 256, (n, d // 4), dtype=np.uint8), rng.random(n, dtype=np.float32),
            rng.random(n, dtype=np.float32), (np.arange(n) % 300).astype(np.float32))


def _collect(path, key, rows=None):
    from scratchtape_b200.memfile import read_mem
    got = []
    meta = read_mem(path, key, rows=rows, on_tile=lambda first, *a: got.append((first,) + tuple(x.copy() for x in a)))
    if meta is None:
        return None, None
    cat = [np.concatenate([g[i] for g in got]) for i in range(1, 5)] if got else None
    return meta, cat


def test_reads_the_reference_layout(tmp_path):
    from scratchtape_b200.memfile import write_mem
    n, d, tile = 1000, 64, 300
    codes, scales, norms, vals = _data(n, d)
    p = tmp_path / "m.mem"
    p.write_bytes(_reference_layout("model-a", 7, d, tile, codes, scales, norms, vals))
    meta, (c, s, nm, v) = _collect(p, "model-a")
    assert (meta["extra"], meta["d"], meta["tile"], meta["n"], meta["first"]) == (7, d, tile, n, 0)
    assert np.array_equal(c, codes) and np.array_equal(s, scales) and np.array_equal(nm, norms)
    assert np.array_equal(v, vals) and meta["ivf"] is None
    # and the writer produces exactly those bytes
    q = tmp_path / "w.mem"
    write_mem(q, "model-a", 7, d, tile, codes, scales, norms, vals)
    assert q.read_bytes() == p.read_bytes()


def test_wrong_key_or_missing_file_reads_as_absent(tmp_path):
    from scratchtape_b200.memfile import read_mem, write_mem
    codes, scales, norms, vals = _data(10, 64)
    p = tmp_path / "m.mem"
    write_mem(p, "a", 0, 64, 16, codes, scales, norms, vals)
    assert read_mem(p, "b") is None
    assert read_mem(tmp_path / "none.mem", "a") is None


def test_sharded_read(tmp_path):
    from scratchtape_b200.memfile import write_mem
    n, d, tile = 1000, 128, 128
    codes, scales, norms, vals = _data(n, d, 3)
    p = tmp_path / "m.mem"
    write_mem(p, "k", 0, d, tile, codes, scales, norms, vals)
    for lo, hi in ((0, 500), (500, 1000), (130, 131), (999, 1000)):
        meta, (c, s, nm, v) = _collect(p, "k", rows=(lo, hi))
        assert meta["first"] == lo and meta["n"] == n
        assert np.array_equal(c, codes[lo:hi]) and np.array_equal(v, vals[lo:hi])


def test_ivf_section_round_trips(tmp_path):
    from scratchtape_b200.memfile import write_mem
    codes, scales, norms, vals = _data(40, 64)
    ivf = {"nlist": 2, "n": 40, "keys": bytes(range(64)), "norm": np.array([1.0, 2.0], np.float32),
           "cells": [[(0, 0, 16, 0)], [(0, 16, 40, 1), (0, 3, 4, 2)]]}
    p = tmp_path / "m.mem"
    write_mem(p, "k", 3, 64, 32, codes, scales, norms, vals, ivf=ivf)
    meta, _ = _collect(p, "k")
    assert meta["ivf"]["nlist"] == 2 and meta["ivf"]["keys"] == ivf["keys"]
    assert meta["ivf"]["cells"] == ivf["cells"]


def test_store_ivf_section_restores_cells(tmp_path):
    """KnnStore's IVF section: cells written as per-tile pieces of consecutive
    store ranges (ivf.rs:451-460) come back as the same cell starts, f16
    centroids and norms; a section whose cells are not consecutive is left
    out rather than misread."""
    import torch
    from scratchtape_b200.knn import KnnStore
    from scratchtape_b200.memfile import read_mem, write_mem
    d, tile, n, nl = 64, 32, 100, 5
    codes, scales, norms, vals = _data(n, d, 4)
    st = KnnStore(d, tile=tile, device="cpu")
    st.codes, st.scales = torch.from_numpy(codes), torch.from_numpy(scales)
    starts = np.array([0, 7, 40, 40, 71, 100], np.int64)
    cent = np.random.default_rng(1).standard_normal((nl, d)).astype(np.float16).astype(np.float32)
    st.ivf = {"cent": torch.from_numpy(cent), "cnorm": torch.from_numpy((cent * cent).sum(1)), "starts": starts,
              "nlist": nl}
    sec = st._ivf_section()
    assert sec["cells"][1] == [(0, 7, 32, 7), (1, 0, 8, 32)] and sec["cells"][2] == []
    p = tmp_path / "m.mem"
    write_mem(p, "k", 0, d, tile, codes, scales, norms, vals, ivf=sec)
    raw = read_mem(p, "k")["ivf"]
    st2 = KnnStore(d, tile=tile, device="cpu")
    st2.codes, st2.scales = st.codes, st.scales
    st2._restore_ivf(raw)
    assert np.array_equal(st2.ivf["starts"], starts)
    assert torch.equal(st2.ivf["cent"], st.ivf["cent"]) and torch.equal(st2.ivf["cnorm"], st.ivf["cnorm"])
    raw["cells"][1] = [(1, 0, 8, 32), (0, 7, 32, 7)]  # out of order: not a consecutive range
    st3 = KnnStore(d, tile=tile, device="cpu")
    st3.codes, st3.scales = st.codes, st.scales
    st3._restore_ivf(raw)
    assert getattr(st3, "ivf", None) is None


def test_f16_flag_round_trips_and_temp_name(tmp_path):
    """The header's f16 flag is written as given and read back (a store that
    was loaded re-saves with the flag it came with), and the temporary file is
    named as path.with_extension("part") names it (cache.rs:36-41): the
    extension replaced, and gone once the write is complete."""
    from scratchtape_b200.memfile import read_header, read_mem, write_mem
    n, d, tile = 100, 64, 64
    codes, scales, norms, vals = _data(n, d, seed=4)
    for flag in (0, 1):
        p = tmp_path / ("f%d.mem" % flag)
        write_mem(p, "k", 3, d, tile, codes, scales, norms, vals, f16=flag)
        with open(p, "rb") as f:
            assert read_header(f, "k")[3] == flag
        assert read_mem(p, "k")["f16"] == flag
        assert not (tmp_path / ("f%d.part" % flag)).exists()
        assert not (tmp_path / ("f%d.mem.part" % flag)).exists()
