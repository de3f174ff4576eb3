"""KnnStore.save / load through the device (src/gpu_step/knn/cache.rs:9-136):
a saved and reloaded store searches exactly as before, flat and IVF (the IVF
section restores the cells), and a sharded load (rows = (lo, hi)) reports
global key indices that agree with the flat search over the same rows."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _store(n, d, seed, tile):
    import scratchtape_b200.knn as K
    rng = np.random.default_rng(seed)
    centers = rng.standard_normal((12, d)).astype(np.float32) * 3
    keys = centers[rng.integers(0, 12, n)] + rng.standard_normal((n, d)).astype(np.float32)
    st = K.KnnStore(d, tile=tile)
    st.set_key_bits(2)
    st.add(keys, np.arange(n) % 251)
    st.add_doc(rng.standard_normal((300, d)).astype(np.float32), np.arange(300) % 7)
    st.finish()
    return st, rng


@pytest.mark.parametrize("mode", ["l2", "dot"])
def test_reload_searches_the_same(dev, tmp_path, mode):
    import scratchtape_b200.knn as K
    st, rng = _store(7000, 128, 3, tile=2048)
    st.build_ivf(12, iters=4)
    path = tmp_path / "m.mem"
    st.save(path, "model-a", extra=77)
    assert K.KnnStore.load(path, "model-b") is None
    st2, extra = K.KnnStore.load(path, "model-a")
    assert extra == 77 and len(st2) == len(st)
    for a, b in ((st.codes, st2.codes), (st.scales, st2.scales), (st.norms, st2.norms), (st.vals, st2.vals)):
        assert torch.equal(a, b)
    q = rng.standard_normal((40, 128)).astype(np.float32)
    s1, v1 = st.search_tagged(q, mode=mode)
    s2, v2 = st2.search_tagged(q, mode=mode)
    assert torch.equal(s1, s2) and torch.equal(v1, v2)
    assert st2.ivf is not None and np.array_equal(st2.ivf["starts"], st.ivf["starts"])
    assert torch.equal(st2.ivf["cent"], st.ivf["cent"]) and torch.equal(st2.ivf["cnorm"], st.ivf["cnorm"])
    s1, i1 = st.search_ivf(q, nprobe=3, mode=mode, with_ids=True)
    s2, i2 = st2.search_ivf(q, nprobe=3, mode=mode, with_ids=True)
    assert torch.equal(s1, s2) and torch.equal(i1, i2)


def test_sharded_load_reports_global_indices(dev, tmp_path):
    import scratchtape_b200.knn as K
    st, rng = _store(9000, 64, 5, tile=1000)
    path = tmp_path / "m.mem"
    st.save(path, "k")
    lo, hi = 2500, 6100
    sh, _ = K.KnnStore.load(path, "k", rows=(lo, hi))
    assert sh.first == lo and len(sh) == hi - lo and sh.ivf_raw is None
    q = torch.from_numpy(rng.standard_normal((20, 64)).astype(np.float32)).cuda()
    s1, i1 = sh.search_ids(q, mode="dot")
    s2, i2 = K.search(st.codes[lo:hi], st.scales[lo:hi], q, mode="dot", index_base=lo)
    assert torch.equal(s1, s2) and torch.equal(i1, i2)
    assert int(i1[i1 >= 0].min()) >= lo and int(i1.max()) < hi
