"""GPU train/add (the build path of IvfUsqIndex) against the CPU oracle.

The global mean, the rotated centroid, the list assignment and every encoded
vector (codes, sign bits, norm, norm_sq, vmax, quant_quality) are bit-exact with
the oracle's restatement of quantizer.rs / ivf_usq.rs; search on the GPU-built
index equals the oracle's search on the exported artifact.  K-means itself is a
seeded GPU implementation (the reference's is entropy-seeded), checked loosely.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_gpu_build_matches_oracle(oracle_mod):
    from hanns_b200.ivf_usq import IvfUsqConfig, IvfUsqIndex, SearchRequest
    from tests.golden.make_golden import mixture
    O = oracle_mod
    rng = np.random.default_rng(77)
    for nbits, metric, d in [(4, 0, 128), (8, 1, 96)]:
        x, _ = mixture(rng, 6000, d, 12, 0.4, metric == 1)
        idx = IvfUsqIndex(IvfUsqConfig(d, 12, nbits, metric_type=metric, rotation_seed=5))
        idx.train(x, kmeans_iters=5, kmeans_seed=1)
        idx.add(x[:4000])
        idx.add(x[4000:], ids=np.arange(4000, 6000, dtype=np.int64) + 10)
        art = idx.export_artifact()
        ids = art["ids"]
        orig = np.where(ids >= 4010, ids - 10, ids)
        assert idx.count() == 6000 and sorted(orig.tolist()) == list(range(6000))
        gm = O.global_mean(x)
        assert np.array_equal(O.rotate(art["rotation"], gm).view(np.uint32),
                              art["rotated_centroid"].view(np.uint32))
        P = art["rotation"]
        assert np.abs(P.astype(np.float64) @ P.T.astype(np.float64) - np.eye(P.shape[0])).max() < 1e-4
        # assignment: every row sits in its nearest list (first strict minimum)
        lists = np.repeat(np.arange(12), np.diff(art["list_offsets"]))
        assert np.array_equal(O.assign(x[orig], art["centroids"]), lists)
        # within a list rows keep insertion order
        for l in range(12):
            seg = orig[art["list_offsets"][l]:art["list_offsets"][l + 1]]
            assert np.all(np.diff(seg) > 0)
        codes, signs, meta = O.encode_batch(P, d, nbits, gm, x[orig])
        assert np.array_equal(codes, art["codes"])
        assert np.array_equal(signs, art["sign_bits"])
        for j, key in enumerate(["norms", "norms_sq", "vmaxs", "quant_qualities"]):
            assert np.array_equal(meta[:, j].view(np.uint32), art[key].view(np.uint32)), key
        # search on the GPU-built index == oracle on its artifact
        q, _ = mixture(rng, 100, d, 12, 0.4, metric == 1)
        r = idx.search(q, SearchRequest(top_k=10, nprobe=4))
        e_ids, e_d, _ = O.OracleIndex(art).search(q, 10, 4)
        assert np.array_equal(r.ids.reshape(e_ids.shape), e_ids)
        assert np.array_equal(r.distances.reshape(e_d.shape).view(np.uint32), e_d.view(np.uint32))
        # k-means produced a sane partition
        sizes = np.diff(art["list_offsets"])
        assert (sizes > 0).sum() >= 10


def test_kmeans_seeding_and_empty_list_restart():
    """k-means++ seeding and the restart of empty centroids (src/quantization/kmeans.rs:
    138-183, 272-290): 64 lists over 8 tight clusters -- random seeding leaves most
    centroids without rows, the reference's scheme keeps every list populated."""
    from hanns_b200.ivf_usq import IvfUsqConfig, IvfUsqIndex
    from tests.golden.make_golden import mixture
    rng = np.random.default_rng(91)
    d, nlist = 64, 64
    x, _ = mixture(rng, 8000, d, 8, 0.05, False)
    idx = IvfUsqIndex(IvfUsqConfig(d, nlist, 4, rotation_seed=3))
    idx.train(x, kmeans_iters=25, kmeans_seed=4)
    idx.add(x)
    art = idx.export_artifact()
    sizes = np.diff(art["list_offsets"])
    assert sizes.sum() == 8000
    assert (sizes == 0).sum() == 0, sizes
    cent = art["centroids"]
    assert len(np.unique(cent.round(6), axis=0)) == nlist
    # same seed, same centroids
    idx2 = IvfUsqIndex(IvfUsqConfig(d, nlist, 4, rotation_seed=3))
    idx2.train(x, kmeans_iters=25, kmeans_seed=4)
    idx2.add(x[:10])
    assert np.array_equal(idx2.export_artifact()["centroids"].view(np.uint32), cent.view(np.uint32))


def test_knowhere_lifecycle_and_persistence(tmp_path):
    """create -> train -> add -> search -> save -> load -> search (C ABI)."""
    from hanns_b200 import _lib
    L = _lib.lib()
    rng = np.random.default_rng(3)
    d, n = 32, 512
    x = rng.uniform(-1, 1, (n, d)).astype(np.float32)
    cfg = _lib.CIndexConfig.default()
    cfg.index_type, cfg.metric_type, cfg.dim = 4, 0, d
    cfg.num_clusters, cfg.nprobe, cfg.prq_nbits = 16, 4, 4
    h = L.knowhere_create_index(cfg)
    assert h, _lib.last_error()
    xp = x.ctypes.data_as(_lib.f32p)
    assert L.knowhere_train_index(h, xp, n, d) == 0
    assert L.knowhere_add_index(h, xp, None, n, d) == 0
    assert L.knowhere_get_index_count(h) == n and L.knowhere_get_index_dim(h) == d
    assert L.knowhere_get_index_type(h) == b"IVF-USQ"
    r = L.knowhere_search(h, xp, 1, 10, d)
    ids = np.ctypeslib.as_array(r.contents.ids, (10,)).copy()
    L.knowhere_free_result(r)
    assert ids[0] == 0  # tests/test_ivf_index_trait.rs:25-51
    path = str(tmp_path / "ivfusq.hgpu").encode()
    assert L.knowhere_save_index(h, path) == 0
    h2 = L.knowhere_create_index(cfg)
    assert L.knowhere_load_index(h2, path) == 0
    r2 = L.knowhere_search(h2, xp, 4, 10, d)
    r1 = L.knowhere_search(h, xp, 4, 10, d)
    a = np.ctypeslib.as_array(r1.contents.ids, (40,)).copy()
    b = np.ctypeslib.as_array(r2.contents.ids, (40,)).copy()
    L.knowhere_free_result(r1)
    L.knowhere_free_result(r2)
    assert np.array_equal(a, b)
    L.knowhere_free_index(h)
    L.knowhere_free_index(h2)


def _ramp(n=100, dim=16):
    i = np.arange(n, dtype=np.float32)[:, None]
    j = np.arange(dim, dtype=np.float32)[None, :]
    return (i * np.float32(0.1) + j * np.float32(0.01)).astype(np.float32)


def test_exrabitq_build_search():
    """src/faiss/exrabitq_ffi.rs:317-355 (build 100x16, nlist 4, 4-bit; search k=10 nprobe=2)."""
    from hanns_b200 import _lib
    L = _lib.lib()
    data = _ramp()
    h = L.knowhere_ivf_exrabitq_build(16, 4, 4, data.ctypes.data_as(_lib.f32p), 100, None)
    assert h, _lib.last_error()
    q = np.full(16, 0.5, np.float32)
    dist = np.zeros(10, np.float32)
    lab = np.zeros(10, np.int64)
    assert L.knowhere_ivf_exrabitq_search(h, q.ctypes.data_as(_lib.f32p), 10, 2,
                                          dist.ctypes.data_as(_lib.f32p), lab.ctypes.data_as(_lib.i64p)) == 0
    L.knowhere_ivf_exrabitq_free(h)


def test_exrabitq_save_load(tmp_path, oracle_mod):
    """src/faiss/exrabitq_ffi.rs:357-394, plus batch_search against the oracle."""
    from hanns_b200 import _lib
    from hanns_b200.ivf_usq import IvfUsqConfig, IvfUsqIndex
    L = _lib.lib()
    data = _ramp()
    h = L.knowhere_ivf_exrabitq_build(16, 4, 4, data.ctypes.data_as(_lib.f32p), 100, None)
    assert h
    path = str(tmp_path / "test_ivf_exrabitq.bin").encode()
    assert L.knowhere_ivf_exrabitq_save(h, path) == 0
    k = 5
    labels = np.zeros(3 * k, np.int64)
    dist = np.zeros(3 * k, np.float32)
    assert L.knowhere_ivf_exrabitq_batch_search(h, data.ctypes.data_as(_lib.f32p), 3, k, 2,
                                                dist.ctypes.data_as(_lib.f32p),
                                                labels.ctypes.data_as(_lib.i64p)) == 0
    art = IvfUsqIndex(IvfUsqConfig(16, 4, 4), _handle=h).export_artifact()
    e_ids, e_d, _ = oracle_mod.OracleIndex(art).search(data[:3], k, 2)
    assert np.array_equal(labels.reshape(3, k), e_ids)
    loaded = L.knowhere_ivf_exrabitq_load(path)
    assert loaded
    assert L.knowhere_ivf_exrabitq_count(loaded) == 100
    assert L.knowhere_ivf_exrabitq_dim(loaded) == 16
    assert L.knowhere_ivf_exrabitq_nlist(loaded) == 4
    L.knowhere_ivf_exrabitq_free(loaded)
