"""The reference's IVF-USQ snapshot file (IvfUsqIndex::save / load,
src/faiss/ivf_usq.rs:131-166, 353-506): "IVFUSQ00", version 3, dim, then the bincode 1.3
encoding (fixed-width little-endian integers, u64 lengths, enum variant index as u32) of
StoredSnapshot.

The writer below restates that layout independently of the library; the library's host
reader must recover every array from it, and the library's writer must produce the same
bytes.  A GPU test loads such a file and searches it against the oracle.
"""
import os
import struct

import numpy as np
import pytest

from tests.golden.make_golden import mixture


def bincode_snapshot(art, nprobe, seed, rerank_k, magic=b"IVFUSQ00", header=True):
    d, nlist = int(art["dim"]), int(art["nlist"])
    off = art["list_offsets"]
    out = bytearray()
    if header:
        out += magic + struct.pack("<II", 3, d)
    out += struct.pack("<QQQ", d, nlist, nprobe)
    out += struct.pack("<I", int(art["metric"]))          # MetricType variant index
    out += struct.pack("<QBQQ", int(art["nbits"]), 0, seed, rerank_k)
    cent = np.ascontiguousarray(art["centroids"], np.float32).reshape(-1)
    out += struct.pack("<Q", cent.size) + cent.tobytes()
    out += struct.pack("<Q", nlist)
    codes = np.ascontiguousarray(art["codes"], np.uint8)
    signs = np.ascontiguousarray(art["sign_bits"], np.uint8)
    for c in range(nlist):
        b, e = int(off[c]), int(off[c + 1])
        ids = np.ascontiguousarray(art["ids"][b:e], np.int64)
        out += struct.pack("<Q", e - b) + ids.tobytes()
        out += struct.pack("<Q", e - b)
        for r in range(b, e):
            out += struct.pack("<Q", codes.shape[1]) + codes[r].tobytes()
            out += struct.pack("<Q", signs.shape[1]) + signs[r].tobytes()
            out += struct.pack("<ffff", art["norms"][r], art["norms_sq"][r], art["vmaxs"][r],
                               art["quant_qualities"][r])
    out += struct.pack("<BQ", 1, len(art["ids"]))
    return bytes(out)


@pytest.fixture(scope="module")
def small_artifact(oracle_mod):
    rng = np.random.default_rng(8)
    x, _ = mixture(rng, 3000, 96, 8, 0.4, False)
    art = oracle_mod.build_artifact(x, 6, 4, oracle_mod.METRIC_L2, rotation_seed=11, kmeans_iters=4,
                                    kmeans_seed=5)
    return art


def read_via_library(path):
    from hanns_b200 import _lib
    L = _lib.lib()
    hdr = np.zeros(10, np.int64)
    assert L.hanns_ivfusq00_read_header(path.encode(), hdr.ctypes.data_as(_lib.i64p)) == 0, _lib.last_error()
    d, D, nbits, nlist, metric, n = (int(v) for v in hdr[:6])
    cb = (D * nbits + 7) // 8
    arrs = dict(centroids=np.zeros(nlist * d, np.float32), rotation=np.zeros(D * D, np.float32),
                rotated_centroid=np.ones(D, np.float32), list_offsets=np.zeros(nlist + 1, np.int64),
                ids=np.zeros(n, np.int64), norms=np.zeros(n, np.float32), norms_sq=np.zeros(n, np.float32),
                vmaxs=np.zeros(n, np.float32), quant_qualities=np.zeros(n, np.float32),
                codes=np.zeros((n, cb), np.uint8), sign_bits=np.zeros((n, D // 8), np.uint8))
    a = _lib.Artifact()
    a.dim, a.padded_dim, a.nbits, a.nlist, a.metric, a.ntotal = d, D, nbits, nlist, metric, n
    for k, v in arrs.items():
        ct = {np.float32: _lib.f32p, np.int64: _lib.i64p, np.uint8: _lib.u8p}[v.dtype.type]
        setattr(a, k, v.ctypes.data_as(ct))
    import ctypes as C
    assert L.hanns_ivfusq00_read(path.encode(), C.byref(a)) == 0, _lib.last_error()
    arrs.update(dim=d, padded_dim=D, nbits=nbits, nlist=nlist, metric=int(a.metric), ntotal=n)
    return hdr, arrs


def test_reader_recovers_every_array(tmp_path, small_artifact):
    art = small_artifact
    p = str(tmp_path / "idx.ivfusq")
    with open(p, "wb") as f:
        f.write(bincode_snapshot(art, nprobe=3, seed=11, rerank_k=64))
    hdr, got = read_via_library(p)
    assert hdr[0] == art["dim"] and hdr[2] == art["nbits"] and hdr[3] == art["nlist"]
    assert hdr[5] == len(art["ids"]) and hdr[6] == 3 and hdr[7] == 11 and hdr[8] == 64 and hdr[9] & 1
    for k in ("list_offsets", "ids", "codes", "sign_bits"):
        assert np.array_equal(got[k].reshape(np.asarray(art[k]).shape), art[k]), k
    for k in ("centroids", "norms", "norms_sq", "vmaxs", "quant_qualities"):
        assert np.array_equal(got[k].view(np.uint32), np.asarray(art[k], np.float32).reshape(-1).view(np.uint32)), k
    # the reference loads with a zero global centroid
    assert not got["rotated_centroid"].any()
    # the rotation comes from the seed: the same matrix the oracle artifact was built with
    assert np.array_equal(got["rotation"].view(np.uint32),
                          np.asarray(art["rotation"], np.float32).reshape(-1).view(np.uint32))


def test_writer_matches_the_restated_layout(tmp_path, small_artifact):
    import ctypes as C

    from hanns_b200 import _lib
    art = small_artifact
    p1 = str(tmp_path / "a.ivfusq")
    with open(p1, "wb") as f:
        f.write(bincode_snapshot(art, nprobe=5, seed=11, rerank_k=32))
    _, got = read_via_library(p1)
    a = _lib.Artifact()
    a.dim, a.padded_dim, a.nbits, a.nlist, a.metric, a.ntotal = (
        got["dim"], got["padded_dim"], got["nbits"], got["nlist"], got["metric"], got["ntotal"])
    keep = {}
    for k in ("centroids", "rotation", "rotated_centroid", "list_offsets", "ids", "norms", "norms_sq",
              "vmaxs", "quant_qualities", "codes", "sign_bits"):
        v = np.ascontiguousarray(got[k])
        keep[k] = v
        ct = {np.float32: _lib.f32p, np.int64: _lib.i64p, np.uint8: _lib.u8p}[v.dtype.type]
        setattr(a, k, v.ctypes.data_as(ct))
    p2 = str(tmp_path / "b.ivfusq")
    assert _lib.lib().hanns_ivfusq00_write(p2.encode(), C.byref(a), 5, 11, 32) == 0, _lib.last_error()
    assert open(p1, "rb").read() == open(p2, "rb").read()


def test_legacy_magic_bare_payload_and_truncation(tmp_path, small_artifact):
    from hanns_b200 import _lib
    art = small_artifact
    body = bincode_snapshot(art, nprobe=2, seed=11, rerank_k=64, header=False)
    for name, blob in (("legacy", b"IVFXRBTQ" + struct.pack("<II", 3, int(art["dim"])) + body),
                       ("bare", body)):
        p = str(tmp_path / name)
        with open(p, "wb") as f:
            f.write(blob)
        _, got = read_via_library(p)
        assert np.array_equal(got["ids"], art["ids"]), name
    p = str(tmp_path / "short")
    with open(p, "wb") as f:
        f.write(bincode_snapshot(art, 2, 11, 64)[:-9])
    hdr = np.zeros(10, np.int64)
    assert _lib.lib().hanns_ivfusq00_read_header(p.encode(), hdr.ctypes.data_as(_lib.i64p)) != 0
    assert "truncated" in _lib.last_error()


@pytest.mark.gpu
def test_gpu_searches_a_reference_snapshot(tmp_path, oracle_mod, small_artifact):
    """hanns_gpu_ivf_usq_load_ivfusq00 and knowhere_load_index open the file; results equal
    the oracle on the artifact as the reference loads it (zero global centroid)."""
    from hanns_b200 import _lib
    from hanns_b200.ivf_usq import IvfUsqIndex, SearchRequest
    O = oracle_mod
    art = small_artifact
    p = str(tmp_path / "idx.ivfusq")
    with open(p, "wb") as f:
        f.write(bincode_snapshot(art, nprobe=3, seed=11, rerank_k=64))
    _, loaded = read_via_library(p)
    exp_art = dict(art)
    exp_art["rotated_centroid"] = np.zeros_like(np.asarray(art["rotated_centroid"], np.float32))
    rng = np.random.default_rng(9)
    q, _ = mixture(rng, 64, int(art["dim"]), 8, 0.4, False)
    e_ids, e_d, _ = O.OracleIndex(exp_art).search(q, 10, 3)
    idx = IvfUsqIndex.load_ivfusq00(p)
    assert idx.config.rotation_seed == 11 and idx.config.nprobe == 3
    r = idx.search(q, SearchRequest(top_k=10, nprobe=3))
    assert np.array_equal(r.ids.reshape(e_ids.shape), e_ids)
    assert np.array_equal(r.distances.reshape(e_ids.shape).view(np.uint32), e_d.view(np.uint32))
    # the GPU index writes the same file back
    p2 = str(tmp_path / "back.ivfusq")
    idx.save_ivfusq00(p2)
    assert open(p, "rb").read() == open(p2, "rb").read()
    # knowhere_load_index on a handle with the same config opens it too
    h = _lib.lib().knowhere_create_index(_knowhere_config(art))
    assert h
    assert _lib.lib().knowhere_load_index(h, p.encode()) == 0, _lib.last_error()
    assert _lib.lib().knowhere_get_index_count(h) == len(art["ids"])
    _lib.lib().knowhere_free_index(h)


def _knowhere_config(art):
    from hanns_b200 import _lib
    c = _lib.CIndexConfig.default()
    c.index_type = 4
    c.metric_type = int(art["metric"])
    c.dim = int(art["dim"])
    c.num_clusters = int(art["nlist"])
    c.prq_nbits = int(art["nbits"])
    c.nprobe = 3
    return c
