"""The reference's own USQ / IVF-USQ tests, restated against the CPU oracle.

The reference holds no numeric golden vectors for this path; its tests are property
tests.  Each test below names the reference test it restates (paths relative to the
reference repository root).  These pin the oracle's structure (sizes, block
geometry, LUT edge cases, selection rule, end-to-end behaviour); numeric parity with
the Rust binary itself stays unpinned because the Rust toolchain is absent.
"""
import numpy as np
import pytest


def sin_data(n, dim, step=0.13):
    i = np.arange(n * dim, dtype=np.float32)
    return np.sin(i * np.float32(step)).astype(np.float32).reshape(n, dim)


def encode_list(O, dim, nbits, n, seed=42):
    D = O.padded_dim(dim)
    P = O.rotation_matrix(seed, D)
    data = sin_data(n, dim)
    codes, signs, meta = O.encode_batch(P, dim, nbits, np.zeros(dim, np.float32), data)
    return P, data, codes, signs, meta


# tests/test_usq_quantizer.rs:21-44
def test_config_sizes(oracle_mod):
    O = oracle_mod
    assert O.padded_dim(128) == 128 and O.padded_dim(100) == 128 and O.padded_dim(65) == 128
    assert O.code_bytes(128, 4) == 64 and O.code_bytes(128, 1) == 16 and O.code_bytes(128, 8) == 128
    L = O.lib()
    assert L.ousq_sign_bytes(128) == 16 and L.ousq_code_bytes(100, 4) == 64


# tests/test_usq_quantizer.rs:46-94 (rotation preserves norm, inverse, determinism)
def test_rotation_properties(oracle_mod):
    O = oracle_mod
    P = O.rotation_matrix(42, 128)
    v = np.sin(np.arange(128, dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    r = O.rotate(P, v)
    assert abs(np.linalg.norm(v) - np.linalg.norm(r)) < 1e-3
    back = P.T.astype(np.float64) @ r.astype(np.float64)
    assert np.abs(back - v).max() < 1e-3
    assert np.array_equal(P, O.rotation_matrix(42, 128))
    assert not np.array_equal(P, O.rotation_matrix(43, 128))


# tests/test_usq_quantizer.rs:98-191, 195-207
@pytest.mark.parametrize("nbits", [1, 2, 4, 8])
def test_encode_sizes(oracle_mod, nbits):
    O = oracle_mod
    dim = 64 if nbits == 8 else 128
    P = O.rotation_matrix(42, O.padded_dim(dim))
    v = np.sin(np.arange(dim, dtype=np.float32) * np.float32(0.37)).astype(np.float32)[None]
    codes, signs, meta = O.encode_batch(P, dim, nbits, np.zeros(dim, np.float32), v)
    assert codes.shape[1] == O.code_bytes(dim, nbits)
    assert signs.shape[1] == O.padded_dim(dim) // 8
    norm, norm_sq, vmax, qq = meta[0]
    assert norm > 0 and vmax > 0 and qq > 0
    if nbits == 1:
        assert np.array_equal(codes, signs)
    if nbits == 8:
        assert codes.shape[1] != signs.shape[1]
    # nonzero centroid still encodes
    c = (np.arange(dim, dtype=np.float32) * np.float32(0.01)).astype(np.float32)
    codes2, _, meta2 = O.encode_batch(P, dim, nbits, c, v)
    assert meta2[0, 0] > 0 and codes2.shape == codes.shape


# tests/test_usq_quantizer.rs:140-159 (self score within 30% of ||v||^2)
def test_self_score_reasonable(oracle_mod):
    O = oracle_mod
    dim = 128
    P = O.rotation_matrix(42, dim)
    v = np.sin(np.arange(dim, dtype=np.float32) * np.float32(0.37)).astype(np.float32)
    codes, signs, meta = O.encode_batch(P, dim, 4, np.zeros(dim, np.float32), v[None])
    art = dict(dim=dim, padded_dim=dim, nbits=4, nlist=1, metric=O.METRIC_L2,
               centroids=np.zeros((1, dim), np.float32), rotation=P,
               rotated_centroid=np.zeros(dim, np.float32), list_offsets=np.array([0, 1], np.int64),
               ids=np.array([0], np.int64), norms=meta[:, 0].copy(), norms_sq=meta[:, 1].copy(),
               vmaxs=meta[:, 2].copy(), quant_qualities=meta[:, 3].copy(), codes=codes, sign_bits=signs)
    s = O.score(art, v, 0)
    true = float(np.sum(v.astype(np.float64) ** 2))
    assert abs(s - true) / true < 0.3


# tests/test_usq_quantizer.rs:234-297 (layout geometry)
def test_layout_block_geometry(oracle_mod):
    O = oracle_mod
    for n, nb in [(100, 4), (64, 2), (1, 1), (32, 1), (33, 2)]:
        _, _, _, signs, _ = encode_list(O, 128, 4, n)
        blocks = O.fastscan_blocks(signs, 128)
        assert blocks.size == nb * (128 // 4) * 16
    assert (128 // 4) * 16 == 512


# tests/test_usq_fastscan.rs:21-32
def test_fastscan_zero_query(oracle_mod):
    O = oracle_mod
    lut, scale = O.fastscan_lut(np.zeros(128, np.float32))
    assert (lut == 0).all()
    assert scale == np.float32(1e-6)


# tests/test_usq_fastscan.rs:34-47
def test_fastscan_topk_returns_at_most_n(oracle_mod):
    O = oracle_mod
    P, _, _, signs, _ = encode_list(O, 128, 4, 100)
    q = np.cos(np.arange(128, dtype=np.float32) * np.float32(0.71)).astype(np.float32)
    lut, _ = O.fastscan_lut(O.rotate(P, q))
    idx, sc = O.fastscan_topk(O.fastscan_blocks(signs, 128), 100, 128, lut, 20)
    assert 0 < len(idx) <= 20
    assert np.all(np.diff(sc) <= 0)


# tests/test_usq_fastscan.rs:49-147 (two-stage top-10 overlaps brute force >= 4/10)
def test_scan_and_rerank_overlap(oracle_mod):
    O = oracle_mod
    dim, n, k = 128, 200, 10
    P, data, codes, signs, meta = encode_list(O, dim, 4, n)
    art = dict(dim=dim, padded_dim=dim, nbits=4, nlist=1, metric=O.METRIC_L2,
               centroids=np.zeros((1, dim), np.float32), rotation=P,
               rotated_centroid=np.zeros(dim, np.float32), list_offsets=np.array([0, n], np.int64),
               ids=np.arange(n, dtype=np.int64), norms=meta[:, 0].copy(), norms_sq=meta[:, 1].copy(),
               vmaxs=meta[:, 2].copy(), quant_qualities=meta[:, 3].copy(), codes=codes, sign_bits=signs)
    q = np.cos(np.arange(dim, dtype=np.float32) * np.float32(0.71)).astype(np.float32)
    st = O.query_state(art, q)
    qn = np.float32(np.sum(st["q_rot"].astype(np.float32) ** 2, dtype=np.float32))
    bf = []
    for i in range(n):
        s = np.float32(O.score(art, q, i))
        bf.append((max(np.float32(qn + meta[i, 1] - np.float32(2) * s), 0.0), i))
    bf_top = [i for _, i in sorted(bf, key=lambda t: t[0])[:k]]
    ncand = O.n_candidates(4, k)
    assert n > ncand == 150
    idx, _ = O.fastscan_topk(O.fastscan_blocks(signs, dim), n, dim, st["lut"], ncand)
    res = sorted(((max(np.float32(qn + meta[i, 1] - np.float32(2) * np.float32(O.score(art, q, i))), 0.0), i)
                  for i in idx), key=lambda t: t[0])[:k]
    overlap = len(set(bf_top) & {i for _, i in res})
    assert overlap >= 4


# tests/test_ivf_index_trait.rs:25-51 (d=32, n=512, nlist=16, nprobe=4, 4-bit, L2)
def test_ivf_train_add_search_self_query(oracle_mod):
    O = oracle_mod
    rng = np.random.default_rng(7)
    data = rng.uniform(-1, 1, (512, 32)).astype(np.float32)
    art = O.build_artifact(data, 16, 4, O.METRIC_L2, rotation_seed=17)
    idx = O.OracleIndex(art)
    ids, dists, _ = idx.search(data[:1], 10, 4)
    assert ids.shape == (1, 10)
    assert ids[0, 0] == 0


# src/faiss/ivf_usq.rs:792-809 (rank_centroids returns the closest in order)
def test_rank_centroids_order(oracle_mod):
    O = oracle_mod
    dim = 2
    P = O.rotation_matrix(42, 64)
    art = dict(dim=dim, padded_dim=64, nbits=4, nlist=3, metric=O.METRIC_L2,
               centroids=np.array([[0, 0], [10, 10], [20, 20]], np.float32), rotation=P,
               rotated_centroid=np.zeros(64, np.float32), list_offsets=np.zeros(4, np.int64),
               ids=np.zeros(0, np.int64), norms=np.zeros(0, np.float32), norms_sq=np.zeros(0, np.float32),
               vmaxs=np.zeros(0, np.float32), quant_qualities=np.zeros(0, np.float32),
               codes=np.zeros((0, 32), np.uint8), sign_bits=np.zeros((0, 8), np.uint8))
    idx = O.OracleIndex(art)
    ids, dists, cnt, probes = idx.search(np.array([1, 1], np.float32), 5, 2, want_probes=True)
    assert probes.tolist() == [[0, 1]]
    assert (ids == -1).all() and np.isinf(dists).all()  # empty lists -> padded rows


# fastscan.rs:123-131 -- the heap replacement rule (history dependent at the boundary)
def test_fastscan_heap_rule(oracle_mod):
    O = oracle_mod
    idx, sc = O.topk_from_scores(np.array([5, 5, 5, 6], np.int32), 2)
    assert sorted(idx.tolist()) == [1, 3]
    assert idx.tolist() == [3, 1] and sc.tolist() == [6, 5]


# fastscan.rs:179-208 -- AVX-512 accumulates in i16 with wraparound; scalar in i32.
def test_fastscan_i16_wraparound(oracle_mod):
    O = oracle_mod
    D = 3072
    q_rot = np.full(D, 1.0, np.float32)  # every group: nibble 15 -> +4 -> LUT 127
    lut, _ = O.fastscan_lut(q_rot)
    signs = np.full((1, D // 8), 0xFF, np.uint8)
    blocks = O.fastscan_blocks(signs, D)
    s_avx = O.fastscan_scores(blocks, 1, D, lut, O.MODE_AVX512)[0]
    s_sc = O.fastscan_scores(blocks, 1, D, lut, O.MODE_SCALAR)[0]
    assert s_sc == 127 * (D // 4)
    assert s_avx == np.int16(np.int32(s_sc).astype(np.int16))
    assert s_avx != s_sc


def test_pack_unpack_roundtrip(oracle_mod):
    O = oracle_mod
    rng = np.random.default_rng(0)
    for nbits in range(1, 9):
        c = rng.integers(0, 1 << nbits, 257).astype(np.uint16)
        b = O.pack_codes(c, nbits)
        assert b.size == (257 * nbits + 7) // 8
        assert np.array_equal(O.unpack_codes(b, 257, nbits), c)
    # 4-bit: low nibble = even dim (packed.rs LSB-first)
    assert O.pack_codes(np.array([1, 2], np.uint16), 4).tolist() == [0x21]


# USQ half of tests/test_usq_quantizer.rs:301-436 (recall@10 > 0.2 on its data)
def test_usq_flat_recall(oracle_mod):
    O = oracle_mod
    dim, n, k = 128, 500, 10
    i = np.arange(n * dim, dtype=np.float32)
    data = (np.sin(i * np.float32(0.037) + np.float32(0.1)) * np.float32(2.0)).astype(np.float32).reshape(n, dim)
    qs = np.stack([np.cos(np.arange(dim, dtype=np.float32) * np.float32(0.71) + np.float32(q * 0.3))
                   for q in range(10)]).astype(np.float32)
    art = O.build_artifact(data, 1, 4, O.METRIC_L2, rotation_seed=42,
                           centroids=np.zeros((1, dim), np.float32))
    idx = O.OracleIndex(art)
    ids, _, _ = idx.search(qs, n, 1)  # whole list reranked (n <= n_candidates)
    gt = np.argsort(((qs[:, None, :].astype(np.float64) - data[None].astype(np.float64)) ** 2).sum(-1), axis=1)[:, :k]
    recall = np.mean([len(set(gt[q]) & set(ids[q, :k])) / k for q in range(10)])
    assert recall > 0.2
