"""Parity of the CUDA search path (through the C ABI) with the CPU oracle.

Bit-exact: coarse probes, q_rot, q_i8, sum(q_i8), the FastScan LUT and its scale,
the per-query scalars, result ids and distances (float bits), fused and post
bitset filtering.  Inputs: the committed golden fixtures (oracle outputs) and
freshly oracle-built artifacts at larger sizes.
"""
import ctypes as C
import glob
import os

import numpy as np
import pytest

from tests.golden.make_golden import load

pytestmark = pytest.mark.gpu

FIXTURES = sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz")))
IDS = [os.path.basename(p)[:-4] for p in FIXTURES]


@pytest.fixture(scope="module")
def gpu():
    from hanns_b200 import _lib
    L = _lib.lib()
    if L.hanns_gpu_device_count() < 1:
        pytest.fail("no CUDA device visible to libhanns_gpu")
    return L


def bits_eq(a, b):
    return np.array_equal(np.asarray(a, np.float32).view(np.uint32), np.asarray(b, np.float32).view(np.uint32))


@pytest.mark.parametrize("path", FIXTURES, ids=IDS)
def test_query_state_and_probes_bit_exact(gpu, path):
    from hanns_b200.ivf_usq import IvfUsqIndex
    art, z = load(path)
    idx = IvfUsqIndex.from_artifact(art)
    st = idx.debug_query(z["queries"], z["nprobe"])
    assert np.array_equal(st["probes"], z["exp_probes"])
    assert bits_eq(st["q_rot"], z["exp_q_rot"])
    assert np.array_equal(st["q_i8"], z["exp_q_i8"])
    assert np.array_equal(st["q_i8_sum"], z["exp_q_i8_sum"])
    assert np.array_equal(st["lut"], z["exp_lut"])
    assert bits_eq(st["q_scale"], z["exp_scalars"][:, 0])
    assert bits_eq(st["centroid_score"], z["exp_scalars"][:, 1])
    assert bits_eq(st["q_norm_sq"], z["exp_scalars"][:, 2])
    assert bits_eq(st["lut_scale"], z["exp_scalars"][:, 3])


@pytest.mark.parametrize("path", FIXTURES, ids=IDS)
def test_search_bit_exact(gpu, path):
    from hanns_b200.ivf_usq import IvfUsqIndex, SearchRequest
    art, z = load(path)
    idx = IvfUsqIndex.from_artifact(art)
    r = idx.search(z["queries"], SearchRequest(top_k=z["k"], nprobe=z["nprobe"]))
    ids = r.ids.reshape(z["exp_ids"].shape)
    d = r.distances.reshape(z["exp_ids"].shape)
    assert np.array_equal(ids, z["exp_ids"])
    assert bits_eq(d, z["exp_dists"])
    # run twice: workspace reuse must not change results
    r2 = idx.search(z["queries"], SearchRequest(top_k=z["k"], nprobe=z["nprobe"]))
    assert np.array_equal(r2.ids, r.ids) and bits_eq(r2.distances, r.distances)


@pytest.mark.parametrize("path", FIXTURES, ids=IDS)
def test_bitset_fused_and_post(gpu, path):
    from hanns_b200.ivf_usq import FILTER_FUSED, FILTER_POST, IvfUsqIndex, SearchRequest
    art, z = load(path)
    idx = IvfUsqIndex.from_artifact(art)
    req = SearchRequest(top_k=z["k"], nprobe=z["nprobe"])
    blen = int(z["bitset_len"][0])
    f = idx.search(z["queries"], req, FILTER_FUSED, z["bitsets"], blen, z["query_bitset"])
    assert np.array_equal(f.ids.reshape(z["exp_fused_ids"].shape), z["exp_fused_ids"])
    assert bits_eq(f.distances.reshape(z["exp_fused_ids"].shape), z["exp_fused_dists"])
    p = idx.search(z["queries"], req, FILTER_POST, z["bitsets"], blen, z["query_bitset"])
    assert np.array_equal(p.counts, z["exp_post_counts"])
    assert np.array_equal(p.ids.reshape(z["exp_post_ids"].shape), z["exp_post_ids"])


def test_knowhere_c_abi_search(gpu):
    """knowhere_search / knowhere_search_with_bitset on an imported index."""
    from hanns_b200 import _lib
    from hanns_b200.ivf_usq import IvfUsqIndex
    art, z = load(FIXTURES[0])
    idx = IvfUsqIndex.from_artifact(art)
    h = idx._h
    assert gpu.knowhere_set_nprobe(h, int(z["nprobe"])) == 0
    q = np.ascontiguousarray(z["queries"], np.float32)
    nq, k = q.shape[0], int(z["k"])
    r = gpu.knowhere_search(h, q.ctypes.data_as(_lib.f32p), nq, k, q.shape[1])
    assert r
    n = r.contents.num_results
    ids = np.ctypeslib.as_array(r.contents.ids, (n,)).copy()
    ds = np.ctypeslib.as_array(r.contents.distances, (n,)).copy()
    gpu.knowhere_free_result(r)
    assert n == nq * k
    assert np.array_equal(ids.reshape(nq, k), z["exp_ids"])
    assert bits_eq(ds.reshape(nq, k), z["exp_dists"])
    # wrong dim -> NULL, no crash
    assert not gpu.knowhere_search(h, q.ctypes.data_as(_lib.f32p), nq, k, q.shape[1] + 1)
    # one bitset for the whole batch, fused (default) semantics
    blen = int(z["bitset_len"][0])
    b = gpu.knowhere_bitset_create(blen)
    words = z["bitsets"][0]
    for i in range(blen):
        if (int(words[i >> 6]) >> (i & 63)) & 1:
            gpu.knowhere_bitset_set(b, i, True)
    r = gpu.knowhere_search_with_bitset(h, q.ctypes.data_as(_lib.f32p), nq, k, q.shape[1], b)
    n = r.contents.num_results
    fid = np.ctypeslib.as_array(r.contents.ids, (n,)).copy()
    gpu.knowhere_free_result(r)
    gpu.knowhere_bitset_free(b)
    from oracle import oracle as O
    oi = O.OracleIndex(art)
    exp, _, _ = oi.search(q, k, int(z["nprobe"]), filter_mode=O.FILTER_FUSED,
                          bitsets=z["bitsets"][:1], bitset_len=blen)
    assert np.array_equal(fid.reshape(nq, k), exp)


@pytest.mark.parametrize("nbits,metric,k,d", [(4, 0, 10, 128), (8, 1, 10, 200), (4, 1, 50, 64),
                                              (8, 0, 100, 96), (4, 1, 10, 1100), (8, 0, 10, 520)])
def test_search_bit_exact_larger(gpu, oracle_mod, nbits, metric, k, d):
    """Oracle-built artifacts with 20k rows: FastScan lists, k up to 100; d = 520 (8-bit,
    padded 576) and d = 1100 (padded 1152) take the rerank without the prefetched code
    registers (query rows in shared memory)."""
    from hanns_b200.ivf_usq import IvfUsqIndex, SearchRequest
    from tests.golden.make_golden import mixture
    O = oracle_mod
    rng = np.random.default_rng(100 + nbits + k)
    x, _ = mixture(rng, 20000, d, 32, 0.4, metric == 1)
    q, _ = mixture(rng, 300, d, 32, 0.4, metric == 1)
    art = O.build_artifact(x, 24, nbits, metric, rotation_seed=9, kmeans_iters=6, kmeans_seed=3)
    oi = O.OracleIndex(art)
    exp_ids, exp_d, _ = oi.search(q, k, 6)
    idx = IvfUsqIndex.from_artifact(art)
    r = idx.search(q, SearchRequest(top_k=k, nprobe=6))
    assert np.array_equal(r.ids.reshape(exp_ids.shape), exp_ids)
    assert bits_eq(r.distances.reshape(exp_ids.shape), exp_d)


@pytest.mark.parametrize("nbits,metric,k,nlist,fused", [(4, 1, 10, 12, False), (8, 0, 10, 40, True),
                                                         (4, 0, 20, 6, True)])
def test_tensor_core_and_simt_scans_agree(gpu, oracle_mod, nbits, metric, k, nlist, fused):
    """Lists above n_cand and up to 1,792 rows take the tcgen05 scan (one-hot FastScan GEMM,
    int8 rerank GEMM), longer ones the SIMT scan: both equal the oracle, with and without
    a fused bitset (HANNS_GPU_SCAN=tc and =simt)."""
    from hanns_b200.ivf_usq import FILTER_FUSED, FILTER_NONE, IvfUsqIndex, SearchRequest
    from tests.golden.make_golden import mixture
    O = oracle_mod
    rng = np.random.default_rng(300 + nbits + nlist)
    d = 192
    x, _ = mixture(rng, 20000, d, 16, 0.4, metric == 1)
    q, _ = mixture(rng, 200, d, 16, 0.4, metric == 1)
    art = O.build_artifact(x, nlist, nbits, metric, rotation_seed=5, kmeans_iters=4, kmeans_seed=1)
    sizes = np.diff(art["list_offsets"])
    n_cand = O.n_candidates(nbits, k)
    assert (sizes > n_cand).any()
    oi = O.OracleIndex(art)
    nprobe = min(4, nlist)
    kw = {}
    okw = {}
    mode = FILTER_NONE
    if fused:
        blen = 20000
        bits = (rng.random(blen) < 0.3)
        words = np.zeros((1, (blen + 63) // 64), np.uint64)
        for i in np.nonzero(bits)[0]:
            words[0, i >> 6] |= np.uint64(1) << np.uint64(i & 63)
        mode = FILTER_FUSED
        kw = dict(bitsets=words, bitset_len=blen, query_bitset=np.zeros(q.shape[0], np.int32))
        okw = dict(filter_mode=O.FILTER_FUSED, bitsets=words, bitset_len=blen,
                   query_bitset=np.zeros(q.shape[0], np.int32))
    e_ids, e_d, _ = oi.search(q, k, nprobe, **okw)
    idx = IvfUsqIndex.from_artifact(art)
    req = SearchRequest(top_k=k, nprobe=nprobe)
    old = os.environ.pop("HANNS_GPU_SCAN", None)
    try:
        res = {}
        for m in ("tc", "simt"):
            os.environ["HANNS_GPU_SCAN"] = m
            if fused:
                r = idx.search(q, req, mode, kw["bitsets"], kw["bitset_len"], kw["query_bitset"])
            else:
                r = idx.search(q, req)
            res[m] = r
            assert np.array_equal(r.ids.reshape(e_ids.shape), e_ids), m
            assert bits_eq(r.distances.reshape(e_ids.shape), e_d), m
    finally:
        os.environ.pop("HANNS_GPU_SCAN", None)
        if old is not None:
            os.environ["HANNS_GPU_SCAN"] = old


def test_host_search_chunked_upload(gpu, oracle_mod):
    """Host-pointer search of 9000 queries: the upload runs in chunks on the copy stream,
    each chunk's per-query stages waiting only for its own copy.  Equal to the oracle and
    to the device-pointer path."""
    import torch
    from hanns_b200.ivf_usq import IvfUsqIndex, SearchRequest
    from tests.golden.make_golden import mixture
    O = oracle_mod
    rng = np.random.default_rng(77)
    d, k, nprobe = 96, 10, 5
    x, _ = mixture(rng, 20000, d, 32, 0.4, False)
    q, _ = mixture(rng, 9000, d, 32, 0.4, False)
    art = O.build_artifact(x, 40, 4, O.METRIC_L2, rotation_seed=4, kmeans_iters=5, kmeans_seed=2)
    e_ids, e_d, _ = O.OracleIndex(art).search(q, k, nprobe)
    idx = IvfUsqIndex.from_artifact(art)
    r = idx.search(q, SearchRequest(top_k=k, nprobe=nprobe))
    assert np.array_equal(r.ids.reshape(e_ids.shape), e_ids)
    assert bits_eq(r.distances.reshape(e_ids.shape), e_d)
    dq = torch.from_numpy(q).cuda()
    ids = torch.empty(q.shape[0], k, dtype=torch.int64, device="cuda")
    dist = torch.empty(q.shape[0], k, dtype=torch.float32, device="cuda")
    idx.search_device(dq.data_ptr(), q.shape[0], k, nprobe, ids.data_ptr(), dist.data_ptr())
    assert np.array_equal(ids.cpu().numpy(), e_ids)
    assert bits_eq(dist.cpu().numpy(), e_d)


def test_stream_ordered_device_search(gpu, oracle_mod):
    """On a created stream the device search returns once enqueued: five back-to-back
    searches of different batches into different outputs, read after one synchronize,
    equal the oracle; the stage-event ring times each of them."""
    import torch
    from hanns_b200.ivf_usq import IvfUsqIndex
    from tests.golden.make_golden import mixture
    O = oracle_mod
    rng = np.random.default_rng(78)
    d, k, nprobe, nq, nb = 96, 10, 5, 700, 5
    x, _ = mixture(rng, 20000, d, 32, 0.4, False)
    q, _ = mixture(rng, nq * nb, d, 32, 0.4, False)
    art = O.build_artifact(x, 40, 4, O.METRIC_IP, rotation_seed=6, kmeans_iters=5, kmeans_seed=3)
    e_ids, e_d, _ = O.OracleIndex(art).search(q, k, nprobe)
    idx = IvfUsqIndex.from_artifact(art)
    dq = torch.from_numpy(q).cuda()
    ids = torch.full((nq * nb, k), -9, dtype=torch.int64, device="cuda")
    dist = torch.empty(nq * nb, k, dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    st = torch.cuda.Stream()
    for b in range(nb):
        idx.search_device(dq.data_ptr() + b * nq * d * 4, nq, k, nprobe,
                          ids.data_ptr() + b * nq * k * 8, dist.data_ptr() + b * nq * k * 4,
                          stream=st.cuda_stream)
    st.synchronize()
    assert np.array_equal(ids.cpu().numpy(), e_ids)
    assert bits_eq(dist.cpu().numpy(), e_d)
    tot, cnt, covered = idx.stage_ms_recent(nb)
    assert covered == nb and cnt[5] == nb and cnt[7] == nb
    assert tot[5] > 0 and tot[7] >= tot[5]


@pytest.mark.parametrize("path", FIXTURES[:3], ids=IDS[:3])
def test_rerank_rows_equals_candidate_distances(gpu, oracle_mod, path):
    """hanns_gpu_ivf_usq_rerank_rows_device on the rows the oracle reranks for each query
    gives the oracle's candidate distances bit for bit; rows outside the index give +inf."""
    from hanns_b200.ivf_usq import IvfUsqIndex
    O = oracle_mod
    art, z = load(path)
    oi = O.OracleIndex(art)
    idx = IvfUsqIndex.from_artifact(art)
    off = np.asarray(art["list_offsets"], np.int64)
    qs = z["queries"][:12]
    rows, exp = [], []
    for qv in qs:
        c = oi.candidates(qv, int(z["k"]), int(z["nprobe"]))
        r = off[np.asarray(c["list"], np.int64)] + np.asarray(c["local"], np.int64)
        rows.append(r[:40])
        exp.append(np.asarray(c["dist"], np.float32)[:40])
    m = max(len(r) for r in rows) + 2
    R = np.full((len(qs), m), -1, np.int64)
    E = np.full((len(qs), m), np.inf, np.float32)
    for i, (r, e) in enumerate(zip(rows, exp)):
        R[i, :len(r)] = r
        E[i, :len(e)] = e
    R[:, -1] = len(art["ids"]) + 5  # beyond the index
    got = idx.rerank_rows(qs, R)
    assert bits_eq(got, E)


def test_empty_and_tiny_index(gpu, oracle_mod):
    """Lists of 0, 1, 31, 32, 33 rows; k larger than everything probed."""
    from hanns_b200.ivf_usq import IvfUsqIndex, SearchRequest
    O = oracle_mod
    rng = np.random.default_rng(1)
    sizes = [0, 1, 31, 32, 33, 0, 2]
    d = 40
    cent = rng.normal(size=(len(sizes), d)).astype(np.float32) * 5
    x = np.concatenate([cent[i] + 0.1 * rng.normal(size=(s, d)) for i, s in enumerate(sizes) if s]).astype(np.float32)
    art = O.build_artifact(x, len(sizes), 4, O.METRIC_L2, centroids=cent)
    assert np.diff(art["list_offsets"]).tolist() == sizes
    q = np.concatenate([cent + 0.05, x[:3]]).astype(np.float32)
    oi = O.OracleIndex(art)
    idx = IvfUsqIndex.from_artifact(art)
    for k, npr in [(5, 1), (200, 7), (40, 3)]:
        e_ids, e_d, _ = oi.search(q, k, npr)
        r = idx.search(q, SearchRequest(top_k=k, nprobe=npr))
        assert np.array_equal(r.ids.reshape(e_ids.shape), e_ids)
        assert bits_eq(r.distances.reshape(e_ids.shape), e_d)


def _empty_artifact(cent, D, nbits=4, metric=0):
    nlist, d = cent.shape
    rng = np.random.default_rng(0)
    P = np.linalg.qr(rng.normal(size=(D, D)))[0].astype(np.float32)
    cb = (D * nbits + 7) // 8
    return dict(dim=d, padded_dim=D, nbits=nbits, nlist=nlist, metric=metric, centroids=cent,
                rotation=P, rotated_centroid=np.zeros(D, np.float32),
                list_offsets=np.zeros(nlist + 1, np.int64), ids=np.zeros(0, np.int64),
                norms=np.zeros(0, np.float32), norms_sq=np.zeros(0, np.float32),
                vmaxs=np.zeros(0, np.float32), quant_qualities=np.zeros(0, np.float32),
                codes=np.zeros((0, cb), np.uint8), sign_bits=np.zeros((0, D // 8), np.uint8))


@pytest.mark.parametrize("nlist,d,nprobe,normalise", [
    (4096, 768, 32, True),     # block-per-query select (row in shared memory)
    (40000, 64, 16, False),    # block-per-query select (row left in global memory)
    (65536, 768, 64, True),    # the 20 M-row configuration's coarse shape (row in global memory)
    (2048, 96, 300, True),     # nprobe > 256: exact kernels
])
def test_coarse_fast_path_equals_exact(gpu, oracle_mod, nlist, d, nprobe, normalise):
    """Approximate-GEMM + exact re-score coarse step == exact sequential L2 selection:
    checked against the exact kernels (static entry point) and the oracle, with 600
    duplicate centroids (exact ties, candidate sets beyond the cap -> fallback)."""
    import torch
    from hanns_b200 import _lib
    from hanns_b200.ivf_usq import IvfUsqIndex
    O = oracle_mod
    rng = np.random.default_rng(5)
    cent = rng.normal(size=(nlist, d)).astype(np.float32)
    if normalise:
        cent /= np.linalg.norm(cent, axis=1, keepdims=True)
    cent[100:700] = cent[99]
    nq = 1000
    q = rng.normal(size=(nq, d)).astype(np.float32)
    if normalise:
        q /= np.linalg.norm(q, axis=1, keepdims=True)
    q[:50] = cent[99] + 0.01 * rng.normal(size=(50, d)).astype(np.float32)
    q[50:60] = cent[5]  # exact hits
    art = _empty_artifact(cent, (d + 63) // 64 * 64)
    idx = IvfUsqIndex.from_artifact(art)
    fast = idx.debug_query(q, nprobe)["probes"]
    qt = torch.from_numpy(q).cuda()
    ct = torch.from_numpy(cent).cuda()
    exact = torch.empty(nq, nprobe, dtype=torch.int32, device="cuda")
    step = max(1, ((16 << 20) - nq * nprobe * 8) // (4 * nlist) - 1)
    for s in range(0, nq, step):
        m = min(step, nq - s)
        rc = gpu.hanns_gpu_coarse_probes_static(qt[s:].data_ptr(), m, ct.data_ptr(), nlist, d, nprobe,
                                                exact[s:].data_ptr(), None)
        assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert np.array_equal(fast, exact.cpu().numpy())
    oi = O.OracleIndex(art)
    _, _, _, op = oi.search(q[:60], 5, nprobe, want_probes=True)
    assert np.array_equal(fast[:60], op)


@pytest.mark.parametrize("d", [768, 128])
def test_coarse_near_ties_order(gpu, oracle_mod, d):
    """Candidates a rounding apart: pairs and triples of equal centroids and centroids one
    ulp apart in one coordinate, with queries next to them, so that the approximate-score
    intervals of several top-nprobe candidates overlap and their order comes from the
    exact sums (ties by centroid id).  Probes equal the exact kernels and the oracle."""
    import torch
    from hanns_b200 import _lib
    from hanns_b200.ivf_usq import IvfUsqIndex
    O = oracle_mod
    rng = np.random.default_rng(15)
    nlist, nprobe, nq = 4096, 32, 800
    cent = rng.normal(size=(nlist, d)).astype(np.float32)
    cent /= np.linalg.norm(cent, axis=1, keepdims=True)
    for i in range(0, 400, 8):
        cent[i + 1] = cent[i]                                   # exact tie
        cent[i + 2] = cent[i]
        cent[i + 2, i % d] = np.nextafter(cent[i, i % d], np.float32(2))   # one ulp
        cent[i + 3] = cent[i]
        cent[i + 3, (i + 1) % d] = np.nextafter(cent[i, (i + 1) % d], np.float32(-2))
    q = rng.normal(size=(nq, d)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    base = rng.integers(0, 50, nq) * 8
    q[:600] = cent[base[:600]] + 0.05 * rng.normal(size=(600, d)).astype(np.float32)
    art = _empty_artifact(cent, (d + 63) // 64 * 64)
    idx = IvfUsqIndex.from_artifact(art)
    fast = idx.debug_query(q, nprobe)["probes"]
    qt = torch.from_numpy(q).cuda()
    ct = torch.from_numpy(cent).cuda()
    exact = torch.empty(nq, nprobe, dtype=torch.int32, device="cuda")
    step = max(1, ((16 << 20) - nq * nprobe * 8) // (4 * nlist) - 1)
    for s in range(0, nq, step):
        m = min(step, nq - s)
        rc = gpu.hanns_gpu_coarse_probes_static(qt[s:].data_ptr(), m, ct.data_ptr(), nlist, d, nprobe,
                                                exact[s:].data_ptr(), None)
        assert rc == 0, _lib.last_error()
    torch.cuda.synchronize()
    assert np.array_equal(fast, exact.cpu().numpy())
    oi = O.OracleIndex(art)
    _, _, _, op = oi.search(q[:40], 5, nprobe, want_probes=True)
    assert np.array_equal(fast[:40], op)


def test_query_split_shards_equal_single_gpu(gpu, oracle_mod):
    """Query-split multi-GPU protocol on one device: two list shards of one index, each
    prepares the state of half of the queries, the halves are concatenated (the NCCL
    all-gather), each shard scans its lists for all queries, and merge_shards gives the
    single-index rows bit for bit."""
    import torch
    from hanns_b200 import _lib
    from hanns_b200.ivf_usq import IvfUsqIndex, SearchRequest
    from tests.golden.make_golden import mixture
    O = oracle_mod
    rng = np.random.default_rng(21)
    d, k, nprobe, nq, world = 128, 10, 6, 600, 2
    x, _ = mixture(rng, 20000, d, 32, 0.4, False)
    q, _ = mixture(rng, nq, d, 32, 0.4, False)
    art = O.build_artifact(x, 24, 4, O.METRIC_L2, rotation_seed=3, kmeans_iters=5, kmeans_seed=2)
    full = IvfUsqIndex.from_artifact(art)
    exp = full.search(q, SearchRequest(top_k=k, nprobe=nprobe))
    shards = []
    for r in range(world):
        s = IvfUsqIndex.from_artifact(art)
        s.shard(r, world)
        shards.append(s)
    L = gpu
    parts = np.zeros(5, np.int64)
    assert L.hanns_gpu_ivf_usq_query_state_bytes(shards[0]._h, nprobe, parts.ctypes.data_as(_lib.i64p)) == 0
    bufs = [torch.zeros(nq * int(b), dtype=torch.uint8, device="cuda") for b in parts]
    dq = torch.from_numpy(q).cuda()
    per = nq // world
    for r, s in enumerate(shards):
        ptrs = [b.data_ptr() + r * per * int(p) for b, p in zip(bufs, parts)]
        assert L.hanns_gpu_ivf_usq_prepare_device(s._h, dq.data_ptr() + r * per * d * 4, per, nprobe,
                                                  *ptrs, None) == 0, _lib.last_error()
    g_d = torch.empty(world, nq, k, dtype=torch.float32, device="cuda")
    g_k = torch.empty(world, nq, k, dtype=torch.int64, device="cuda")
    g_i = torch.empty(world, nq, k, dtype=torch.int64, device="cuda")
    for r, s in enumerate(shards):
        assert L.hanns_gpu_ivf_usq_search_prepared_shard_device(
            s._h, nq, k, nprobe, *[b.data_ptr() for b in bufs], g_d[r].data_ptr(), g_k[r].data_ptr(),
            g_i[r].data_ptr(), None) == 0, _lib.last_error()
    out_i = torch.empty(nq, k, dtype=torch.int64, device="cuda")
    out_d = torch.empty(nq, k, dtype=torch.float32, device="cuda")
    assert L.hanns_gpu_merge_shards_device(g_d.data_ptr(), g_k.data_ptr(), g_i.data_ptr(), world, nq, k,
                                           out_i.data_ptr(), out_d.data_ptr(), None) == 0
    assert np.array_equal(out_i.cpu().numpy(), exp.ids.reshape(nq, k))
    assert bits_eq(out_d.cpu().numpy(), exp.distances.reshape(nq, k))


def _gpu_built(d, nlist, nbits, metric, n, comps, sigma, seed):
    from hanns_b200.ivf_usq import IvfUsqConfig, IvfUsqIndex
    from tests.golden.make_golden import mixture
    rng = np.random.default_rng(seed)
    x, _ = mixture(rng, n, d, comps, sigma, metric == 1)
    idx = IvfUsqIndex(IvfUsqConfig(d, nlist, nbits, metric_type=metric, rotation_seed=seed))
    idx.train(x, kmeans_iters=6, kmeans_seed=seed)
    idx.add(x)
    return idx, rng


def test_config_8bit_k100_deletion_bitsets(gpu, oracle_mod):
    """The shape of the 8-bit configuration: 8-bit codes, inner product, d = 768, k = 100,
    10 % of the queries with a deletion bitset masking ids with probability 0.2; fused
    and reference post filtering equal the oracle on the GPU-built index."""
    from hanns_b200.ivf_usq import FILTER_FUSED, FILTER_POST, SearchRequest
    from tests.golden.make_golden import mixture
    O = oracle_mod
    idx, rng = _gpu_built(768, 32, 8, 1, 12000, 64, 0.5, 11)
    art = idx.export_artifact()
    q, _ = mixture(rng, 200, 768, 64, 0.5, True)
    k, nprobe, n = 100, 8, 12000
    n_bs = 20
    bitsets = np.zeros((n_bs, (n + 63) // 64), np.uint64)  # bit id & 63 of word id >> 6
    for b in range(n_bs):
        dead = np.nonzero(rng.random(n) < 0.2)[0].astype(np.uint64)
        np.bitwise_or.at(bitsets[b], (dead >> np.uint64(6)).astype(np.int64),
                         np.uint64(1) << (dead & np.uint64(63)))
    qb = np.full(q.shape[0], -1, np.int32)
    qb[rng.choice(q.shape[0], q.shape[0] // 10, replace=False)] = np.arange(q.shape[0] // 10) % n_bs
    oi = O.OracleIndex(art)
    req = SearchRequest(top_k=k, nprobe=nprobe)
    for mode, fm in ((FILTER_FUSED, O.FILTER_FUSED), (FILTER_POST, O.FILTER_POST)):
        e_ids, e_d, e_c = oi.search(q, k, nprobe, filter_mode=fm, bitsets=bitsets, bitset_len=n,
                                    query_bitset=qb)
        r = idx.search(q, req, mode, bitsets, n, qb)
        if mode == FILTER_FUSED:
            assert np.array_equal(r.ids.reshape(e_ids.shape), e_ids)
            assert bits_eq(r.distances.reshape(e_ids.shape), e_d)
        else:
            assert np.array_equal(r.counts, e_c)
            got = r.ids.reshape(e_ids.shape)
            assert all(np.array_equal(got[i, :c], e_ids[i, :c]) for i, c in enumerate(e_c))


def test_config_3072_dims_8bit(gpu, oracle_mod):
    """The shape of the 3,072-dimension configuration (8-bit codes, inner product, k = 10)
    on a GPU-built index: 12 lists of ~500 rows, so that lists exceed the 8-bit n_cand of
    300 and FastScan runs (nprobe 8); D > 1024 takes the 8 x 8 rotation tiles."""
    from hanns_b200.ivf_usq import SearchRequest
    from tests.golden.make_golden import mixture
    O = oracle_mod
    idx, rng = _gpu_built(3072, 12, 8, 1, 6000, 16, 0.4, 3)
    art = idx.export_artifact()
    assert (np.diff(art["list_offsets"]) > O.n_candidates(8, 10)).sum() >= 4
    q, _ = mixture(rng, 64, 3072, 16, 0.4, True)
    e_ids, e_d, _ = O.OracleIndex(art).search(q, 10, 8)
    r = idx.search(q, SearchRequest(top_k=10, nprobe=8))
    assert np.array_equal(r.ids.reshape(e_ids.shape), e_ids)
    assert bits_eq(r.distances.reshape(e_ids.shape), e_d)


@pytest.mark.parametrize("nbits,metric", [(1, 0), (2, 1), (3, 0), (6, 1), (7, 0)])
def test_search_bit_exact_other_widths(gpu, oracle_mod, nbits, metric):
    """Code widths other than 4 and 8 (single-GPU search): FastScan and the kept sets as for
    every width, then the reference's f32 reranks on the SIMT scan -- the 1-bit sixteen
    chains and tree, the scalar dequantised sum in dimension order for the others.  Ids,
    distance bits and every kept candidate equal the oracle's."""
    from hanns_b200.ivf_usq import IvfUsqIndex, SearchRequest
    from tests.golden.make_golden import mixture
    O = oracle_mod
    rng = np.random.default_rng(600 + nbits)
    x, _ = mixture(rng, 3000, 96, 8, 0.4, metric == 1)
    q, _ = mixture(rng, 40, 96, 8, 0.4, metric == 1)
    art = O.build_artifact(x, 6, nbits, metric, rotation_seed=4, kmeans_iters=4, kmeans_seed=1)
    assert (np.diff(art["list_offsets"]) > O.n_candidates(nbits, 10)).any()  # FastScan runs
    idx = IvfUsqIndex.from_artifact(art)
    oi = O.OracleIndex(art)
    e_ids, e_d, _ = oi.search(q, 10, 3)
    r = idx.search(q, SearchRequest(top_k=10, nprobe=3))
    assert np.array_equal(r.ids.reshape(e_ids.shape), e_ids)
    assert bits_eq(r.distances.reshape(e_ids.shape), e_d)
    got = idx.debug_candidates(q[:8], 10, 3)
    for i in range(8):
        exp = oi.candidates(q[i], 10, 3)
        for key in ("list", "local", "fs", "int_ip"):
            assert np.array_equal(got[i][key], exp[key]), (i, key)
        assert np.array_equal(got[i]["dist"].view(np.uint32), exp["dist"].view(np.uint32)), i
