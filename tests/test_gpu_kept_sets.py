"""Kept sets of the list scan against the oracle, candidate by candidate.

The reference's search_single (src/faiss/ivf_usq.rs:547-588) builds one candidate vector
per query: per probed list, every row when |list| <= n_cand, else the FastScan heap's kept
set in (score descending, position) order (src/quantization/usq/fastscan.rs:86-146); each
candidate then gets its VNNI int_ip (quantizer.rs:382-400) and distance.  The GPU's
debug entry returns exactly those tuples from the scan's candidate regions, so a wrong
kept set (an off-by-one at the heap boundary, a missed tie) fails here even where the
final top-k would hide it.  Both scans are covered: the tensor-core scan (default) and
the SIMT scan (HANNS_GPU_SCAN=simt).  The i16 case builds 3,072-dimension 4-bit lists
whose FastScan sums leave the i16 range, so the reference's wraparound decides the kept
sets.
"""
import glob
import os

import numpy as np
import pytest

from tests.golden.make_golden import load, mixture

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


def assert_same_candidates(got, exp, what):
    assert got["list"].shape == exp["list"].shape, f"{what}: {got['list'].size} vs {exp['list'].size} candidates"
    assert np.array_equal(got["list"], exp["list"]), what
    assert np.array_equal(got["local"], exp["local"]), what
    assert np.array_equal(got["fs"], exp["fs"]), what
    assert np.array_equal(got["int_ip"], exp["int_ip"]), what
    assert np.array_equal(got["dist"].view(np.uint32), exp["dist"].view(np.uint32)), what


def check_queries(idx, oi, q, k, nprobe, **filt):
    got = idx.debug_candidates(q, k, nprobe, **filt)
    ofilt = {}
    if filt:
        ofilt = dict(filter_mode=filt["filter_mode"], bitset=filt["bitsets"][0],
                     bitset_len=filt["bitset_len"])
    for i in range(q.shape[0]):
        exp = oi.candidates(q[i], k, nprobe, **ofilt)
        assert_same_candidates(got[i], exp, f"query {i}")
    return got


@pytest.fixture(params=["tc", "simt"])
def scan_mode(request):
    old = os.environ.pop("HANNS_GPU_SCAN", None)
    if request.param == "simt":
        os.environ["HANNS_GPU_SCAN"] = "simt"
    yield request.param
    os.environ.pop("HANNS_GPU_SCAN", None)
    if old is not None:
        os.environ["HANNS_GPU_SCAN"] = old


@pytest.mark.parametrize("path", FIXTURES, ids=IDS)
def test_kept_sets_golden(gpu, oracle_mod, scan_mode, path):
    from hanns_b200.ivf_usq import IvfUsqIndex
    art, z = load(path)
    idx = IvfUsqIndex.from_artifact(art)
    check_queries(idx, oracle_mod.OracleIndex(art), z["queries"], int(z["k"]), int(z["nprobe"]))


@pytest.mark.parametrize("nlist,fused", [(12, False), (12, True), (40, True), (6, False)])
def test_kept_sets_item_splits_and_bitsets(gpu, oracle_mod, scan_mode, nlist, fused):
    """20,000 rows, d = 192, 4-bit L2: nlist 12 gives ~1,700-row lists (14 row tiles, items
    of 16 queries, several items per list), 40 ~500 rows, 6 ~3,300 rows (SIMT lists);
    a fused bitset masks 30 % of the ids."""
    from hanns_b200.ivf_usq import FILTER_FUSED, IvfUsqIndex
    O = oracle_mod
    rng = np.random.default_rng(500 + nlist)
    x, _ = mixture(rng, 20000, 192, 16, 0.4, False)
    q, _ = mixture(rng, 96, 192, 16, 0.4, False)
    art = O.build_artifact(x, nlist, 4, O.METRIC_L2, rotation_seed=5, kmeans_iters=4, kmeans_seed=1)
    assert (np.diff(art["list_offsets"]) > O.n_candidates(4, 10)).any()
    idx = IvfUsqIndex.from_artifact(art)
    filt = {}
    if fused:
        blen = 20000
        dead = np.nonzero(rng.random(blen) < 0.3)[0].astype(np.uint64)
        words = np.zeros((1, (blen + 63) // 64), np.uint64)
        np.bitwise_or.at(words[0], (dead >> np.uint64(6)).astype(np.int64),
                         np.uint64(1) << (dead & np.uint64(63)))
        filt = dict(filter_mode=FILTER_FUSED, bitsets=words, bitset_len=blen,
                    query_bitset=np.zeros(q.shape[0], np.int32))
    check_queries(idx, O.OracleIndex(art), q, 10, 4, **filt)


def test_fastscan_i16_wraparound(gpu, oracle_mod, scan_mode):
    """d = 3,072 (768 FastScan groups), 4-bit, lists of ~500 rows (FastScan runs above 150):
    queries that are near-copies of stored rows score well above 32,767 on their own row
    (checked with the oracle's i32 scalar-path scores), so the reference's i16 accumulation
    wraps and can drop the best row from the kept set.  The GPU's kept sets, raw scores and
    search results equal the oracle's AVX-512 (wrapping) path."""
    from hanns_b200.ivf_usq import IvfUsqConfig, IvfUsqIndex, SearchRequest
    O = oracle_mod
    rng = np.random.default_rng(3072)
    d, n, nlist = 3072, 4000, 8
    x, _ = mixture(rng, n, d, 8, 0.4, True)
    # GPU build path (bit-exact with the oracle's encoder; much faster at this dimension)
    idx = IvfUsqIndex(IvfUsqConfig(d, nlist, 4, metric_type=O.METRIC_IP, rotation_seed=3))
    idx.train(x, kmeans_iters=4, kmeans_seed=2)
    idx.add(x)
    art = idx.export_artifact()
    src = rng.choice(n, 24, replace=False)
    q = x[src] + 0.01 * rng.normal(size=(24, d)).astype(np.float32)
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    q = q.astype(np.float32)
    D = int(art["padded_dim"])
    off = np.asarray(art["list_offsets"])
    oi = O.OracleIndex(art)
    # the wrap occurs: the unwrapped (scalar-path, i32) score of some probed row leaves i16
    wrapped = 0
    for i in range(q.shape[0]):
        st = O.query_state(art, q[i])
        for l in oi.search(q[i:i + 1], 10, 3, want_probes=True)[3][0]:
            rows = slice(off[l], off[l + 1])
            nl = off[l + 1] - off[l]
            if nl == 0:
                continue
            blocks = O.fastscan_blocks(art["sign_bits"][rows], D)
            s32 = O.fastscan_scores(blocks, nl, D, st["lut"], mode=O.MODE_SCALAR)
            s16 = O.fastscan_scores(blocks, nl, D, st["lut"], mode=O.MODE_AVX512)
            assert np.array_equal(s16, s32.astype(np.int16).astype(np.int32))
            wrapped += int((np.abs(s32) > 32767).sum())
    assert wrapped > 0
    got = check_queries(idx, oi, q, 10, 3)
    assert any((g["fs"] != np.iinfo(np.int32).min).any() for g in got)
    e_ids, e_d, _ = oi.search(q, 10, 3)
    r = idx.search(q, SearchRequest(top_k=10, nprobe=3))
    assert np.array_equal(r.ids.reshape(e_ids.shape), e_ids)
    assert np.array_equal(r.distances.reshape(e_ids.shape).view(np.uint32), e_d.view(np.uint32))
