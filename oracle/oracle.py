"""ctypes wrapper around the CPU oracle (oracle/build/libusq_oracle.so).

TEST INFRASTRUCTURE ONLY.  Imported by tests/, __graft_entry__.smoke() and the
CPU-baseline leg of bench.py as the checker; the product (hanns_b200) never uses it.

An *artifact* is a dict of numpy arrays describing a frozen IVF-USQ index in list
order (the same fields as ``hanns_ivf_usq_artifact_t`` in include/hanns_gpu.h):
  dim, padded_dim, nbits, nlist, metric (ints); centroids [nlist,d] f32;
  rotation [D,D] f32; rotated_centroid [D] f32; list_offsets [nlist+1] i64;
  ids [n] i64; norms, norms_sq, vmaxs, quant_qualities [n] f32;
  codes [n, code_bytes] u8; sign_bits [n, D/8] u8.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "build", "libusq_oracle.so")

MODE_AVX512, MODE_SCALAR = 0, 1
FILTER_NONE, FILTER_POST, FILTER_FUSED = 0, 1, 2
METRIC_L2, METRIC_IP = 0, 1

_f32p = C.POINTER(C.c_float)
_i64p = C.POINTER(C.c_int64)
_i32p = C.POINTER(C.c_int32)
_u8p = C.POINTER(C.c_uint8)
_i8p = C.POINTER(C.c_int8)
_u16p = C.POINTER(C.c_uint16)
_u64p = C.POINTER(C.c_uint64)


class Artifact(C.Structure):
    _fields_ = [
        ("dim", C.c_int32), ("padded_dim", C.c_int32), ("nbits", C.c_int32),
        ("nlist", C.c_int32), ("metric", C.c_int32), ("reserved", C.c_int32),
        ("ntotal", C.c_int64),
        ("centroids", _f32p), ("rotation", _f32p), ("rotated_centroid", _f32p),
        ("list_offsets", _i64p), ("ids", _i64p),
        ("norms", _f32p), ("norms_sq", _f32p), ("vmaxs", _f32p), ("quant_qualities", _f32p),
        ("codes", _u8p), ("sign_bits", _u8p),
    ]


def build_lib() -> None:
    subprocess.run(["make", "-s", "-C", HERE], check=True)


_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build_lib()
        L = C.CDLL(LIB_PATH)
        L.ousq_padded_dim.restype = C.c_int32
        L.ousq_code_bytes.restype = C.c_int32
        L.ousq_sign_bytes.restype = C.c_int32
        L.ousq_n_candidates.restype = C.c_int32
        L.ousq_fastscan_topk.restype = C.c_int64
        L.ousq_int_ip.restype = C.c_int32
        L.ousq_score.restype = C.c_float
        L.ousq_index_create.restype = C.c_void_p
        L.ousq_index_create.argtypes = [C.POINTER(Artifact)]
        L.ousq_index_free.argtypes = [C.c_void_p]
        L.ousq_search.restype = C.c_int32
        L.ousq_candidates.restype = C.c_int64
        L.ousq_rotation_matrix.argtypes = [C.c_uint64, C.c_int32, _f32p]
        L.ousq_kmeans.argtypes = [_f32p, C.c_int64, C.c_int32, C.c_int32, C.c_int32,
                                  C.c_uint64, _f32p, C.c_int32]
        _lib = L
    return _lib


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


def padded_dim(d: int) -> int:
    return (d + 63) // 64 * 64


def code_bytes(d: int, nbits: int) -> int:
    return (padded_dim(d) * nbits + 7) // 8


def n_candidates(nbits: int, k: int) -> int:
    return int(lib().ousq_n_candidates(nbits, k))


# ---------------------------------------------------------------- build helpers
def rotation_matrix(seed: int, D: int) -> np.ndarray:
    P = np.empty((D, D), np.float32)
    lib().ousq_rotation_matrix(C.c_uint64(seed), D, _p(P, _f32p))
    return P


def rotate(P: np.ndarray, x: np.ndarray, mode: int = MODE_AVX512) -> np.ndarray:
    P = np.ascontiguousarray(P, np.float32)
    D = P.shape[0]
    xp = np.zeros(D, np.float32)
    xp[: x.shape[0]] = x
    out = np.empty(D, np.float32)
    lib().ousq_rotate(_p(P, _f32p), D, _p(xp, _f32p), _p(out, _f32p), mode)
    return out


def global_mean(data: np.ndarray) -> np.ndarray:
    data = np.ascontiguousarray(data, np.float32)
    out = np.empty(data.shape[1], np.float32)
    lib().ousq_global_mean(_p(data, _f32p), C.c_int64(data.shape[0]), data.shape[1], _p(out, _f32p))
    return out


def kmeans(data: np.ndarray, k: int, iters: int, seed: int, nthreads: int = 0) -> np.ndarray:
    data = np.ascontiguousarray(data, np.float32)
    cent = np.empty((k, data.shape[1]), np.float32)
    lib().ousq_kmeans(_p(data, _f32p), data.shape[0], data.shape[1], k, iters, seed,
                      _p(cent, _f32p), nthreads)
    return cent


def assign(data: np.ndarray, centroids: np.ndarray, nthreads: int = 0) -> np.ndarray:
    data = np.ascontiguousarray(data, np.float32)
    centroids = np.ascontiguousarray(centroids, np.float32)
    out = np.empty(data.shape[0], np.int32)
    lib().ousq_assign(_p(data, _f32p), C.c_int64(data.shape[0]), data.shape[1],
                      _p(centroids, _f32p), centroids.shape[0], _p(out, _i32p), nthreads)
    return out


def encode_batch(P, dim, nbits, centroid, x, mode=MODE_AVX512, nthreads=0):
    x = np.ascontiguousarray(x, np.float32)
    n = x.shape[0]
    D = padded_dim(dim)
    codes = np.zeros((n, code_bytes(dim, nbits)), np.uint8)
    signs = np.zeros((n, D // 8), np.uint8)
    meta = np.zeros((n, 4), np.float32)
    P = np.ascontiguousarray(P, np.float32)
    centroid = np.ascontiguousarray(centroid, np.float32)
    lib().ousq_encode_batch(_p(P, _f32p), dim, nbits, _p(centroid, _f32p), _p(x, _f32p),
                            C.c_int64(n), mode, _p(codes, _u8p), _p(signs, _u8p),
                            _p(meta, _f32p), nthreads)
    return codes, signs, meta


def pack_codes(codes: np.ndarray, nbits: int) -> np.ndarray:
    codes = np.ascontiguousarray(codes, np.uint16)
    out = np.zeros((codes.size * nbits + 7) // 8, np.uint8)
    lib().ousq_pack_codes(_p(codes, _u16p), C.c_int64(codes.size), nbits, _p(out, _u8p))
    return out


def unpack_codes(b: np.ndarray, n: int, nbits: int) -> np.ndarray:
    b = np.ascontiguousarray(b, np.uint8)
    out = np.zeros(n, np.uint16)
    lib().ousq_unpack_codes(_p(b, _u8p), C.c_int64(n), nbits, _p(out, _u16p))
    return out


def build_artifact(data: np.ndarray, nlist: int, nbits: int, metric: int = METRIC_L2,
                   rotation_seed: int = 42, kmeans_iters: int = 10, kmeans_seed: int = 1,
                   ids: np.ndarray | None = None, train: np.ndarray | None = None,
                   centroids: np.ndarray | None = None, rotation: np.ndarray | None = None,
                   nthreads: int = 0) -> dict:
    """Oracle-side IVF-USQ build (train + add) following ivf_usq.rs:228-320 with a
    seeded k-means in place of the reference's entropy-seeded one."""
    data = np.ascontiguousarray(data, np.float32)
    n, d = data.shape
    D = padded_dim(d)
    train = data if train is None else np.ascontiguousarray(train, np.float32)
    if centroids is None:
        centroids = kmeans(train, nlist, kmeans_iters, kmeans_seed, nthreads)
    centroids = np.ascontiguousarray(centroids, np.float32)
    P = rotation_matrix(rotation_seed, D) if rotation is None else np.ascontiguousarray(rotation, np.float32)
    gmean = global_mean(train)
    rc = rotate(P, gmean)
    lists = assign(data, centroids, nthreads)
    codes, signs, meta = encode_batch(P, d, nbits, gmean, data, MODE_AVX512, nthreads)
    if ids is None:
        ids = np.arange(n, dtype=np.int64)
    order = np.argsort(lists, kind="stable")
    counts = np.bincount(lists, minlength=nlist).astype(np.int64)
    offs = np.zeros(nlist + 1, np.int64)
    offs[1:] = np.cumsum(counts)
    return dict(
        dim=d, padded_dim=D, nbits=nbits, nlist=nlist, metric=metric,
        centroids=centroids, rotation=P, rotated_centroid=rc, global_centroid=gmean,
        list_offsets=offs, ids=np.ascontiguousarray(np.asarray(ids, np.int64)[order]),
        norms=np.ascontiguousarray(meta[order, 0]), norms_sq=np.ascontiguousarray(meta[order, 1]),
        vmaxs=np.ascontiguousarray(meta[order, 2]), quant_qualities=np.ascontiguousarray(meta[order, 3]),
        codes=np.ascontiguousarray(codes[order]), sign_bits=np.ascontiguousarray(signs[order]),
    )


def to_struct(art: dict) -> tuple[Artifact, list]:
    """Returns the ctypes struct and the list of arrays it points into (keep alive)."""
    keep = []

    def arr(name, dt):
        a = np.ascontiguousarray(art[name], dt)
        keep.append(a)
        return a

    s = Artifact()
    s.dim, s.padded_dim, s.nbits = int(art["dim"]), int(art["padded_dim"]), int(art["nbits"])
    s.nlist, s.metric, s.reserved = int(art["nlist"]), int(art["metric"]), 0
    s.ntotal = int(np.asarray(art["ids"]).shape[0])
    s.centroids = _p(arr("centroids", np.float32), _f32p)
    s.rotation = _p(arr("rotation", np.float32), _f32p)
    s.rotated_centroid = _p(arr("rotated_centroid", np.float32), _f32p)
    s.list_offsets = _p(arr("list_offsets", np.int64), _i64p)
    s.ids = _p(arr("ids", np.int64), _i64p)
    s.norms = _p(arr("norms", np.float32), _f32p)
    s.norms_sq = _p(arr("norms_sq", np.float32), _f32p)
    s.vmaxs = _p(arr("vmaxs", np.float32), _f32p)
    s.quant_qualities = _p(arr("quant_qualities", np.float32), _f32p)
    s.codes = _p(arr("codes", np.uint8), _u8p)
    s.sign_bits = _p(arr("sign_bits", np.uint8), _u8p)
    return s, keep


class OracleIndex:
    """IVF-USQ search on a frozen artifact, reference semantics."""

    def __init__(self, art: dict):
        self.art = art
        self._s, self._keep = to_struct(art)
        self._h = lib().ousq_index_create(C.byref(self._s))

    def close(self):
        if self._h:
            lib().ousq_index_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def search(self, queries, k, nprobe, mode=MODE_AVX512, filter_mode=FILTER_NONE,
               bitsets=None, bitset_len=0, query_bitset=None, nthreads=0, want_probes=False):
        q = np.ascontiguousarray(queries, np.float32).reshape(-1, int(self.art["dim"]))
        nq = q.shape[0]
        kk = max(int(k), 1)
        ids = np.empty((nq, kk), np.int64)
        dists = np.empty((nq, kk), np.float32)
        counts = np.empty(nq, np.int64)
        npr = min(max(int(nprobe), 1), int(self.art["nlist"]))
        probes = np.empty((nq, npr), np.int32) if want_probes else None
        bs_p, nbs = None, 0
        if bitsets is not None:
            bitsets = np.ascontiguousarray(bitsets, np.uint64)
            if bitsets.ndim == 1:
                bitsets = bitsets[None, :]
            nbs = bitsets.shape[0]
            bs_p = _p(bitsets, _u64p)
        qb_p = None
        if query_bitset is not None:
            query_bitset = np.ascontiguousarray(query_bitset, np.int32)
            qb_p = _p(query_bitset, _i32p)
        rc = lib().ousq_search(C.c_void_p(self._h), _p(q, _f32p), C.c_int64(nq), kk, npr, mode,
                               filter_mode, bs_p, C.c_int64(bitset_len), C.c_int64(nbs), qb_p,
                               nthreads, _p(ids, _i64p), _p(dists, _f32p), _p(counts, _i64p),
                               _p(probes, _i32p) if probes is not None else None)
        if rc != 0:
            raise RuntimeError("oracle search failed")
        if want_probes:
            return ids, dists, counts, probes
        return ids, dists, counts

    def candidates(self, query, k, nprobe, mode=MODE_AVX512, filter_mode=FILTER_NONE,
                   bitset=None, bitset_len=0, cap=1 << 20):
        q = np.ascontiguousarray(query, np.float32)
        lst = np.empty(cap, np.int32)
        loc = np.empty(cap, np.int64)
        fs = np.empty(cap, np.int32)
        iip = np.empty(cap, np.int32)
        dist = np.empty(cap, np.float32)
        bp = None
        if bitset is not None:
            bitset = np.ascontiguousarray(bitset, np.uint64)
            bp = _p(bitset, _u64p)
        n = lib().ousq_candidates(C.c_void_p(self._h), _p(q, _f32p), int(k), int(nprobe), mode,
                                  filter_mode, bp, C.c_int64(bitset_len), C.c_int64(cap),
                                  _p(lst, _i32p), _p(loc, _i64p), _p(fs, _i32p), _p(iip, _i32p),
                                  _p(dist, _f32p))
        n = min(n, cap)
        return dict(list=lst[:n], local=loc[:n], fs=fs[:n], int_ip=iip[:n], dist=dist[:n])


def query_state(art: dict, q: np.ndarray, mode: int = MODE_AVX512) -> dict:
    s, keep = to_struct(art)
    D = int(art["padded_dim"])
    q = np.ascontiguousarray(q, np.float32)
    q_rot = np.empty(D, np.float32)
    q_i8 = np.empty(D, np.int8)
    sc = np.empty(4, np.float32)
    qs = C.c_int32(0)
    lib().ousq_query_state(C.byref(s), _p(q, _f32p), mode, _p(q_rot, _f32p), _p(q_i8, _i8p),
                           _p(sc, _f32p), C.byref(qs))
    lut = np.empty(D // 4 * 16, np.int8)
    ls = C.c_float(0)
    lib().ousq_fastscan_lut(_p(q_rot, _f32p), D, _p(lut, _i8p), C.byref(ls))
    return dict(q_rot=q_rot, q_i8=q_i8, q_sum=sc[0], q_scale=sc[1], centroid_score=sc[2],
                q_norm_sq=sc[3], q_i8_sum=qs.value, lut=lut, lut_scale=np.float32(ls.value))


def fastscan_lut(q_rot: np.ndarray) -> tuple[np.ndarray, np.float32]:
    q_rot = np.ascontiguousarray(q_rot, np.float32)
    D = q_rot.shape[0]
    lut = np.empty(D // 4 * 16, np.int8)
    ls = C.c_float(0)
    lib().ousq_fastscan_lut(_p(q_rot, _f32p), D, _p(lut, _i8p), C.byref(ls))
    return lut, np.float32(ls.value)


def fastscan_blocks(sign_bits: np.ndarray, D: int) -> np.ndarray:
    sign_bits = np.ascontiguousarray(sign_bits, np.uint8)
    n = sign_bits.shape[0]
    out = np.zeros(((n + 31) // 32) * (D // 4) * 16, np.uint8)
    lib().ousq_fastscan_blocks(_p(sign_bits, _u8p), C.c_int64(n), D, _p(out, _u8p))
    return out


def fastscan_scores(blocks, n, D, lut, mode=MODE_AVX512) -> np.ndarray:
    out = np.empty(n, np.int32)
    lut = np.ascontiguousarray(lut, np.int8)
    lib().ousq_fastscan_scores(_p(blocks, _u8p), C.c_int64(n), D, _p(lut, _i8p), mode, _p(out, _i32p))
    return out


def fastscan_topk(blocks, n, D, lut, top_n, mode=MODE_AVX512):
    idx = np.empty(max(top_n, 1), np.int64)
    sc = np.empty(max(top_n, 1), np.int32)
    lut = np.ascontiguousarray(lut, np.int8)
    m = lib().ousq_fastscan_topk(_p(blocks, _u8p), C.c_int64(n), D, _p(lut, _i8p),
                                 C.c_int64(top_n), mode, _p(idx, _i64p), _p(sc, _i32p))
    return idx[:m], sc[:m]


def topk_from_scores(scores, top_n):
    scores = np.ascontiguousarray(scores, np.int32)
    idx = np.empty(max(top_n, 1), np.int64)
    sc = np.empty(max(top_n, 1), np.int32)
    lib().ousq_topk_from_scores.restype = C.c_int64
    m = lib().ousq_topk_from_scores(_p(scores, _i32p), C.c_int64(scores.size), C.c_int64(top_n),
                                    _p(idx, _i64p), _p(sc, _i32p))
    return idx[:m], sc[:m]


def int_ip(codes: np.ndarray, D: int, nbits: int, q_i8: np.ndarray) -> int:
    codes = np.ascontiguousarray(codes, np.uint8)
    q_i8 = np.ascontiguousarray(q_i8, np.int8)
    return int(lib().ousq_int_ip(_p(codes, _u8p), D, nbits, _p(q_i8, _i8p)))


def score(art: dict, q: np.ndarray, row: int, mode: int = MODE_AVX512) -> float:
    s, keep = to_struct(art)
    q = np.ascontiguousarray(q, np.float32)
    return float(lib().ousq_score(C.byref(s), _p(q, _f32p), C.c_int64(row), mode))
