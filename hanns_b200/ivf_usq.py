"""IvfUsqIndex: the reference's Rust IVF-USQ API, backed by libhanns_gpu.so.

Mirrors src/faiss/ivf_usq.rs (IvfUsqConfig :24-110, IvfUsqIndex :170-352, the Index
trait :639-756) and src/api/search.rs (SearchRequest :7-18, SearchResult :22-43).
Errors the reference reports as KnowhereError::InvalidArg raise ValueError; GPU
failures raise RuntimeError.  Every call goes through the C ABI.
"""
from __future__ import annotations

import ctypes as C
import time
from dataclasses import dataclass, field

import numpy as np

from . import _lib as L

METRIC_L2, METRIC_IP = 0, 1
FILTER_NONE, FILTER_POST, FILTER_FUSED = 0, 1, 2


@dataclass
class IvfUsqConfig:
    """IvfUsqConfig (src/faiss/ivf_usq.rs:24-47)."""
    dim: int
    nlist: int
    bits_per_dim: int
    nprobe: int = 1
    metric_type: int = METRIC_L2
    use_high_accuracy_scan: bool = False  # stored, unused by search (as in the reference)
    rotation_seed: int = 42
    rerank_k: int = 64  # stored, unused by search (as in the reference)

    def with_nprobe(self, n): self.nprobe = n; return self
    def with_metric(self, m): self.metric_type = m; return self
    def with_rotation_seed(self, s): self.rotation_seed = s; return self
    def with_high_accuracy_scan(self, b): self.use_high_accuracy_scan = b; return self
    def with_rerank_k(self, k): self.rerank_k = k; return self


@dataclass
class SearchRequest:
    """SearchRequest (src/api/search.rs:7-18); filter/params/radius are unused by IVF-USQ."""
    top_k: int = 10
    nprobe: int = 8
    filter: object = None
    params: object = None
    radius: float | None = None


@dataclass
class SearchResult:
    """SearchResult (src/api/search.rs:22-43): row-major nq*top_k ids and distances."""
    ids: np.ndarray
    distances: np.ndarray
    elapsed_ms: float = 0.0
    num_visited: int = 0
    counts: np.ndarray | None = field(default=None, repr=False)


def _p(a, t):
    return a.ctypes.data_as(t)


def _check(rc: int, what: str):
    if rc != 0:
        msg = L.last_error()
        if rc == 2:
            raise ValueError(f"{what}: {msg}")
        raise RuntimeError(f"{what} failed ({rc}): {msg}")


class IvfUsqIndex:
    """GPU IVF-USQ index on one device."""

    def __init__(self, config: IvfUsqConfig, device: int = 0, _handle=None):
        self.config = config
        self.device = device
        lib = L.lib()
        if _handle is not None:
            self._h = _handle
        else:
            self._h = lib.hanns_gpu_ivf_usq_create(config.dim, config.nlist, config.bits_per_dim,
                                                   config.metric_type, config.rotation_seed,
                                                   max(config.nprobe, 1), device)
            if not self._h:
                raise ValueError(f"IvfUsqIndex::new: {L.last_error()}")

    # ------------------------------------------------------------ lifecycle
    def close(self):
        if getattr(self, "_h", None):
            L.lib().hanns_gpu_ivf_usq_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @classmethod
    def from_artifact(cls, art: dict, device: int = 0) -> "IvfUsqIndex":
        """Uploads a frozen index (dict of arrays, list order; see oracle/oracle.py)."""
        keep = []

        def arr(name, dt):
            a = np.ascontiguousarray(art[name], dt)
            keep.append(a)
            return a

        s = L.Artifact()
        s.dim, s.padded_dim, s.nbits = int(art["dim"]), int(art["padded_dim"]), int(art["nbits"])
        s.nlist, s.metric, s.reserved = int(art["nlist"]), int(art["metric"]), 0
        s.ntotal = int(np.asarray(art["ids"]).shape[0])
        s.centroids = _p(arr("centroids", np.float32), L.f32p)
        s.rotation = _p(arr("rotation", np.float32), L.f32p)
        s.rotated_centroid = _p(arr("rotated_centroid", np.float32), L.f32p)
        s.list_offsets = _p(arr("list_offsets", np.int64), L.i64p)
        s.ids = _p(arr("ids", np.int64), L.i64p)
        s.norms = _p(arr("norms", np.float32), L.f32p)
        s.norms_sq = _p(arr("norms_sq", np.float32), L.f32p)
        s.vmaxs = _p(arr("vmaxs", np.float32), L.f32p)
        s.quant_qualities = _p(arr("quant_qualities", np.float32), L.f32p)
        s.codes = _p(arr("codes", np.uint8), L.u8p)
        s.sign_bits = _p(arr("sign_bits", np.uint8), L.u8p)
        h = L.lib().hanns_gpu_ivf_usq_import(C.byref(s), device)
        if not h:
            raise ValueError(f"import: {L.last_error()}")
        cfg = IvfUsqConfig(s.dim, s.nlist, s.nbits, metric_type=s.metric)
        return cls(cfg, device, _handle=h)

    @classmethod
    def load_ivfusq00(cls, path: str, device: int = 0) -> "IvfUsqIndex":
        """Opens a snapshot written by the reference's IvfUsqIndex::save ("IVFUSQ00",
        src/faiss/ivf_usq.rs:353-406); loaded like IvfUsqIndex::load (zero global centroid)."""
        hdr = np.zeros(10, np.int64)
        _check(L.lib().hanns_ivfusq00_read_header(str(path).encode(), _p(hdr, L.i64p)), "IVFUSQ00 header")
        h = L.lib().hanns_gpu_ivf_usq_load_ivfusq00(str(path).encode(), device)
        if not h:
            raise ValueError(f"load IVFUSQ00: {L.last_error()}")
        cfg = IvfUsqConfig(int(hdr[0]), int(hdr[3]), int(hdr[2]), nprobe=int(hdr[6]), metric_type=int(hdr[4]),
                           rotation_seed=int(hdr[7]))
        return cls(cfg, device, _handle=h)

    def save_ivfusq00(self, path: str, rerank_k: int = 64):
        """Writes the index in the reference's snapshot format."""
        _check(L.lib().hanns_gpu_ivf_usq_save_ivfusq00(self._h, str(path).encode(),
                                                        self.config.rotation_seed, rerank_k),
               "save IVFUSQ00")

    def save(self, path: str):
        """IvfUsqIndex::save (src/faiss/ivf_usq.rs:354-406): the "IVFUSQ00" snapshot, with
        the config's rerank_k stored as the reference stores it."""
        self.save_ivfusq00(path, rerank_k=self.config.rerank_k)

    # IvfUsqIndex::load (src/faiss/ivf_usq.rs:411-506)
    load = load_ivfusq00

    def export_artifact(self) -> dict:
        shp = np.zeros(6, np.int64)
        _check(L.lib().hanns_gpu_ivf_usq_shape(self._h, _p(shp, L.i64p)), "shape")
        d, D, nbits, nlist, metric, n = (int(v) for v in shp)
        cb = (D * nbits + 7) // 8
        art = dict(dim=d, padded_dim=D, nbits=nbits, nlist=nlist, metric=metric,
                   centroids=np.zeros((nlist, d), np.float32), rotation=np.zeros((D, D), np.float32),
                   rotated_centroid=np.zeros(D, np.float32), list_offsets=np.zeros(nlist + 1, np.int64),
                   ids=np.zeros(n, np.int64), norms=np.zeros(n, np.float32),
                   norms_sq=np.zeros(n, np.float32), vmaxs=np.zeros(n, np.float32),
                   quant_qualities=np.zeros(n, np.float32), codes=np.zeros((n, cb), np.uint8),
                   sign_bits=np.zeros((n, D // 8), np.uint8))
        s = L.Artifact()
        for name, t in [("centroids", L.f32p), ("rotation", L.f32p), ("rotated_centroid", L.f32p),
                        ("list_offsets", L.i64p), ("ids", L.i64p), ("norms", L.f32p),
                        ("norms_sq", L.f32p), ("vmaxs", L.f32p), ("quant_qualities", L.f32p),
                        ("codes", L.u8p), ("sign_bits", L.u8p)]:
            setattr(s, name, _p(art[name], t))
        _check(L.lib().hanns_gpu_ivf_usq_export(self._h, C.byref(s)), "export")
        return art

    # ------------------------------------------------------------ build
    def train(self, data: np.ndarray, kmeans_iters: int = 25, kmeans_seed: int = 42):
        data = np.ascontiguousarray(data, np.float32).reshape(-1, self.config.dim)
        _check(L.lib().hanns_gpu_ivf_usq_train(self._h, _p(data, L.f32p), data.shape[0],
                                               kmeans_iters, kmeans_seed), "train")

    def add(self, data: np.ndarray, ids: np.ndarray | None = None) -> int:
        data = np.ascontiguousarray(data, np.float32).reshape(-1, self.config.dim)
        idp = None
        if ids is not None:
            ids = np.ascontiguousarray(ids, np.int64)
            if ids.shape[0] != data.shape[0]:
                raise ValueError("ids length does not match vector count")
            idp = _p(ids, L.i64p)
        _check(L.lib().hanns_gpu_ivf_usq_add(self._h, _p(data, L.f32p), data.shape[0], idp), "add")
        return data.shape[0]

    # ------------------------------------------------------------ search
    def search(self, query: np.ndarray, req: SearchRequest, filter_mode: int = FILTER_NONE,
               bitsets: np.ndarray | None = None, bitset_len: int = 0,
               query_bitset: np.ndarray | None = None) -> SearchResult:
        """IvfUsqIndex::search (src/faiss/ivf_usq.rs:322-352), batched on the GPU."""
        q = np.ascontiguousarray(query, np.float32)
        if q.size == 0 or q.size % self.config.dim:
            raise ValueError("query dimension mismatch")
        q = q.reshape(-1, self.config.dim)
        nq = q.shape[0]
        k = max(int(req.top_k), 1)
        ids = np.empty((nq, k), np.int64)
        dists = np.empty((nq, k), np.float32)
        counts = np.empty(nq, np.int64)
        bp, nbs, qbp = None, 0, None
        if bitsets is not None and filter_mode != FILTER_NONE:
            bitsets = np.ascontiguousarray(bitsets, np.uint64)
            if bitsets.ndim == 1:
                bitsets = bitsets[None, :]
            nbs = bitsets.shape[0]
            bp = _p(bitsets, L.u64p)
            if query_bitset is not None:
                query_bitset = np.ascontiguousarray(query_bitset, np.int32)
                qbp = _p(query_bitset, L.i32p)
        t0 = time.perf_counter()
        _check(L.lib().hanns_gpu_ivf_usq_search(self._h, _p(q, L.f32p), nq, k, max(int(req.nprobe), 1),
                                                filter_mode if bp is not None else 0, bp, bitset_len,
                                                nbs, qbp, _p(ids, L.i64p), _p(dists, L.f32p),
                                                _p(counts, L.i64p)), "search")
        ms = (time.perf_counter() - t0) * 1e3
        return SearchResult(ids.reshape(-1), dists.reshape(-1), ms, 0, counts)

    def search_with_bitset(self, query: np.ndarray, top_k: int, bitset: np.ndarray,
                           bitset_len: int) -> SearchResult:
        """Index::search_with_bitset (src/faiss/ivf_usq.rs:688-715): search with the index's
        nprobe, then drop (id, d) whose id < len has its bit set; rows are concatenated."""
        r = self.search(query, SearchRequest(top_k=top_k, nprobe=self.config.nprobe),
                        FILTER_POST, bitset, bitset_len)
        k = max(int(top_k), 1)
        ids = r.ids.reshape(-1, k)
        d = r.distances.reshape(-1, k)
        keep_i = np.concatenate([ids[q, :c] for q, c in enumerate(r.counts)])
        keep_d = np.concatenate([d[q, :c] for q, c in enumerate(r.counts)])
        return SearchResult(keep_i, keep_d, r.elapsed_ms)

    def search_device(self, d_queries: int, nq: int, k: int, nprobe: int, d_ids: int, d_dists: int,
                      d_counts: int = 0, stream: int = 0, filter_mode: int = FILTER_NONE,
                      d_bitsets: int = 0, bitset_len: int = 0, n_bitsets: int = 0,
                      d_query_bitset: int = 0):
        """Search with device pointers (ints, e.g. torch tensor.data_ptr())."""
        _check(L.lib().hanns_gpu_ivf_usq_search_device(
            self._h, d_queries, nq, k, nprobe, filter_mode, d_bitsets or None, bitset_len,
            n_bitsets, d_query_bitset or None, d_ids, d_dists, d_counts or None, stream or None),
            "search_device")

    def rerank_rows(self, queries: np.ndarray, rows: np.ndarray) -> np.ndarray:
        """USQ distances of stored rows (storage order, as export_artifact lists them):
        rows[q, j] for query q; rows outside [0, count) give +inf.  The score_with_meta
        rerank the reference's graph indexes reuse (faiss/hnsw_pca_usq.rs:55-63)."""
        import torch
        q = np.ascontiguousarray(queries, np.float32).reshape(-1, self.config.dim)
        r = np.ascontiguousarray(rows, np.int64).reshape(q.shape[0], -1)
        dq = torch.from_numpy(q).to(f"cuda:{self.device}")
        dr = torch.from_numpy(r).to(f"cuda:{self.device}")
        out = torch.empty(r.shape, dtype=torch.float32, device=dq.device)
        _check(L.lib().hanns_gpu_ivf_usq_rerank_rows_device(self._h, dq.data_ptr(), q.shape[0],
                                                            dr.data_ptr(), r.shape[1],
                                                            out.data_ptr(), None), "rerank_rows")
        return out.cpu().numpy()

    STAGES = ("coarse_gemm", "coarse_select", "rotate", "query_state", "group", "scan", "merge",
              "total")

    def stage_ms(self) -> np.ndarray:
        """Device ms of the last search per stage (names in STAGES); waits for it."""
        out = np.zeros(8, np.float32)
        _check(L.lib().hanns_gpu_ivf_usq_stage_ms(self._h, _p(out, L.f32p)), "stage_ms")
        return out

    def stage_ms_recent(self, n_calls: int):
        """(sum of device ms per stage, batches that timed each stage, calls covered) over
        the last n_calls search / prepare calls."""
        out = np.zeros(8, np.float32)
        cnt = np.zeros(8, np.int32)
        rc = L.lib().hanns_gpu_ivf_usq_stage_ms_recent(self._h, int(n_calls), _p(out, L.f32p),
                                                       _p(cnt, L.i32p))
        if rc < 0:
            _check(-rc, "stage_ms_recent")
        return out, cnt, int(rc)

    SCAN_KERNELS = ("scan_tc", "scan_simt", "fs_select")

    def scan_kernel_ms_recent(self, n_calls: int):
        """(sum of device ms per list-scan kernel (names in SCAN_KERNELS), batches timed)
        over the last n_calls search calls."""
        out = np.zeros(3, np.float32)
        cnt = np.zeros(3, np.int32)
        rc = L.lib().hanns_gpu_ivf_usq_scan_kernel_ms_recent(self._h, int(n_calls), _p(out, L.f32p),
                                                             _p(cnt, L.i32p))
        if rc < 0:
            _check(-rc, "scan_kernel_ms_recent")
        return out, cnt

    def last_launches(self) -> int:
        return int(L.lib().hanns_gpu_ivf_usq_last_launches(self._h))

    def debug_query(self, queries: np.ndarray, nprobe: int) -> dict:
        q = np.ascontiguousarray(queries, np.float32).reshape(-1, self.config.dim)
        nq = q.shape[0]
        D = (self.config.dim + 63) // 64 * 64
        npr = min(max(nprobe, 1), self.config.nlist)
        probes = np.zeros((nq, npr), np.int32)
        q_rot = np.zeros((nq, D), np.float32)
        q_i8 = np.zeros((nq, D), np.int8)
        lut = np.zeros((nq, D // 4 * 16), np.int8)
        sc = np.zeros((nq, 5), np.float32)
        _check(L.lib().hanns_gpu_ivf_usq_debug_query(self._h, _p(q, L.f32p), nq, npr,
                                                     _p(probes, L.i32p), _p(q_rot, L.f32p),
                                                     _p(q_i8, L.i8p), _p(lut, L.i8p),
                                                     _p(sc, L.f32p)), "debug_query")
        return dict(probes=probes, q_rot=q_rot, q_i8=q_i8, lut=lut, q_scale=sc[:, 0],
                    centroid_score=sc[:, 1], q_norm_sq=sc[:, 2], lut_scale=sc[:, 3],
                    q_i8_sum=sc[:, 4].copy().view(np.int32))

    def debug_candidates(self, query: np.ndarray, k: int, nprobe: int, filter_mode: int = FILTER_NONE,
                         bitsets: np.ndarray | None = None, bitset_len: int = 0,
                         query_bitset: np.ndarray | None = None, cap: int = 1 << 16) -> list:
        """The list scan's kept candidates of each query, in the reference's candidate order
        (the oracle's `candidates` format: list, local, fs, int_ip, dist per query)."""
        q = np.ascontiguousarray(query, np.float32).reshape(-1, self.config.dim)
        nq = q.shape[0]
        counts = np.zeros(nq, np.int64)
        lists = np.zeros((nq, cap), np.int32)
        local = np.zeros((nq, cap), np.int64)
        fs = np.zeros((nq, cap), np.int32)
        iip = np.zeros((nq, cap), np.int32)
        dist = np.zeros((nq, cap), np.float32)
        bp, nbs, qbp = None, 0, None
        if bitsets is not None and filter_mode != FILTER_NONE:
            bitsets = np.ascontiguousarray(bitsets, np.uint64)
            if bitsets.ndim == 1:
                bitsets = bitsets[None, :]
            nbs = bitsets.shape[0]
            bp = _p(bitsets, L.u64p)
            if query_bitset is not None:
                query_bitset = np.ascontiguousarray(query_bitset, np.int32)
                qbp = _p(query_bitset, L.i32p)
        _check(L.lib().hanns_gpu_ivf_usq_debug_candidates(
            self._h, _p(q, L.f32p), nq, max(int(k), 1), max(int(nprobe), 1),
            filter_mode if bp is not None else 0, bp, bitset_len, nbs, qbp, cap,
            _p(counts, L.i64p), _p(lists, L.i32p), _p(local, L.i64p), _p(fs, L.i32p),
            _p(iip, L.i32p), _p(dist, L.f32p)), "debug_candidates")
        return [dict(list=lists[i, :c], local=local[i, :c], fs=fs[i, :c], int_ip=iip[i, :c],
                     dist=dist[i, :c]) for i, c in enumerate(counts)]

    # ------------------------------------------------------------ misc
    def set_nprobe(self, nprobe: int):
        """set_nprobe (src/faiss/ivf_usq.rs:224-226): clamp to 1..=nlist."""
        self.config.nprobe = max(1, min(int(nprobe), self.config.nlist))
        _check(L.lib().hanns_gpu_ivf_usq_set_nprobe(self._h, self.config.nprobe), "set_nprobe")

    def shard(self, rank: int, world: int):
        _check(L.lib().hanns_gpu_ivf_usq_shard(self._h, rank, world), "shard")

    def count(self) -> int:
        return int(L.lib().hanns_gpu_ivf_usq_count(self._h))

    ntotal = count

    def dim(self) -> int:
        return self.config.dim

    def has_raw_data(self) -> bool:
        return False

    def size(self) -> int:
        """IvfUsqIndex::size (src/faiss/ivf_usq.rs:208-222): centroid bytes plus, per stored
        row, its id (8), four f32 factors (16) and packed code bytes."""
        D = -(-self.config.dim // 64) * 64
        code_bytes = (D * self.config.bits_per_dim + 7) // 8
        return self.config.nlist * self.config.dim * 4 + self.count() * (8 + 16 + code_bytes)
