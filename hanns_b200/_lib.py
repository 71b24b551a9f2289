"""ctypes binding of libhanns_gpu.so (the C ABI declared in include/hanns_gpu.h).

The library is the product: loading fails loudly (ImportError) when it is missing;
there is no fallback implementation.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
# HANNS_GPU_LIB: another build of the same library (an experiment's variant)
LIB_PATH = os.environ.get("HANNS_GPU_LIB") or os.path.join(HERE, "lib", "libhanns_gpu.so")

f32p = C.POINTER(C.c_float)
i64p = C.POINTER(C.c_int64)
i32p = C.POINTER(C.c_int32)
u8p = C.POINTER(C.c_uint8)
i8p = C.POINTER(C.c_int8)
u64p = C.POINTER(C.c_uint64)
vp = C.c_void_p


class CIndexConfig(C.Structure):
    """CIndexConfig of the reference C ABI (src/ffi.rs:113-143)."""
    _fields_ = [
        ("index_type", C.c_int32), ("metric_type", C.c_int32), ("dim", C.c_size_t),
        ("ef_construction", C.c_size_t), ("ef_search", C.c_size_t),
        ("num_partitions", C.c_size_t), ("num_centroids", C.c_size_t),
        ("reorder_k", C.c_size_t), ("prq_nsplits", C.c_size_t), ("prq_msub", C.c_size_t),
        ("prq_nbits", C.c_size_t), ("num_clusters", C.c_size_t), ("nprobe", C.c_size_t),
        ("data_type", C.c_int32), ("pq_code_budget_gb", C.c_float),
        ("build_dram_budget_gb", C.c_float), ("disk_pq_dims", C.c_size_t),
        ("beamwidth", C.c_size_t), ("pq_m", C.c_size_t), ("pq_nbits", C.c_size_t),
        ("pca_dim", C.c_size_t),
    ]

    @classmethod
    def default(cls) -> "CIndexConfig":
        # Default for CIndexConfig (src/ffi.rs:145-171)
        c = cls()
        c.index_type, c.metric_type, c.dim = 0, 0, 0
        c.ef_construction, c.ef_search, c.num_partitions = 200, 64, 16
        c.num_centroids, c.reorder_k, c.prq_nsplits, c.prq_msub, c.prq_nbits = 256, 100, 2, 4, 8
        c.num_clusters, c.nprobe, c.data_type = 256, 8, 101
        c.pq_code_budget_gb, c.build_dram_budget_gb, c.disk_pq_dims, c.beamwidth = 0.0, 0.0, 0, 8
        c.pq_m, c.pq_nbits, c.pca_dim = 32, 8, 0
        return c


class CSearchResult(C.Structure):
    _fields_ = [("ids", i64p), ("distances", f32p), ("num_results", C.c_size_t),
                ("elapsed_ms", C.c_float)]


class CBitset(C.Structure):
    _fields_ = [("data", u64p), ("len", C.c_size_t), ("cap_words", C.c_size_t)]


class Artifact(C.Structure):
    """hanns_ivf_usq_artifact_t."""
    _fields_ = [
        ("dim", C.c_int32), ("padded_dim", C.c_int32), ("nbits", C.c_int32),
        ("nlist", C.c_int32), ("metric", C.c_int32), ("reserved", C.c_int32),
        ("ntotal", C.c_int64),
        ("centroids", f32p), ("rotation", f32p), ("rotated_centroid", f32p),
        ("list_offsets", i64p), ("ids", i64p),
        ("norms", f32p), ("norms_sq", f32p), ("vmaxs", f32p), ("quant_qualities", f32p),
        ("codes", u8p), ("sign_bits", u8p),
    ]


# Every symbol declared in include/hanns_gpu.h: (name, restype, argtypes)
SIGNATURES = [
    ("knowhere_create_index", vp, [CIndexConfig]),
    ("knowhere_free_index", None, [vp]),
    ("knowhere_train_index", C.c_int32, [vp, f32p, C.c_size_t, C.c_size_t]),
    ("knowhere_add_index", C.c_int32, [vp, f32p, i64p, C.c_size_t, C.c_size_t]),
    ("knowhere_search", C.POINTER(CSearchResult), [vp, f32p, C.c_size_t, C.c_size_t, C.c_size_t]),
    ("knowhere_search_with_bitset", C.POINTER(CSearchResult),
     [vp, f32p, C.c_size_t, C.c_size_t, C.c_size_t, C.POINTER(CBitset)]),
    ("knowhere_set_nprobe", C.c_int32, [vp, C.c_size_t]),
    ("knowhere_free_result", None, [C.POINTER(CSearchResult)]),
    ("knowhere_get_index_count", C.c_size_t, [vp]),
    ("knowhere_get_index_dim", C.c_size_t, [vp]),
    ("knowhere_get_index_size", C.c_size_t, [vp]),
    ("knowhere_get_index_type", C.c_char_p, [vp]),
    ("knowhere_get_index_metric", C.c_char_p, [vp]),
    ("knowhere_has_raw_data", C.c_bool, [vp]),
    ("knowhere_save_index", C.c_int32, [vp, C.c_char_p]),
    ("knowhere_load_index", C.c_int32, [vp, C.c_char_p]),
    ("knowhere_bitset_create", C.POINTER(CBitset), [C.c_size_t]),
    ("knowhere_bitset_free", None, [C.POINTER(CBitset)]),
    ("knowhere_bitset_set", None, [C.POINTER(CBitset), C.c_size_t, C.c_bool]),
    ("knowhere_bitset_get", C.c_bool, [C.POINTER(CBitset), C.c_size_t]),
    ("knowhere_bitset_count", C.c_size_t, [C.POINTER(CBitset)]),
    ("knowhere_bitset_size", C.c_size_t, [C.POINTER(CBitset)]),
    ("knowhere_bitset_data", u64p, [C.POINTER(CBitset)]),
    ("knowhere_ivf_exrabitq_build", vp, [C.c_uint32, C.c_uint32, C.c_uint32, f32p, C.c_uint64, i64p]),
    ("knowhere_ivf_exrabitq_load", vp, [C.c_char_p]),
    ("knowhere_ivf_exrabitq_save", C.c_int32, [vp, C.c_char_p]),
    ("knowhere_ivf_exrabitq_search", C.c_int32, [vp, f32p, C.c_uint32, C.c_uint32, f32p, i64p]),
    ("knowhere_ivf_exrabitq_batch_search", C.c_int32,
     [vp, f32p, C.c_uint64, C.c_uint32, C.c_uint32, f32p, i64p]),
    ("knowhere_ivf_exrabitq_has_raw_data", C.c_int32, [vp]),
    ("knowhere_ivf_exrabitq_count", C.c_uint64, [vp]),
    ("knowhere_ivf_exrabitq_size", C.c_uint64, [vp]),
    ("knowhere_ivf_exrabitq_free", None, [vp]),
    ("knowhere_ivf_exrabitq_set_nprobe", C.c_int32, [vp, C.c_uint32]),
    ("knowhere_ivf_exrabitq_dim", C.c_uint32, [vp]),
    ("knowhere_ivf_exrabitq_nlist", C.c_uint32, [vp]),
    ("hanns_gpu_last_error", C.c_char_p, []),
    ("hanns_gpu_device_count", C.c_int32, []),
    ("hanns_gpu_ivf_usq_create", vp,
     [C.c_int32, C.c_int32, C.c_int32, C.c_int32, C.c_uint64, C.c_int32, C.c_int32]),
    ("hanns_gpu_ivf_usq_import", vp, [C.POINTER(Artifact), C.c_int32]),
    ("hanns_gpu_ivf_usq_shape", C.c_int32, [vp, i64p]),
    ("hanns_gpu_ivf_usq_export", C.c_int32, [vp, C.POINTER(Artifact)]),
    ("hanns_gpu_ivf_usq_train", C.c_int32, [vp, f32p, C.c_int64, C.c_int32, C.c_uint64]),
    ("hanns_gpu_ivf_usq_add", C.c_int32, [vp, f32p, C.c_int64, i64p]),
    ("hanns_gpu_ivf_usq_search", C.c_int32,
     [vp, f32p, C.c_int64, C.c_int32, C.c_int32, C.c_int32, u64p, C.c_int64, C.c_int64, i32p,
      i64p, f32p, i64p]),
    ("hanns_gpu_ivf_usq_search_device", C.c_int32,
     [vp, vp, C.c_int64, C.c_int32, C.c_int32, C.c_int32, vp, C.c_int64, C.c_int64, vp, vp, vp,
      vp, vp]),
    ("hanns_gpu_ivf_usq_stage_ms", C.c_int32, [vp, f32p]),
    ("hanns_gpu_ivf_usq_stage_ms_recent", C.c_int32, [vp, C.c_int32, f32p, i32p]),
    ("hanns_gpu_ivf_usq_scan_kernel_ms_recent", C.c_int32, [vp, C.c_int32, f32p, i32p]),
    ("hanns_gpu_ivf_usq_last_launches", C.c_int64, [vp]),
    ("hanns_gpu_ivf_usq_set_nprobe", C.c_int32, [vp, C.c_int32]),
    ("hanns_gpu_ivf_usq_count", C.c_int64, [vp]),
    ("hanns_gpu_ivf_usq_free", None, [vp]),
    ("hanns_gpu_ivf_usq_debug_query", C.c_int32,
     [vp, f32p, C.c_int64, C.c_int32, i32p, f32p, i8p, i8p, f32p]),
    ("hanns_gpu_ivf_usq_debug_candidates", C.c_int32,
     [vp, f32p, C.c_int64, C.c_int32, C.c_int32, C.c_int32, u64p, C.c_int64, C.c_int64, i32p,
      C.c_int64, i64p, i32p, i64p, i32p, i32p, f32p]),
    ("hanns_gpu_ivf_usq_set_scan_wait_ns", C.c_int32, [vp, C.c_uint64]),
    ("hanns_gpu_debug_inject_fault", C.c_int32, [C.c_char_p]),
    ("hanns_gpu_ivf_usq_shard", C.c_int32, [vp, C.c_int32, C.c_int32]),
    ("hanns_gpu_ivf_usq_search_shard_device", C.c_int32,
     [vp, vp, C.c_int64, C.c_int32, C.c_int32, vp, vp, vp, vp]),
    ("hanns_gpu_merge_shards_device", C.c_int32,
     [vp, vp, vp, C.c_int32, C.c_int64, C.c_int32, vp, vp, vp]),
    ("hanns_gpu_ivf_usq_query_state_bytes", C.c_int32, [vp, C.c_int32, i64p]),
    ("hanns_gpu_ivf_usq_rerank_rows_device", C.c_int32, [vp, vp, C.c_int64, vp, C.c_int32, vp, vp]),
    ("hanns_gpu_ivf_usq_prepare_device", C.c_int32,
     [vp, vp, C.c_int64, C.c_int32, vp, vp, vp, vp, vp, vp]),
    ("hanns_gpu_ivf_usq_search_prepared_shard_device", C.c_int32,
     [vp, C.c_int64, C.c_int32, C.c_int32, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
    ("hanns_gpu_shard_owners", C.c_int32, [i64p, C.c_int32, C.c_int32, i32p]),
    ("hanns_ivfusq00_read_header", C.c_int32, [C.c_char_p, i64p]),
    ("hanns_ivfusq00_read", C.c_int32, [C.c_char_p, C.POINTER(Artifact)]),
    ("hanns_ivfusq00_write", C.c_int32, [C.c_char_p, C.POINTER(Artifact), C.c_int64, C.c_uint64,
                                         C.c_int64]),
    ("hanns_gpu_ivf_usq_load_ivfusq00", vp, [C.c_char_p, C.c_int32]),
    ("hanns_gpu_ivf_usq_save_ivfusq00", C.c_int32, [vp, C.c_char_p, C.c_uint64, C.c_int64]),
    ("hanns_gpu_coarse_probes_static", C.c_int32,
     [vp, C.c_int64, vp, C.c_int32, C.c_int32, C.c_int32, vp, vp]),
]

_lib = None


def lib():
    """Loads libhanns_gpu.so; raises ImportError when it has not been built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: run `python -m hanns_b200.build` "
                              "(the CUDA library is required; there is no CPU path)")
        L = C.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    e = lib().hanns_gpu_last_error()
    return e.decode() if e else ""
