/*
 * hanns_gpu.h -- C ABI of libhanns_gpu.so, the B200 (sm_100a) IVF-USQ search library.
 *
 * Three groups of entry points:
 *  1. The KnowHere C ABI of Hanns (reference src/ffi.rs), for the IVF-USQ index kind.
 *     Signatures, struct layouts, error codes and ownership rules are those of the
 *     reference; each declaration cites the reference item it replaces.
 *  2. The per-index IVF-USQ C ABI of Hanns (reference src/faiss/exrabitq_ffi.rs).
 *  3. hanns_gpu_* extras with no counterpart in the reference: artifact import and
 *     export (parity testing on a frozen index), device-pointer search, per-query
 *     bitsets, list sharding for multi-GPU and per-stage timings.
 *
 * Every call returns NULL / an error code on failure and never aborts the process;
 * hanns_gpu_last_error() describes the last failure of the calling thread.
 * Concurrent calls on one handle are serialised by the handle (one CUDA stream each).
 */
#ifndef HANNS_GPU_H
#define HANNS_GPU_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------ KnowHere ABI */

/* CError (src/ffi.rs:62-71). */
typedef enum {
    HANNS_OK = 0,
    HANNS_NOT_FOUND = 1,
    HANNS_INVALID_ARG = 2,
    HANNS_INTERNAL = 3,
    HANNS_NOT_IMPLEMENTED = 4,
    HANNS_OUT_OF_MEMORY = 5
} CError;

/* CIndexType (src/ffi.rs:74-100).  IVF-USQ is built for kind 4 (IvfRabitq, which the
 * reference maps to IndexType::IvfUsq at src/ffi.rs:449) and for the new value 23.
 * Every other kind makes knowhere_create_index return NULL. */
typedef int32_t CIndexType;
#define CINDEX_IVF_RABITQ 4
#define CINDEX_IVF_USQ 23

/* CMetricType (src/ffi.rs:103-110).  IVF-USQ: L2 => ||q||^2+||x||^2-2s, anything
 * else => -s (src/faiss/ivf_usq.rs:581-586). */
typedef int32_t CMetricType;
#define CMETRIC_L2 0
#define CMETRIC_IP 1
#define CMETRIC_COSINE 2
#define CMETRIC_HAMMING 3

/* CIndexConfig (src/ffi.rs:113-143), same field order and types.  IVF-USQ reads
 * dim, metric_type, num_clusters (nlist), nprobe and prq_nbits (bits per dim, 1..8). */
typedef struct {
    CIndexType index_type;
    CMetricType metric_type;
    size_t dim;
    size_t ef_construction;
    size_t ef_search;
    size_t num_partitions;
    size_t num_centroids;
    size_t reorder_k;
    size_t prq_nsplits;
    size_t prq_msub;
    size_t prq_nbits;
    size_t num_clusters;
    size_t nprobe;
    int32_t data_type;
    float pq_code_budget_gb;
    float build_dram_budget_gb;
    size_t disk_pq_dims;
    size_t beamwidth;
    size_t pq_m;
    size_t pq_nbits;
    size_t pca_dim;
} CIndexConfig;

/* CSearchResult (src/ffi.rs:183-190).  Owned by the library; free with
 * knowhere_free_result. */
typedef struct {
    int64_t* ids;
    float* distances;
    size_t num_results;
    float elapsed_ms;
} CSearchResult;

/* CBitset (src/ffi.rs:3657-3662): u64 words, bit=1 => filtered (deleted). */
typedef struct {
    uint64_t* data;
    size_t len;
    size_t cap_words;
} CBitset;

/* knowhere_create_index (src/ffi.rs:2252). */
void* knowhere_create_index(CIndexConfig config);
/* knowhere_free_index (src/ffi.rs:2264). */
void knowhere_free_index(void* index);
/* knowhere_train_index (src/ffi.rs:2304): k-means (nlist) + global mean, on the GPU. */
int32_t knowhere_train_index(void* index, const float* vectors, size_t count, size_t dim);
/* knowhere_add_index (src/ffi.rs:2274): assign + USQ encode on the GPU; ids may be NULL
 * (then ids continue from the current count). */
int32_t knowhere_add_index(void* index, const float* vectors, const int64_t* ids,
                           size_t count, size_t dim);
/* knowhere_search (src/ffi.rs:2328): count queries, rows of top_k (id, distance) padded
 * with (-1, +inf); nprobe = the handle's nprobe. */
CSearchResult* knowhere_search(const void* index, const float* query, size_t count,
                               size_t top_k, size_t dim);
/* knowhere_search_with_bitset (src/ffi.rs:2453).  Default: filtered ids are removed
 * before FastScan and rerank and rows stay padded to top_k (num_results = count*top_k).
 * With HANNS_GPU_BITSET_MODE=post the reference post-filter of
 * src/faiss/ivf_usq.rs:688-715 is reproduced (unfiltered search, filtered ids dropped,
 * rows concatenated).  nprobe = the handle's nprobe. */
CSearchResult* knowhere_search_with_bitset(const void* index, const float* query, size_t count,
                                           size_t top_k, size_t dim, const CBitset* bitset);
/* knowhere_set_nprobe (src/ffi.rs:2401). */
int32_t knowhere_set_nprobe(void* index, size_t nprobe);
/* knowhere_free_result (src/ffi.rs:2975). */
void knowhere_free_result(CSearchResult* result);
/* knowhere_get_index_count / _dim / _size (src/ffi.rs:2748,2761,2791). */
size_t knowhere_get_index_count(const void* index);
size_t knowhere_get_index_dim(const void* index);
size_t knowhere_get_index_size(const void* index);
/* knowhere_get_index_type (src/ffi.rs:2820) -> "IVF-USQ" (static string). */
const char* knowhere_get_index_type(const void* index);
/* knowhere_get_index_metric (src/ffi.rs) -> "L2" / "IP" (static string). */
const char* knowhere_get_index_metric(const void* index);
/* knowhere_has_raw_data (src/ffi.rs) -> false for USQ (lossy codes). */
bool knowhere_has_raw_data(const void* index);
/* knowhere_save_index / knowhere_load_index (src/ffi.rs:3445,3493), HGPUUSQ1 format. */
int32_t knowhere_save_index(const void* index, const char* path);
int32_t knowhere_load_index(void* index, const char* path);

/* Bitset helpers (src/ffi.rs:3693-3900; header include/knowhere_bitset.h). */
CBitset* knowhere_bitset_create(size_t len);
void knowhere_bitset_free(CBitset* bitset);
void knowhere_bitset_set(CBitset* bitset, size_t index, bool value);
bool knowhere_bitset_get(const CBitset* bitset, size_t index);
size_t knowhere_bitset_count(const CBitset* bitset);
size_t knowhere_bitset_size(const CBitset* bitset);
const uint64_t* knowhere_bitset_data(const CBitset* bitset);

/* ------------------------------------------------------- per-index IVF-USQ ABI */
typedef struct HannsIvfUsqHandle HannsIvfUsqHandle;

/* knowhere_ivf_exrabitq_build (src/faiss/exrabitq_ffi.rs:23-55): train + add, L2,
 * nprobe 1, rotation seed 42 (IvfUsqConfig::new defaults, src/faiss/ivf_usq.rs:36-47). */
HannsIvfUsqHandle* knowhere_ivf_exrabitq_build(uint32_t dim, uint32_t nlist, uint32_t bits_per_dim,
                                               const float* data, uint64_t n, const int64_t* ids);
/* knowhere_ivf_exrabitq_load / _save (exrabitq_ffi.rs:61-101), HGPUUSQ1 format. */
HannsIvfUsqHandle* knowhere_ivf_exrabitq_load(const char* path);
int32_t knowhere_ivf_exrabitq_save(HannsIvfUsqHandle* index, const char* path);
/* knowhere_ivf_exrabitq_search (exrabitq_ffi.rs:108-146): one query, caller-owned
 * outputs of k, padded with (-1, FLT_MAX); 0 or -1. */
int32_t knowhere_ivf_exrabitq_search(const HannsIvfUsqHandle* index, const float* query, uint32_t k,
                                     uint32_t nprobe, float* distances, int64_t* labels);
/* knowhere_ivf_exrabitq_batch_search (exrabitq_ffi.rs:153-210): nq queries. */
int32_t knowhere_ivf_exrabitq_batch_search(const HannsIvfUsqHandle* index, const float* queries,
                                           uint64_t nq, uint32_t k, uint32_t nprobe,
                                           float* distances, int64_t* labels);
int32_t knowhere_ivf_exrabitq_has_raw_data(const HannsIvfUsqHandle* index); /* :216 */
uint64_t knowhere_ivf_exrabitq_count(const HannsIvfUsqHandle* index);       /* :235 */
uint64_t knowhere_ivf_exrabitq_size(const HannsIvfUsqHandle* index);        /* :248 */
void knowhere_ivf_exrabitq_free(HannsIvfUsqHandle* index);                  /* :261 */
int32_t knowhere_ivf_exrabitq_set_nprobe(HannsIvfUsqHandle* index, uint32_t nprobe); /* :272 */
uint32_t knowhere_ivf_exrabitq_dim(const HannsIvfUsqHandle* index);         /* :289 */
uint32_t knowhere_ivf_exrabitq_nlist(const HannsIvfUsqHandle* index);       /* :302 */

/* ------------------------------------------------------------- hanns_gpu extras */
/* No counterpart in the reference. */

/* Frozen index in list order (same fields as the CPU oracle's artifact). */
typedef struct {
    int32_t dim, padded_dim, nbits, nlist, metric, reserved;
    int64_t ntotal;
    const float* centroids;        /* nlist*dim */
    const float* rotation;         /* padded_dim^2, row-major */
    const float* rotated_centroid; /* padded_dim */
    const int64_t* list_offsets;   /* nlist+1 */
    const int64_t* ids;            /* ntotal */
    const float* norms;
    const float* norms_sq;
    const float* vmaxs;
    const float* quant_qualities;
    const uint8_t* codes;          /* ntotal*code_bytes */
    const uint8_t* sign_bits;      /* ntotal*padded_dim/8 */
} hanns_ivf_usq_artifact_t;

#define HANNS_FILTER_NONE 0
#define HANNS_FILTER_POST 1
#define HANNS_FILTER_FUSED 2

const char* hanns_gpu_last_error(void);
int32_t hanns_gpu_device_count(void);

/* New empty IVF-USQ index on `device` (rotation seed as in IvfUsqConfig). */
HannsIvfUsqHandle* hanns_gpu_ivf_usq_create(int32_t dim, int32_t nlist, int32_t nbits,
                                            int32_t metric, uint64_t rotation_seed,
                                            int32_t nprobe, int32_t device);
/* Uploads a frozen artifact (copied; the caller keeps ownership of its arrays). */
HannsIvfUsqHandle* hanns_gpu_ivf_usq_import(const hanns_ivf_usq_artifact_t* artifact,
                                            int32_t device);
/* Artifact sizes: out6 = {dim, padded_dim, nbits, nlist, metric, ntotal}. */
int32_t hanns_gpu_ivf_usq_shape(const HannsIvfUsqHandle* h, int64_t* out6);
/* Copies the artifact into caller arrays sized from hanns_gpu_ivf_usq_shape
 * (pointer fields of *out are the destinations). */
int32_t hanns_gpu_ivf_usq_export(const HannsIvfUsqHandle* h, hanns_ivf_usq_artifact_t* out);
int32_t hanns_gpu_ivf_usq_train(HannsIvfUsqHandle* h, const float* data, int64_t n,
                                int32_t kmeans_iters, uint64_t kmeans_seed);
int32_t hanns_gpu_ivf_usq_add(HannsIvfUsqHandle* h, const float* data, int64_t n,
                              const int64_t* ids);
/* Batched search with host buffers (copies inside).  ids/dists: nq*k row-major.
 * counts (may be NULL): entries per row (k, or fewer under FILTER_POST).
 * Bitsets: pool of n_bitsets bitsets, each bitset_len bits ((len+63)/64 u64 words);
 * query_bitset[q] picks one or -1; NULL => every query uses bitset 0. */
int32_t hanns_gpu_ivf_usq_search(HannsIvfUsqHandle* h, const float* queries, int64_t nq,
                                 int32_t k, int32_t nprobe, int32_t filter_mode,
                                 const uint64_t* bitsets, int64_t bitset_len, int64_t n_bitsets,
                                 const int32_t* query_bitset, int64_t* ids, float* dists,
                                 int64_t* counts);
/* Same with every buffer in device memory of the handle's GPU, on `stream` (cudaStream_t).
 * With a stream the call is stream-ordered: it returns once the work is enqueued (the
 * opt-in tensor-core scan waits for its error flag).  NULL = the handle's own stream,
 * and the call returns when the search has finished. */
int32_t hanns_gpu_ivf_usq_search_device(HannsIvfUsqHandle* h, const float* d_queries, int64_t nq,
                                        int32_t k, int32_t nprobe, int32_t filter_mode,
                                        const uint64_t* d_bitsets, int64_t bitset_len,
                                        int64_t n_bitsets, const int32_t* d_query_bitset,
                                        int64_t* d_ids, float* d_dists, int64_t* d_counts,
                                        void* stream);
/* Device time (ms) of the stages of the last search, out8 = {coarse GEMM, coarse select,
 * rotation, query state, list grouping, list scan, merge, total}; waits for that search. */
int32_t hanns_gpu_ivf_usq_stage_ms(HannsIvfUsqHandle* h, float* out8);
/* The same summed over the last n_calls search / prepare calls (their stage events sit in
 * a ring of 64 batches); counts8 (may be NULL) = how many batches timed each stage.
 * Returns how many calls it covered, or -(error code). */
int32_t hanns_gpu_ivf_usq_stage_ms_recent(HannsIvfUsqHandle* h, int32_t n_calls, float* out8,
                                          int32_t* counts8);
/* Device time (ms) of the list scan's kernels, out3 = {tensor-core list scan, SIMT list scan,
 * FastScan kept-set selection}, summed over the batches of the last n_calls search calls;
 * counts3 = batches timed.  Returns how many calls it covered, or -(error code). */
int32_t hanns_gpu_ivf_usq_scan_kernel_ms_recent(HannsIvfUsqHandle* h, int32_t n_calls, float* out3,
                                                int32_t* counts3);
/* Number of kernel launches of the last search. */
int64_t hanns_gpu_ivf_usq_last_launches(const HannsIvfUsqHandle* h);
int32_t hanns_gpu_ivf_usq_set_nprobe(HannsIvfUsqHandle* h, int32_t nprobe);
int64_t hanns_gpu_ivf_usq_count(const HannsIvfUsqHandle* h);
void hanns_gpu_ivf_usq_free(HannsIvfUsqHandle* h);

/* Debug: per-query coarse probes [nq*nprobe] and query state
 * (q_rot [nq*D] f32, q_i8 [nq*D] natural order, lut [nq*D/4*16] i8,
 *  scalars [nq*5] = {q_scale, centroid_score, q_norm_sq, lut_scale, q_i8_sum (as f32 bits)}). */
int32_t hanns_gpu_ivf_usq_debug_query(HannsIvfUsqHandle* h, const float* queries, int64_t nq,
                                      int32_t nprobe, int32_t* probes, float* q_rot, int8_t* q_i8,
                                      int8_t* lut, float* scalars);

/* Debug: the list scan's kept candidates of each query -- the reference's candidate vector
 * of search_single (src/faiss/ivf_usq.rs:547-588: probe order, FastScan order inside a list
 * that ran it, fastscan.rs:140-144) -- written at q * cap: list, position in the list,
 * FastScan score (INT32_MIN where FastScan did not select the row), int_ip (quantizer.rs
 * :382-400) and distance; counts[q] = entries of query q.  filter_mode as in
 * hanns_gpu_ivf_usq_search (fused filtering removes rows before the selection).  All
 * queries must fit one internal batch; HANNS_INVALID_ARG / an error if cap is too small. */
int32_t hanns_gpu_ivf_usq_debug_candidates(HannsIvfUsqHandle* h, const float* queries, int64_t nq,
                                           int32_t k, int32_t nprobe, int32_t filter_mode,
                                           const uint64_t* bitsets, int64_t bitset_len,
                                           int64_t n_bitsets, const int32_t* query_bitset,
                                           int64_t cap, int64_t* counts, int32_t* lists,
                                           int64_t* local, int32_t* fs, int32_t* int_ip,
                                           float* dists);

/* Failure testing (no counterpart in the reference, which has no device): the limit of
 * each bounded wait inside the tensor-core list scan (2 s by default).  A wait that runs
 * out makes the scan record an error, finish the MMAs it issued, free its tensor memory
 * and return; the search then fails with an error code (once) and the next search runs
 * normally. */
int32_t hanns_gpu_ivf_usq_set_scan_wait_ns(HannsIvfUsqHandle* h, uint64_t ns);
/* Failure testing: make the library's next device allocations ("alloc") or host-to-device
 * copies ("h2d") fail as if CUDA had returned an error, or stop doing so ("none").  Only
 * the host sees the fault; no kernel runs on bad memory.  HANNS_GPU_FAULT=alloc|h2d sets
 * the same at load. */
int32_t hanns_gpu_debug_inject_fault(const char* what);

/* Multi-GPU list sharding: keep only lists l with owner[l] == rank, where owner is a
 * longest-processing-time assignment of lists (by size) to world ranks.  Search then
 * returns this shard's top-k with merge keys. */
int32_t hanns_gpu_ivf_usq_shard(HannsIvfUsqHandle* h, int32_t rank, int32_t world);
/* Sharded search: per query k entries of (dist, key) where key = probe_rank<<48 |
 * fastscan_key<<32 | local_index, plus ids; device buffers. */
int32_t hanns_gpu_ivf_usq_search_shard_device(HannsIvfUsqHandle* h, const float* d_queries,
                                              int64_t nq, int32_t k, int32_t nprobe,
                                              float* d_dists, uint64_t* d_keys, int64_t* d_ids,
                                              void* stream);
/* The reference's snapshot file (IvfUsqIndex::save, src/faiss/ivf_usq.rs:353-406:
 * "IVFUSQ00", version 3, bincode 1.3 StoredSnapshot); no counterpart in the reference's
 * C ABI.  Host only, no GPU:
 *   hanns_ivfusq00_read_header: out10 = {dim, padded_dim, nbits, nlist, metric, ntotal,
 *     nprobe, rotation_seed, rerank_k, flags (bit 0 trained, bit 1 high-accuracy scan)}.
 *   hanns_ivfusq00_read: fills the caller's artifact arrays (shape fields must match the
 *     header).  As IvfUsqIndex::load does (:408-506), the global centroid is zero, so
 *     rotated_centroid = 0; the rotation is regenerated from rotation_seed by this
 *     library's generator (parity of P with the Rust build is not claimed).
 *   hanns_ivfusq00_write: writes an artifact in that format (list order = clusters).
 * On the GPU: hanns_gpu_ivf_usq_load_ivfusq00 opens such a file as a new index;
 * knowhere_load_index also accepts it (the shape must match the handle's config);
 * hanns_gpu_ivf_usq_save_ivfusq00 writes an index in that format. */
int32_t hanns_ivfusq00_read_header(const char* path, int64_t* out10);
int32_t hanns_ivfusq00_read(const char* path, hanns_ivf_usq_artifact_t* out);
int32_t hanns_ivfusq00_write(const char* path, const hanns_ivf_usq_artifact_t* artifact,
                             int64_t nprobe, uint64_t rotation_seed, int64_t rerank_k);
HannsIvfUsqHandle* hanns_gpu_ivf_usq_load_ivfusq00(const char* path, int32_t device);
int32_t hanns_gpu_ivf_usq_save_ivfusq00(HannsIvfUsqHandle* h, const char* path,
                                        uint64_t rotation_seed, int64_t rerank_k);
/* Query-split multi-GPU search (no counterpart in the reference, whose search runs on one
 * host).  Each rank prepares the per-query state of its share of the queries, the ranks
 * all-gather it, and every rank scans its own lists for all queries:
 *   hanns_gpu_ivf_usq_query_state_bytes: bytes per query of the five state arrays
 *     (probes int32[nprobe], scalars, FastScan LUT, q_i8 dp4a layout, q_i8 in dimension
 *     order) into out5.
 *   hanns_gpu_ivf_usq_prepare_device: coarse probes, rotation and query state of nq
 *     device-resident queries into the caller's device arrays (d_qi8n may be NULL).
 *   hanns_gpu_ivf_usq_search_prepared_shard_device: grouping, list scan and merge of nq
 *     queries from such arrays (concatenated over the ranks); output as
 *     hanns_gpu_ivf_usq_search_shard_device.
 * Both are stream-ordered like hanns_gpu_ivf_usq_search_device (NULL stream: synchronous). */
int32_t hanns_gpu_ivf_usq_query_state_bytes(HannsIvfUsqHandle* h, int32_t nprobe, int64_t* out5);
int32_t hanns_gpu_ivf_usq_prepare_device(HannsIvfUsqHandle* h, const float* d_queries, int64_t nq,
                                         int32_t nprobe, void* d_probes, void* d_qp, void* d_lut,
                                         void* d_qi8p, void* d_qi8n, void* stream);
int32_t hanns_gpu_ivf_usq_search_prepared_shard_device(
    HannsIvfUsqHandle* h, int64_t nq, int32_t k, int32_t nprobe, const void* d_probes,
    const void* d_qp, const void* d_lut, const void* d_qi8p, const void* d_qi8n, float* d_dists,
    uint64_t* d_keys, int64_t* d_ids, void* stream);
/* Batched USQ rerank of caller-chosen stored rows: for each of nq device queries and each
 * of its m rows (d_rows[q*m + j], positions in the index's storage order as exported;
 * rows outside [0, count) give +inf), the distance the search computes for that row --
 * query state (quantizer.rs:236-270), integer inner product and score_with_meta
 * (quantizer.rs:274-288, 382-400), L2 / IP distance (ivf_usq.rs:581-586).  The arithmetic
 * the reference reuses in HNSW-HVQ (faiss/hnsw_hvq.rs:601), HNSW-PCA-USQ
 * (faiss/hnsw_pca_usq.rs:55-63) and DiskANN-PCA-USQ (faiss/diskann_pca_usq.rs:77-85) to
 * rerank graph candidates.  Stream-ordered like hanns_gpu_ivf_usq_search_device. */
int32_t hanns_gpu_ivf_usq_rerank_rows_device(HannsIvfUsqHandle* h, const float* d_queries,
                                              int64_t nq, const int64_t* d_rows, int32_t m,
                                              float* d_dists, void* stream);
/* The list -> rank owner map that hanns_gpu_ivf_usq_shard uses (host only, no GPU):
 * longest-processing-time on |L|^2 (scan work ~ list size x probes of the list), lists
 * by decreasing weight, each to the least-loaded rank. */
int32_t hanns_gpu_shard_owners(const int64_t* list_sizes, int32_t nlist, int32_t world,
                               int32_t* owner);
/* Merges world shard results laid out [world][nq][k] into the global top-k
 * (ties broken by key, matching the single-GPU stable order); device buffers. */
int32_t hanns_gpu_merge_shards_device(const float* d_dists, const uint64_t* d_keys,
                                      const int64_t* d_ids, int32_t world, int64_t nq, int32_t k,
                                      int64_t* d_out_ids, float* d_out_dists, void* stream);

/* Coarse-probe step without any device allocation.  No counterpart in the reference.
 * For callers that cannot call cudaMalloc: processes that give all GPU memory to their
 * own pool at start-up, and latency-critical paths where cudaMalloc/cudaFree (which may
 * synchronise the device) are not allowed.  Computes, for nq device-resident queries,
 * the exact L2 to the nlist device-resident centroids (dim floats each) and writes the
 * nprobe nearest list ids per query, in order, to d_probes[nq*nprobe] -- the same
 * probes the search path uses.  Scratch is a fixed 16 MiB array inside the library (held
 * on every GPU that loads it until exit); nq*nlist*4 + nq*nprobe*8 bytes (distances
 * rounded up to 256) must fit, else HANNS_INVALID_ARG and nothing runs.  The first call
 * on a device looks up the scratch address (make it before any stream capture).
 * Asynchronous on `stream`; all calls share the scratch, so calls that overlap on the
 * GPU race -- order them on one stream. */
int32_t hanns_gpu_coarse_probes_static(const float* d_queries, int64_t nq,
                                       const float* d_centroids, int32_t nlist, int32_t dim,
                                       int32_t nprobe, int32_t* d_probes, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* HANNS_GPU_H */
