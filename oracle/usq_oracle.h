/*
 * usq_oracle.h -- CPU restatement of Hanns' IVF-USQ search arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * hanns_b200/csrc.  Only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.  The product library never links or calls it.
 *
 * Parity status: UNPINNED against the Rust binary.  The reference (Rust) cannot be
 * compiled in this environment (no rustc/cargo, crates not vendored) and its own
 * tests hold no numeric golden vectors for this path, only property tests
 * (tests/test_usq_quantizer.rs, tests/test_usq_fastscan.rs,
 * tests/test_ivf_index_trait.rs, src/faiss/ivf_usq.rs:792-809).  Those property
 * tests are ported against this oracle in tests/test_oracle_reference_props.py.
 *
 * Semantics restated (reference = benwuhua/Hanns, paths relative to its root):
 *   src/quantization/usq/config.rs            padded_dim / code_bytes / sign_bytes
 *   src/quantization/usq/rotator.rs:56-120     rotate (AVX-512F 16-lane FMA + reduce)
 *   src/quantization/usq/quantizer.rs:124-270  encode, precompute_query_state
 *   src/quantization/usq/quantizer.rs:274-400  score_with_meta / compute_ip (VNNI, 1-bit, scalar)
 *   src/quantization/usq/quantizer.rs:442-672  greedy / threshold-sweep quantisers
 *   src/quantization/usq/fastscan.rs:22-227    LUT, fastscan_topk heap, block scans
 *   src/quantization/usq/layout.rs:139-197     FastScan block transpose
 *   src/quantization/turboquant/packed.rs:1-59 pack_codes / unpack_codes
 *   src/faiss/ivf_usq.rs:322-352,527-635       search, search_single, rank_centroids
 *   src/faiss/ivf_usq.rs:688-715               search_with_bitset post-filter
 *
 * Two semantic switches:
 *   mode  OUSQ_MODE_AVX512 (0): the x86 AVX-512BW/VNNI path the reference takes on
 *                               its authority machine (i16-wrapped FastScan sums,
 *                               integer VNNI rerank for 4/8 bit, 16-lane FMA rotation).
 *         OUSQ_MODE_SCALAR (1): the reference's portable fallback (i32 FastScan sums,
 *                               float dequantised rerank, sequential rotation).
 *   filter OUSQ_FILTER_NONE / POST (reference post-filter) / FUSED (filtered ids are
 *          removed from each list before FastScan and rerank; rows padded to k).
 */
#ifndef HANNS_USQ_ORACLE_H
#define HANNS_USQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { OUSQ_MODE_AVX512 = 0, OUSQ_MODE_SCALAR = 1 };
enum { OUSQ_FILTER_NONE = 0, OUSQ_FILTER_POST = 1, OUSQ_FILTER_FUSED = 2 };
enum { OUSQ_METRIC_L2 = 0, OUSQ_METRIC_IP = 1 };

/* A frozen IVF-USQ index: every array in list order (list l owns rows
 * list_offsets[l] .. list_offsets[l+1]).  Same field meaning as the GPU library's
 * import struct. */
typedef struct {
    int32_t dim;          /* d */
    int32_t padded_dim;   /* D = ceil(d/64)*64 */
    int32_t nbits;        /* 1..8 */
    int32_t nlist;
    int32_t metric;       /* OUSQ_METRIC_* */
    int32_t reserved;
    int64_t ntotal;
    const float* centroids;         /* nlist*d   IVF centroids */
    const float* rotation;          /* D*D       row-major orthogonal P */
    const float* rotated_centroid;  /* D         P * pad(global mean) */
    const int64_t* list_offsets;    /* nlist+1 */
    const int64_t* ids;             /* ntotal */
    const float* norms;             /* ntotal    ||rotated residual|| */
    const float* norms_sq;          /* ntotal    ||x||^2 (raw vector) */
    const float* vmaxs;             /* ntotal */
    const float* quant_qualities;   /* ntotal */
    const uint8_t* codes;           /* ntotal*code_bytes, pack_codes LSB-first */
    const uint8_t* sign_bits;       /* ntotal*(D/8), 1 bit per padded dim, LSB-first */
} ousq_artifact_t;

/* ---- config helpers (config.rs) ---- */
int32_t ousq_padded_dim(int32_t dim);
int32_t ousq_code_bytes(int32_t dim, int32_t nbits);
int32_t ousq_sign_bytes(int32_t dim);
int32_t ousq_n_candidates(int32_t nbits, int32_t top_k);

/* ---- build-side helpers (fixtures only) ---- */
void ousq_rotation_matrix(uint64_t seed, int32_t D, float* out);
void ousq_rotate(const float* P, int32_t D, const float* x, float* out, int32_t mode);
void ousq_encode(const float* P, int32_t dim, int32_t nbits, const float* centroid,
                 const float* x, int32_t mode, uint8_t* codes, uint8_t* sign_bits,
                 float* meta4 /* norm, norm_sq, vmax, quant_quality */);
void ousq_encode_batch(const float* P, int32_t dim, int32_t nbits, const float* centroid,
                       const float* x, int64_t n, int32_t mode, uint8_t* codes,
                       uint8_t* sign_bits, float* meta4, int32_t nthreads);
void ousq_kmeans(const float* data, int64_t n, int32_t dim, int32_t k, int32_t iters,
                 uint64_t seed, float* centroids, int32_t nthreads);
void ousq_assign(const float* data, int64_t n, int32_t dim, const float* centroids,
                 int32_t nlist, int32_t* out_list, int32_t nthreads);
/* Global mean in the order of ivf_usq.rs:253-263 (row-sequential f32 sums, * (1/n)). */
void ousq_global_mean(const float* data, int64_t n, int32_t dim, float* out);
void ousq_pack_codes(const uint16_t* codes, int64_t n, int32_t nbits, uint8_t* out);
void ousq_unpack_codes(const uint8_t* bytes, int64_t n, int32_t nbits, uint16_t* out);

/* ---- query-side stages ---- */
void ousq_query_state(const ousq_artifact_t* a, const float* q, int32_t mode,
                      float* q_rot /* D */, int8_t* q_i8 /* D */,
                      float* scalars4 /* q_sum, q_scale, centroid_score, q_norm_sq */,
                      int32_t* q_i8_sum);
void ousq_fastscan_lut(const float* q_rot, int32_t D, int8_t* lut /* D/4*16 */,
                       float* lut_scale);
/* Builds the reference FastScan blocks for n vectors (sign bits in, blocks out,
 * ceil(n/32) * (D/4)*16 bytes). */
void ousq_fastscan_blocks(const uint8_t* sign_bits, int64_t n, int32_t D, uint8_t* blocks);
/* Raw FastScan scores of all n vectors of one list (no selection). */
void ousq_fastscan_scores(const uint8_t* blocks, int64_t n, int32_t D, const int8_t* lut,
                          int32_t mode, int32_t* scores);
/* fastscan_topk: returns the number of candidates written (<= top_n), sorted by
 * (score desc, idx asc). */
int64_t ousq_fastscan_topk(const uint8_t* blocks, int64_t n, int32_t D, const int8_t* lut,
                           int64_t top_n, int32_t mode, int64_t* out_idx,
                           int32_t* out_score);
/* The fastscan_topk selection rule applied to precomputed scores of vids 0..n-1. */
int64_t ousq_topk_from_scores(const int32_t* scores, int64_t n, int64_t top_n,
                              int64_t* out_idx, int32_t* out_score);
/* Integer rerank dot product sum(code_u8 * q_i8) (VNNI path, nbits 4 or 8). */
int32_t ousq_int_ip(const uint8_t* codes, int32_t D, int32_t nbits, const int8_t* q_i8);
/* score_with_meta for one stored vector. */
float ousq_score(const ousq_artifact_t* a, const float* q, int64_t row, int32_t mode);

/* ---- whole search ---- */
typedef struct ousq_index ousq_index_t;
ousq_index_t* ousq_index_create(const ousq_artifact_t* a);
void ousq_index_free(ousq_index_t* idx);

/* Batched search (queries are independent; threaded over queries).
 * out_ids/out_dists: nq*k, row-major.  Rows are padded to k with (-1, +inf)
 * except in POST mode, where each row holds its kept entries left-aligned and
 * out_counts[q] says how many (the reference concatenates those rows).
 * Bitsets: a pool of n_bitsets bitsets of bitset_len bits each (u64 words,
 * bit=1 => filtered); query_bitset[q] indexes the pool or is -1 (no filter).
 * query_bitset == NULL means every query uses bitset 0.
 * Debug outputs (may be NULL): probes[nq*nprobe] coarse order. */
int32_t ousq_search(const ousq_index_t* idx, const float* queries, int64_t nq, int32_t k,
                    int32_t nprobe, int32_t mode, int32_t filter_mode,
                    const uint64_t* bitsets, int64_t bitset_len, int64_t n_bitsets,
                    const int32_t* query_bitset, int32_t nthreads, int64_t* out_ids,
                    float* out_dists, int64_t* out_counts, int32_t* out_probes);

/* Per-query candidate dump for parity debugging: for query q, writes up to cap
 * (list, local_idx, fastscan_score_or_INT32_MIN, int_ip, distance) tuples in the
 * reference's candidate order.  Returns the candidate count. */
int64_t ousq_candidates(const ousq_index_t* idx, const float* query, int32_t k, int32_t nprobe,
                        int32_t mode, int32_t filter_mode, const uint64_t* bitset,
                        int64_t bitset_len, int64_t cap, int32_t* out_list,
                        int64_t* out_local, int32_t* out_fs, int32_t* out_int_ip,
                        float* out_dist);

#ifdef __cplusplus
}
#endif
#endif
