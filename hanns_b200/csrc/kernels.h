// kernels.h -- kernel argument blocks and launch wrappers shared by the host code.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

namespace hanns {

struct QueryParams;

struct CudaError : std::runtime_error {
    cudaError_t code;
    CudaError(cudaError_t c, const char* expr, const char* file, int line)
        : std::runtime_error(std::string(cudaGetErrorString(c)) + " in " + expr + " at " + file +
                             ":" + std::to_string(line)),
          code(c) {}
};

struct ScanArgs {
    // index (device)
    int D, nbits, code_bytes, nchunks, G, metric_l2;
    const int64_t* list_off;
    const int64_t* fs_blk_off;
    const uint2* fs;        // FastScan sign codes: [block][D/64][32 slots] x 8 bytes
    const uint8_t* codes;   // [ntotal][code_bytes]
    const float4* meta;     // [ntotal] {norm, norm_sq, vmax, quant_quality}
    const int64_t* ids;     // [ntotal]
    // queries
    const QueryParams* qp;
    const uint8_t* lut;     // [nq][G*16] offset-binary
    const uint8_t* q_i8p;   // [nq][D] dp4a layout
    // (list, query) grouping
    const int2* lq;         // (query, probe rank) grouped by list
    const int4* items;      // (list, first lq index, count, 0)
    const int* n_items;
    int* item_counter;
    // selection
    int k, n_cand, nprobe;
    int fused;
    const uint64_t* bitsets;
    int64_t bitset_len, bitset_words, n_bitsets;
    const int32_t* query_bitset;
    // outputs: every kept candidate of a (query, probe) pair, at
    // cand_*[q * q_stride + pair_off[q * (nprobe + 1) + rank] + j]; tie = rank << 48 |
    // FastScan key << 32 | list position; unused entries hold key ~0u, tie ~0ull
    const int* pair_off;
    int64_t q_stride;
    uint32_t* cand_key;
    uint64_t* cand_tie;
    // nullable (parity debugging): (int_ip, FastScan score or INT32_MIN when FastScan did
    // not select the row) of every kept candidate, at the same index as cand_key
    int2* cand_dbg;
    // FastScan scores scratch: per CTA, kScanWarps rows of max_len (the longest list)
    int16_t* scores;
    const float* q_rot;  // [nq][D]: the f32 rerank of nbits other than 4 and 8
    int max_len;
};

#ifdef __CUDACC__
#define HANNS_HD __host__ __device__
#else
#define HANNS_HD
#endif

// Lists of at most kTcMaxRows rows are scanned by the tensor-core kernel (scan_tc.cu),
// longer ones by the SIMT kernel.  A tensor-core item holds one list's rows in T =
// ceil(n / 128) tiles of 128 (the MMA's M) and up to 128 queries (the MMA's N, a multiple
// of 16).  Its GEMMs run over groups of G = min(T, kTcItemCols / N) tiles, whose
// accumulators fit in half of the TMEM.  A FastScan list (more than n_cand rows) takes
// 128 queries per item whatever its length; a rerank-only list at most kTcItemCols / T
// (one group: the kept-row bitmaps of all T tiles fit in shared memory).
constexpr int kTcMaxRows = 2048;
constexpr int kTcItemCols = 256;
HANNS_HD inline int tc_queries_per_item(long long n, bool fastscan) {
    if (fastscan) return 128;
    const int t = (int)((n + 127) / 128);
    const int q = (kTcItemCols / (t < 1 ? 1 : t)) & ~15;
    return q > 128 ? 128 : q;
}

// Tensor-core list scan (scan_tc.cu): the items flagged for it by the grouping step.
struct TcScanArgs {
    int D, nbits, code_bytes, G, metric_l2, nchunks;
    const int64_t* list_off;
    const int64_t* fs_blk_off;
    const uint2* fs;        // FastScan sign codes: [block][D/64][32 slots] x 8 bytes
    const uint8_t* codes;   // [ntotal][code_bytes]
    const float4* meta;
    const int64_t* ids;
    const QueryParams* qp;
    const uint8_t* lut;     // [nq][G*16] offset-binary
    const uint8_t* q_i8p;   // [nq][D] dp4a layout (4-bit: even then odd dims per 8)
    const int2* lq;
    const int4* items;
    const int* n_items;
    int* item_counter;
    int k, n_cand, nprobe, fused;
    const uint64_t* bitsets;
    int64_t bitset_len, bitset_words, n_bitsets;
    const int32_t* query_bitset;
    const int* pair_off;
    int64_t q_stride;
    uint32_t* cand_key;
    uint64_t* cand_tie;
    int2* cand_dbg;         // nullable, as in ScanArgs
    // FastScan pairs (|list| > n_cand): every row's score and int_ip to the FastScan scratch
    // at query * fs_stride + fs_off[query * nprobe + rank] (fs_select_kernel takes it from there)
    const int* fs_off;
    int64_t fs_stride;
    int16_t* fs_sc;
    int32_t* fs_ip;
    // nullable: per CTA kTcProfSlots nanosecond counters of where each role spends its time
    // (HANNS_GPU_SCAN_PROFILE=1; see scan_tc.cu)
    unsigned long long* prof;
    int* err_flag;          // set to a nonzero code when a bounded wait expired
    uint64_t wait_ns;       // limit of every wait on another role (2 s by default)
};

// Kept sets of the tensor-core FastScan pairs from the FastScan scratch (warp per pair): the
// reference heap's kept set of the 16-bit scores, each kept row's distance (from its int_ip)
// and tie to the pair's candidate region.
struct FsSelectArgs {
    int64_t nq;
    int nprobe, n_cand, nbits, metric_l2, fused;
    const int32_t* probes;
    const int64_t* list_off;
    const int64_t* ids;
    const float4* meta;
    const QueryParams* qp;
    const int* fs_off;
    int64_t fs_stride;
    const int16_t* fs_sc;
    const int32_t* fs_ip;
    const int* pair_off;
    int64_t q_stride;
    const uint64_t* bitsets;
    int64_t bitset_len, bitset_words, n_bitsets;
    const int32_t* query_bitset;
    uint32_t* cand_key;
    uint64_t* cand_tie;
    int2* cand_dbg;  // nullable
    // the grouping step's pairs (this rank's, grouped by list) and their number
    const int2* lq;
    const int* n_lq;
};
void launch_fs_select(const FsSelectArgs& a, int grid, cudaStream_t s);

// USQ rerank of caller-chosen stored rows: out[q * m + j] = distance of row rows[q*m+j]
// (+inf for rows outside [0, ntotal)).
struct RerankRowsArgs {
    int D, nbits, code_bytes, metric_l2;
    const uint8_t* codes;
    const float4* meta;
    int64_t ntotal;
    const QueryParams* qp;
    const uint8_t* q_i8p;
    const int64_t* rows;
    int64_t nq;
    int m;
    float* out;
};
void launch_rerank_rows(const RerankRowsArgs& a, cudaStream_t s);

// Per (query, probe) pair top-k of the scan's candidate regions into a compact region
// of nprobe * k entries per query (slot rank * k).
struct CompactArgs {
    int64_t nq;
    int nprobe, k;
    const uint32_t* cand_key;
    const uint64_t* cand_tie;
    const int* pair_off;
    int64_t q_stride;
    uint32_t* out_key;
    uint64_t* out_tie;
};

struct MergeArgs {
    int64_t nq;
    int nprobe, k, nlist;
    const uint32_t* cand_key;  // candidate regions written by the list scan (or compacted)
    const uint64_t* cand_tie;
    const int* pair_off;
    int64_t q_stride;
    int fixed_total;  // > 0: every query has this many entries (compact regions)
    const int32_t* probes;
    const int64_t* list_off;
    const int64_t* ids;
    uint32_t* sel_key;  // [nq][k] scratch
    uint64_t* sel_tie;  // [nq][k] scratch
    int64_t* out_ids;
    float* out_dists;
    int64_t* out_counts;
    // post filter (reference semantics) -- NULL when unused
    const uint64_t* post_bitsets;
    int64_t bitset_len, bitset_words, n_bitsets;
    const int32_t* query_bitset;
    // shard mode: also emit merge keys
    int shard_mode;
    uint64_t* out_keys;
};

// Records the message returned by hanns_gpu_last_error() on this thread.
void set_last_error(const std::string& msg);

// search stages
void launch_coarse_l2(const float* q, int64_t nq, const float* cent, int nlist, int d, float* dist,
                      cudaStream_t s);
void launch_select_probes(const float* dist, int64_t nq, int nlist, int nprobe, int32_t* probes,
                          uint32_t* scratch, cudaStream_t s);
// Approximate-then-exact coarse step (same probes as the two launches above).
void launch_coarse_gemm(const float* q, int64_t nq, const float* cent, const float* cn, int nlist,
                        int d, float* approx, cudaStream_t s);
// Candidates per query handed from the select kernel to the ordering kernel; rs holds
// nq x kCoarseRsStride ints (count, ||q||^2 bits, kCoarseRescoreMax centroid ids,
// kCoarseRescoreMax approximate-score bits).  rs may be null (the select kernel then
// re-scores every candidate itself).
constexpr int kCoarseRescoreMax = 64;
constexpr int kCoarseRsStride = 2 + 2 * kCoarseRescoreMax;
int launch_coarse_select(float* approx, const float* q, int64_t nq, const float* cent, int nlist,
                          int d, int nprobe, float cmax, float dot_rel, const int* tc_err,
                          int32_t* probes, int* fallbacks, int* rs, cudaStream_t s);
// Tensor-core approximation of the coarse scores (coarse_tc.cu).
int coarse_tc_k(int d);
void launch_split_bf16(const float* x, int64_t rows, int d, int K, void* hi, void* lo,
                       cudaStream_t s);
bool launch_coarse_tc(const void* qh, const void* ql, int64_t nq, const void* ch, const void* cl,
                      int nlist, int K, const float* cn, float* out, int* err_flag,
                      cudaStream_t s);
void launch_centroid_norms(const float* cent, int nlist, int d, float* cn, cudaStream_t s);
// q_rot = P * pad(x) in the reference's FMA order; Pc is P in chain-major order
// (launch_rotation_chain_major).
void launch_rotation_chain_major(const float* P, int D, float* Pc, cudaStream_t s);
void launch_rotate(const float* x, int64_t nq, int d, int D, const float* Pc, float* out,
                   cudaStream_t s);
void launch_query_state(const float* x, const float* q_rot, int64_t nq, int d, int D,
                        const float* rc, int nbits, QueryParams* qp, uint8_t* q_i8p,
                        int8_t* q_i8n, uint8_t* lut, cudaStream_t s);
// Items (list, first lq index, queries, kind): lists of at most tc_max_rows rows (0:
// none) become tensor-core items (kind 1) of tc_queries_per_item(|list|, |list| > n_cand)
// queries, the
// others SIMT items (kind 0) of qpi queries.  Items and pairs are laid out list by list in
// `order` (a permutation of the lists, or null for list order); every item and pair
// writes to places fixed by its (query, probe), so the order changes no result, only
// which items the persistent scans claim first.
void launch_group_pairs(const int32_t* probes, int64_t nq, int nprobe, int nlist,
                        const uint8_t* owned, const int64_t* list_off, const int* order,
                        int tc_max_rows, int n_cand,
                        int qpi, int* cnt, int* cursor, int* lq_off, int* item_off, int* n_items,
                        int2* lq, int4* items, cudaStream_t s);
// pair_off[q][r] = sum over earlier probes of min(|list|, n_cand) (0 for lists this
// index does not own); pair_off[q][nprobe] = the query's candidate total
// pair_off: per query the candidate regions of its probes (min(|list|, n_cand) entries each,
// min(|list|, n_cand, fs_keep) for the FastScan pairs PairTrunc truncates).
// fs_off (nullable): per (query, probe) the offset of a tensor-core FastScan pair (n_cand <
// |list| <= tc_rows) in the query's region of the FastScan scratch (|list| entries each), -1
// for other pairs.
// Lists of at most kFsRegRows rows take fs_select's register path (scores in registers,
// kept rows in a per-warp shared buffer of kFsRegRows entries).
constexpr int kFsRegRows = 1024;
// Region truncation of the FastScan pairs: with fs_keep > 0 (k < n_cand <= kFsRegRows / 2,
// no debug candidates) every FastScan pair on fs_select's register path -- |list| <=
// kFsRegRows and no fused filter for its query -- gets a region of min(n_cand, fs_keep)
// entries, and fs_select writes the pair's top fs_keep there.
struct PairTrunc {
    int fs_keep = 0;
    int fused = 0;
    const uint64_t* bitsets = nullptr;
    int64_t n_bitsets = 0;
    const int32_t* query_bitset = nullptr;
};
void launch_pair_offsets(const int32_t* probes, int64_t nq, int nprobe, const int64_t* list_off,
                         int nlist, const uint8_t* owned, int n_cand, int* pair_off, int tc_rows,
                         int* fs_off, const PairTrunc& tr, cudaStream_t s);
size_t scan_smem_bytes(int D);
size_t scan_tc_smem_bytes();
constexpr int kTcProfSlots = 16;
void launch_scan_tc(const TcScanArgs& a, int grid, cudaStream_t s);
int scan_grid_size(int D);
void launch_scan(const ScanArgs& a, int grid, cudaStream_t s);
void launch_compact_pairs(const CompactArgs& a, cudaStream_t s);
void launch_merge(const MergeArgs& a, cudaStream_t s);
// Over the scan's candidate regions (no compaction), eight queries per block; k <= kMergeMaxK.
// sel_key / sel_tie: [nq][k] scratch.
constexpr int kMergeMaxK = 1024;
void launch_merge_direct(const MergeArgs& a, cudaStream_t s);
void launch_merge_shards(const float* dists, const uint64_t* keys, const int64_t* ids, int world,
                         int64_t nq, int k, int64_t* out_ids, float* out_dists, cudaStream_t s);

// build stages
void launch_global_mean(const float* x, int64_t n, int d, float* out, cudaStream_t s);
void launch_row_norm_sq(const float* x, int64_t n, int d, float* out, cudaStream_t s);
void launch_residual_pad(const float* x, int64_t n, int d, int D, const float* centroid, float* out,
                         cudaStream_t s);
void launch_encode_rotated(const float* rotated, int64_t n, int D, int nbits,
                           const float* norm_sq_raw, uint8_t* codes, uint8_t* signs, float4* meta,
                           cudaStream_t s);
void launch_argmin_rows(const float* dist, int64_t n, int nlist, int32_t* out, cudaStream_t s);
void launch_kmeans_accumulate(const float* x, int64_t n, int d, const int32_t* assign,
                              long long* sums, int* counts, cudaStream_t s);
void launch_kmeans_update(const long long* sums, const int* counts, int nlist, int d,
                          float* centroids, float* shift, cudaStream_t s);
// k-means++ seeding steps (build_kernels.cu): blocks of the distance pass for n rows, the
// min-distance reset, and one step (distances to centroid slot-1, draw of centroid slot).
int kpp_blocks(int64_t n, int64_t* per);
void launch_kpp_init_min(float* min_d, int64_t n, cudaStream_t s);
void launch_kpp_step(const float* x, int64_t n, int d, float* cent, int slot, float* min_d,
                     double* block_sum, double u_target, double u_uniform, cudaStream_t s);
void launch_build_fastscan(const uint8_t* signs, const int64_t* list_off, const int64_t* blk_off,
                           int nlist, int D, uint2* fs, cudaStream_t s);
void launch_gather_rows(const uint8_t* src, const int64_t* perm, int64_t n, int64_t row_bytes,
                        uint8_t* dst, cudaStream_t s);

}  // namespace hanns
