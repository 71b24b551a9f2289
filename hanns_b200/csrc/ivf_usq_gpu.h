// ivf_usq_gpu.h -- host-side IVF-USQ index living on one B200.
//
// Mirrors IvfUsqIndex (reference src/faiss/ivf_usq.rs:118-127, 170-352): config,
// train (k-means + global mean), add (assign + USQ encode + per-list layout), search.
// The search path runs entirely on the GPU; there is no CPU fallback.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <deque>
#include <mutex>
#include <string>
#include <vector>

#include "kernels.h"

namespace hanns {

struct QueryParams;

// Host-side fault injection (tests of the error paths; no device is ever faulted): a bit
// set here makes the next device allocations (kFaultAlloc) or host-to-device copies
// (kFaultH2D) fail as if the CUDA call had returned an error.  Set by
// hanns_gpu_debug_inject_fault or, at load, by HANNS_GPU_FAULT=alloc|h2d.
constexpr int kFaultAlloc = 1, kFaultH2D = 2;
bool fault_injected(int what);
void set_fault_injection(int mask);

// Grow-only device buffer.
template <class T>
struct DevBuf {
    T* p = nullptr;
    size_t n = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    ~DevBuf() { release(); }
    void release() {
        if (p) cudaFree(p);
        p = nullptr;
        n = 0;
    }
    void reserve(size_t count) {
        if (count <= n && p) return;
        release();
        if (count == 0) count = 1;
        cudaError_t e = fault_injected(kFaultAlloc) ? cudaErrorMemoryAllocation
                                                    : cudaMalloc(&p, count * sizeof(T));
        if (e != cudaSuccess) {
            p = nullptr;
            throw CudaError(e, "cudaMalloc", __FILE__, __LINE__);
        }
        n = count;
    }
    void swap(DevBuf& o) {
        std::swap(p, o.p);
        std::swap(n, o.n);
    }
};

struct SearchOptions {
    int k = 10;
    int nprobe = 8;
    int filter_mode = 0;  // 0 none, 1 post (reference), 2 fused
    const uint64_t* d_bitsets = nullptr;  // device
    int64_t bitset_len = 0;
    int64_t n_bitsets = 0;
    const int32_t* d_query_bitset = nullptr;  // device or null
    bool shard_output = false;                // emit merge keys (multi-GPU)
};

// Per-query search state of a batch (device pointers): probes [nq][nprobe], scalars [nq],
// FastScan LUT [nq][D/4*16] (offset-binary), q_i8 in the dp4a layout [nq][D], q_i8 in
// dimension order [nq][D].
struct QueryState {
    int32_t* probes;
    QueryParams* qp;
    uint8_t* lut;
    uint8_t* q_i8p;
    int8_t* q_i8n;
};

class IvfUsqGpu {
   public:
    IvfUsqGpu(int dim, int nlist, int nbits, int metric, uint64_t rotation_seed, int nprobe,
              int device);
    ~IvfUsqGpu();

    // Frozen-artifact import / export (list order).
    void import_artifact(const void* artifact /* hanns_ivf_usq_artifact_t* */);
    void export_artifact(void* artifact /* hanns_ivf_usq_artifact_t* (destinations) */) const;

    void train(const float* h_data, int64_t n, int kmeans_iters, uint64_t kmeans_seed);
    void add(const float* h_data, int64_t n, const int64_t* h_ids);

    // All pointers device; synchronises the stream before returning.
    void search_device(const float* d_queries, int64_t nq, const SearchOptions& opt, int64_t* d_ids,
                       float* d_dists, int64_t* d_counts, uint64_t* d_keys, cudaStream_t stream);
    // Host pointers (copies in and out).
    void search_host(const float* h_queries, int64_t nq, const SearchOptions& opt,
                     const uint64_t* h_bitsets, const int32_t* h_query_bitset, int64_t* h_ids,
                     float* h_dists, int64_t* h_counts);

    // Per-query stages only (coarse probes, rotation, query state) into st (q_i8n may be
    // null); synchronises the stream.
    void prepare_device(const float* d_queries, int64_t nq, int nprobe, QueryState st,
                        cudaStream_t stream);
    // Grouping, list scan and merge over query state made by prepare_device (of this index
    // or of another shard of it); synchronises the stream.
    // USQ distances of caller-chosen stored rows (storage order) for nq device queries:
    // query state (rotation, q_i8, scalars) then the integer rerank and score epilogue.
    void rerank_rows_device(const float* d_queries, int64_t nq, const int64_t* d_rows, int m,
                            float* d_dists, cudaStream_t stream);
    void search_prepared_device(int64_t nq, const SearchOptions& opt, QueryState st,
                                int64_t* d_ids, float* d_dists, int64_t* d_counts,
                                uint64_t* d_keys, cudaStream_t stream);
    // Bytes per query of the five QueryState arrays.
    void query_state_bytes(int nprobe, int64_t* parts) const;

    void debug_query(const float* h_queries, int64_t nq, int nprobe, int32_t* probes, float* q_rot,
                     int8_t* q_i8, int8_t* lut, float* scalars);
    // The list scan's kept candidates of nq host queries (one internal batch), each query's
    // in the reference's candidate order (probe order; inside a list that ran FastScan,
    // score descending then position): list, position in the list, FastScan score
    // (INT32_MIN where FastScan did not select the row), int_ip and distance, at q * cap;
    // counts[q] = the query's candidates.  Throws if a query has more than cap.
    void debug_candidates(const float* h_queries, int64_t nq, const SearchOptions& opt,
                          const uint64_t* h_bitsets, const int32_t* h_query_bitset, int64_t cap,
                          int64_t* counts, int32_t* lists, int64_t* local, int32_t* fs,
                          int32_t* int_ip, float* dists);

    void shard(int rank, int world);
    void save(const std::string& path) const;
    void load(const std::string& path);

    int dim() const { return dim_; }
    int padded_dim() const { return D_; }
    int nbits() const { return nbits_; }
    int nlist() const { return nlist_; }
    int metric() const { return metric_; }
    int nprobe() const { return nprobe_; }
    void set_nprobe(int p) { nprobe_ = p < 1 ? 1 : (p > nlist_ ? nlist_ : p); }
    void set_scan_wait_ns(uint64_t ns) { scan_wait_ns_ = ns; }
    bool trained() const { return trained_; }
    int64_t count() const { return ntotal_; }
    int64_t size_bytes() const;
    int device() const { return device_; }
    // Per-stage device ms (coarse GEMM, coarse select, rotate, query state, group, scan,
    // merge, total) summed over the last n_calls search / prepare calls; waits for their
    // events.  counts (nullable): batches that timed each stage.  Returns the number of
    // calls covered (calls older than the event ring are not).
    int stage_ms(int n_calls, float* out, int* counts = nullptr);
    // device ms of the list scan's kernels {tensor-core scan, SIMT scan, FastScan selection}
    // summed over the batches of the last n_calls calls; counts3: batches timed
    int scan_kernel_ms(int n_calls, float* out3, int* counts3);
    int64_t last_launches() const { return last_launches_; }
    std::mutex& mutex() { return mu_; }

   private:
    void check_supported() const;
    void check_int_rerank(const char* what) const;  // 4-bit / 8-bit only
    void upload_rotation_centroid();
    void rebuild_fastscan();
    void ensure_stream();
    // d_q: device query rows.  h_q (nullable): host rows to upload into d_q first, in chunks
    // on copy_stream_ that overlap the per-query stages of the preceding chunk.
    void search_batch(const float* d_q, const float* h_q, int64_t nb, const SearchOptions& opt,
                      int64_t* d_ids, float* d_dists, int64_t* d_counts, uint64_t* d_keys,
                      cudaStream_t s, bool time_it);
    int64_t prepare_batch(const float* d_q, const float* h_q, int64_t nb, int nprobe,
                          const QueryState& st, cudaStream_t s, bool time_it);
    int64_t scan_merge_batch(int64_t nb, const SearchOptions& opt, const QueryState& st,
                             int64_t* d_ids, float* d_dists, int64_t* d_counts, uint64_t* d_keys,
                             cudaStream_t s, bool time_it);
    // Stage events: each search batch takes the next slot of a ring (ev_ / ev_aux_ point into
    // it), so that calls need not wait for the device before their events are reused.
    void begin_call();
    void next_slot(int first, int last);
    void check_tc_scan();
    void run_search(const float* d_queries, const float* h_queries, int64_t nq,
                    const SearchOptions& opt, int64_t* d_ids, float* d_dists, int64_t* d_counts,
                    uint64_t* d_keys, cudaStream_t stream);
    void set_list_layout(const std::vector<int64_t>& h_off);
    int64_t cand_stride(int nprobe, int k) const;
    // lists of at most this many rows take the tensor-core scan (HANNS_GPU_SCAN: default all
    // lists up to kTcMaxRows, =hybrid only those without FastScan, =simt none)
    int scan_tc_rows(int n_cand) const;
    // entries of one query's region of the FastScan scratch: the nprobe longest lists that
    // the tensor-core scan runs FastScan on (n_cand < |list| <= tc_rows); cached
    int64_t fs_stride(int nprobe, int n_cand, int tc_rows);
    // queries per internal batch: candidate regions and FastScan scratch within budget
    int64_t batch_limit(int nprobe, int k);
    int fs_stride_key_[3] = {-1, -1, -1};
    int64_t fs_stride_val_ = 0;
    void update_centroid_norms();
    // returns the number of kernels launched
    int64_t coarse_probes(const float* d_q, int64_t nb, int nprobe, int32_t* d_probes,
                          cudaStream_t s, cudaEvent_t mid_event = nullptr);

    int dim_, D_, nbits_, nlist_, metric_, nprobe_, device_;
    uint64_t rotation_seed_;
    bool trained_ = false;
    int64_t ntotal_ = 0;
    int code_bytes_;

    // device artifact (list order)
    DevBuf<float> centroids_, P_, rc_, gmean_, cn_;
    DevBuf<float> Pc_;  // P in the rotation kernel's chain-major order (refresh_rotation())
    void refresh_rotation();
    float cmax_ = 0.0f;  // max ||centroid|| (bound of the approximate coarse step)
    DevBuf<uint16_t> cent_hi_, cent_lo_;  // bf16 split of the centroids [nlist][tc_k_]
    int tc_k_ = 64;
    DevBuf<int64_t> list_off_, fs_blk_off_, ids_;
    // the lists by decreasing length (stable): the order in which the grouping step lays
    // out the scan's items, so the persistent scans claim the longest lists first
    DevBuf<int> list_order_;
    DevBuf<float4> meta_;
    DevBuf<uint8_t> codes_, signs_, owned_;
    DevBuf<uint2> fs_;
    std::vector<int64_t> h_list_off_;
    int max_list_ = 0;
    bool sharded_ = false;

    // search workspace
    DevBuf<float> w_dist_, w_qrot_, w_pad_queries_;
    DevBuf<uint32_t> w_sel_, w_mkey_;
    DevBuf<int32_t> w_probes_;
    DevBuf<QueryParams> w_qp_;
    DevBuf<uint8_t> w_qi8p_, w_lut_;
    DevBuf<int8_t> w_qi8n_;
    DevBuf<int> w_cnt_, w_cursor_, w_lq_off_, w_item_off_, w_counters_, w_pair_off_, w_rs_;
    DevBuf<int2> w_lq_;
    DevBuf<int4> w_items_;
    DevBuf<uint64_t> w_mtie_, w_cand_tie_, w_bits_;
    DevBuf<int16_t> w_scores_;
    DevBuf<uint32_t> w_cand_key_;
    DevBuf<uint32_t> w_cmp_key_;  // per (query, probe) top-k, nprobe * k per query
    DevBuf<uint64_t> w_cmp_tie_;
    DevBuf<int32_t> w_qbits_;
    DevBuf<int64_t> w_out_ids_, w_out_counts_;
    DevBuf<float> w_out_dists_;

    cudaStream_t stream_ = nullptr;
    cudaStream_t copy_stream_ = nullptr;  // host->device query upload
    cudaStream_t aux_stream_ = nullptr;   // rotation + query state, beside the coarse step
    cudaEvent_t ev_fork_ = nullptr, ev_join_ = nullptr;

    static constexpr int kMaxUploadChunks = 8;
    cudaEvent_t ev_up_[kMaxUploadChunks] = {};
    cudaEvent_t ev_ready_ = nullptr;  // copy_stream_ waits for earlier work on the search stream
    int* h_scan_err_ = nullptr;       // pinned: error code of the tensor-core list scan
    cudaEvent_t ev_scan_err_ = nullptr;  // completes when h_scan_err_ holds the last scan's code
    bool debug_candidates_ = false;      // scans also write (int_ip, FastScan score) per candidate
    uint64_t scan_wait_ns_ = 2000000000ull;  // tensor-core scan: limit of each wait on a role
    DevBuf<int2> w_cand_dbg_;
    DevBuf<int> w_fs_off_;       // per (query, probe): place in the FastScan scratch, -1: none
    DevBuf<int16_t> w_fs_sc_;    // FastScan scratch: scores of every row of FastScan pairs
    DevBuf<int32_t> w_fs_ip_;    //                   and their int_ip
    DevBuf<unsigned long long> w_tc_prof_;  // tensor-core scan: role time counters (profiling)
    DevBuf<int> w_scan_err_;
    int sm_count_ = 0;
    // stages: coarse GEMM, coarse select, rotate, query state, group, scan, merge; then total
    static constexpr int kStages = 7;
    static constexpr int kEvRing = 64;
    struct StageSlot {
        cudaEvent_t ev[kStages + 1] = {};
        cudaEvent_t aux[3] = {};  // rotation start / end, query state end (aux stream)
        bool aux_timed = false;
        // inside the list scan: before the tensor-core kernel, after it, after the SIMT scan,
        // after the FastScan selection
        cudaEvent_t kt[4] = {};
        bool kt_timed = false;
        int first = 0, last = 0;  // events first..last were recorded
    };
    StageSlot ring_[kEvRing];
    int64_t slot_seq_ = 0;                           // slots handed out so far
    std::deque<std::pair<int64_t, int>> calls_;      // (first slot, slot count) per call
    StageSlot* cur_ = &ring_[0];
    cudaEvent_t* ev_ = ring_[0].ev;
    cudaEvent_t* ev_aux_ = ring_[0].aux;
    bool used_tc_ = false;  // the last scan ran the tensor-core kernel (host reads its error flag)
    int64_t last_launches_ = 0;
    DevBuf<int> w_fallbacks_;  // [0] exact fallbacks, [1] tensor-core error flag
    DevBuf<uint16_t> w_qhi_, w_qlo_;
    int scan_grid_ = 0;
    std::mutex mu_;
};

// Seeded uniform [-1,1) matrix -> Householder QR -> Q (row-major, f32), the method of
// src/quantization/usq/rotator.rs:15-39 with this library's own random stream.
void rotation_matrix(uint64_t seed, int D, float* out);

// List -> rank assignment used by IvfUsqGpu::shard (host only).
void shard_owners(const int64_t* sizes, int nlist, int world, int32_t* owner);

}  // namespace hanns
