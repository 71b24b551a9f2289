// ivf_usq_gpu.cu -- host orchestration of the IVF-USQ index on one GPU.
#include "ivf_usq_gpu.h"

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <fstream>
#include <numeric>
#include <stdexcept>

#include "common.cuh"
#include "hanns_gpu.h"

namespace hanns {

namespace {
// Candidate regions of one internal batch: 12 bytes per entry, at most 16 GiB (of the
// 180 GB HBM); per-query kernels index queries in grid.y in tiles of >= 8, so 262,144
// queries per batch stay inside the 65,535 grid.y limit.
constexpr int64_t kCandBudget = 16ll << 30;
constexpr int64_t kFsBudget = 16ll << 30;  // FastScan scratch: 6 bytes per entry
constexpr int64_t kMaxBatch = 262144;
}  // namespace

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) HANNS_CUDA_OK(cudaSetDevice(dev));
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

int padded_of(int d) { return (d + 63) / 64 * 64; }

int64_t n_candidates(int nbits, int64_t k) {
    if (nbits == 1) return std::max<int64_t>(k * 20, 200);
    if (nbits >= 2 && nbits <= 4) return std::max<int64_t>(k * 15, 150);
    return std::max<int64_t>(k * 30, 300);
}

template <class T>
void h2d(DevBuf<T>& b, const T* src, size_t count, cudaStream_t s) {
    b.reserve(count);
    if (count && fault_injected(kFaultH2D))
        throw CudaError(cudaErrorInvalidValue, "cudaMemcpyAsync (injected host-to-device fault)",
                        __FILE__, __LINE__);
    if (count) HANNS_CUDA_OK(cudaMemcpyAsync(b.p, src, count * sizeof(T), cudaMemcpyHostToDevice, s));
}

std::atomic<int>& fault_mask() {
    static std::atomic<int> m{[] {
        const char* e = std::getenv("HANNS_GPU_FAULT");
        if (!e) return 0;
        return (std::strcmp(e, "alloc") == 0 ? kFaultAlloc : 0) | (std::strcmp(e, "h2d") == 0 ? kFaultH2D : 0);
    }()};
    return m;
}

constexpr int kQueriesPerItem = 32;

}  // namespace

// Entries of one query's candidate region: the probes' min(|list|, n_cand) summed is at
// most nprobe * min(n_cand, longest list) and at most the index size.
bool fault_injected(int what) { return (fault_mask().load(std::memory_order_relaxed) & what) != 0; }
void set_fault_injection(int mask) { fault_mask().store(mask); }

int64_t IvfUsqGpu::cand_stride(int nprobe, int k) const {
    const int64_t per = std::min<int64_t>(n_candidates(nbits_, k), std::max(max_list_, 1));
    const int64_t st = std::max<int64_t>(1, std::min<int64_t>((int64_t)nprobe * per, std::max<int64_t>(ntotal_, 1)));
    if (st > (int64_t)INT32_MAX) throw std::invalid_argument("nprobe x candidates per probe too large");
    return st;
}

int IvfUsqGpu::scan_tc_rows(int n_cand) const {
    if (nbits_ != 4 && nbits_ != 8) return 0;  // (the f32 reranks run on the SIMT scan)
    const char* mode = std::getenv("HANNS_GPU_SCAN");
    if (mode && std::strcmp(mode, "simt") == 0) return 0;
    if (mode && std::strcmp(mode, "hybrid") == 0) return std::min(kTcMaxRows, n_cand);
    return kTcMaxRows;
}

int64_t IvfUsqGpu::fs_stride(int nprobe, int n_cand, int tc_rows) {
    if (tc_rows <= n_cand) return 0;
    if (fs_stride_key_[0] == nprobe && fs_stride_key_[1] == n_cand && fs_stride_key_[2] == tc_rows)
        return fs_stride_val_;
    std::vector<int64_t> sz;
    for (int l = 0; l < nlist_; ++l) {
        const int64_t n = h_list_off_[l + 1] - h_list_off_[l];
        if (n > n_cand && n <= tc_rows) sz.push_back((n + 7) & ~7ll);  // (regions padded to 8)
    }
    const size_t m = std::min<size_t>(sz.size(), (size_t)nprobe);
    std::partial_sort(sz.begin(), sz.begin() + m, sz.end(), std::greater<int64_t>());
    int64_t sum = 0;
    for (size_t i = 0; i < m; ++i) sum += sz[i];
    fs_stride_key_[0] = nprobe;
    fs_stride_key_[1] = n_cand;
    fs_stride_key_[2] = tc_rows;
    fs_stride_val_ = sum;
    return sum;
}

int64_t IvfUsqGpu::batch_limit(int nprobe, int k) {
    // candidate regions: 12 bytes per entry; FastScan scratch: 6 bytes per entry
    int64_t nb = std::max<int64_t>(1, kCandBudget / (cand_stride(nprobe, k) * 12));
    const int n_cand = (int)n_candidates(nbits_, k);
    const int64_t fs = fs_stride(nprobe, n_cand, scan_tc_rows(n_cand));
    if (fs > 0) nb = std::min<int64_t>(nb, std::max<int64_t>(1, kFsBudget / (fs * 6)));
    return std::min<int64_t>(nb, kMaxBatch);
}

IvfUsqGpu::IvfUsqGpu(int dim, int nlist, int nbits, int metric, uint64_t rotation_seed, int nprobe,
                     int device)
    : dim_(dim), nbits_(nbits), nlist_(nlist), metric_(metric), device_(device),
      rotation_seed_(rotation_seed) {
    if (dim <= 0) throw std::invalid_argument("dim must be > 0");
    if (nlist <= 0) throw std::invalid_argument("nlist must be > 0");
    if (nbits < 1 || nbits > 8) throw std::invalid_argument("nbits must be 1..=8");
    D_ = padded_of(dim);
    code_bytes_ = (D_ * nbits + 7) / 8;
    nprobe_ = std::max(1, std::min(nprobe, nlist));
    DeviceGuard g(device_);
    ensure_stream();
    set_list_layout(std::vector<int64_t>(nlist_ + 1, 0));
    owned_.reserve(nlist_);
    HANNS_CUDA_OK(cudaMemsetAsync(owned_.p, 1, nlist_, stream_));
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
}

IvfUsqGpu::~IvfUsqGpu() {
    cudaSetDevice(device_);
    for (auto& sl : ring_) {
        for (auto& e : sl.ev)
            if (e) cudaEventDestroy(e);
        for (auto& e : sl.aux)
            if (e) cudaEventDestroy(e);
    }
    for (auto& e : ev_up_)
        if (e) cudaEventDestroy(e);
    if (ev_ready_) cudaEventDestroy(ev_ready_);
    if (ev_scan_err_) cudaEventDestroy(ev_scan_err_);
    if (ev_fork_) cudaEventDestroy(ev_fork_);
    if (ev_join_) cudaEventDestroy(ev_join_);
    if (aux_stream_) cudaStreamDestroy(aux_stream_);
    if (h_scan_err_) cudaFreeHost(h_scan_err_);
    if (copy_stream_) cudaStreamDestroy(copy_stream_);
    if (stream_) cudaStreamDestroy(stream_);
}

void IvfUsqGpu::ensure_stream() {
    if (!stream_) {
        HANNS_CUDA_OK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
        HANNS_CUDA_OK(cudaStreamCreateWithFlags(&copy_stream_, cudaStreamNonBlocking));
        HANNS_CUDA_OK(cudaStreamCreateWithFlags(&aux_stream_, cudaStreamNonBlocking));
        HANNS_CUDA_OK(cudaEventCreateWithFlags(&ev_fork_, cudaEventDisableTiming));
        HANNS_CUDA_OK(cudaEventCreateWithFlags(&ev_join_, cudaEventDisableTiming));
        for (auto& sl : ring_) {
            for (auto& e : sl.aux) HANNS_CUDA_OK(cudaEventCreate(&e));
            for (auto& e : sl.kt) HANNS_CUDA_OK(cudaEventCreate(&e));
            for (auto& e : sl.ev) HANNS_CUDA_OK(cudaEventCreate(&e));
        }
        for (auto& e : ev_up_) HANNS_CUDA_OK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        HANNS_CUDA_OK(cudaEventCreateWithFlags(&ev_ready_, cudaEventDisableTiming));
        HANNS_CUDA_OK(cudaEventCreateWithFlags(&ev_scan_err_, cudaEventDisableTiming));
        HANNS_CUDA_OK(cudaHostAlloc(reinterpret_cast<void**>(&h_scan_err_), sizeof(int),
                                    cudaHostAllocDefault));
        *h_scan_err_ = 0;
        HANNS_CUDA_OK(cudaDeviceGetAttribute(&sm_count_, cudaDevAttrMultiProcessorCount, device_));
    }
}

void IvfUsqGpu::check_supported() const {
    if (nbits_ < 1 || nbits_ > 8) throw std::domain_error("IVF-USQ codes of 1 to 8 bits only");
}

void IvfUsqGpu::check_int_rerank(const char* what) const {
    check_supported();
    if (nbits_ != 4 && nbits_ != 8)
        throw std::domain_error(std::string(what) + ": 4-bit and 8-bit codes only in this build "
                                "(other widths: single-GPU search)");
}

int64_t IvfUsqGpu::size_bytes() const {
    // Same accounting as IvfUsqIndex::size (src/faiss/ivf_usq.rs:208-222).
    return (int64_t)nlist_ * dim_ * 4 + ntotal_ * (8 + 16 + (int64_t)code_bytes_);
}

void IvfUsqGpu::set_list_layout(const std::vector<int64_t>& h_off) {
    h_list_off_ = h_off;
    fs_stride_key_[0] = -1;
    max_list_ = 1;
    std::vector<int64_t> blk(nlist_ + 1, 0);
    for (int l = 0; l < nlist_; ++l) {
        const int64_t len = h_off[l + 1] - h_off[l];
        max_list_ = (int)std::max<int64_t>(max_list_, len);
        blk[l + 1] = blk[l] + (len + 31) / 32;
    }
    std::vector<int> order(nlist_);
    for (int l = 0; l < nlist_; ++l) order[l] = l;
    std::stable_sort(order.begin(), order.end(), [&](int x, int y) {
        return h_off[x + 1] - h_off[x] > h_off[y + 1] - h_off[y];
    });
    h2d(list_off_, h_off.data(), h_off.size(), stream_);
    h2d(fs_blk_off_, blk.data(), blk.size(), stream_);
    if (nlist_ > 0) h2d(list_order_, order.data(), order.size(), stream_);
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
}

void IvfUsqGpu::rebuild_fastscan() {
    int64_t blocks = 0;
    for (int l = 0; l < nlist_; ++l) blocks += (h_list_off_[l + 1] - h_list_off_[l] + 31) / 32;
    const size_t words = (size_t)std::max<int64_t>(blocks, 1) * (D_ / 64) * 32;
    fs_.reserve(words);
    HANNS_CUDA_OK(cudaMemsetAsync(fs_.p, 0, words * sizeof(uint2), stream_));
    launch_build_fastscan(signs_.p, list_off_.p, fs_blk_off_.p, nlist_, D_, fs_.p, stream_);
    HANNS_CUDA_OK(cudaGetLastError());
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
}

void IvfUsqGpu::update_centroid_norms() {
    cn_.reserve(nlist_);
    launch_centroid_norms(centroids_.p, nlist_, dim_, cn_.p, stream_);
    // bf16 hi/lo split of the centroids for the tensor-core coarse approximation
    tc_k_ = coarse_tc_k(dim_);
    cent_hi_.reserve((size_t)nlist_ * tc_k_);
    cent_lo_.reserve((size_t)nlist_ * tc_k_);
    launch_split_bf16(centroids_.p, nlist_, dim_, tc_k_, cent_hi_.p, cent_lo_.p, stream_);
    HANNS_CUDA_OK(cudaGetLastError());
    std::vector<float> h(nlist_);
    HANNS_CUDA_OK(cudaMemcpyAsync(h.data(), cn_.p, sizeof(float) * nlist_, cudaMemcpyDeviceToHost,
                                  stream_));
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
    float m = 0.0f;
    for (float v : h) m = (v != v) ? INFINITY : std::max(m, v);
    cmax_ = std::sqrt(m);
}

// Probes of nb device queries: approximate scores (tcgen05 bf16x3 GEMM, or the FP32 SIMT
// GEMM) + exact re-score, in chunks bounded by the approximation matrix (1 GiB).
int64_t IvfUsqGpu::coarse_probes(const float* d_q, int64_t nb, int nprobe, int32_t* d_probes,
                                  cudaStream_t s, cudaEvent_t mid_event) {
    int64_t launches = 0;
    const int64_t cchunk = std::max<int64_t>(1, std::min<int64_t>(nb, (1ll << 28) / nlist_));
    w_dist_.reserve((size_t)cchunk * nlist_);
    w_fallbacks_.reserve(2);
    w_rs_.reserve((size_t)cchunk * kCoarseRsStride);
    HANNS_CUDA_OK(cudaMemsetAsync(w_fallbacks_.p, 0, 2 * sizeof(int), s));
    if (nprobe > 256) {  // candidate buffers hold 512: large nprobe takes the exact kernels
        w_sel_.reserve((size_t)cchunk * 2 * nprobe);
        for (int64_t c = 0; c < nb; c += cchunk) {
            const int64_t m = std::min(cchunk, nb - c);
            launch_coarse_l2(d_q + c * dim_, m, centroids_.p, nlist_, dim_, w_dist_.p, s);
            if (mid_event && c == 0) HANNS_CUDA_OK(cudaEventRecord(mid_event, s));
            launch_select_probes(w_dist_.p, m, nlist_, nprobe, d_probes + c * nprobe, w_sel_.p, s);
            launches += 2;
        }
        return launches;
    }
    const char* mode = std::getenv("HANNS_GPU_COARSE");
    bool tc = !(mode && std::strcmp(mode, "simt") == 0);
    // |computed q.c - q.c| <= dot_rel * sum|q_i c_i|:
    //   SIMT FP32 FMA chain: (d + 8) 2^-24;
    //   bf16 hi/lo x3: representation 3.2 * 2^-16 plus tensor-core accumulation, taken as
    //   2^-21 per K16 step (3K/16 steps), both doubled.
    const float rel_simt = (float)((dim_ + 8) * 5.9604644775390625e-8);
    const float rel_tc =
        (float)(2.0 * (3.2 * 1.52587890625e-5 + (3.0 * tc_k_ / 16.0 + 2.0) * 4.76837158203125e-7));
    if (tc) {
        w_qhi_.reserve((size_t)cchunk * tc_k_);
        w_qlo_.reserve((size_t)cchunk * tc_k_);
    }
    for (int64_t c = 0; c < nb; c += cchunk) {
        const int64_t m = std::min(cchunk, nb - c);
        bool used_tc = false;
        if (tc) {
            launch_split_bf16(d_q + c * dim_, m, dim_, tc_k_, w_qhi_.p, w_qlo_.p, s);
            used_tc = launch_coarse_tc(w_qhi_.p, w_qlo_.p, m, cent_hi_.p, cent_lo_.p, nlist_, tc_k_,
                                       cn_.p, w_dist_.p, w_fallbacks_.p + 1, s);
            tc = used_tc;
            launches += used_tc ? 2 : 1;
        }
        if (!used_tc)
            launch_coarse_gemm(d_q + c * dim_, m, centroids_.p, cn_.p, nlist_, dim_, w_dist_.p, s);
        if (mid_event && c == 0) HANNS_CUDA_OK(cudaEventRecord(mid_event, s));
        launches += launch_coarse_select(w_dist_.p, d_q + c * dim_, m, centroids_.p, nlist_, dim_,
                                         nprobe, cmax_, used_tc ? rel_tc : rel_simt,
                                         used_tc ? w_fallbacks_.p + 1 : nullptr,
                                         d_probes + c * nprobe, w_fallbacks_.p, w_rs_.p, s);
        launches += used_tc ? 0 : 1;
    }
    return launches;
}

void IvfUsqGpu::refresh_rotation() {
    Pc_.reserve((size_t)D_ * D_);
    launch_rotation_chain_major(P_.p, D_, Pc_.p, stream_);
    HANNS_CUDA_OK(cudaGetLastError());
}

void IvfUsqGpu::upload_rotation_centroid() {
    std::vector<float> P((size_t)D_ * D_);
    rotation_matrix(rotation_seed_, D_, P.data());
    h2d(P_, P.data(), P.size(), stream_);
    refresh_rotation();
    rc_.reserve(D_);
    // rotated_centroid = P * pad(global mean)  (quantizer.rs:107-121)
    launch_rotate(gmean_.p, 1, dim_, D_, Pc_.p, rc_.p, stream_);
    HANNS_CUDA_OK(cudaGetLastError());
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
}

// ---------------------------------------------------------------- import/export
void IvfUsqGpu::import_artifact(const void* art_) {
    const auto* a = static_cast<const hanns_ivf_usq_artifact_t*>(art_);
    DeviceGuard g(device_);
    if (a->dim != dim_ || a->nbits != nbits_ || a->nlist != nlist_ || a->padded_dim != D_)
        throw std::invalid_argument("artifact shape does not match the index");
    metric_ = a->metric;
    ntotal_ = a->ntotal;
    h2d(centroids_, a->centroids, (size_t)nlist_ * dim_, stream_);
    update_centroid_norms();
    h2d(P_, a->rotation, (size_t)D_ * D_, stream_);
    refresh_rotation();
    h2d(rc_, a->rotated_centroid, (size_t)D_, stream_);
    std::vector<int64_t> off(a->list_offsets, a->list_offsets + nlist_ + 1);
    if (off[0] != 0 || off[nlist_] != ntotal_) throw std::invalid_argument("bad list offsets");
    for (int l = 0; l < nlist_; ++l)
        if (off[l + 1] < off[l]) throw std::invalid_argument("list offsets not monotone");
    const size_t n = (size_t)ntotal_;
    h2d(ids_, a->ids, n, stream_);
    std::vector<float4> meta(n);
    for (size_t i = 0; i < n; ++i)
        meta[i] = make_float4(a->norms[i], a->norms_sq[i], a->vmaxs[i], a->quant_qualities[i]);
    h2d(meta_, meta.data(), n, stream_);
    h2d(codes_, a->codes, n * code_bytes_, stream_);
    h2d(signs_, a->sign_bits, n * (D_ / 8), stream_);
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
    set_list_layout(off);
    rebuild_fastscan();
    gmean_.reserve(dim_);
    HANNS_CUDA_OK(cudaMemset(gmean_.p, 0, sizeof(float) * dim_));  // not part of the artifact
    trained_ = true;
}

void IvfUsqGpu::export_artifact(void* out_) const {
    auto* o = static_cast<hanns_ivf_usq_artifact_t*>(out_);
    DeviceGuard g(device_);
    const size_t n = (size_t)ntotal_;
    auto d2h = [&](void* dst, const void* src, size_t bytes) {
        if (dst && bytes) HANNS_CUDA_OK(cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost));
    };
    o->dim = dim_;
    o->padded_dim = D_;
    o->nbits = nbits_;
    o->nlist = nlist_;
    o->metric = metric_;
    o->ntotal = ntotal_;
    d2h((void*)o->centroids, centroids_.p, sizeof(float) * nlist_ * dim_);
    d2h((void*)o->rotation, P_.p, sizeof(float) * D_ * D_);
    d2h((void*)o->rotated_centroid, rc_.p, sizeof(float) * D_);
    if (o->list_offsets)
        std::memcpy((void*)o->list_offsets, h_list_off_.data(), sizeof(int64_t) * (nlist_ + 1));
    d2h((void*)o->ids, ids_.p, sizeof(int64_t) * n);
    if (n && (o->norms || o->norms_sq || o->vmaxs || o->quant_qualities)) {
        std::vector<float4> meta(n);
        d2h(meta.data(), meta_.p, sizeof(float4) * n);
        for (size_t i = 0; i < n; ++i) {
            if (o->norms) ((float*)o->norms)[i] = meta[i].x;
            if (o->norms_sq) ((float*)o->norms_sq)[i] = meta[i].y;
            if (o->vmaxs) ((float*)o->vmaxs)[i] = meta[i].z;
            if (o->quant_qualities) ((float*)o->quant_qualities)[i] = meta[i].w;
        }
    }
    d2h((void*)o->codes, codes_.p, n * code_bytes_);
    d2h((void*)o->sign_bits, signs_.p, n * (D_ / 8));
}

// ---------------------------------------------------------------- train / add
void IvfUsqGpu::train(const float* h_data, int64_t n, int kmeans_iters, uint64_t kmeans_seed) {
    DeviceGuard g(device_);
    if (n < nlist_) throw std::invalid_argument("training data too small: n < nlist");
    DevBuf<float> x;
    h2d(x, h_data, (size_t)n * dim_, stream_);
    // Seeded uniform stream in [0, 1) (the reference draws from an entropy-seeded StdRng).
    uint64_t s = kmeans_seed ^ 0xD1B54A32D192ED03ull;
    auto uniform = [&s]() {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        return (double)(s >> 11) * (1.0 / 9007199254740992.0);
    };
    // k-means++ seeding (kmeans.rs:138-183): the first centroid a uniform row, each next one
    // a row drawn with probability proportional to its squared distance to the nearest
    // centroid so far.
    centroids_.reserve((size_t)nlist_ * dim_);
    {
        const int64_t first = std::min<int64_t>(n - 1, (int64_t)(uniform() * (double)n));
        HANNS_CUDA_OK(cudaMemcpyAsync(centroids_.p, x.p + first * dim_, sizeof(float) * dim_,
                                      cudaMemcpyDeviceToDevice, stream_));
        DevBuf<float> min_d;
        min_d.reserve(n);
        int64_t per = 0;
        DevBuf<double> block_sum;
        block_sum.reserve(kpp_blocks(n, &per));
        launch_kpp_init_min(min_d.p, n, stream_);
        for (int c = 1; c < nlist_; ++c) {
            const double ut = uniform(), uu = uniform();
            launch_kpp_step(x.p, n, dim_, centroids_.p, c, min_d.p, block_sum.p, ut, uu, stream_);
        }
        HANNS_CUDA_OK(cudaGetLastError());
        HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
    }
    DevBuf<int32_t> assign;
    assign.reserve(n);
    DevBuf<long long> sums;
    sums.reserve((size_t)nlist_ * dim_);
    DevBuf<int> counts;
    counts.reserve(nlist_);
    DevBuf<float> shift;
    shift.reserve(nlist_);
    std::vector<int> h_counts(nlist_);
    std::vector<float> h_shift(nlist_);
    std::vector<int32_t> h_assign;
    std::vector<float> row(dim_);
    constexpr float kTolerance = 1e-2f;  // KMeans::new (kmeans.rs:44-56)
    for (int it = 0; it < kmeans_iters; ++it) {
        // nearest centroid of every row: the search's coarse step with one probe (the
        // lowest id among equally near centroids, as a strict-less argmin keeps)
        update_centroid_norms();
        coarse_probes(x.p, n, 1, assign.p, stream_);
        HANNS_CUDA_OK(cudaMemsetAsync(sums.p, 0, sizeof(long long) * nlist_ * dim_, stream_));
        HANNS_CUDA_OK(cudaMemsetAsync(counts.p, 0, sizeof(int) * nlist_, stream_));
        launch_kmeans_accumulate(x.p, n, dim_, assign.p, sums.p, counts.p, stream_);
        launch_kmeans_update(sums.p, counts.p, nlist_, dim_, centroids_.p, shift.p, stream_);
        HANNS_CUDA_OK(cudaGetLastError());
        HANNS_CUDA_OK(cudaMemcpyAsync(h_counts.data(), counts.p, sizeof(int) * nlist_,
                                      cudaMemcpyDeviceToHost, stream_));
        HANNS_CUDA_OK(cudaMemcpyAsync(h_shift.data(), shift.p, sizeof(float) * nlist_,
                                      cudaMemcpyDeviceToHost, stream_));
        HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
        // empty centroids restart at a random row of the largest list (the last one among
        // equal counts), scaled by 1 + 1e-4 (u - 0.5) per element (kmeans.rs:272-290)
        int largest = 0;
        for (int c = 0; c < nlist_; ++c)
            if (h_counts[c] >= h_counts[largest]) largest = c;
        std::vector<int64_t> members;
        for (int c = 0; c < nlist_; ++c) {
            if (h_counts[c] > 0) continue;
            if (members.empty()) {
                h_assign.resize(n);
                HANNS_CUDA_OK(cudaMemcpy(h_assign.data(), assign.p, sizeof(int32_t) * n,
                                         cudaMemcpyDeviceToHost));
                for (int64_t i = 0; i < n; ++i)
                    if (h_assign[i] == largest) members.push_back(i);
                if (members.empty()) break;
            }
            const int64_t pick = members[std::min<size_t>(
                members.size() - 1, (size_t)(uniform() * (double)members.size()))];
            for (int j = 0; j < dim_; ++j)
                row[j] = h_data[pick * dim_ + j] * (1.0f + 1e-4f * ((float)uniform() - 0.5f));
            HANNS_CUDA_OK(cudaMemcpy(centroids_.p + (int64_t)c * dim_, row.data(),
                                     sizeof(float) * dim_, cudaMemcpyHostToDevice));
        }
        float max_shift = 0.0f;
        for (int c = 0; c < nlist_; ++c) max_shift = std::max(max_shift, h_shift[c]);
        if (max_shift < kTolerance) break;
    }
    update_centroid_norms();
    gmean_.reserve(dim_);
    launch_global_mean(x.p, n, dim_, gmean_.p, stream_);
    HANNS_CUDA_OK(cudaGetLastError());
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
    upload_rotation_centroid();
    // A retrain discards stored vectors, as a fresh IvfUsqIndex would hold none.
    ntotal_ = 0;
    set_list_layout(std::vector<int64_t>(nlist_ + 1, 0));
    trained_ = true;
}

void IvfUsqGpu::add(const float* h_data, int64_t n, const int64_t* h_ids) {
    DeviceGuard g(device_);
    if (!trained_) throw std::invalid_argument("index not trained, call train() first");
    check_int_rerank("GPU encoder");
    if (n <= 0) return;
    const int64_t chunk = 65536;
    DevBuf<float> x, res, nsq;
    DevBuf<float> rot;  // chunk*D floats followed by chunk*D code bytes (encode scratch)
    DevBuf<int32_t> asg;
    DevBuf<uint8_t> ncodes, nsigns;
    DevBuf<float4> nmeta;
    ncodes.reserve((size_t)n * code_bytes_);
    nsigns.reserve((size_t)n * (D_ / 8));
    nmeta.reserve((size_t)n);
    asg.reserve((size_t)n);
    for (int64_t b = 0; b < n; b += chunk) {
        const int64_t m = std::min(chunk, n - b);
        h2d(x, h_data + b * dim_, (size_t)m * dim_, stream_);
        nsq.reserve(m);
        launch_row_norm_sq(x.p, m, dim_, nsq.p, stream_);
        res.reserve((size_t)m * D_);
        launch_residual_pad(x.p, m, dim_, D_, gmean_.p, res.p, stream_);
        rot.reserve((size_t)m * D_ + ((size_t)m * D_ + 3) / 4);
        launch_rotate(res.p, m, D_, D_, Pc_.p, rot.p, stream_);
        launch_encode_rotated(rot.p, m, D_, nbits_, nsq.p, ncodes.p + b * code_bytes_,
                              nsigns.p + b * (D_ / 8), nmeta.p + b, stream_);
        // nearest centroid (find_best_centroid, ivf_usq.rs:611-625): the search's coarse
        // step with one probe -- the same centroid, lowest id among equally near ones
        coarse_probes(x.p, m, 1, asg.p + b, stream_);
        HANNS_CUDA_OK(cudaGetLastError());
    }
    std::vector<int32_t> h_asg(n);
    HANNS_CUDA_OK(cudaMemcpyAsync(h_asg.data(), asg.p, sizeof(int32_t) * n, cudaMemcpyDeviceToHost,
                                  stream_));
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
    // New list order: every list keeps its old rows, then the new rows in insertion order.
    const int64_t old_n = ntotal_, tot = old_n + n;
    std::vector<int64_t> cnt(nlist_ + 1, 0);
    for (int l = 0; l < nlist_; ++l) cnt[l + 1] = h_list_off_[l + 1] - h_list_off_[l];
    for (int64_t i = 0; i < n; ++i) cnt[h_asg[i] + 1]++;
    std::vector<int64_t> off(nlist_ + 1, 0);
    for (int l = 0; l < nlist_; ++l) off[l + 1] = off[l] + cnt[l + 1];
    std::vector<int64_t> cursor(off.begin(), off.end() - 1), perm(tot);
    for (int l = 0; l < nlist_; ++l)
        for (int64_t r = h_list_off_[l]; r < h_list_off_[l + 1]; ++r) perm[cursor[l]++] = r;
    for (int64_t i = 0; i < n; ++i) perm[cursor[h_asg[i]]++] = old_n + i;
    // concatenated sources [old ; new]
    DevBuf<uint8_t> cat_codes, cat_signs;
    DevBuf<float4> cat_meta;
    DevBuf<int64_t> cat_ids, d_perm;
    cat_codes.reserve((size_t)tot * code_bytes_);
    cat_signs.reserve((size_t)tot * (D_ / 8));
    cat_meta.reserve(tot);
    cat_ids.reserve(tot);
    if (old_n) {
        HANNS_CUDA_OK(cudaMemcpyAsync(cat_codes.p, codes_.p, (size_t)old_n * code_bytes_,
                                      cudaMemcpyDeviceToDevice, stream_));
        HANNS_CUDA_OK(cudaMemcpyAsync(cat_signs.p, signs_.p, (size_t)old_n * (D_ / 8),
                                      cudaMemcpyDeviceToDevice, stream_));
        HANNS_CUDA_OK(cudaMemcpyAsync(cat_meta.p, meta_.p, sizeof(float4) * old_n,
                                      cudaMemcpyDeviceToDevice, stream_));
        HANNS_CUDA_OK(cudaMemcpyAsync(cat_ids.p, ids_.p, sizeof(int64_t) * old_n,
                                      cudaMemcpyDeviceToDevice, stream_));
    }
    HANNS_CUDA_OK(cudaMemcpyAsync(cat_codes.p + old_n * code_bytes_, ncodes.p,
                                  (size_t)n * code_bytes_, cudaMemcpyDeviceToDevice, stream_));
    HANNS_CUDA_OK(cudaMemcpyAsync(cat_signs.p + old_n * (D_ / 8), nsigns.p, (size_t)n * (D_ / 8),
                                  cudaMemcpyDeviceToDevice, stream_));
    HANNS_CUDA_OK(cudaMemcpyAsync(cat_meta.p + old_n, nmeta.p, sizeof(float4) * n,
                                  cudaMemcpyDeviceToDevice, stream_));
    std::vector<int64_t> new_ids(n);
    for (int64_t i = 0; i < n; ++i) new_ids[i] = h_ids ? h_ids[i] : old_n + i;
    HANNS_CUDA_OK(cudaMemcpyAsync(cat_ids.p + old_n, new_ids.data(), sizeof(int64_t) * n,
                                  cudaMemcpyHostToDevice, stream_));
    h2d(d_perm, perm.data(), perm.size(), stream_);
    DevBuf<uint8_t> o_codes, o_signs;
    DevBuf<float4> o_meta;
    DevBuf<int64_t> o_ids;
    o_codes.reserve((size_t)tot * code_bytes_);
    o_signs.reserve((size_t)tot * (D_ / 8));
    o_meta.reserve(tot);
    o_ids.reserve(tot);
    launch_gather_rows(cat_codes.p, d_perm.p, tot, code_bytes_, o_codes.p, stream_);
    launch_gather_rows(cat_signs.p, d_perm.p, tot, D_ / 8, o_signs.p, stream_);
    launch_gather_rows(reinterpret_cast<const uint8_t*>(cat_meta.p), d_perm.p, tot, 16,
                       reinterpret_cast<uint8_t*>(o_meta.p), stream_);
    launch_gather_rows(reinterpret_cast<const uint8_t*>(cat_ids.p), d_perm.p, tot, 8,
                       reinterpret_cast<uint8_t*>(o_ids.p), stream_);
    HANNS_CUDA_OK(cudaGetLastError());
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
    codes_.swap(o_codes);
    signs_.swap(o_signs);
    meta_.swap(o_meta);
    ids_.swap(o_ids);
    ntotal_ = tot;
    set_list_layout(off);
    rebuild_fastscan();
}

// ---------------------------------------------------------------- sharding
// Longest-processing-time assignment: lists in decreasing size (ties: lower id first) go
// to the currently least-loaded rank (ties: lower rank).  Host-only and deterministic, so
// every rank computes the same owners.
void shard_owners(const int64_t* sizes, int nlist, int world, int32_t* owner) {
    // expected scan work of a list ~ |L| x (queries that probe it, ~ |L| when queries
    // follow the data): longest-processing-time on |L|^2
    std::vector<int64_t> weights(nlist);
    for (int l = 0; l < nlist; ++l) weights[l] = sizes[l] * sizes[l];
    std::vector<int> order(nlist);
    std::iota(order.begin(), order.end(), 0);
    std::stable_sort(order.begin(), order.end(),
                     [&](int a, int b) { return weights[a] > weights[b]; });
    std::vector<int64_t> load(world, 0);
    for (int l : order) {
        int best = 0;
        for (int r = 1; r < world; ++r)
            if (load[r] < load[best]) best = r;
        load[best] += weights[l];
        owner[l] = best;
    }
}

void IvfUsqGpu::shard(int rank, int world) {
    DeviceGuard g(device_);
    if (world < 1 || rank < 0 || rank >= world) throw std::invalid_argument("bad rank/world");
    std::vector<int64_t> sizes(nlist_);
    for (int l = 0; l < nlist_; ++l) sizes[l] = h_list_off_[l + 1] - h_list_off_[l];
    std::vector<int32_t> owner(nlist_);
    shard_owners(sizes.data(), nlist_, world, owner.data());
    std::vector<uint8_t> owned(nlist_, 0);
    for (int l = 0; l < nlist_; ++l) owned[l] = owner[l] == rank ? 1 : 0;
    // keep only owned lists' rows
    std::vector<int64_t> perm, off(nlist_ + 1, 0);
    for (int l = 0; l < nlist_; ++l) {
        if (owned[l])
            for (int64_t r = h_list_off_[l]; r < h_list_off_[l + 1]; ++r) perm.push_back(r);
        off[l + 1] = (int64_t)perm.size();
    }
    const int64_t tot = (int64_t)perm.size();
    DevBuf<int64_t> d_perm;
    h2d(d_perm, perm.data(), perm.size(), stream_);
    DevBuf<uint8_t> o_codes, o_signs;
    DevBuf<float4> o_meta;
    DevBuf<int64_t> o_ids;
    o_codes.reserve((size_t)tot * code_bytes_);
    o_signs.reserve((size_t)tot * (D_ / 8));
    o_meta.reserve(tot);
    o_ids.reserve(tot);
    launch_gather_rows(codes_.p, d_perm.p, tot, code_bytes_, o_codes.p, stream_);
    launch_gather_rows(signs_.p, d_perm.p, tot, D_ / 8, o_signs.p, stream_);
    launch_gather_rows(reinterpret_cast<const uint8_t*>(meta_.p), d_perm.p, tot, 16,
                       reinterpret_cast<uint8_t*>(o_meta.p), stream_);
    launch_gather_rows(reinterpret_cast<const uint8_t*>(ids_.p), d_perm.p, tot, 8,
                       reinterpret_cast<uint8_t*>(o_ids.p), stream_);
    h2d(owned_, owned.data(), owned.size(), stream_);
    HANNS_CUDA_OK(cudaGetLastError());
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
    codes_.swap(o_codes);
    signs_.swap(o_signs);
    meta_.swap(o_meta);
    ids_.swap(o_ids);
    ntotal_ = tot;
    sharded_ = true;
    set_list_layout(off);
    rebuild_fastscan();
}

// ---------------------------------------------------------------- search
void IvfUsqGpu::search_batch(const float* d_q, const float* h_q, int64_t nb,
                             const SearchOptions& opt, int64_t* d_ids, float* d_dists,
                             int64_t* d_counts, uint64_t* d_keys, cudaStream_t s, bool time_it) {
    const int nprobe = std::max(1, std::min(opt.nprobe, nlist_));
    const int G = D_ / 4;
    if (time_it) HANNS_CUDA_OK(cudaEventRecord(ev_[0], s));
    w_probes_.reserve((size_t)nb * nprobe);
    w_qp_.reserve(nb);
    w_qi8p_.reserve((size_t)nb * D_);
    w_qi8n_.reserve((size_t)nb * D_);
    w_lut_.reserve((size_t)nb * G * 16);
    const QueryState st{w_probes_.p, w_qp_.p, w_lut_.p, w_qi8p_.p, w_qi8n_.p};
    int64_t launches = prepare_batch(d_q, h_q, nb, nprobe, st, s, time_it);
    launches += scan_merge_batch(nb, opt, st, d_ids, d_dists, d_counts, d_keys, s, time_it);
    last_launches_ += launches;
}

int64_t IvfUsqGpu::prepare_batch(const float* d_q, const float* h_q, int64_t nb, int nprobe,
                                 const QueryState& st, cudaStream_t s, bool time_it) {
    const int G = D_ / 4;
    int64_t launches = 0;
    w_qrot_.reserve((size_t)nb * D_);
    // 1-2. per-query stages: coarse probes, rotation, query state.  Host queries are uploaded
    // in up to kMaxUploadChunks chunks on copy_stream_; chunk c's per-query stages wait only
    // for chunk c's copy, so the copy of chunk c+1 runs under them.
    w_sel_.reserve((size_t)nb * 2 * nprobe);
    int nchunks = 1;
    if (h_q) nchunks = (int)std::min<int64_t>(kMaxUploadChunks, std::max<int64_t>(1, nb / 1024));
    const int64_t per = (nb + nchunks - 1) / nchunks;
    if (h_q) {
        HANNS_CUDA_OK(cudaEventRecord(ev_ready_, s));
        HANNS_CUDA_OK(cudaStreamWaitEvent(copy_stream_, ev_ready_, 0));
        for (int c = 0; c < nchunks; ++c) {
            const int64_t q0 = c * per, m = std::min(per, nb - q0);
            if (m <= 0) break;
            if (fault_injected(kFaultH2D))
                throw CudaError(cudaErrorInvalidValue, "cudaMemcpyAsync (injected host-to-device fault)",
                                __FILE__, __LINE__);
            HANNS_CUDA_OK(cudaMemcpyAsync(const_cast<float*>(d_q) + q0 * dim_, h_q + q0 * dim_,
                                          sizeof(float) * m * dim_, cudaMemcpyHostToDevice,
                                          copy_stream_));
            HANNS_CUDA_OK(cudaEventRecord(ev_up_[c], copy_stream_));
        }
    }
    // the coarse step runs on s, rotation + query state on aux_stream_ (independent work on
    // the same queries, so the two latency-bound chains overlap); s joins aux before grouping
    const bool per_stage = time_it && nchunks == 1;
    cur_->aux_timed = per_stage;
    HANNS_CUDA_OK(cudaEventRecord(ev_fork_, s));
    HANNS_CUDA_OK(cudaStreamWaitEvent(aux_stream_, ev_fork_, 0));
    if (per_stage) HANNS_CUDA_OK(cudaEventRecord(ev_aux_[0], aux_stream_));
    for (int c = 0; c < nchunks; ++c) {
        const int64_t q0 = c * per, m = std::min(per, nb - q0);
        if (m <= 0) break;
        const float* q = d_q + q0 * dim_;
        if (h_q) {
            HANNS_CUDA_OK(cudaStreamWaitEvent(s, ev_up_[c], 0));
            HANNS_CUDA_OK(cudaStreamWaitEvent(aux_stream_, ev_up_[c], 0));
        }
        launches += coarse_probes(q, m, nprobe, st.probes + q0 * nprobe, s,
                                  per_stage ? ev_[1] : nullptr);
        launch_rotate(q, m, dim_, D_, Pc_.p, w_qrot_.p + q0 * D_, aux_stream_);
        if (per_stage) HANNS_CUDA_OK(cudaEventRecord(ev_aux_[1], aux_stream_));
        launch_query_state(q, w_qrot_.p + q0 * D_, m, dim_, D_, rc_.p, nbits_, st.qp + q0,
                           st.q_i8p + q0 * D_, st.q_i8n + q0 * D_, st.lut + q0 * G * 16,
                           aux_stream_);
        launches += 2;
    }
    if (per_stage) {
        HANNS_CUDA_OK(cudaEventRecord(ev_aux_[2], aux_stream_));
        HANNS_CUDA_OK(cudaEventRecord(ev_[2], s));  // coarse step done
    }
    HANNS_CUDA_OK(cudaEventRecord(ev_join_, aux_stream_));
    HANNS_CUDA_OK(cudaStreamWaitEvent(s, ev_join_, 0));
    if (time_it) {
        if (!per_stage) {  // chunked upload: the first stage spans upload + per-query stages
            HANNS_CUDA_OK(cudaEventRecord(ev_[1], s));
            HANNS_CUDA_OK(cudaEventRecord(ev_[2], s));
        }
        HANNS_CUDA_OK(cudaEventRecord(ev_[3], s));  // per-query stages done
    }
    return launches;
}

int64_t IvfUsqGpu::scan_merge_batch(int64_t nb, const SearchOptions& opt, const QueryState& st,
                                    int64_t* d_ids, float* d_dists, int64_t* d_counts,
                                    uint64_t* d_keys, cudaStream_t s, bool time_it) {
    const int k = std::max(opt.k, 1);
    const int nprobe = std::max(1, std::min(opt.nprobe, nlist_));
    const int G = D_ / 4;
    int64_t launches = 0;
    if (time_it) HANNS_CUDA_OK(cudaEventRecord(ev_[4], s));
    // 3. group (query, probe) pairs by list
    w_cnt_.reserve(nlist_ + 1);
    w_cursor_.reserve(nlist_ + 1);
    w_lq_off_.reserve(nlist_ + 1);
    w_item_off_.reserve(nlist_ + 1);
    w_counters_.reserve(4);
    w_lq_.reserve((size_t)nb * nprobe);
    w_items_.reserve((size_t)nb * nprobe);
    HANNS_CUDA_OK(cudaMemsetAsync(w_counters_.p, 0, 4 * sizeof(int), s));
    // lists of at most kTcMaxRows rows take the tensor-core scan; HANNS_GPU_SCAN=simt: none,
    // =hybrid: only lists without FastScan (|list| <= n_cand)
    const int n_cand = (int)n_candidates(nbits_, k);
    const int tc_rows = scan_tc_rows(n_cand);
    const bool use_tc = tc_rows > 0;
    const int64_t fss = fs_stride(nprobe, n_cand, tc_rows);
    launch_group_pairs(st.probes, nb, nprobe, nlist_, sharded_ ? owned_.p : nullptr, list_off_.p,
                       list_order_.p, tc_rows, n_cand, kQueriesPerItem, w_cnt_.p, w_cursor_.p, w_lq_off_.p,
                       w_item_off_.p, w_counters_.p, w_lq_.p, w_items_.p, s);
    const int64_t q_stride = cand_stride(nprobe, k);
    w_pair_off_.reserve((size_t)nb * (nprobe + 1));
    if (fss > 0) {
        w_fs_off_.reserve((size_t)nb * nprobe);
        w_fs_sc_.reserve((size_t)nb * fss);
        w_fs_ip_.reserve((size_t)nb * fss);
    }
    // a FastScan pair's region holds only its top k when that cannot change the query's
    // top k (every entry of the top k is in its own pair's top k); the debug entry wants
    // every kept candidate
    PairTrunc tr;
    tr.fs_keep = (!debug_candidates_ && k < n_cand && n_cand <= kFsRegRows / 2) ? k : 0;
    tr.fused = opt.filter_mode == 2 ? 1 : 0;
    tr.bitsets = opt.d_bitsets;
    tr.n_bitsets = opt.d_bitsets ? opt.n_bitsets : 0;
    tr.query_bitset = opt.d_query_bitset;
    launch_pair_offsets(st.probes, nb, nprobe, list_off_.p, nlist_, sharded_ ? owned_.p : nullptr,
                        n_cand, w_pair_off_.p, tc_rows, fss > 0 ? w_fs_off_.p : nullptr, tr, s);
    launches += 5;
    if (time_it) HANNS_CUDA_OK(cudaEventRecord(ev_[5], s));
    // 4. list scan: kept candidates of every (query, probe) pair with their distance keys
    w_cand_key_.reserve((size_t)nb * q_stride);
    w_cand_tie_.reserve((size_t)nb * q_stride);
    if (!scan_grid_) scan_grid_ = scan_grid_size(D_);
    const int grid = scan_grid_;
    const size_t per_warp = (size_t)max_list_;
    w_scores_.reserve((size_t)grid * 8 * per_warp);
    ScanArgs a{};
    a.D = D_;
    a.nbits = nbits_;
    a.code_bytes = code_bytes_;
    a.nchunks = D_ / 64;
    a.G = G;
    a.metric_l2 = metric_ == 0 ? 1 : 0;
    a.list_off = list_off_.p;
    a.fs_blk_off = fs_blk_off_.p;
    a.fs = fs_.p;
    a.codes = codes_.p;
    a.meta = meta_.p;
    a.ids = ids_.p;
    a.qp = st.qp;
    a.lut = st.lut;
    a.q_i8p = st.q_i8p;
    a.lq = w_lq_.p;
    a.items = w_items_.p;
    a.n_items = w_counters_.p;
    a.item_counter = w_counters_.p + 1;
    a.k = k;
    a.n_cand = n_cand;
    a.nprobe = nprobe;
    a.fused = opt.filter_mode == 2 ? 1 : 0;
    a.bitsets = opt.d_bitsets;
    a.bitset_len = opt.bitset_len;
    a.bitset_words = (opt.bitset_len + 63) / 64;
    a.n_bitsets = opt.d_bitsets ? opt.n_bitsets : 0;
    a.query_bitset = opt.d_query_bitset;
    a.pair_off = w_pair_off_.p;
    a.q_stride = q_stride;
    a.cand_key = w_cand_key_.p;
    a.cand_tie = w_cand_tie_.p;
    a.scores = w_scores_.p;
    a.q_rot = w_qrot_.p;  // (this batch's rotated queries, from prepare_batch)
    a.max_len = (int)per_warp;
    if (debug_candidates_) {
        w_cand_dbg_.reserve((size_t)nb * q_stride);
        a.cand_dbg = w_cand_dbg_.p;
    }
    if (use_tc) {
        if (!w_scan_err_.p) {
            // sticky: an expired bounded wait stays visible to every later check
            w_scan_err_.reserve(1);
            HANNS_CUDA_OK(cudaMemsetAsync(w_scan_err_.p, 0, sizeof(int), s));
        }
        TcScanArgs t{};
        t.D = D_;
        t.nbits = nbits_;
        t.code_bytes = code_bytes_;
        t.G = G;
        t.metric_l2 = a.metric_l2;
        t.nchunks = D_ / 64;
        t.list_off = list_off_.p;
        t.fs_blk_off = fs_blk_off_.p;
        t.fs = fs_.p;
        t.codes = codes_.p;
        t.meta = meta_.p;
        t.ids = ids_.p;
        t.qp = st.qp;
        t.lut = st.lut;
        t.q_i8p = st.q_i8p;
        t.cand_dbg = a.cand_dbg;
        t.fs_off = w_fs_off_.p;
        t.fs_stride = fss;
        t.fs_sc = w_fs_sc_.p;
        t.fs_ip = w_fs_ip_.p;
        t.wait_ns = scan_wait_ns_;
        const char* prof_env = std::getenv("HANNS_GPU_SCAN_PROFILE");
        const bool prof = prof_env && prof_env[0] == '1';
        if (prof) {
            w_tc_prof_.reserve((size_t)sm_count_ * kTcProfSlots);
            HANNS_CUDA_OK(cudaMemsetAsync(w_tc_prof_.p, 0, sizeof(unsigned long long) * sm_count_ * kTcProfSlots, s));
            t.prof = w_tc_prof_.p;
        }
        t.lq = w_lq_.p;
        t.items = w_items_.p;
        t.n_items = w_counters_.p;
        t.item_counter = w_counters_.p + 2;
        t.k = k;
        t.n_cand = n_cand;
        t.nprobe = nprobe;
        t.fused = a.fused;
        t.bitsets = a.bitsets;
        t.bitset_len = a.bitset_len;
        t.bitset_words = a.bitset_words;
        t.n_bitsets = a.n_bitsets;
        t.query_bitset = a.query_bitset;
        t.pair_off = w_pair_off_.p;
        t.q_stride = q_stride;
        t.cand_key = w_cand_key_.p;
        t.cand_tie = w_cand_tie_.p;
        t.err_flag = w_scan_err_.p;
        if (time_it) HANNS_CUDA_OK(cudaEventRecord(cur_->kt[0], s));
        launch_scan_tc(t, sm_count_, s);
        launches += 1;
        if (t.prof) {
            // per-CTA averages of the role counters (scan_tc.cu), one line on stderr
            std::vector<unsigned long long> h((size_t)sm_count_ * kTcProfSlots);
            HANNS_CUDA_OK(cudaMemcpyAsync(h.data(), w_tc_prof_.p, sizeof(unsigned long long) * h.size(),
                                          cudaMemcpyDeviceToHost, s));
            HANNS_CUDA_OK(cudaStreamSynchronize(s));
            static const char* names[] = {"build", "build_wait_slot", "build_wait_item", "mma_wait_full",
                                          "mma_wait_free", "mma", "epi_wait_acc", "epi_copy",
                                          "epi_select", "epi_rerank", "epi_wait_item", "epi",
                                          "items", "stages", "mma_wait_b", "unused"};
            std::fprintf(stderr, "TC_SCAN_PROFILE ctas=%d", sm_count_);
            for (int k = 0; k < 16; ++k) {
                double sum = 0;
                for (int c = 0; c < sm_count_; ++c) sum += (double)h[(size_t)c * kTcProfSlots + k];
                const bool count = k == 12 || k == 13;
                std::fprintf(stderr, count ? " %s=%.1f" : " %s=%.3fms", names[k],
                             count ? sum / sm_count_ : sum / sm_count_ / 1e6);
            }
            std::fprintf(stderr, "\n");
        }
    }
    if (time_it) {
        if (!use_tc) HANNS_CUDA_OK(cudaEventRecord(cur_->kt[0], s));
        HANNS_CUDA_OK(cudaEventRecord(cur_->kt[1], s));
    }
    launch_scan(a, grid, s);
    launches += 1;
    if (time_it) HANNS_CUDA_OK(cudaEventRecord(cur_->kt[2], s));
    if (fss > 0) {
        // kept sets and distances of the tensor-core FastScan pairs
        FsSelectArgs f{};
        f.nq = nb;
        f.nprobe = nprobe;
        f.n_cand = n_cand;
        f.nbits = nbits_;
        f.metric_l2 = a.metric_l2;
        f.fused = a.fused;
        f.probes = st.probes;
        f.list_off = list_off_.p;
        f.ids = ids_.p;
        f.meta = meta_.p;
        f.qp = st.qp;
        f.fs_off = w_fs_off_.p;
        f.fs_stride = fss;
        f.fs_sc = w_fs_sc_.p;
        f.fs_ip = w_fs_ip_.p;
        f.pair_off = w_pair_off_.p;
        f.q_stride = q_stride;
        f.bitsets = a.bitsets;
        f.bitset_len = a.bitset_len;
        f.bitset_words = a.bitset_words;
        f.n_bitsets = a.n_bitsets;
        f.query_bitset = a.query_bitset;
        f.cand_key = w_cand_key_.p;
        f.cand_tie = w_cand_tie_.p;
        f.cand_dbg = a.cand_dbg;
        f.lq = w_lq_.p;
        f.n_lq = w_lq_off_.p + nlist_;
        launch_fs_select(f, sm_count_ * 4, s);
        launches += 1;
    }
    if (time_it) {
        HANNS_CUDA_OK(cudaEventRecord(cur_->kt[3], s));
        cur_->kt_timed = true;
    }
    if (time_it) HANNS_CUDA_OK(cudaEventRecord(ev_[6], s));
    // 5-6. the top k of each query over its candidate regions: one block per query
    // (k <= kMergeMaxK), else each (query, probe) pair's top-k into a compact region of
    // nprobe * k entries and a warp per query over those
    const bool direct = k <= kMergeMaxK;
    if (!direct) {
        w_cmp_key_.reserve((size_t)nb * nprobe * k);
        w_cmp_tie_.reserve((size_t)nb * nprobe * k);
        CompactArgs c{};
        c.nq = nb;
        c.nprobe = nprobe;
        c.k = k;
        c.cand_key = w_cand_key_.p;
        c.cand_tie = w_cand_tie_.p;
        c.pair_off = w_pair_off_.p;
        c.q_stride = q_stride;
        c.out_key = w_cmp_key_.p;
        c.out_tie = w_cmp_tie_.p;
        launch_compact_pairs(c, s);
        launches += 1;
    }
    w_mkey_.reserve((size_t)nb * k);
    w_mtie_.reserve((size_t)nb * k);
    MergeArgs m{};
    m.nq = nb;
    m.nprobe = nprobe;
    m.k = k;
    m.nlist = nlist_;
    if (direct) {
        m.cand_key = w_cand_key_.p;
        m.cand_tie = w_cand_tie_.p;
        m.pair_off = w_pair_off_.p;
        m.q_stride = q_stride;
    } else {
        m.cand_key = w_cmp_key_.p;
        m.cand_tie = w_cmp_tie_.p;
        m.pair_off = nullptr;
        m.q_stride = (int64_t)nprobe * k;
        m.fixed_total = nprobe * k;
    }
    m.probes = st.probes;
    m.list_off = list_off_.p;
    m.ids = ids_.p;
    m.sel_key = w_mkey_.p;
    m.sel_tie = w_mtie_.p;
    m.out_ids = d_ids;
    m.out_dists = d_dists;
    m.out_counts = d_counts;
    if (opt.filter_mode == 1 && opt.d_bitsets) {
        m.post_bitsets = opt.d_bitsets;
        m.bitset_len = opt.bitset_len;
        m.bitset_words = (opt.bitset_len + 63) / 64;
        m.n_bitsets = opt.n_bitsets;
        m.query_bitset = opt.d_query_bitset;
    }
    m.shard_mode = d_keys ? 1 : 0;
    m.out_keys = d_keys;
    if (direct)
        launch_merge_direct(m, s);
    else
        launch_merge(m, s);
    launches += 1;
    used_tc_ = used_tc_ || use_tc;
    if (use_tc) {
        HANNS_CUDA_OK(cudaMemcpyAsync(h_scan_err_, w_scan_err_.p, sizeof(int), cudaMemcpyDeviceToHost, s));
        HANNS_CUDA_OK(cudaEventRecord(ev_scan_err_, s));
    }
    HANNS_CUDA_OK(cudaGetLastError());
    if (time_it) HANNS_CUDA_OK(cudaEventRecord(ev_[7], s));
    return launches;
}


void IvfUsqGpu::search_device(const float* d_queries, int64_t nq, const SearchOptions& opt,
                              int64_t* d_ids, float* d_dists, int64_t* d_counts, uint64_t* d_keys,
                              cudaStream_t stream) {
    DeviceGuard g(device_);
    run_search(d_queries, nullptr, nq, opt, d_ids, d_dists, d_counts, d_keys, stream);
    if (!stream) {
        HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
        check_tc_scan();
    }
}

void IvfUsqGpu::run_search(const float* d_queries, const float* h_queries, int64_t nq,
                           const SearchOptions& opt, int64_t* d_ids, float* d_dists,
                           int64_t* d_counts, uint64_t* d_keys, cudaStream_t stream) {
    if (!trained_) throw std::invalid_argument("index not trained");
    check_supported();
    if (nq <= 0) throw std::invalid_argument("query dimension mismatch");
    cudaStream_t s = stream ? stream : stream_;
    const int k = std::max(opt.k, 1);
    const int nprobe = std::max(1, std::min(opt.nprobe, nlist_));
    const int64_t nb_max = batch_limit(nprobe, k);
    last_launches_ = 0;
    begin_call();
    for (int64_t b = 0; b < nq; b += nb_max) {
        const int64_t nb = std::min(nb_max, nq - b);
        SearchOptions o = opt;
        if (o.d_query_bitset) o.d_query_bitset += b;
        // stages 0-1 (coarse step) and 2-3 (rotation, query state) overlap on two streams;
        // ev_[3] -> ev_[4] is empty (the join)
        next_slot(0, kStages);
        search_batch(d_queries + b * dim_, h_queries ? h_queries + b * dim_ : nullptr, nb, o,
                     d_ids + b * k, d_dists + b * k, d_counts ? d_counts + b : nullptr,
                     d_keys ? d_keys + b * k : nullptr, s, true);
        check_tc_scan();
    }
}

void IvfUsqGpu::query_state_bytes(int nprobe, int64_t* parts) const {
    nprobe = std::max(1, std::min(nprobe, nlist_));
    parts[0] = (int64_t)nprobe * sizeof(int32_t);
    parts[1] = sizeof(QueryParams);
    parts[2] = (int64_t)(D_ / 4) * 16;
    parts[3] = D_;
    parts[4] = D_;
}

void IvfUsqGpu::begin_call() {
    calls_.emplace_back(slot_seq_, 0);
    while ((int)calls_.size() > kEvRing) calls_.pop_front();
}

void IvfUsqGpu::next_slot(int first, int last) {
    cur_ = &ring_[slot_seq_ % kEvRing];
    cur_->first = first;
    cur_->last = last;
    cur_->aux_timed = false;
    cur_->kt_timed = false;
    ev_ = cur_->ev;
    ev_aux_ = cur_->aux;
    ++slot_seq_;
    if (!calls_.empty()) ++calls_.back().second;
}

// The tensor-core scan reports an expired bounded wait through a sticky device flag that
// each scan copies to pinned memory.  The check does not wait for the device: it reads the
// copy once the event behind it has completed (a stream-ordered call returns once
// enqueued, and a later call or a synchronising one reports the error).
void IvfUsqGpu::check_tc_scan() {
    if (!used_tc_) return;
    if (cudaEventQuery(ev_scan_err_) != cudaSuccess) return;
    const int code = *h_scan_err_;
    if (code != 0) {
        // reported once: the flag is cleared so that the next search starts clean (the
        // kernel freed its TMEM and returned; the context stays usable)
        HANNS_CUDA_OK(cudaMemsetAsync(w_scan_err_.p, 0, sizeof(int), stream_));
        HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
        *h_scan_err_ = 0;
        throw std::runtime_error("tensor-core list scan: a bounded wait expired (code " +
                                 std::to_string(code) + ")");
    }
}

// stage e = ev[e] -> ev[e + 1] for first <= e < last (stages 2-3 from the rotation stream's
// events), total = ev[first] -> ev[last]; summed over the slots of the last n_calls calls.
int IvfUsqGpu::stage_ms(int n_calls, float* out, int* counts) {
    for (int e = 0; e < kStages + 1; ++e) {
        out[e] = 0;
        if (counts) counts[e] = 0;
    }
    int covered = 0;
    for (auto it = calls_.rbegin(); it != calls_.rend() && covered < n_calls; ++it, ++covered) {
        if (slot_seq_ - it->first > kEvRing) break;  // its slots were reused
        for (int j = 0; j < it->second; ++j) {
            const StageSlot& sl = ring_[(it->first + j) % kEvRing];
            HANNS_CUDA_OK(cudaEventSynchronize(sl.ev[sl.last]));
            float t;
            for (int e = sl.first; e < sl.last; ++e) {
                if (e == 2 || e == 3) {
                    if (sl.aux_timed) {
                        HANNS_CUDA_OK(cudaEventElapsedTime(&t, sl.aux[e - 2], sl.aux[e - 1]));
                        out[e] += t;
                        if (counts) ++counts[e];
                    }
                    continue;
                }
                HANNS_CUDA_OK(cudaEventElapsedTime(&t, sl.ev[e], sl.ev[e + 1]));
                out[e] += t;
                if (counts) ++counts[e];
            }
            HANNS_CUDA_OK(cudaEventElapsedTime(&t, sl.ev[sl.first], sl.ev[sl.last]));
            out[kStages] += t;
            if (counts) ++counts[kStages];
        }
    }
    return covered;
}

int IvfUsqGpu::scan_kernel_ms(int n_calls, float* out3, int* counts3) {
    for (int e = 0; e < 3; ++e) {
        out3[e] = 0;
        counts3[e] = 0;
    }
    int covered = 0;
    for (auto it = calls_.rbegin(); it != calls_.rend() && covered < n_calls; ++it, ++covered) {
        if (slot_seq_ - it->first > kEvRing) break;  // its slots were reused
        for (int j = 0; j < it->second; ++j) {
            const StageSlot& sl = ring_[(it->first + j) % kEvRing];
            if (!sl.kt_timed) continue;
            HANNS_CUDA_OK(cudaEventSynchronize(sl.kt[3]));
            for (int e = 0; e < 3; ++e) {
                float t;
                HANNS_CUDA_OK(cudaEventElapsedTime(&t, sl.kt[e], sl.kt[e + 1]));
                out3[e] += t;
                ++counts3[e];
            }
        }
    }
    return covered;
}

void IvfUsqGpu::rerank_rows_device(const float* d_queries, int64_t nq, const int64_t* d_rows,
                                   int m, float* d_dists, cudaStream_t stream) {
    DeviceGuard g(device_);
    if (!trained_) throw std::invalid_argument("index not trained");
    check_int_rerank("rerank_rows");
    if (nq <= 0 || m <= 0) throw std::invalid_argument("empty rerank request");
    cudaStream_t s = stream ? stream : stream_;
    const int G = D_ / 4;
    w_qrot_.reserve((size_t)nq * D_);
    w_qp_.reserve(nq);
    w_qi8p_.reserve((size_t)nq * D_);
    w_qi8n_.reserve((size_t)nq * D_);
    w_lut_.reserve((size_t)nq * G * 16);
    launch_rotate(d_queries, nq, dim_, D_, Pc_.p, w_qrot_.p, s);
    launch_query_state(d_queries, w_qrot_.p, nq, dim_, D_, rc_.p, nbits_, w_qp_.p, w_qi8p_.p,
                       w_qi8n_.p, w_lut_.p, s);
    RerankRowsArgs a{};
    a.D = D_;
    a.nbits = nbits_;
    a.code_bytes = code_bytes_;
    a.metric_l2 = metric_ == 0 ? 1 : 0;
    a.codes = codes_.p;
    a.meta = meta_.p;
    a.ntotal = ntotal_;
    a.qp = w_qp_.p;
    a.q_i8p = w_qi8p_.p;
    a.rows = d_rows;
    a.nq = nq;
    a.m = m;
    a.out = d_dists;
    launch_rerank_rows(a, s);
    HANNS_CUDA_OK(cudaGetLastError());
    last_launches_ = 3;
    if (!stream) HANNS_CUDA_OK(cudaStreamSynchronize(s));
}

void IvfUsqGpu::prepare_device(const float* d_queries, int64_t nq, int nprobe, QueryState st,
                               cudaStream_t stream) {
    DeviceGuard g(device_);
    if (!trained_) throw std::invalid_argument("index not trained");
    check_int_rerank("prepared (sharded) search");
    if (nq <= 0) throw std::invalid_argument("query dimension mismatch");
    if (!st.probes || !st.qp || !st.lut || !st.q_i8p) throw std::invalid_argument("null query state");
    cudaStream_t s = stream ? stream : stream_;
    nprobe = std::max(1, std::min(nprobe, nlist_));
    if (!st.q_i8n) {
        w_qi8n_.reserve((size_t)nq * D_);
        st.q_i8n = w_qi8n_.p;
    }
    begin_call();
    next_slot(0, 4);
    HANNS_CUDA_OK(cudaEventRecord(ev_[0], s));
    last_launches_ = prepare_batch(d_queries, nullptr, nq, nprobe, st, s, true);
    HANNS_CUDA_OK(cudaEventRecord(ev_[4], s));
    if (!stream) HANNS_CUDA_OK(cudaStreamSynchronize(s));
}

void IvfUsqGpu::search_prepared_device(int64_t nq, const SearchOptions& opt, QueryState st,
                                       int64_t* d_ids, float* d_dists, int64_t* d_counts,
                                       uint64_t* d_keys, cudaStream_t stream) {
    DeviceGuard g(device_);
    if (!trained_) throw std::invalid_argument("index not trained");
    check_int_rerank("prepared (sharded) search");
    if (nq <= 0) throw std::invalid_argument("query dimension mismatch");
    if (!st.probes || !st.qp || !st.lut || !st.q_i8p) throw std::invalid_argument("null query state");
    cudaStream_t s = stream ? stream : stream_;
    const int k = std::max(opt.k, 1);
    const int nprobe = std::max(1, std::min(opt.nprobe, nlist_));
    const int G = D_ / 4;
    const int64_t nb_max = batch_limit(nprobe, k);
    last_launches_ = 0;
    begin_call();
    for (int64_t b = 0; b < nq; b += nb_max) {
        const int64_t nb = std::min(nb_max, nq - b);
        SearchOptions o = opt;
        if (o.d_query_bitset) o.d_query_bitset += b;
        const QueryState sb{st.probes + b * nprobe, st.qp + b, st.lut + b * G * 16,
                            st.q_i8p + b * D_, st.q_i8n ? st.q_i8n + b * D_ : nullptr};
        next_slot(4, kStages);
        HANNS_CUDA_OK(cudaEventRecord(ev_[4], s));
        last_launches_ += scan_merge_batch(nb, o, sb, d_ids + b * k, d_dists + b * k,
                                           d_counts ? d_counts + b : nullptr,
                                           d_keys ? d_keys + b * k : nullptr, s, true);
        check_tc_scan();
    }
    if (!stream) {
        HANNS_CUDA_OK(cudaStreamSynchronize(s));
        check_tc_scan();
    }
}

void IvfUsqGpu::search_host(const float* h_queries, int64_t nq, const SearchOptions& opt_in,
                            const uint64_t* h_bitsets, const int32_t* h_query_bitset,
                            int64_t* h_ids, float* h_dists, int64_t* h_counts) {
    DeviceGuard g(device_);
    SearchOptions opt = opt_in;
    const int k = std::max(opt.k, 1);
    opt.k = k;
    if (!trained_) throw std::invalid_argument("index not trained");
    if (nq <= 0) throw std::invalid_argument("query dimension mismatch");
    w_pad_queries_.reserve((size_t)nq * dim_);
    if (h_bitsets && opt.n_bitsets > 0 && opt.filter_mode != 0) {
        const size_t words = (size_t)((opt.bitset_len + 63) / 64) * opt.n_bitsets;
        h2d(w_bits_, h_bitsets, words, stream_);
        opt.d_bitsets = w_bits_.p;
        if (h_query_bitset) {
            h2d(w_qbits_, h_query_bitset, (size_t)nq, stream_);
            opt.d_query_bitset = w_qbits_.p;
        } else {
            opt.d_query_bitset = nullptr;
        }
    } else {
        opt.d_bitsets = nullptr;
        opt.n_bitsets = 0;
        opt.d_query_bitset = nullptr;
    }
    w_out_ids_.reserve((size_t)nq * k);
    w_out_dists_.reserve((size_t)nq * k);
    w_out_counts_.reserve((size_t)nq);
    run_search(w_pad_queries_.p, h_queries, nq, opt, w_out_ids_.p, w_out_dists_.p, w_out_counts_.p,
               nullptr, stream_);
    HANNS_CUDA_OK(cudaMemcpyAsync(h_ids, w_out_ids_.p, sizeof(int64_t) * nq * k,
                                  cudaMemcpyDeviceToHost, stream_));
    HANNS_CUDA_OK(cudaMemcpyAsync(h_dists, w_out_dists_.p, sizeof(float) * nq * k,
                                  cudaMemcpyDeviceToHost, stream_));
    if (h_counts)
        HANNS_CUDA_OK(cudaMemcpyAsync(h_counts, w_out_counts_.p, sizeof(int64_t) * nq,
                                      cudaMemcpyDeviceToHost, stream_));
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
    check_tc_scan();
}

void IvfUsqGpu::debug_candidates(const float* h_queries, int64_t nq, const SearchOptions& opt_in,
                                 const uint64_t* h_bitsets, const int32_t* h_query_bitset,
                                 int64_t cap, int64_t* counts, int32_t* lists, int64_t* local,
                                 int32_t* fs, int32_t* int_ip, float* dists) {
    DeviceGuard g(device_);
    SearchOptions opt = opt_in;
    const int k = std::max(opt.k, 1);
    const int nprobe = std::max(1, std::min(opt.nprobe, nlist_));
    const int64_t stride = cand_stride(nprobe, k);
    (void)stride;
    if (nq > batch_limit(nprobe, k))
        throw std::invalid_argument("debug_candidates: more queries than one internal batch");
    std::vector<int64_t> ids((size_t)nq * k), cnt(nq);
    std::vector<float> d((size_t)nq * k);
    debug_candidates_ = true;
    try {
        search_host(h_queries, nq, opt, h_bitsets, h_query_bitset, ids.data(), d.data(), cnt.data());
    } catch (...) {
        debug_candidates_ = false;
        throw;
    }
    debug_candidates_ = false;
    std::vector<int> off((size_t)nq * (nprobe + 1));
    std::vector<int32_t> probes((size_t)nq * nprobe);
    std::vector<uint32_t> key((size_t)nq * stride);
    std::vector<uint64_t> tie((size_t)nq * stride);
    std::vector<int2> dbg((size_t)nq * stride);
    HANNS_CUDA_OK(cudaMemcpy(off.data(), w_pair_off_.p, sizeof(int) * off.size(), cudaMemcpyDeviceToHost));
    HANNS_CUDA_OK(cudaMemcpy(probes.data(), w_probes_.p, sizeof(int32_t) * probes.size(), cudaMemcpyDeviceToHost));
    HANNS_CUDA_OK(cudaMemcpy(key.data(), w_cand_key_.p, sizeof(uint32_t) * key.size(), cudaMemcpyDeviceToHost));
    HANNS_CUDA_OK(cudaMemcpy(tie.data(), w_cand_tie_.p, sizeof(uint64_t) * tie.size(), cudaMemcpyDeviceToHost));
    HANNS_CUDA_OK(cudaMemcpy(dbg.data(), w_cand_dbg_.p, sizeof(int2) * dbg.size(), cudaMemcpyDeviceToHost));
    std::vector<int64_t> order;
    for (int64_t q = 0; q < nq; ++q) {
        const int64_t base = q * stride;
        const int total = off[q * (nprobe + 1) + nprobe];
        order.clear();
        for (int e = 0; e < total; ++e)
            if (tie[base + e] != ~0ull) order.push_back(base + e);
        // tie = probe rank << 48 | FastScan key (32767 - score, 0 without FastScan) << 32 |
        // position: increasing ties are the reference's candidate order
        std::sort(order.begin(), order.end(), [&](int64_t x, int64_t y) { return tie[x] < tie[y]; });
        if ((int64_t)order.size() > cap) throw std::invalid_argument("debug_candidates: cap too small");
        counts[q] = (int64_t)order.size();
        for (size_t j = 0; j < order.size(); ++j) {
            const int64_t e = order[j], o = q * cap + (int64_t)j;
            const uint64_t t = tie[e];
            lists[o] = probes[q * nprobe + (int)(t >> 48)];
            local[o] = (int64_t)(t & 0xFFFFFFFFull);
            fs[o] = dbg[e].y;
            int_ip[o] = dbg[e].x;
            const uint32_t kk = key[e];
            const uint32_t bits = (kk & 0x80000000u) ? (kk & 0x7FFFFFFFu) : ~kk;
            std::memcpy(&dists[o], &bits, 4);
        }
    }
}

void IvfUsqGpu::debug_query(const float* h_queries, int64_t nq, int nprobe, int32_t* probes,
                            float* q_rot, int8_t* q_i8, int8_t* lut, float* scalars) {
    DeviceGuard g(device_);
    if (!trained_) throw std::invalid_argument("index not trained");
    nprobe = std::max(1, std::min(nprobe, nlist_));
    const int G = D_ / 4;
    h2d(w_pad_queries_, h_queries, (size_t)nq * dim_, stream_);
    w_probes_.reserve((size_t)nq * nprobe);
    w_sel_.reserve((size_t)nq * 2 * nprobe);
    coarse_probes(w_pad_queries_.p, nq, nprobe, w_probes_.p, stream_);
    w_qrot_.reserve((size_t)nq * D_);
    w_qp_.reserve(nq);
    w_qi8p_.reserve((size_t)nq * D_);
    w_qi8n_.reserve((size_t)nq * D_);
    w_lut_.reserve((size_t)nq * G * 16);
    launch_rotate(w_pad_queries_.p, nq, dim_, D_, Pc_.p, w_qrot_.p, stream_);
    launch_query_state(w_pad_queries_.p, w_qrot_.p, nq, dim_, D_, rc_.p, nbits_, w_qp_.p,
                       w_qi8p_.p, w_qi8n_.p, w_lut_.p, stream_);
    HANNS_CUDA_OK(cudaGetLastError());
    HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
    if (probes)
        HANNS_CUDA_OK(cudaMemcpy(probes, w_probes_.p, sizeof(int32_t) * nq * nprobe,
                                 cudaMemcpyDeviceToHost));
    if (q_rot)
        HANNS_CUDA_OK(cudaMemcpy(q_rot, w_qrot_.p, sizeof(float) * nq * D_, cudaMemcpyDeviceToHost));
    if (q_i8)
        HANNS_CUDA_OK(cudaMemcpy(q_i8, w_qi8n_.p, (size_t)nq * D_, cudaMemcpyDeviceToHost));
    if (lut) {
        std::vector<uint8_t> u((size_t)nq * G * 16);
        HANNS_CUDA_OK(cudaMemcpy(u.data(), w_lut_.p, u.size(), cudaMemcpyDeviceToHost));
        for (size_t i = 0; i < u.size(); ++i) lut[i] = (int8_t)((int)u[i] - 128);
    }
    if (scalars) {
        std::vector<QueryParams> qp(nq);
        HANNS_CUDA_OK(cudaMemcpy(qp.data(), w_qp_.p, sizeof(QueryParams) * nq, cudaMemcpyDeviceToHost));
        for (int64_t i = 0; i < nq; ++i) {
            scalars[i * 5 + 0] = qp[i].q_scale;
            scalars[i * 5 + 1] = qp[i].centroid_score;
            scalars[i * 5 + 2] = qp[i].q_norm_sq;
            scalars[i * 5 + 3] = qp[i].lut_scale;
            std::memcpy(&scalars[i * 5 + 4], &qp[i].q_i8_sum, 4);
        }
    }
}

// ---------------------------------------------------------------- persistence
namespace {
const char kMagic[8] = {'H', 'G', 'P', 'U', 'U', 'S', 'Q', '1'};
}

void IvfUsqGpu::save(const std::string& path) const {
    DeviceGuard g(device_);
    std::ofstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open " + path);
    const int64_t hdr[10] = {dim_, nbits_, nlist_, metric_, nprobe_, (int64_t)rotation_seed_,
                             ntotal_, trained_ ? 1 : 0, D_, 0};
    f.write(kMagic, 8);
    f.write(reinterpret_cast<const char*>(hdr), sizeof(hdr));
    auto put = [&](const void* dptr, size_t bytes) {
        std::vector<char> h(bytes);
        if (bytes) HANNS_CUDA_OK(cudaMemcpy(h.data(), dptr, bytes, cudaMemcpyDeviceToHost));
        f.write(h.data(), (std::streamsize)bytes);
    };
    const size_t n = (size_t)ntotal_;
    put(centroids_.p, trained_ ? sizeof(float) * nlist_ * dim_ : 0);
    put(P_.p, trained_ ? sizeof(float) * D_ * D_ : 0);
    put(rc_.p, trained_ ? sizeof(float) * D_ : 0);
    put(gmean_.p, trained_ ? sizeof(float) * dim_ : 0);
    f.write(reinterpret_cast<const char*>(h_list_off_.data()), sizeof(int64_t) * (nlist_ + 1));
    put(ids_.p, sizeof(int64_t) * n);
    put(meta_.p, sizeof(float4) * n);
    put(codes_.p, n * code_bytes_);
    put(signs_.p, n * (D_ / 8));
    if (!f) throw std::runtime_error("write failed: " + path);
}

void IvfUsqGpu::load(const std::string& path) {
    DeviceGuard g(device_);
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open " + path);
    char magic[8];
    int64_t hdr[10];
    f.read(magic, 8);
    f.read(reinterpret_cast<char*>(hdr), sizeof(hdr));
    if (!f || std::memcmp(magic, kMagic, 8) != 0) throw std::runtime_error("not an HGPUUSQ1 file");
    if (hdr[0] != dim_ || hdr[1] != nbits_ || hdr[2] != nlist_)
        throw std::invalid_argument("saved index shape does not match the handle");
    metric_ = (int)hdr[3];
    nprobe_ = (int)hdr[4];
    rotation_seed_ = (uint64_t)hdr[5];
    ntotal_ = hdr[6];
    trained_ = hdr[7] != 0;
    auto get = [&](auto& buf, size_t count) {
        using T = typename std::remove_reference<decltype(*buf.p)>::type;
        std::vector<T> h(count);
        f.read(reinterpret_cast<char*>(h.data()), (std::streamsize)(sizeof(T) * count));
        if (!f) throw std::runtime_error("truncated file: " + path);
        h2d(buf, h.data(), count, stream_);
        HANNS_CUDA_OK(cudaStreamSynchronize(stream_));
    };
    const size_t n = (size_t)ntotal_;
    if (trained_) {
        get(centroids_, (size_t)nlist_ * dim_);
        update_centroid_norms();
        get(P_, (size_t)D_ * D_);
        refresh_rotation();
        get(rc_, (size_t)D_);
        get(gmean_, (size_t)dim_);
    }
    std::vector<int64_t> off(nlist_ + 1);
    f.read(reinterpret_cast<char*>(off.data()), sizeof(int64_t) * (nlist_ + 1));
    get(ids_, n);
    get(meta_, n);
    get(codes_, n * code_bytes_);
    get(signs_, n * (D_ / 8));
    set_list_layout(off);
    rebuild_fastscan();
}

}  // namespace hanns
