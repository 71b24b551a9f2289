// capi.cu -- the C ABI of libhanns_gpu.so (declarations and citations: include/hanns_gpu.h).
#include <cfloat>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <fstream>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "hanns_gpu.h"
#include "ivf_usq_gpu.h"

struct HannsIvfUsqHandle {
    std::unique_ptr<hanns::IvfUsqGpu> idx;
};

namespace {

thread_local std::string g_last_error;

void set_error(const std::string& msg) { g_last_error = msg; }

}  // namespace

namespace hanns {
void set_last_error(const std::string& msg) { set_error(msg); }
}  // namespace hanns

namespace {

// Maps exceptions to CError codes (src/ffi.rs:62-71).
int32_t code_of(const std::exception& e) {
    if (dynamic_cast<const std::invalid_argument*>(&e)) return HANNS_INVALID_ARG;
    if (dynamic_cast<const std::domain_error*>(&e)) return HANNS_NOT_IMPLEMENTED;
    if (auto* ce = dynamic_cast<const hanns::CudaError*>(&e))
        return ce->code == cudaErrorMemoryAllocation ? HANNS_OUT_OF_MEMORY : HANNS_INTERNAL;
    return HANNS_INTERNAL;
}

template <class F>
int32_t guarded(F&& f) {
    try {
        f();
        return HANNS_OK;
    } catch (const std::exception& e) {
        set_error(e.what());
        return code_of(e);
    } catch (...) {
        set_error("unknown error");
        return HANNS_INTERNAL;
    }
}

int default_device() {
    const char* e = std::getenv("HANNS_GPU_DEVICE");
    return e ? std::atoi(e) : 0;
}

int kmeans_iters() {
    const char* e = std::getenv("HANNS_GPU_KMEANS_ITERS");
    return e ? std::atoi(e) : 25;
}

hanns::IvfUsqGpu* as_index(const void* p) {
    return p ? static_cast<const HannsIvfUsqHandle*>(p)->idx.get() : nullptr;
}

CSearchResult* make_result(const std::vector<int64_t>& ids, const std::vector<float>& d,
                           float ms) {
    auto* r = static_cast<CSearchResult*>(std::malloc(sizeof(CSearchResult)));
    if (!r) return nullptr;
    r->num_results = ids.size();
    r->ids = static_cast<int64_t*>(std::malloc(sizeof(int64_t) * std::max<size_t>(ids.size(), 1)));
    r->distances = static_cast<float*>(std::malloc(sizeof(float) * std::max<size_t>(d.size(), 1)));
    if (!r->ids || !r->distances) {
        std::free(r->ids);
        std::free(r->distances);
        std::free(r);
        return nullptr;
    }
    if (!ids.empty()) std::memcpy(r->ids, ids.data(), sizeof(int64_t) * ids.size());
    if (!d.empty()) std::memcpy(r->distances, d.data(), sizeof(float) * d.size());
    r->elapsed_ms = ms;
    return r;
}

CSearchResult* search_common(const void* index, const float* query, size_t count, size_t top_k,
                             size_t dim, const CBitset* bitset) {
    auto* idx = as_index(index);
    if (!idx || !query || count == 0 || top_k == 0 || dim == 0) return nullptr;
    if ((int)dim != idx->dim()) {
        set_error("query dimension mismatch");
        return nullptr;
    }
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<int64_t> ids(count * top_k), counts(count);
    std::vector<float> dists(count * top_k);
    bool post = false;
    int32_t rc = guarded([&] {
        std::lock_guard<std::mutex> lk(idx->mutex());
        hanns::SearchOptions opt;
        opt.k = (int)top_k;
        opt.nprobe = idx->nprobe();
        const uint64_t* words = nullptr;
        if (bitset && bitset->data && bitset->len > 0) {
            const char* mode = std::getenv("HANNS_GPU_BITSET_MODE");
            post = mode && std::strcmp(mode, "post") == 0;
            opt.filter_mode = post ? HANNS_FILTER_POST : HANNS_FILTER_FUSED;
            opt.bitset_len = (int64_t)bitset->len;
            opt.n_bitsets = 1;
            words = bitset->data;
        }
        idx->search_host(query, (int64_t)count, opt, words, nullptr, ids.data(), dists.data(),
                         counts.data());
    });
    if (rc != HANNS_OK) return nullptr;
    const double us =
        std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
    if (std::getenv("HANNS_TRACE_SEARCH")) {
        float st[8];
        idx->stage_ms(1, st);
        std::fprintf(stderr,
                     "TRACE_SEARCH nq=%zu elapsed_us=%.0f coarse_ms=%.3f prep_ms=%.3f "
                     "group_ms=%.3f scan_ms=%.3f merge_ms=%.3f\n",
                     count, us, st[0] + st[1], st[2] + st[3], st[4], st[5], st[6]);
    }
    if (post) {  // reference post-filter: rows concatenated, filtered entries dropped
        std::vector<int64_t> fid;
        std::vector<float> fd;
        for (size_t q = 0; q < count; ++q)
            for (int64_t j = 0; j < counts[q]; ++j) {
                fid.push_back(ids[q * top_k + j]);
                fd.push_back(dists[q * top_k + j]);
            }
        return make_result(fid, fd, (float)(us / 1000.0));
    }
    return make_result(ids, dists, (float)(us / 1000.0));
}

}  // namespace

extern "C" {

const char* hanns_gpu_last_error(void) { return g_last_error.c_str(); }

int32_t hanns_gpu_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
    return n;
}

// ------------------------------------------------------------------ KnowHere ABI
void* knowhere_create_index(CIndexConfig config) {
    if (config.index_type != CINDEX_IVF_RABITQ && config.index_type != CINDEX_IVF_USQ) {
        set_error("libhanns_gpu builds the IVF-USQ index kind only");
        return nullptr;
    }
    if (config.dim == 0) {
        set_error("dimension must be > 0");
        return nullptr;
    }
    HannsIvfUsqHandle* h = nullptr;
    guarded([&] {
        const int nlist = config.num_clusters ? (int)config.num_clusters : 100;
        const int nbits = config.prq_nbits ? (int)config.prq_nbits : 4;
        const int metric = config.metric_type == CMETRIC_L2 ? 0 : 1;
        auto idx = std::make_unique<hanns::IvfUsqGpu>((int)config.dim, nlist, nbits, metric, 42ull,
                                                      config.nprobe ? (int)config.nprobe : 8,
                                                      default_device());
        h = new HannsIvfUsqHandle{std::move(idx)};
    });
    return h;
}

void knowhere_free_index(void* index) { delete static_cast<HannsIvfUsqHandle*>(index); }

int32_t knowhere_train_index(void* index, const float* vectors, size_t count, size_t dim) {
    auto* idx = as_index(index);
    if (!idx || !vectors || count == 0 || dim == 0) return HANNS_INVALID_ARG;
    if ((int)dim != idx->dim()) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(idx->mutex());
        idx->train(vectors, (int64_t)count, kmeans_iters(), 42ull);
    });
}

int32_t knowhere_add_index(void* index, const float* vectors, const int64_t* ids, size_t count,
                           size_t dim) {
    auto* idx = as_index(index);
    if (!idx || !vectors || count == 0 || dim == 0) return HANNS_INVALID_ARG;
    if ((int)dim != idx->dim()) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(idx->mutex());
        idx->add(vectors, (int64_t)count, ids);
    });
}

CSearchResult* knowhere_search(const void* index, const float* query, size_t count, size_t top_k,
                               size_t dim) {
    return search_common(index, query, count, top_k, dim, nullptr);
}

CSearchResult* knowhere_search_with_bitset(const void* index, const float* query, size_t count,
                                           size_t top_k, size_t dim, const CBitset* bitset) {
    if (!bitset) return nullptr;
    return search_common(index, query, count, top_k, dim, bitset);
}

int32_t knowhere_set_nprobe(void* index, size_t nprobe) {
    auto* idx = as_index(index);
    if (!idx || nprobe == 0) return HANNS_INVALID_ARG;
    idx->set_nprobe((int)std::min<size_t>(nprobe, 1u << 30));
    return HANNS_OK;
}

void knowhere_free_result(CSearchResult* result) {
    if (!result) return;
    std::free(result->ids);
    std::free(result->distances);
    std::free(result);
}

size_t knowhere_get_index_count(const void* index) {
    auto* idx = as_index(index);
    return idx ? (size_t)idx->count() : 0;
}
size_t knowhere_get_index_dim(const void* index) {
    auto* idx = as_index(index);
    return idx ? (size_t)idx->dim() : 0;
}
size_t knowhere_get_index_size(const void* index) {
    auto* idx = as_index(index);
    return idx ? (size_t)idx->size_bytes() : 0;
}
const char* knowhere_get_index_type(const void* index) { return index ? "IVF-USQ" : "Unknown"; }
const char* knowhere_get_index_metric(const void* index) {
    auto* idx = as_index(index);
    if (!idx) return "Unknown";
    return idx->metric() == 0 ? "L2" : "IP";
}
bool knowhere_has_raw_data(const void* index) { return false; }

int32_t knowhere_save_index(const void* index, const char* path) {
    auto* idx = as_index(index);
    if (!idx || !path) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(idx->mutex());
        idx->save(path);
    });
}
namespace {

// Host copy of an IVFUSQ00 snapshot in artifact form (owning arrays).
struct Ivfusq00Artifact {
    int64_t hdr[10];
    std::vector<float> cent, rot, rc, norms, norms_sq, vmaxs, quals;
    std::vector<int64_t> off, ids;
    std::vector<uint8_t> codes, signs;
    hanns_ivf_usq_artifact_t art{};
};

bool is_ivfusq00(const char* path) {
    std::ifstream f(path, std::ios::binary);
    char m[8] = {};
    f.read(m, 8);
    return f && (std::memcmp(m, "IVFUSQ00", 8) == 0 || std::memcmp(m, "IVFXRBTQ", 8) == 0);
}

void read_ivfusq00(const char* path, Ivfusq00Artifact& s) {
    if (hanns_ivfusq00_read_header(path, s.hdr) != HANNS_OK)
        throw std::invalid_argument(hanns_gpu_last_error());
    const int64_t d = s.hdr[0], D = s.hdr[1], nbits = s.hdr[2], nlist = s.hdr[3], n = s.hdr[5];
    const int64_t cb = (D * nbits + 7) / 8;
    s.cent.resize(nlist * d);
    s.rot.resize(D * D);
    s.rc.resize(D);
    s.off.resize(nlist + 1);
    s.ids.resize(n);
    s.norms.resize(n);
    s.norms_sq.resize(n);
    s.vmaxs.resize(n);
    s.quals.resize(n);
    s.codes.resize(n * cb);
    s.signs.resize(n * (D / 8));
    hanns_ivf_usq_artifact_t& a = s.art;
    a.dim = (int32_t)d;
    a.padded_dim = (int32_t)D;
    a.nbits = (int32_t)nbits;
    a.nlist = (int32_t)nlist;
    a.metric = (int32_t)s.hdr[4];
    a.ntotal = n;
    a.centroids = s.cent.data();
    a.rotation = s.rot.data();
    a.rotated_centroid = s.rc.data();
    a.list_offsets = s.off.data();
    a.ids = s.ids.data();
    a.norms = s.norms.data();
    a.norms_sq = s.norms_sq.data();
    a.vmaxs = s.vmaxs.data();
    a.quant_qualities = s.quals.data();
    a.codes = s.codes.data();
    a.sign_bits = s.signs.data();
    if (hanns_ivfusq00_read(path, &a) != HANNS_OK) throw std::invalid_argument(hanns_gpu_last_error());
    if (!(s.hdr[9] & 1)) throw std::invalid_argument("IVFUSQ00 snapshot of an untrained index");
    if (a.metric > 2) throw std::invalid_argument("IVFUSQ00: Hamming metric is not an IVF-USQ search metric");
}

}  // namespace

int32_t knowhere_load_index(void* index, const char* path) {
    auto* idx = as_index(index);
    if (!idx || !path) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(idx->mutex());
        if (is_ivfusq00(path)) {  // the reference's IvfUsqIndex::save format
            Ivfusq00Artifact s;
            read_ivfusq00(path, s);
            if (s.art.dim != idx->dim() || s.art.nlist != idx->nlist() || s.art.nbits != idx->nbits())
                throw std::invalid_argument("IVFUSQ00 snapshot shape differs from the index config");
            idx->import_artifact(&s.art);
            idx->set_nprobe((int)s.hdr[6]);
        } else {
            idx->load(path);
        }
    });
}

CBitset* knowhere_bitset_create(size_t len) {
    auto* b = static_cast<CBitset*>(std::malloc(sizeof(CBitset)));
    if (!b) return nullptr;
    b->len = len;
    b->cap_words = (len + 63) / 64;
    b->data = static_cast<uint64_t*>(std::calloc(std::max<size_t>(b->cap_words, 1), 8));
    if (!b->data) {
        std::free(b);
        return nullptr;
    }
    return b;
}
void knowhere_bitset_free(CBitset* b) {
    if (!b) return;
    std::free(b->data);
    std::free(b);
}
void knowhere_bitset_set(CBitset* b, size_t i, bool v) {
    if (!b || i >= b->len) return;
    if (v)
        b->data[i >> 6] |= 1ull << (i & 63);
    else
        b->data[i >> 6] &= ~(1ull << (i & 63));
}
bool knowhere_bitset_get(const CBitset* b, size_t i) {
    if (!b || i >= b->len) return false;
    return (b->data[i >> 6] >> (i & 63)) & 1ull;
}
size_t knowhere_bitset_count(const CBitset* b) {
    if (!b) return 0;
    size_t c = 0;
    for (size_t w = 0; w < (b->len + 63) / 64; ++w) {
        uint64_t x = b->data[w];
        if (w == (b->len - 1) / 64 && (b->len & 63)) x &= (1ull << (b->len & 63)) - 1;
        c += (size_t)__builtin_popcountll(x);
    }
    return c;
}
size_t knowhere_bitset_size(const CBitset* b) { return b ? b->len : 0; }
const uint64_t* knowhere_bitset_data(const CBitset* b) { return b ? b->data : nullptr; }

// ------------------------------------------------------------ per-index ABI
HannsIvfUsqHandle* knowhere_ivf_exrabitq_build(uint32_t dim, uint32_t nlist, uint32_t bits_per_dim,
                                               const float* data, uint64_t n, const int64_t* ids) {
    if (!data || dim == 0 || nlist == 0 || bits_per_dim == 0 || n == 0) return nullptr;
    HannsIvfUsqHandle* h = nullptr;
    guarded([&] {
        auto idx = std::make_unique<hanns::IvfUsqGpu>((int)dim, (int)nlist, (int)bits_per_dim, 0,
                                                      42ull, 1, default_device());
        idx->train(data, (int64_t)n, kmeans_iters(), 42ull);
        idx->add(data, (int64_t)n, ids);
        h = new HannsIvfUsqHandle{std::move(idx)};
    });
    return h;
}

HannsIvfUsqHandle* knowhere_ivf_exrabitq_load(const char* path) {
    if (!path) return nullptr;
    HannsIvfUsqHandle* h = nullptr;
    guarded([&] {
        std::FILE* f = std::fopen(path, "rb");
        if (!f) throw std::runtime_error(std::string("cannot open ") + path);
        char magic[8];
        int64_t hdr[10];
        const bool ok = std::fread(magic, 1, 8, f) == 8 && std::fread(hdr, 8, 10, f) == 10;
        std::fclose(f);
        if (!ok) throw std::runtime_error("truncated index file");
        auto idx = std::make_unique<hanns::IvfUsqGpu>((int)hdr[0], (int)hdr[2], (int)hdr[1],
                                                      (int)hdr[3], (uint64_t)hdr[5], (int)hdr[4],
                                                      default_device());
        idx->load(path);
        h = new HannsIvfUsqHandle{std::move(idx)};
    });
    return h;
}

int32_t knowhere_ivf_exrabitq_save(HannsIvfUsqHandle* index, const char* path) {
    if (!index || !path) return -1;
    return guarded([&] { index->idx->save(path); }) == HANNS_OK ? 0 : -1;
}

int32_t knowhere_ivf_exrabitq_batch_search(const HannsIvfUsqHandle* index, const float* queries,
                                           uint64_t nq, uint32_t k, uint32_t nprobe,
                                           float* distances, int64_t* labels) {
    if (!index || !queries || !distances || !labels || nq == 0 || k == 0) return -1;
    auto* idx = index->idx.get();
    const int32_t rc = guarded([&] {
        std::lock_guard<std::mutex> lk(idx->mutex());
        hanns::SearchOptions opt;
        opt.k = (int)k;
        opt.nprobe = (int)nprobe;
        idx->search_host(queries, (int64_t)nq, opt, nullptr, nullptr, labels, distances, nullptr);
    });
    if (rc != HANNS_OK) {
        // the reference fills failed rows with (-1, f32::MAX) and still returns 0
        for (uint64_t i = 0; i < nq * k; ++i) {
            labels[i] = -1;
            distances[i] = FLT_MAX;
        }
    }
    return 0;
}

int32_t knowhere_ivf_exrabitq_search(const HannsIvfUsqHandle* index, const float* query, uint32_t k,
                                     uint32_t nprobe, float* distances, int64_t* labels) {
    if (!index || !query || !distances || !labels || k == 0) return -1;
    auto* idx = index->idx.get();
    return guarded([&] {
               std::lock_guard<std::mutex> lk(idx->mutex());
               hanns::SearchOptions opt;
               opt.k = (int)k;
               opt.nprobe = (int)nprobe;
               idx->search_host(query, 1, opt, nullptr, nullptr, labels, distances, nullptr);
           }) == HANNS_OK
               ? 0
               : -1;
}

int32_t knowhere_ivf_exrabitq_has_raw_data(const HannsIvfUsqHandle* index) { return 0; }
uint64_t knowhere_ivf_exrabitq_count(const HannsIvfUsqHandle* index) {
    return index ? (uint64_t)index->idx->count() : 0;
}
uint64_t knowhere_ivf_exrabitq_size(const HannsIvfUsqHandle* index) {
    return index ? (uint64_t)index->idx->size_bytes() : 0;
}
void knowhere_ivf_exrabitq_free(HannsIvfUsqHandle* index) { delete index; }
int32_t knowhere_ivf_exrabitq_set_nprobe(HannsIvfUsqHandle* index, uint32_t nprobe) {
    if (!index) return -1;
    index->idx->set_nprobe((int)std::max<uint32_t>(nprobe, 1));
    return 0;
}
uint32_t knowhere_ivf_exrabitq_dim(const HannsIvfUsqHandle* index) {
    return index ? (uint32_t)index->idx->dim() : 0;
}
uint32_t knowhere_ivf_exrabitq_nlist(const HannsIvfUsqHandle* index) {
    return index ? (uint32_t)index->idx->nlist() : 0;
}

// ------------------------------------------------------------ hanns_gpu extras
HannsIvfUsqHandle* hanns_gpu_ivf_usq_create(int32_t dim, int32_t nlist, int32_t nbits,
                                            int32_t metric, uint64_t rotation_seed, int32_t nprobe,
                                            int32_t device) {
    HannsIvfUsqHandle* h = nullptr;
    guarded([&] {
        h = new HannsIvfUsqHandle{std::make_unique<hanns::IvfUsqGpu>(
            dim, nlist, nbits, metric, rotation_seed, nprobe, device < 0 ? default_device() : device)};
    });
    return h;
}

HannsIvfUsqHandle* hanns_gpu_ivf_usq_import(const hanns_ivf_usq_artifact_t* a, int32_t device) {
    if (!a) return nullptr;
    HannsIvfUsqHandle* h = nullptr;
    guarded([&] {
        auto idx = std::make_unique<hanns::IvfUsqGpu>(a->dim, a->nlist, a->nbits, a->metric, 42ull,
                                                      1, device < 0 ? default_device() : device);
        idx->import_artifact(a);
        h = new HannsIvfUsqHandle{std::move(idx)};
    });
    return h;
}

HannsIvfUsqHandle* hanns_gpu_ivf_usq_load_ivfusq00(const char* path, int32_t device) {
    if (!path) return nullptr;
    HannsIvfUsqHandle* h = nullptr;
    guarded([&] {
        Ivfusq00Artifact s;
        read_ivfusq00(path, s);
        auto idx = std::make_unique<hanns::IvfUsqGpu>(s.art.dim, s.art.nlist, s.art.nbits, s.art.metric,
                                                      (uint64_t)s.hdr[7], (int)s.hdr[6],
                                                      device < 0 ? default_device() : device);
        idx->import_artifact(&s.art);
        h = new HannsIvfUsqHandle{std::move(idx)};
    });
    return h;
}

int32_t hanns_gpu_ivf_usq_save_ivfusq00(HannsIvfUsqHandle* h, const char* path, uint64_t rotation_seed,
                                        int64_t rerank_k) {
    if (!h || !path) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        auto* i = h->idx.get();
        const int64_t n = i->count(), D = i->padded_dim(), cb = (D * i->nbits() + 7) / 8;
        std::vector<float> cent((size_t)i->nlist() * i->dim()), rot((size_t)D * D), rc(D), norms(n),
            norms_sq(n), vmaxs(n), quals(n);
        std::vector<int64_t> off(i->nlist() + 1), ids(n);
        std::vector<uint8_t> codes(n * cb), signs(n * (D / 8));
        hanns_ivf_usq_artifact_t a{};
        a.centroids = cent.data();
        a.rotation = rot.data();
        a.rotated_centroid = rc.data();
        a.list_offsets = off.data();
        a.ids = ids.data();
        a.norms = norms.data();
        a.norms_sq = norms_sq.data();
        a.vmaxs = vmaxs.data();
        a.quant_qualities = quals.data();
        a.codes = codes.data();
        a.sign_bits = signs.data();
        i->export_artifact(&a);
        if (hanns_ivfusq00_write(path, &a, i->nprobe(), rotation_seed, rerank_k) != HANNS_OK)
            throw std::invalid_argument(hanns_gpu_last_error());
    });
}

int32_t hanns_gpu_ivf_usq_shape(const HannsIvfUsqHandle* h, int64_t* out6) {
    if (!h || !out6) return HANNS_INVALID_ARG;
    auto* i = h->idx.get();
    out6[0] = i->dim();
    out6[1] = i->padded_dim();
    out6[2] = i->nbits();
    out6[3] = i->nlist();
    out6[4] = i->metric();
    out6[5] = i->count();
    return HANNS_OK;
}

int32_t hanns_gpu_ivf_usq_export(const HannsIvfUsqHandle* h, hanns_ivf_usq_artifact_t* out) {
    if (!h || !out) return HANNS_INVALID_ARG;
    return guarded([&] { h->idx->export_artifact(out); });
}

int32_t hanns_gpu_ivf_usq_train(HannsIvfUsqHandle* h, const float* data, int64_t n, int32_t iters,
                                uint64_t seed) {
    if (!h || !data || n <= 0) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        h->idx->train(data, n, iters, seed);
    });
}

int32_t hanns_gpu_ivf_usq_add(HannsIvfUsqHandle* h, const float* data, int64_t n,
                              const int64_t* ids) {
    if (!h || !data || n <= 0) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        h->idx->add(data, n, ids);
    });
}

int32_t hanns_gpu_ivf_usq_search(HannsIvfUsqHandle* h, const float* queries, int64_t nq, int32_t k,
                                 int32_t nprobe, int32_t filter_mode, const uint64_t* bitsets,
                                 int64_t bitset_len, int64_t n_bitsets,
                                 const int32_t* query_bitset, int64_t* ids, float* dists,
                                 int64_t* counts) {
    if (!h || !queries || nq <= 0 || k <= 0 || !ids || !dists) return HANNS_INVALID_ARG;
    if (filter_mode < 0 || filter_mode > 2) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        hanns::SearchOptions opt;
        opt.k = k;
        opt.nprobe = nprobe;
        opt.filter_mode = bitsets ? filter_mode : 0;
        opt.bitset_len = bitset_len;
        opt.n_bitsets = n_bitsets;
        h->idx->search_host(queries, nq, opt, bitsets, query_bitset, ids, dists, counts);
    });
}

int32_t hanns_gpu_ivf_usq_search_device(HannsIvfUsqHandle* h, const float* d_queries, int64_t nq,
                                        int32_t k, int32_t nprobe, int32_t filter_mode,
                                        const uint64_t* d_bitsets, int64_t bitset_len,
                                        int64_t n_bitsets, const int32_t* d_query_bitset,
                                        int64_t* d_ids, float* d_dists, int64_t* d_counts,
                                        void* stream) {
    if (!h || !d_queries || nq <= 0 || k <= 0 || !d_ids || !d_dists) return HANNS_INVALID_ARG;
    if (filter_mode < 0 || filter_mode > 2) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        hanns::SearchOptions opt;
        opt.k = k;
        opt.nprobe = nprobe;
        opt.filter_mode = d_bitsets ? filter_mode : 0;
        opt.d_bitsets = d_bitsets;
        opt.bitset_len = bitset_len;
        opt.n_bitsets = n_bitsets;
        opt.d_query_bitset = d_query_bitset;
        h->idx->search_device(d_queries, nq, opt, d_ids, d_dists, d_counts, nullptr,
                              static_cast<cudaStream_t>(stream));
    });
}

int32_t hanns_gpu_ivf_usq_stage_ms(HannsIvfUsqHandle* h, float* out8) {
    if (!h || !out8) return HANNS_INVALID_ARG;
    return guarded([&] { h->idx->stage_ms(1, out8); });
}

int32_t hanns_gpu_ivf_usq_stage_ms_recent(HannsIvfUsqHandle* h, int32_t n_calls, float* out8,
                                          int32_t* counts8) {
    if (!h || !out8 || n_calls <= 0) return HANNS_INVALID_ARG;
    int covered = 0;
    const int32_t rc = guarded([&] { covered = h->idx->stage_ms(n_calls, out8, counts8); });
    return rc == HANNS_OK ? covered : -rc;
}

int32_t hanns_gpu_ivf_usq_scan_kernel_ms_recent(HannsIvfUsqHandle* h, int32_t n_calls, float* out3,
                                                int32_t* counts3) {
    if (!h || !out3 || !counts3 || n_calls <= 0) return HANNS_INVALID_ARG;
    int covered = 0;
    const int32_t rc = guarded([&] { covered = h->idx->scan_kernel_ms(n_calls, out3, counts3); });
    return rc == HANNS_OK ? covered : -rc;
}

int64_t hanns_gpu_ivf_usq_last_launches(const HannsIvfUsqHandle* h) {
    return h ? h->idx->last_launches() : 0;
}

int32_t hanns_gpu_ivf_usq_set_nprobe(HannsIvfUsqHandle* h, int32_t nprobe) {
    if (!h || nprobe <= 0) return HANNS_INVALID_ARG;
    h->idx->set_nprobe(nprobe);
    return HANNS_OK;
}

int64_t hanns_gpu_ivf_usq_count(const HannsIvfUsqHandle* h) { return h ? h->idx->count() : 0; }

void hanns_gpu_ivf_usq_free(HannsIvfUsqHandle* h) { delete h; }

int32_t hanns_gpu_ivf_usq_debug_query(HannsIvfUsqHandle* h, const float* queries, int64_t nq,
                                      int32_t nprobe, int32_t* probes, float* q_rot, int8_t* q_i8,
                                      int8_t* lut, float* scalars) {
    if (!h || !queries || nq <= 0) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        h->idx->debug_query(queries, nq, nprobe, probes, q_rot, q_i8, lut, scalars);
    });
}

int32_t hanns_gpu_ivf_usq_debug_candidates(HannsIvfUsqHandle* h, const float* queries, int64_t nq,
                                           int32_t k, int32_t nprobe, int32_t filter_mode,
                                           const uint64_t* bitsets, int64_t bitset_len,
                                           int64_t n_bitsets, const int32_t* query_bitset,
                                           int64_t cap, int64_t* counts, int32_t* lists,
                                           int64_t* local, int32_t* fs, int32_t* int_ip,
                                           float* dists) {
    if (!h || !queries || nq <= 0 || k <= 0 || cap <= 0 || !counts || !lists || !local || !fs ||
        !int_ip || !dists)
        return HANNS_INVALID_ARG;
    if (filter_mode < 0 || filter_mode > 2) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        hanns::SearchOptions opt;
        opt.k = k;
        opt.nprobe = nprobe;
        opt.filter_mode = bitsets ? filter_mode : 0;
        opt.bitset_len = bitset_len;
        opt.n_bitsets = n_bitsets;
        h->idx->debug_candidates(queries, nq, opt, bitsets, query_bitset, cap, counts, lists, local,
                                 fs, int_ip, dists);
    });
}

int32_t hanns_gpu_ivf_usq_set_scan_wait_ns(HannsIvfUsqHandle* h, uint64_t ns) {
    if (!h || ns == 0) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        h->idx->set_scan_wait_ns(ns);
    });
}

int32_t hanns_gpu_debug_inject_fault(const char* what) {
    if (!what) return HANNS_INVALID_ARG;
    int mask = 0;
    if (std::strcmp(what, "alloc") == 0)
        mask = hanns::kFaultAlloc;
    else if (std::strcmp(what, "h2d") == 0)
        mask = hanns::kFaultH2D;
    else if (std::strcmp(what, "none") != 0)
        return HANNS_INVALID_ARG;
    hanns::set_fault_injection(mask);
    return HANNS_OK;
}

int32_t hanns_gpu_ivf_usq_shard(HannsIvfUsqHandle* h, int32_t rank, int32_t world) {
    if (!h) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        h->idx->shard(rank, world);
    });
}

int32_t hanns_gpu_ivf_usq_search_shard_device(HannsIvfUsqHandle* h, const float* d_queries,
                                              int64_t nq, int32_t k, int32_t nprobe,
                                              float* d_dists, uint64_t* d_keys, int64_t* d_ids,
                                              void* stream) {
    if (!h || !d_queries || nq <= 0 || k <= 0 || !d_dists || !d_keys || !d_ids)
        return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        hanns::SearchOptions opt;
        opt.k = k;
        opt.nprobe = nprobe;
        h->idx->search_device(d_queries, nq, opt, d_ids, d_dists, nullptr, d_keys,
                              static_cast<cudaStream_t>(stream));
    });
}

int32_t hanns_gpu_shard_owners(const int64_t* list_sizes, int32_t nlist, int32_t world,
                               int32_t* owner) {
    if (!list_sizes || !owner || nlist <= 0 || world < 1) return HANNS_INVALID_ARG;
    return guarded([&] { hanns::shard_owners(list_sizes, nlist, world, owner); });
}

int32_t hanns_gpu_ivf_usq_query_state_bytes(HannsIvfUsqHandle* h, int32_t nprobe, int64_t* out5) {
    if (!h || !out5) return HANNS_INVALID_ARG;
    return guarded([&] { h->idx->query_state_bytes(nprobe, out5); });
}

int32_t hanns_gpu_ivf_usq_prepare_device(HannsIvfUsqHandle* h, const float* d_queries, int64_t nq,
                                         int32_t nprobe, void* d_probes, void* d_qp, void* d_lut,
                                         void* d_qi8p, void* d_qi8n, void* stream) {
    if (!h || !d_queries || nq <= 0 || !d_probes || !d_qp || !d_lut || !d_qi8p)
        return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        hanns::QueryState st{static_cast<int32_t*>(d_probes), static_cast<hanns::QueryParams*>(d_qp),
                             static_cast<uint8_t*>(d_lut), static_cast<uint8_t*>(d_qi8p),
                             static_cast<int8_t*>(d_qi8n)};
        h->idx->prepare_device(d_queries, nq, nprobe, st, static_cast<cudaStream_t>(stream));
    });
}

int32_t hanns_gpu_ivf_usq_rerank_rows_device(HannsIvfUsqHandle* h, const float* d_queries,
                                              int64_t nq, const int64_t* d_rows, int32_t m,
                                              float* d_dists, void* stream) {
    if (!h || !d_queries || nq <= 0 || !d_rows || m <= 0 || !d_dists) return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        h->idx->rerank_rows_device(d_queries, nq, d_rows, m, d_dists,
                                   static_cast<cudaStream_t>(stream));
    });
}

int32_t hanns_gpu_ivf_usq_search_prepared_shard_device(
    HannsIvfUsqHandle* h, int64_t nq, int32_t k, int32_t nprobe, const void* d_probes,
    const void* d_qp, const void* d_lut, const void* d_qi8p, const void* d_qi8n, float* d_dists,
    uint64_t* d_keys, int64_t* d_ids, void* stream) {
    if (!h || nq <= 0 || k <= 0 || !d_probes || !d_qp || !d_lut || !d_qi8p || !d_dists ||
        !d_keys || !d_ids)
        return HANNS_INVALID_ARG;
    return guarded([&] {
        std::lock_guard<std::mutex> lk(h->idx->mutex());
        hanns::SearchOptions opt;
        opt.k = k;
        opt.nprobe = nprobe;
        hanns::QueryState st{const_cast<int32_t*>(static_cast<const int32_t*>(d_probes)),
                             const_cast<hanns::QueryParams*>(static_cast<const hanns::QueryParams*>(d_qp)),
                             const_cast<uint8_t*>(static_cast<const uint8_t*>(d_lut)),
                             const_cast<uint8_t*>(static_cast<const uint8_t*>(d_qi8p)),
                             const_cast<int8_t*>(static_cast<const int8_t*>(d_qi8n))};
        h->idx->search_prepared_device(nq, opt, st, d_ids, d_dists, nullptr, d_keys,
                                       static_cast<cudaStream_t>(stream));
    });
}

int32_t hanns_gpu_merge_shards_device(const float* d_dists, const uint64_t* d_keys,
                                      const int64_t* d_ids, int32_t world, int64_t nq, int32_t k,
                                      int64_t* d_out_ids, float* d_out_dists, void* stream) {
    if (!d_dists || !d_keys || !d_ids || world < 1 || world > 32 || nq <= 0 || k <= 0)
        return HANNS_INVALID_ARG;
    return guarded([&] {
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        hanns::launch_merge_shards(d_dists, d_keys, d_ids, world, nq, k, d_out_ids, d_out_dists, s);
        HANNS_CUDA_OK(cudaGetLastError());
        HANNS_CUDA_OK(cudaStreamSynchronize(s));
    });
}

}  // extern "C"
