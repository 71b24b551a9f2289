// ivfusq00.cpp -- the reference's IVF-USQ snapshot file ("IVFUSQ00", version 3), host only.
//
// Layout written by IvfUsqIndex::save (src/faiss/ivf_usq.rs:353-406): the 8-byte magic,
// the version (u32 LE), dim (u32 LE), then the bincode 1.3 (fixed-width integers, little
// endian, lengths as u64) encoding of StoredSnapshot (ivf_usq.rs:131-166):
//   config   dim u64, nlist u64, nprobe u64, metric_type u32 (variant index: L2, Ip,
//            Cosine, Hamming), bits_per_dim u64, use_high_accuracy_scan u8,
//            rotation_seed u64, rerank_k u64
//   centroids        u64 length + f32 values (nlist x dim)
//   clusters         u64 count; per cluster: ids (u64 + i64 values), encoded (u64 count;
//                    per vector packed_bits (u64 + bytes), sign_bits (u64 + bytes), norm,
//                    norm_sq, vmax, quant_quality as f32)
//   trained u8, ntotal u64
// IvfUsqIndex::load (ivf_usq.rs:408-506) also accepts the legacy magic "IVFXRBTQ" and a
// bare payload; it rebuilds the quantizer from (dim, bits, rotation_seed) with a zero
// global centroid, so the loaded index scores with rotated_centroid = 0.  The reader
// does the same; the rotation matrix is regenerated from the seed with this library's
// generator (rotation.cpp), which is not the Rust crates' random stream.
#include <cstdint>
#include <cstring>
#include <fstream>
#include <stdexcept>
#include <string>
#include <vector>

#include "hanns_gpu.h"

namespace hanns {
void rotation_matrix(uint64_t seed, int D, float* out);
void set_last_error(const std::string& msg);
}  // namespace hanns

namespace {

const char kMagic[8] = {'I', 'V', 'F', 'U', 'S', 'Q', '0', '0'};
const char kLegacyMagic[8] = {'I', 'V', 'F', 'X', 'R', 'B', 'T', 'Q'};
constexpr uint32_t kVersion = 3;

struct Reader {
    const uint8_t* p;
    size_t n, off = 0;
    void need(size_t k) {
        if (off + k > n) throw std::runtime_error("IVFUSQ00: truncated snapshot");
    }
    template <class T>
    T get() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, p + off, sizeof(T));
        off += sizeof(T);
        return v;
    }
    uint64_t len(uint64_t max_elems) {
        const uint64_t v = get<uint64_t>();
        if (v > max_elems) throw std::runtime_error("IVFUSQ00: implausible length");
        return v;
    }
};

struct Writer {
    std::vector<uint8_t> b;
    template <class T>
    void put(T v) {
        const size_t o = b.size();
        b.resize(o + sizeof(T));
        std::memcpy(b.data() + o, &v, sizeof(T));
    }
    void bytes(const void* src, size_t k) {
        const size_t o = b.size();
        b.resize(o + k);
        if (k) std::memcpy(b.data() + o, src, k);
    }
};

struct Snapshot {
    uint64_t dim = 0, nlist = 0, nprobe = 0, bits = 0, seed = 0, rerank_k = 0, ntotal = 0;
    uint32_t metric = 0;
    uint8_t high_accuracy = 0, trained = 0;
    std::vector<float> centroids;
    std::vector<int64_t> offsets, ids;
    std::vector<float> norms, norms_sq, vmaxs, quals;
    std::vector<uint8_t> codes, signs;
};

Snapshot parse(const std::string& path) {
    std::ifstream f(path, std::ios::binary);
    if (!f) throw std::runtime_error("cannot open " + path);
    std::vector<uint8_t> all((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    size_t start = 0;
    if (all.size() >= 16 && (std::memcmp(all.data(), kMagic, 8) == 0 ||
                             std::memcmp(all.data(), kLegacyMagic, 8) == 0))
        start = 16;
    Reader r{all.data() + start, all.size() - start};
    Snapshot s;
    s.dim = r.get<uint64_t>();
    s.nlist = r.get<uint64_t>();
    s.nprobe = r.get<uint64_t>();
    s.metric = r.get<uint32_t>();
    s.bits = r.get<uint64_t>();
    s.high_accuracy = r.get<uint8_t>();
    s.seed = r.get<uint64_t>();
    s.rerank_k = r.get<uint64_t>();
    if (s.dim == 0 || s.dim > (1u << 20) || s.nlist == 0 || s.nlist > (1u << 28) || s.bits < 1 ||
        s.bits > 8 || s.metric > 3)
        throw std::runtime_error("IVFUSQ00: bad config");
    const uint64_t D = (s.dim + 63) / 64 * 64;
    const uint64_t code_bytes = (D * s.bits + 7) / 8, sign_bytes = D / 8;
    const uint64_t nc = r.len(r.n / 4);
    s.centroids.resize(nc);
    r.need(nc * 4);
    std::memcpy(s.centroids.data(), r.p + r.off, nc * 4);
    r.off += nc * 4;
    const uint64_t ncl = r.len(1ull << 28);
    if (ncl != s.nlist) throw std::runtime_error("IVFUSQ00: cluster count differs from nlist");
    s.offsets.assign(1, 0);
    for (uint64_t c = 0; c < ncl; ++c) {
        const uint64_t nid = r.len(r.n / 8);
        const size_t i0 = s.ids.size();
        s.ids.resize(i0 + nid);
        r.need(nid * 8);
        std::memcpy(s.ids.data() + i0, r.p + r.off, nid * 8);
        r.off += nid * 8;
        const uint64_t nenc = r.len(r.n / 32);
        if (nenc != nid) throw std::runtime_error("IVFUSQ00: ids and codes differ in count");
        for (uint64_t e = 0; e < nenc; ++e) {
            const uint64_t pb = r.len(r.n);
            if (pb != code_bytes) throw std::runtime_error("IVFUSQ00: packed_bits length mismatch");
            r.need(pb);
            s.codes.insert(s.codes.end(), r.p + r.off, r.p + r.off + pb);
            r.off += pb;
            const uint64_t sb = r.len(r.n);
            if (sb != sign_bytes) throw std::runtime_error("IVFUSQ00: sign_bits length mismatch");
            r.need(sb);
            s.signs.insert(s.signs.end(), r.p + r.off, r.p + r.off + sb);
            r.off += sb;
            s.norms.push_back(r.get<float>());
            s.norms_sq.push_back(r.get<float>());
            s.vmaxs.push_back(r.get<float>());
            s.quals.push_back(r.get<float>());
        }
        s.offsets.push_back((int64_t)s.ids.size());
    }
    s.trained = r.get<uint8_t>();
    s.ntotal = r.get<uint64_t>();
    if (nc != s.nlist * s.dim && !(nc == 0 && !s.trained))
        throw std::runtime_error("IVFUSQ00: centroid count differs from nlist x dim");
    if (s.ntotal != s.ids.size()) throw std::runtime_error("IVFUSQ00: ntotal differs from the clusters");
    return s;
}

template <class F>
int32_t guard(F&& f) {
    try {
        f();
        return HANNS_OK;
    } catch (const std::exception& e) {
        hanns::set_last_error(e.what());
        return HANNS_INVALID_ARG;
    }
}

}  // namespace

extern "C" {

int32_t hanns_ivfusq00_read_header(const char* path, int64_t* out10) {
    if (!path || !out10) return HANNS_INVALID_ARG;
    return guard([&] {
        const Snapshot s = parse(path);
        const int64_t D = (int64_t)(s.dim + 63) / 64 * 64;
        const int64_t v[10] = {(int64_t)s.dim, D, (int64_t)s.bits, (int64_t)s.nlist,
                               (int64_t)s.metric, (int64_t)s.ntotal, (int64_t)s.nprobe,
                               (int64_t)s.seed, (int64_t)s.rerank_k,
                               (int64_t)(s.trained ? 1 : 0) | ((int64_t)s.high_accuracy << 1)};
        std::memcpy(out10, v, sizeof(v));
    });
}

int32_t hanns_ivfusq00_read(const char* path, hanns_ivf_usq_artifact_t* out) {
    if (!path || !out) return HANNS_INVALID_ARG;
    return guard([&] {
        const Snapshot s = parse(path);
        const int D = (int)((s.dim + 63) / 64 * 64);
        if (out->dim != (int32_t)s.dim || out->padded_dim != D || out->nbits != (int32_t)s.bits ||
            out->nlist != (int32_t)s.nlist || out->ntotal != (int64_t)s.ntotal)
            throw std::runtime_error("IVFUSQ00: destination shape differs from the file");
        out->metric = (int32_t)s.metric;
        auto put = [](const void* dst, const void* src, size_t bytes) {
            if (bytes) {
                if (!dst) throw std::runtime_error("IVFUSQ00: null destination array");
                std::memcpy(const_cast<void*>(dst), src, bytes);
            }
        };
        put(out->centroids, s.centroids.data(), s.centroids.size() * 4);
        std::vector<float> P((size_t)D * D);
        hanns::rotation_matrix(s.seed, D, P.data());
        put(out->rotation, P.data(), P.size() * 4);
        std::vector<float> rc((size_t)D, 0.0f);  // zero global centroid, as the reference loads
        put(out->rotated_centroid, rc.data(), rc.size() * 4);
        put(out->list_offsets, s.offsets.data(), s.offsets.size() * 8);
        put(out->ids, s.ids.data(), s.ids.size() * 8);
        put(out->norms, s.norms.data(), s.norms.size() * 4);
        put(out->norms_sq, s.norms_sq.data(), s.norms_sq.size() * 4);
        put(out->vmaxs, s.vmaxs.data(), s.vmaxs.size() * 4);
        put(out->quant_qualities, s.quals.data(), s.quals.size() * 4);
        put(out->codes, s.codes.data(), s.codes.size());
        put(out->sign_bits, s.signs.data(), s.signs.size());
    });
}

int32_t hanns_ivfusq00_write(const char* path, const hanns_ivf_usq_artifact_t* a, int64_t nprobe,
                             uint64_t rotation_seed, int64_t rerank_k) {
    if (!path || !a || a->dim <= 0 || a->nlist <= 0 || a->nbits < 1 || a->nbits > 8 ||
        a->metric < 0 || a->metric > 3)
        return HANNS_INVALID_ARG;
    return guard([&] {
        const int D = a->padded_dim;
        const uint64_t code_bytes = ((uint64_t)D * a->nbits + 7) / 8, sign_bytes = D / 8;
        Writer w;
        w.bytes(kMagic, 8);
        w.put<uint32_t>(kVersion);
        w.put<uint32_t>((uint32_t)a->dim);
        w.put<uint64_t>((uint64_t)a->dim);
        w.put<uint64_t>((uint64_t)a->nlist);
        w.put<uint64_t>((uint64_t)nprobe);
        w.put<uint32_t>((uint32_t)a->metric);
        w.put<uint64_t>((uint64_t)a->nbits);
        w.put<uint8_t>(0);  // use_high_accuracy_scan
        w.put<uint64_t>(rotation_seed);
        w.put<uint64_t>((uint64_t)rerank_k);
        w.put<uint64_t>((uint64_t)a->nlist * a->dim);
        w.bytes(a->centroids, (size_t)a->nlist * a->dim * 4);
        w.put<uint64_t>((uint64_t)a->nlist);
        for (int c = 0; c < a->nlist; ++c) {
            const int64_t b = a->list_offsets[c], e = a->list_offsets[c + 1];
            if (e < b) throw std::runtime_error("list offsets not monotone");
            w.put<uint64_t>((uint64_t)(e - b));
            w.bytes(a->ids + b, (size_t)(e - b) * 8);
            w.put<uint64_t>((uint64_t)(e - b));
            for (int64_t r = b; r < e; ++r) {
                w.put<uint64_t>(code_bytes);
                w.bytes(a->codes + r * code_bytes, code_bytes);
                w.put<uint64_t>(sign_bytes);
                w.bytes(a->sign_bits + r * sign_bytes, sign_bytes);
                w.put<float>(a->norms[r]);
                w.put<float>(a->norms_sq[r]);
                w.put<float>(a->vmaxs[r]);
                w.put<float>(a->quant_qualities[r]);
            }
        }
        w.put<uint8_t>(1);  // trained
        w.put<uint64_t>((uint64_t)a->ntotal);
        std::ofstream f(path, std::ios::binary);
        if (!f) throw std::runtime_error(std::string("cannot write ") + path);
        f.write(reinterpret_cast<const char*>(w.b.data()), (std::streamsize)w.b.size());
        if (!f) throw std::runtime_error(std::string("write failed: ") + path);
    });
}

}  // extern "C"
