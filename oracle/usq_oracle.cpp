// usq_oracle.cpp -- CPU restatement of Hanns' IVF-USQ search arithmetic.
//
// TEST INFRASTRUCTURE ONLY: the checker for the CUDA path and the timed CPU
// baseline.  The product library (hanns_b200/csrc) never links or calls this code.
// Parity against the Rust binary is UNPINNED (see usq_oracle.h for why and for
// the list of reference files restated here).
//
// Build: oracle/Makefile (g++ -O2 -ffp-contract=off -fno-fast-math -fopenmp).
// Floating point follows Rust semantics: no contraction, no reassociation,
// round() = half away from zero, sums start from -0.0 (Rust >= 1.82 Sum<f32>).
#include "usq_oracle.h"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <limits>
#include <vector>

#include <immintrin.h>
#include <omp.h>

namespace {

constexpr float kNegZero = -0.0f;

inline int32_t padded_dim_of(int32_t d) { return (d + 63) / 64 * 64; }

inline uint32_t total_order_key(float f) {
    // Rust f32::total_cmp as an unsigned key: negatives reversed, -0 < +0.
    uint32_t b;
    std::memcpy(&b, &f, 4);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

inline float rust_max(float a, float b) { return std::fmax(a, b); }  // NaN-ignoring like f32::max

// (v).round().clamp(lo, hi) as iN   (NaN -> 0, Rust saturating cast)
inline int32_t round_clamp(float v, float lo, float hi) {
    float r = std::round(v);
    if (std::isnan(r)) return 0;
    if (r < lo) r = lo;
    if (r > hi) r = hi;
    return (int32_t)r;
}

bool cpu_has_avx512() {
    static int cached = -1;
    if (cached < 0) {
        __builtin_cpu_init();
        cached = (__builtin_cpu_supports("avx512f") && __builtin_cpu_supports("avx512bw") &&
                  __builtin_cpu_supports("avx512vnni"))
                     ? 1
                     : 0;
    }
    return cached == 1;
}

// ---------------------------------------------------------------------------
// Rotation  (rotator.rs:56-120)
// AVX-512 path: lane j (0..15) accumulates fma(P[r][c], x[c], acc) over
// c = j, j+16, ...; the 16 lanes are then summed by the halving tree
// s8[i]=a[i]+a[i+8], s4[i]=s8[i]+s8[i+4], s2[i]=s4[i]+s4[i+2], s2[0]+s2[1]
// (the order of _mm512_reduce_add_ps).  Scalar path: sequential sum of
// unfused products starting from -0.0.
// ---------------------------------------------------------------------------
inline float tree16(const float* a) {
    float s8[8], s4[4], s2[2];
    for (int i = 0; i < 8; ++i) s8[i] = a[i] + a[i + 8];
    for (int i = 0; i < 4; ++i) s4[i] = s8[i] + s8[i + 4];
    for (int i = 0; i < 2; ++i) s2[i] = s4[i] + s4[i + 2];
    return s2[0] + s2[1];
}

__attribute__((target("avx512f"))) void rotate_avx512(const float* P, int D, const float* x,
                                                       float* out) {
    for (int r = 0; r < D; ++r) {
        const float* row = P + (size_t)r * D;
        __m512 acc = _mm512_setzero_ps();
        for (int c = 0; c < D; c += 16)
            acc = _mm512_fmadd_ps(_mm512_loadu_ps(row + c), _mm512_loadu_ps(x + c), acc);
        alignas(64) float lanes[16];
        _mm512_store_ps(lanes, acc);
        out[r] = tree16(lanes);
    }
}

void rotate_fma_portable(const float* P, int D, const float* x, float* out) {
    for (int r = 0; r < D; ++r) {
        const float* row = P + (size_t)r * D;
        float lanes[16];
        for (int j = 0; j < 16; ++j) lanes[j] = 0.0f;
        for (int c = 0; c < D; c += 16)
            for (int j = 0; j < 16; ++j) lanes[j] = std::fma(row[c + j], x[c + j], lanes[j]);
        out[r] = tree16(lanes);
    }
}

void rotate_scalar(const float* P, int D, const float* x, float* out) {
    for (int r = 0; r < D; ++r) {
        const float* row = P + (size_t)r * D;
        float s = kNegZero;
        for (int c = 0; c < D; ++c) s = s + row[c] * x[c];
        out[r] = s;
    }
}

void rotate(const float* P, int D, const float* x, float* out, int mode) {
    if (mode == OUSQ_MODE_SCALAR) {
        rotate_scalar(P, D, x, out);
    } else if (cpu_has_avx512()) {
        rotate_avx512(P, D, x, out);
    } else {
        rotate_fma_portable(P, D, x, out);
    }
}

// ---------------------------------------------------------------------------
// Bit packing  (turboquant/packed.rs:1-59): LSB-first bit stream.
// ---------------------------------------------------------------------------
void pack_codes(const uint16_t* codes, int64_t n, int nbits, uint8_t* out) {
    int64_t total_bytes = (n * nbits + 7) / 8;
    std::memset(out, 0, (size_t)total_bytes);
    int64_t bit_offset = 0;
    for (int64_t i = 0; i < n; ++i) {
        uint32_t value = codes[i];
        int remaining = nbits;
        while (remaining > 0) {
            int64_t byte_idx = bit_offset / 8;
            int bit_idx = (int)(bit_offset % 8);
            int take = std::min(remaining, 8 - bit_idx);
            uint32_t mask = (1u << take) - 1;
            out[byte_idx] |= (uint8_t)((value & mask) << bit_idx);
            value >>= take;
            bit_offset += take;
            remaining -= take;
        }
    }
}

void unpack_codes(const uint8_t* bytes, int64_t n, int nbits, uint16_t* out) {
    int64_t bit_offset = 0;
    for (int64_t i = 0; i < n; ++i) {
        uint32_t value = 0;
        int written = 0, remaining = nbits;
        while (remaining > 0) {
            int64_t byte_idx = bit_offset / 8;
            int bit_idx = (int)(bit_offset % 8);
            int take = std::min(remaining, 8 - bit_idx);
            uint32_t mask = (1u << take) - 1;
            uint32_t chunk = ((uint32_t)bytes[byte_idx] >> bit_idx) & mask;
            value |= chunk << written;
            written += take;
            bit_offset += take;
            remaining -= take;
        }
        out[i] = (uint16_t)value;
    }
}

// ---------------------------------------------------------------------------
// Encode  (quantizer.rs:124-230, 421-437, 442-672)
// ---------------------------------------------------------------------------
float unit_vmax(const float* o, int D) {
    float m = 0.0f;
    for (int i = 0; i < D; ++i) m = rust_max(m, std::fabs(o[i]));
    return rust_max(m, 1e-6f);
}

inline float objective(float ip, float qed) { return qed > 1e-12f ? ip * ip / qed : 0.0f; }

// greedy_quantize_into (quantizer.rs:442-541); returns (ip, qed_length).
void greedy_quantize(const float* o_hat, int D, int nbits, int nrefine, uint16_t* codes,
                     float* out_ip, float* out_qed) {
    float max_v = 0.0f;
    for (int i = 0; i < D; ++i) max_v = rust_max(max_v, std::fabs(o_hat[i]));
    max_v = rust_max(max_v, 1e-6f);
    const float levels = (float)(1u << nbits);
    float scale = (2.0f * max_v) / std::fmax(levels, 1.0f);
    if (std::fabs(scale) < 1e-6f) scale = 1e-6f;
    const float offset = -max_v;
    const int max_code = (1 << nbits) - 1;
    auto dequant = [&](int c) { return (float)c * scale + offset; };

    for (int i = 0; i < D; ++i)
        codes[i] = (uint16_t)round_clamp((o_hat[i] - offset) / scale, 0.0f, (float)max_code);

    float ip = kNegZero;
    for (int i = 0; i < D; ++i) ip = ip + dequant(codes[i]) * o_hat[i];
    float qed = kNegZero;
    for (int i = 0; i < D; ++i) {
        float v = dequant(codes[i]);
        qed = qed + v * v;
    }
    float obj = objective(ip, qed);

    const int max_refine = std::min(nrefine, 6);
    for (int round = 0; round < max_refine; ++round) {
        bool improved = false;
        for (int i = 0; i < D; ++i) {
            const int current = codes[i];
            const float old_val = dequant(current);
            const float target_val = std::fabs(ip) > 1e-12f ? o_hat[i] * qed / ip : o_hat[i];
            const int target_code =
                round_clamp((target_val - offset) / scale, 0.0f, (float)max_code);
            int cands[5];
            int nc = 0;
            auto push = [&](int c) {
                if (c < 0 || c > max_code) return;
                if (c == current) return;
                for (int j = 0; j < nc; ++j)
                    if (cands[j] == c) return;
                cands[nc++] = c;
            };
            push(target_code - 1);
            push(target_code);
            push(target_code + 1);
            push(current - 1);
            push(current + 1);

            int best_code = current;
            float best_ip = ip, best_qed = qed, best_obj = obj;
            for (int j = 0; j < nc; ++j) {
                const float new_val = dequant(cands[j]);
                const float new_ip = ip - o_hat[i] * old_val + o_hat[i] * new_val;
                const float new_qed = qed - old_val * old_val + new_val * new_val;
                if (new_qed <= 1e-12f) continue;
                const float new_obj = objective(new_ip, new_qed);
                if (new_obj > best_obj + 1e-10f) {
                    best_code = cands[j];
                    best_ip = new_ip;
                    best_qed = new_qed;
                    best_obj = new_obj;
                }
            }
            if (best_code != current) {
                codes[i] = (uint16_t)best_code;
                ip = best_ip;
                qed = best_qed;
                obj = best_obj;
                improved = true;
            }
        }
        if (!improved) break;
    }
    *out_ip = ip;
    *out_qed = qed;
}

// fast_quantize_into (quantizer.rs:546-650), threshold sweep for nbits < 4.
void fast_quantize(const float* o_hat, int D, int nbits, uint16_t* codes, float* out_ip,
                   float* out_qed) {
    const int levels = 1 << nbits;
    const int half = levels / 2;
    const float half_f = (float)half;
    const int max_code = half;
    const float vmax = unit_vmax(o_hat, D);
    std::vector<float> abs_o(D);
    std::vector<char> non_neg(D);
    std::vector<int> max_level(D);
    for (int i = 0; i < D; ++i) {
        const bool nn = o_hat[i] >= 0.0f;
        abs_o[i] = std::fabs(o_hat[i]);
        non_neg[i] = nn;
        max_level[i] = nn ? std::max(half - 1, 0) : max_code;
    }
    float max_abs = 0.0f;
    for (int i = 0; i < D; ++i) max_abs = rust_max(max_abs, abs_o[i]);
    if (max_abs < 1e-12f) {
        for (int i = 0; i < D; ++i) codes[i] = (uint16_t)half;
        *out_ip = 0.0f;
        *out_qed = 0.0f;
        return;
    }
    struct Ev {
        float t;
        int i, k;
    };
    std::vector<Ev> ev;
    for (int i = 0; i < D; ++i) {
        const float a = abs_o[i];
        if (a < 1e-12f) continue;
        for (int k = 1; k <= max_level[i]; ++k) ev.push_back({((float)k - 0.5f) / a, i, k});
    }
    std::sort(ev.begin(), ev.end(), [](const Ev& x, const Ev& y) {
        uint32_t kx = total_order_key(x.t), ky = total_order_key(y.t);
        if (kx != ky) return kx < ky;
        if (x.i != y.i) return x.i < y.i;
        return x.k < y.k;
    });
    std::vector<int> lev(D, 0);
    float sum_sq = 0.0f, sum_xc = 0.0f, best_obj = 0.0f, best_t = 0.0f, best_sum_sq = 0.0f,
          best_sum_xc = 0.0f;
    size_t ei = 0;
    while (ei < ev.size()) {
        const float cur_t = ev[ei].t;
        uint32_t cur_bits;
        std::memcpy(&cur_bits, &cur_t, 4);
        while (ei < ev.size()) {
            uint32_t b;
            std::memcpy(&b, &ev[ei].t, 4);
            if (b != cur_bits) break;
            const int idx = ev[ei].i, nl = ev[ei].k, ol = lev[idx];
            if (nl > ol) {
                sum_sq += (float)nl * (float)nl - (float)ol * (float)ol;
                sum_xc += (float)(nl - ol) * abs_o[idx];
                lev[idx] = nl;
            }
            ++ei;
        }
        const float obj = sum_sq > 0.0f ? (sum_xc * sum_xc) / sum_sq : 0.0f;
        if (obj > best_obj + 1e-10f) {
            best_obj = obj;
            best_t = cur_t;
            best_sum_sq = sum_sq;
            best_sum_xc = sum_xc;
        }
    }
    const float scale = vmax / std::fmax(half_f, 1.0f);
    *out_ip = scale * best_sum_xc;
    *out_qed = scale * scale * best_sum_sq;
    for (int i = 0; i < D; ++i) {
        int mag = 0;
        if (abs_o[i] > 1e-12f) {
            float f = std::floor(best_t * abs_o[i] + 0.5f);
            int m = std::isnan(f) ? 0 : (f < 0 ? 0 : (f > 65535.0f ? 65535 : (int)f));
            mag = std::min(m, max_level[i]);
        }
        codes[i] = (uint16_t)(non_neg[i] ? half + mag : half - mag);
    }
}

void encode_one(const float* P, int dim, int nbits, const float* centroid, const float* x,
                int mode, uint8_t* codes_out, uint8_t* sign_out, float* meta4) {
    const int D = padded_dim_of(dim);
    float norm_sq_raw = kNegZero;
    for (int i = 0; i < dim; ++i) norm_sq_raw = norm_sq_raw + x[i] * x[i];
    std::vector<float> residual(D, 0.0f), rotated(D), o_hat(D);
    std::vector<uint16_t> codes(D), signs(D);
    for (int i = 0; i < dim; ++i) residual[i] = x[i] - centroid[i];
    rotate(P, D, residual.data(), rotated.data(), mode);

    float nsq = kNegZero;
    for (int i = 0; i < D; ++i) nsq = nsq + rotated[i] * rotated[i];
    const float norm = std::sqrt(nsq);
    if (norm > 1e-12f) {
        const float inv = 1.0f / norm;
        for (int i = 0; i < D; ++i) o_hat[i] = rotated[i] * inv;
    } else {
        for (int i = 0; i < D; ++i) o_hat[i] = rotated[i];
    }
    float ip, qed;
    if (nbits >= 4)
        greedy_quantize(o_hat.data(), D, nbits, 6, codes.data(), &ip, &qed);
    else
        fast_quantize(o_hat.data(), D, nbits, codes.data(), &ip, &qed);
    const float vmax = unit_vmax(o_hat.data(), D);
    const float qq = std::fmax(std::sqrt(qed), 1e-12f);
    pack_codes(codes.data(), D, nbits, codes_out);
    if (nbits == 1) {
        std::memcpy(sign_out, codes_out, (size_t)D / 8);
    } else {
        for (int i = 0; i < D; ++i) signs[i] = o_hat[i] >= 0.0f ? 1 : 0;
        pack_codes(signs.data(), D, 1, sign_out);
    }
    meta4[0] = norm;
    meta4[1] = norm_sq_raw;
    meta4[2] = vmax;
    meta4[3] = qq;
}

// ---------------------------------------------------------------------------
// Query state  (quantizer.rs:236-270) and FastScan LUT (fastscan.rs:22-66)
// ---------------------------------------------------------------------------
struct QueryState {
    std::vector<float> q_rot;
    std::vector<int8_t> q_i8;
    float q_sum = 0, q_scale = 0, centroid_score = 0, q_norm_sq = 0;
    int32_t q_i8_sum = 0;
    std::vector<int8_t> lut;
    float lut_scale = 0;
};

void fastscan_lut(const float* q_rot, int D, int8_t* lut, float* lut_scale) {
    const int G = D / 4;
    std::vector<float> lf((size_t)G * 16);
    for (int g = 0; g < G; ++g) {
        const float* q = q_rot + 4 * g;
        for (int nib = 0; nib < 16; ++nib) {
            float val = 0.0f;
            for (int bit = 0; bit < 4; ++bit) {
                const float sign = ((nib >> bit) & 1) ? 1.0f : -1.0f;
                val += q[bit] * sign;
            }
            lf[(size_t)g * 16 + nib] = val;
        }
    }
    float max_abs = 0.0f;
    for (float v : lf) max_abs = rust_max(max_abs, std::fabs(v));
    max_abs = rust_max(max_abs, 1e-6f);
    const float scale = rust_max(max_abs / 127.0f, 1e-6f);
    for (size_t i = 0; i < lf.size(); ++i)
        lut[i] = (int8_t)round_clamp(lf[i] / scale, -127.0f, 127.0f);
    *lut_scale = scale;
}

void query_state(const ousq_artifact_t* a, const float* q, int mode, QueryState& st) {
    const int d = a->dim, D = a->padded_dim;
    std::vector<float> pad(D, 0.0f);
    std::memcpy(pad.data(), q, sizeof(float) * d);
    st.q_rot.resize(D);
    rotate(a->rotation, D, pad.data(), st.q_rot.data(), mode);
    float s = kNegZero;
    for (int i = 0; i < D; ++i) s = s + st.q_rot[i];
    st.q_sum = s;
    float qm = 0.0f;
    for (int i = 0; i < D; ++i) qm = rust_max(qm, std::fabs(st.q_rot[i]));
    qm = rust_max(qm, 1e-6f);
    st.q_scale = qm / 127.0f;
    st.q_i8.resize(D);
    int32_t qs = 0;
    for (int i = 0; i < D; ++i) {
        st.q_i8[i] = (int8_t)round_clamp(st.q_rot[i] / st.q_scale, -127.0f, 127.0f);
        qs += st.q_i8[i];
    }
    st.q_i8_sum = qs;
    float cs = kNegZero;
    for (int i = 0; i < D; ++i) cs = cs + st.q_rot[i] * a->rotated_centroid[i];
    st.centroid_score = cs;
    float qn = kNegZero;
    for (int i = 0; i < d; ++i) qn = qn + q[i] * q[i];
    st.q_norm_sq = qn;
    st.lut.resize((size_t)D / 4 * 16);
    fastscan_lut(st.q_rot.data(), D, st.lut.data(), &st.lut_scale);
}

// ---------------------------------------------------------------------------
// FastScan blocks (layout.rs:139-197) and block scan (fastscan.rs:150-227)
// ---------------------------------------------------------------------------
void build_blocks(const uint8_t* sign_bits, int64_t n, int D, uint8_t* blocks) {
    const int G = D / 4;
    const int64_t nb = (n + 31) / 32;
    const int sb = D / 8;
    std::memset(blocks, 0, (size_t)(nb * G * 16));
    for (int64_t b = 0; b < nb; ++b) {
        uint8_t* blk = blocks + b * G * 16;
        for (int g = 0; g < G; ++g) {
            for (int slot = 0; slot < 32; ++slot) {
                const int64_t vid = b * 32 + slot;
                uint8_t nib = 0;
                if (vid < n) {
                    const uint8_t* s = sign_bits + vid * sb;
                    for (int bp = 0; bp < 4; ++bp) {
                        const int di = g * 4 + bp;
                        nib |= (uint8_t)(((s[di / 8] >> (di % 8)) & 1) << bp);
                    }
                }
                blk[g * 16 + slot / 2] |= (slot % 2 == 0) ? nib : (uint8_t)(nib << 4);
            }
        }
    }
}

void block_scores_exact(const uint8_t* blk, int G, const int8_t* lut, bool wrap16,
                        int32_t* scores) {
    int32_t acc[32] = {0};
    for (int g = 0; g < G; ++g) {
        const int8_t* l = lut + g * 16;
        for (int slot = 0; slot < 32; ++slot) {
            const uint8_t byte = blk[g * 16 + slot / 2];
            const int nib = (slot % 2 == 0) ? (byte & 0x0F) : ((byte >> 4) & 0x0F);
            acc[slot] += l[nib];
        }
    }
    for (int s = 0; s < 32; ++s) scores[s] = wrap16 ? (int32_t)(int16_t)acc[s] : acc[s];
}

// AVX-512BW version of the i16-wrapped scan; same result as block_scores_exact(wrap16).
__attribute__((target("avx512bw,avx512f,avx2"))) void block_scores_avx512(const uint8_t* blk,
                                                                           int G,
                                                                           const int8_t* lut,
                                                                           int32_t* scores) {
    __m512i acc = _mm512_setzero_si512();
    const __m128i low4 = _mm_set1_epi8(0x0F);
    for (int g = 0; g < G; ++g) {
        const __m128i bytes = _mm_loadu_si128((const __m128i*)(blk + g * 16));
        const __m128i tab = _mm_loadu_si128((const __m128i*)(lut + g * 16));
        const __m128i lo = _mm_and_si128(bytes, low4);
        const __m128i hi = _mm_and_si128(_mm_srli_epi16(bytes, 4), low4);
        // slot 2j <- low nibble of byte j, slot 2j+1 <- high nibble
        const __m128i idx0 = _mm_unpacklo_epi8(lo, hi);  // slots 0..15
        const __m128i idx1 = _mm_unpackhi_epi8(lo, hi);  // slots 16..31
        const __m128i v0 = _mm_shuffle_epi8(tab, idx0);
        const __m128i v1 = _mm_shuffle_epi8(tab, idx1);
        const __m256i v = _mm256_inserti128_si256(_mm256_castsi128_si256(v0), v1, 1);
        acc = _mm512_add_epi16(acc, _mm512_cvtepi8_epi16(v));
    }
    alignas(64) int16_t tmp[32];
    _mm512_store_si512((__m512i*)tmp, acc);
    for (int s = 0; s < 32; ++s) scores[s] = tmp[s];
}

void list_scores(const uint8_t* blocks, int64_t n, int D, const int8_t* lut, int mode,
                 int32_t* scores) {
    const int G = D / 4;
    const int64_t nb = (n + 31) / 32;
    int32_t tmp[32];
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* blk = blocks + b * G * 16;
        if (mode == OUSQ_MODE_AVX512 && cpu_has_avx512())
            block_scores_avx512(blk, G, lut, tmp);
        else
            block_scores_exact(blk, G, lut, mode == OUSQ_MODE_AVX512, tmp);
        for (int s = 0; s < 32; ++s) {
            const int64_t vid = b * 32 + s;
            if (vid < n) scores[vid] = tmp[s];
        }
    }
}

// fastscan_topk (fastscan.rs:86-146): min-heap of (score, vid); a newcomer replaces
// the heap minimum iff score > worst or (score == worst and vid < worst vid).
struct HeapItem {
    int32_t score;
    int64_t vid;
};
inline bool heap_less(const HeapItem& a, const HeapItem& b) {  // a < b lexicographically
    return a.score != b.score ? a.score < b.score : a.vid < b.vid;
}
// std::*_heap with comparator "greater" builds a min-heap.
inline bool heap_greater(const HeapItem& a, const HeapItem& b) { return heap_less(b, a); }

int64_t topk_from_scores(const int32_t* scores, const int64_t* vids, int64_t n, int64_t top_n,
                         int64_t* out_idx, int32_t* out_score) {
    if (top_n <= 0 || n == 0) return 0;
    std::vector<HeapItem> heap;
    heap.reserve((size_t)top_n + 1);
    for (int64_t i = 0; i < n; ++i) {
        HeapItem it{scores[i], vids ? vids[i] : i};
        if ((int64_t)heap.size() < top_n) {
            heap.push_back(it);
            std::push_heap(heap.begin(), heap.end(), heap_greater);
        } else {
            const HeapItem& worst = heap.front();
            if (it.score > worst.score || (it.score == worst.score && it.vid < worst.vid)) {
                std::pop_heap(heap.begin(), heap.end(), heap_greater);
                heap.back() = it;
                std::push_heap(heap.begin(), heap.end(), heap_greater);
            }
        }
    }
    std::sort(heap.begin(), heap.end(), [](const HeapItem& a, const HeapItem& b) {
        return a.score != b.score ? a.score > b.score : a.vid < b.vid;
    });
    for (size_t i = 0; i < heap.size(); ++i) {
        out_idx[i] = heap[i].vid;
        if (out_score) out_score[i] = heap[i].score;
    }
    return (int64_t)heap.size();
}

// ---------------------------------------------------------------------------
// Rerank  (quantizer.rs:274-400, 685-736)
// ---------------------------------------------------------------------------
__attribute__((target("avx512f,avx512vnni,avx512bw"))) int32_t dot_u8_i8_avx512(
    const uint8_t* a, const int8_t* b, int n) {
    __m512i acc = _mm512_setzero_si512();
    for (int i = 0; i < n; i += 64)
        acc = _mm512_dpbusd_epi32(acc, _mm512_loadu_si512(a + i), _mm512_loadu_si512(b + i));
    return _mm512_reduce_add_epi32(acc);
}

int32_t int_ip(const uint8_t* codes, int D, int nbits, const int8_t* q_i8) {
    alignas(64) uint8_t buf[8192];
    std::vector<uint8_t> big;
    const uint8_t* u8 = codes;
    if (nbits == 4) {
        uint8_t* dst = buf;
        if (D > (int)sizeof(buf)) {
            big.resize(D);
            dst = big.data();
        }
        for (int i = 0; i < D / 2; ++i) {
            dst[2 * i] = codes[i] & 0x0F;
            dst[2 * i + 1] = (codes[i] >> 4) & 0x0F;
        }
        u8 = dst;
    }
    if (cpu_has_avx512()) return dot_u8_i8_avx512(u8, q_i8, D);
    int32_t s = 0;
    for (int i = 0; i < D; ++i) s += (int32_t)u8[i] * (int32_t)q_i8[i];
    return s;
}

float compute_ip_scalar(const float* q_rot, int D, int nbits, float vmax, const uint8_t* packed,
                        int code_bytes) {
    const float levels = (float)(1u << nbits);
    const float scale = (2.0f * vmax) / std::fmax(levels, 1.0f);
    const float offset = -vmax;
    const uint32_t mask = (1u << nbits) - 1;
    uint32_t buf = 0;
    int bits = 0, byte_idx = 0;
    float ip = 0.0f;
    for (int i = 0; i < D; ++i) {
        while (bits < nbits) {
            uint32_t next = byte_idx < code_bytes ? packed[byte_idx] : 0;
            buf |= next << bits;
            bits += 8;
            ++byte_idx;
        }
        const uint32_t raw = buf & mask;
        buf >>= nbits;
        bits -= nbits;
        const float decoded = (float)raw * scale + offset;
        ip += q_rot[i] * decoded;
    }
    return ip;
}

float compute_ip_1bit(const QueryState& st, int D, float vmax, const uint8_t* packed) {
    float lanes[16];
    for (int j = 0; j < 16; ++j) lanes[j] = 0.0f;
    for (int c = 0; c < D / 16; ++c) {
        const uint32_t m = (uint32_t)packed[2 * c] | ((uint32_t)packed[2 * c + 1] << 8);
        for (int j = 0; j < 16; ++j) lanes[j] = lanes[j] + (((m >> j) & 1) ? st.q_rot[c * 16 + j] : 0.0f);
    }
    const float fs = tree16(lanes);
    return vmax * (fs - st.q_sum);
}

struct Rerank {
    float score;
    int32_t iip;  // integer dot (VNNI path) or INT32_MIN when not used
};

Rerank score_with_meta(const ousq_artifact_t* a, const QueryState& st, int64_t row, int mode) {
    const int D = a->padded_dim, nbits = a->nbits;
    const int cb = (D * nbits + 7) / 8;
    const float norm = a->norms[row], vmax = a->vmaxs[row], qq = a->quant_qualities[row];
    const uint8_t* codes = a->codes + row * cb;
    Rerank r{0.0f, std::numeric_limits<int32_t>::min()};
    if (qq <= 1e-12f) {
        r.score = st.centroid_score;
        return r;
    }
    float ip;
    if (mode == OUSQ_MODE_AVX512 && nbits == 1) {
        ip = compute_ip_1bit(st, D, vmax, codes);
    } else if (mode == OUSQ_MODE_AVX512 && (nbits == 4 || nbits == 8)) {
        const float levels = (float)(1u << nbits);
        const float code_scale = (2.0f * vmax) / std::fmax(levels, 1.0f);
        const float offset = -vmax;
        const int32_t iip = int_ip(codes, D, nbits, st.q_i8.data());
        r.iip = iip;
        ip = st.q_scale * (code_scale * (float)iip + offset * (float)st.q_i8_sum);
    } else {
        ip = compute_ip_scalar(st.q_rot.data(), D, nbits, vmax, codes, cb);
    }
    r.score = st.centroid_score + norm * ip / qq;
    return r;
}

inline bool bit_filtered(const uint64_t* words, int64_t len, int64_t id) {
    // Kept iff (id as usize) >= len || !bit  (ivf_usq.rs:708-710)
    const uint64_t u = (uint64_t)id;
    if (u >= (uint64_t)len) return false;
    return (words[u >> 6] >> (u & 63)) & 1ull;
}

int64_t n_candidates(int nbits, int64_t top_k) {
    if (nbits == 1) return std::max<int64_t>(top_k * 20, 200);
    if (nbits >= 2 && nbits <= 4) return std::max<int64_t>(top_k * 15, 150);
    return std::max<int64_t>(top_k * 30, 300);
}

}  // namespace

// ---------------------------------------------------------------------------
// Index object: reference FastScan blocks per list, built once.
// ---------------------------------------------------------------------------
struct ousq_index {
    ousq_artifact_t a;
    std::vector<std::vector<uint8_t>> blocks;  // per list
};

namespace {

struct Cand {
    int32_t list;
    int64_t local;
    int32_t fs;   // FastScan score or INT32_MIN
    int32_t iip;  // integer dot or INT32_MIN
    float dist;
    int64_t id;
};

// rank_centroids (ivf_usq.rs:596-609): sequential L2 on the raw query, stable sort.
void rank_centroids(const ousq_artifact_t* a, const float* q, int nprobe, std::vector<int>& out) {
    const int d = a->dim;
    std::vector<std::pair<uint32_t, int>> r(a->nlist);
    for (int c = 0; c < a->nlist; ++c) {
        const float* ce = a->centroids + (size_t)c * d;
        float s = kNegZero;
        for (int i = 0; i < d; ++i) {
            const float diff = q[i] - ce[i];
            s = s + diff * diff;
        }
        r[c] = {total_order_key(s), c};
    }
    std::stable_sort(r.begin(), r.end(),
                     [](const std::pair<uint32_t, int>& x, const std::pair<uint32_t, int>& y) {
                         return x.first < y.first;
                     });
    out.resize(nprobe);
    for (int i = 0; i < nprobe; ++i) out[i] = r[i].second;
}

// search_single (ivf_usq.rs:527-594); fused filtering removes filtered rows first.
void search_single(const ousq_index* idx, const float* q, int top_k, int nprobe, int mode,
                   const uint64_t* fused_words, int64_t fused_len, std::vector<Cand>& cands,
                   std::vector<int>& probes) {
    const ousq_artifact_t* a = &idx->a;
    rank_centroids(a, q, nprobe, probes);
    QueryState st;
    query_state(a, q, mode, st);
    const int64_t ncand = n_candidates(a->nbits, top_k);
    const int D = a->padded_dim;
    cands.clear();
    std::vector<int32_t> scores;
    std::vector<int64_t> vids, sel_idx;
    std::vector<int32_t> sel_score;
    for (int cl : probes) {
        const int64_t beg = a->list_offsets[cl], end = a->list_offsets[cl + 1];
        const int64_t len = end - beg;
        if (len == 0) continue;
        // live rows (all rows unless fused filtering is on)
        vids.clear();
        for (int64_t v = 0; v < len; ++v)
            if (!fused_words || !bit_filtered(fused_words, fused_len, a->ids[beg + v]))
                vids.push_back(v);
        const int64_t live = (int64_t)vids.size();
        if (live <= ncand) {
            for (int64_t v : vids)
                cands.push_back({cl, v, std::numeric_limits<int32_t>::min(), 0, 0.0f, 0});
        } else {
            scores.resize(len);
            list_scores(idx->blocks[cl].data(), len, D, st.lut.data(), mode, scores.data());
            std::vector<int32_t> live_scores(live);
            for (int64_t i = 0; i < live; ++i) live_scores[i] = scores[vids[i]];
            sel_idx.resize(ncand);
            sel_score.resize(ncand);
            const int64_t m = topk_from_scores(live_scores.data(), vids.data(), live, ncand,
                                               sel_idx.data(), sel_score.data());
            for (int64_t i = 0; i < m; ++i)
                cands.push_back({cl, sel_idx[i], sel_score[i], 0, 0.0f, 0});
        }
    }
    const bool use_l2 = a->metric == OUSQ_METRIC_L2;
    for (Cand& c : cands) {
        const int64_t row = a->list_offsets[c.list] + c.local;
        Rerank r = score_with_meta(a, st, row, mode);
        c.iip = r.iip;
        c.dist = use_l2 ? st.q_norm_sq + a->norms_sq[row] - 2.0f * r.score : -r.score;
        c.id = a->ids[row];
    }
}

}  // namespace

extern "C" {

int32_t ousq_padded_dim(int32_t dim) { return padded_dim_of(dim); }
int32_t ousq_code_bytes(int32_t dim, int32_t nbits) {
    return (padded_dim_of(dim) * nbits + 7) / 8;
}
int32_t ousq_sign_bytes(int32_t dim) { return padded_dim_of(dim) / 8; }
int32_t ousq_n_candidates(int32_t nbits, int32_t top_k) {
    return (int32_t)n_candidates(nbits, std::max(top_k, 1));
}

// Seeded uniform [-1,1) matrix -> Householder QR (double) -> Q as f32.  Same method
// as rotator.rs:15-39 (random matrix, QR, keep Q); not the same random stream.
void ousq_rotation_matrix(uint64_t seed, int32_t D, float* out) {
    std::vector<double> A((size_t)D * D);
    uint64_t s = seed;
    auto next = [&]() {
        s += 0x9E3779B97F4A7C15ull;
        uint64_t z = s;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    for (size_t i = 0; i < A.size(); ++i)
        A[i] = (double)(next() >> 40) * (1.0 / 16777216.0) * 2.0 - 1.0;  // row-major
    // Householder: A = Q R; accumulate Q explicitly.
    std::vector<double> Q((size_t)D * D, 0.0), v(D);
    for (int i = 0; i < D; ++i) Q[(size_t)i * D + i] = 1.0;
    for (int k = 0; k < D - 1; ++k) {
        double nrm = 0;
        for (int i = k; i < D; ++i) nrm += A[(size_t)i * D + k] * A[(size_t)i * D + k];
        nrm = std::sqrt(nrm);
        if (nrm == 0) continue;
        const double alpha = A[(size_t)k * D + k] > 0 ? -nrm : nrm;
        double vn = 0;
        for (int i = 0; i < D; ++i) v[i] = i < k ? 0.0 : A[(size_t)i * D + k];
        v[k] -= alpha;
        for (int i = k; i < D; ++i) vn += v[i] * v[i];
        if (vn == 0) continue;
        // A <- (I - 2vv^T/vn) A  (columns k..)
        for (int j = k; j < D; ++j) {
            double dot = 0;
            for (int i = k; i < D; ++i) dot += v[i] * A[(size_t)i * D + j];
            const double f = 2.0 * dot / vn;
            for (int i = k; i < D; ++i) A[(size_t)i * D + j] -= f * v[i];
        }
        // Q <- Q (I - 2vv^T/vn)
        for (int r = 0; r < D; ++r) {
            double dot = 0;
            for (int i = k; i < D; ++i) dot += Q[(size_t)r * D + i] * v[i];
            const double f = 2.0 * dot / vn;
            for (int i = k; i < D; ++i) Q[(size_t)r * D + i] -= f * v[i];
        }
    }
    for (size_t i = 0; i < Q.size(); ++i) out[i] = (float)Q[i];
}

void ousq_rotate(const float* P, int32_t D, const float* x, float* out, int32_t mode) {
    rotate(P, D, x, out, mode);
}

void ousq_encode(const float* P, int32_t dim, int32_t nbits, const float* centroid,
                 const float* x, int32_t mode, uint8_t* codes, uint8_t* sign_bits,
                 float* meta4) {
    encode_one(P, dim, nbits, centroid, x, mode, codes, sign_bits, meta4);
}

void ousq_encode_batch(const float* P, int32_t dim, int32_t nbits, const float* centroid,
                       const float* x, int64_t n, int32_t mode, uint8_t* codes,
                       uint8_t* sign_bits, float* meta4, int32_t nthreads) {
    const int cb = ousq_code_bytes(dim, nbits), sb = ousq_sign_bytes(dim);
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t i = 0; i < n; ++i)
        encode_one(P, dim, nbits, centroid, x + i * dim, mode, codes + i * cb, sign_bits + i * sb,
                   meta4 + i * 4);
}

void ousq_assign(const float* data, int64_t n, int32_t dim, const float* centroids,
                 int32_t nlist, int32_t* out_list, int32_t nthreads) {
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
    for (int64_t i = 0; i < n; ++i) {
        // find_best_centroid (ivf_usq.rs:611-624): first strict minimum.
        const float* x = data + i * dim;
        int best = 0;
        float bd = std::numeric_limits<float>::infinity();
        for (int c = 0; c < nlist; ++c) {
            const float* ce = centroids + (size_t)c * dim;
            float s = kNegZero;
            for (int j = 0; j < dim; ++j) {
                const float df = x[j] - ce[j];
                s = s + df * df;
            }
            if (s < bd) {
                bd = s;
                best = c;
            }
        }
        out_list[i] = best;
    }
}

// Seeded Lloyd k-means for fixtures (distinct random init, double sums).
void ousq_kmeans(const float* data, int64_t n, int32_t dim, int32_t k, int32_t iters,
                 uint64_t seed, float* centroids, int32_t nthreads) {
    std::vector<int64_t> perm(n);
    for (int64_t i = 0; i < n; ++i) perm[i] = i;
    uint64_t s = seed ^ 0xD1B54A32D192ED03ull;
    for (int64_t i = 0; i < k && i < n; ++i) {
        s = s * 6364136223846793005ull + 1442695040888963407ull;
        const int64_t j = i + (int64_t)((s >> 33) % (uint64_t)(n - i));
        std::swap(perm[i], perm[j]);
    }
    for (int c = 0; c < k; ++c)
        std::memcpy(centroids + (size_t)c * dim, data + perm[c % n] * dim, sizeof(float) * dim);
    std::vector<int32_t> asg(n);
    std::vector<double> sums((size_t)k * dim);
    std::vector<int64_t> cnt(k);
    for (int it = 0; it < iters; ++it) {
        ousq_assign(data, n, dim, centroids, k, asg.data(), nthreads);
        std::fill(sums.begin(), sums.end(), 0.0);
        std::fill(cnt.begin(), cnt.end(), 0);
        for (int64_t i = 0; i < n; ++i) {
            const int c = asg[i];
            cnt[c]++;
            for (int j = 0; j < dim; ++j) sums[(size_t)c * dim + j] += data[i * dim + j];
        }
        for (int c = 0; c < k; ++c)
            if (cnt[c] > 0)
                for (int j = 0; j < dim; ++j)
                    centroids[(size_t)c * dim + j] = (float)(sums[(size_t)c * dim + j] / cnt[c]);
    }
}

void ousq_global_mean(const float* data, int64_t n, int32_t dim, float* out) {
    for (int j = 0; j < dim; ++j) out[j] = 0.0f;
    for (int64_t i = 0; i < n; ++i)
        for (int j = 0; j < dim; ++j) out[j] += data[i * dim + j];
    const float inv_n = 1.0f / (float)n;
    for (int j = 0; j < dim; ++j) out[j] *= inv_n;
}

void ousq_pack_codes(const uint16_t* codes, int64_t n, int32_t nbits, uint8_t* out) {
    pack_codes(codes, n, nbits, out);
}
void ousq_unpack_codes(const uint8_t* bytes, int64_t n, int32_t nbits, uint16_t* out) {
    unpack_codes(bytes, n, nbits, out);
}

void ousq_query_state(const ousq_artifact_t* a, const float* q, int32_t mode, float* q_rot,
                      int8_t* q_i8, float* scalars4, int32_t* q_i8_sum) {
    QueryState st;
    query_state(a, q, mode, st);
    std::memcpy(q_rot, st.q_rot.data(), sizeof(float) * a->padded_dim);
    std::memcpy(q_i8, st.q_i8.data(), (size_t)a->padded_dim);
    scalars4[0] = st.q_sum;
    scalars4[1] = st.q_scale;
    scalars4[2] = st.centroid_score;
    scalars4[3] = st.q_norm_sq;
    *q_i8_sum = st.q_i8_sum;
}

void ousq_fastscan_lut(const float* q_rot, int32_t D, int8_t* lut, float* lut_scale) {
    fastscan_lut(q_rot, D, lut, lut_scale);
}

void ousq_fastscan_blocks(const uint8_t* sign_bits, int64_t n, int32_t D, uint8_t* blocks) {
    build_blocks(sign_bits, n, D, blocks);
}

void ousq_fastscan_scores(const uint8_t* blocks, int64_t n, int32_t D, const int8_t* lut,
                          int32_t mode, int32_t* scores) {
    list_scores(blocks, n, D, lut, mode, scores);
}

int64_t ousq_fastscan_topk(const uint8_t* blocks, int64_t n, int32_t D, const int8_t* lut,
                           int64_t top_n, int32_t mode, int64_t* out_idx, int32_t* out_score) {
    if (top_n <= 0 || n <= 0) return 0;
    std::vector<int32_t> sc(n);
    list_scores(blocks, n, D, lut, mode, sc.data());
    return topk_from_scores(sc.data(), nullptr, n, top_n, out_idx, out_score);
}

int64_t ousq_topk_from_scores(const int32_t* scores, int64_t n, int64_t top_n, int64_t* out_idx,
                              int32_t* out_score) {
    return topk_from_scores(scores, nullptr, n, top_n, out_idx, out_score);
}

int32_t ousq_int_ip(const uint8_t* codes, int32_t D, int32_t nbits, const int8_t* q_i8) {
    return int_ip(codes, D, nbits, q_i8);
}

float ousq_score(const ousq_artifact_t* a, const float* q, int64_t row, int32_t mode) {
    QueryState st;
    query_state(a, q, mode, st);
    return score_with_meta(a, st, row, mode).score;
}

ousq_index_t* ousq_index_create(const ousq_artifact_t* a) {
    ousq_index* idx = new ousq_index();
    idx->a = *a;
    idx->blocks.resize(a->nlist);
    const int D = a->padded_dim, sb = D / 8;
    for (int l = 0; l < a->nlist; ++l) {
        const int64_t beg = a->list_offsets[l], len = a->list_offsets[l + 1] - beg;
        idx->blocks[l].resize((size_t)((len + 31) / 32) * (D / 4) * 16);
        if (len > 0) build_blocks(a->sign_bits + beg * sb, len, D, idx->blocks[l].data());
    }
    return idx;
}

void ousq_index_free(ousq_index_t* idx) { delete idx; }

int32_t ousq_search(const ousq_index_t* idx, const float* queries, int64_t nq, int32_t k,
                    int32_t nprobe_req, int32_t mode, int32_t filter_mode,
                    const uint64_t* bitsets, int64_t bitset_len, int64_t n_bitsets,
                    const int32_t* query_bitset, int32_t nthreads, int64_t* out_ids,
                    float* out_dists, int64_t* out_counts, int32_t* out_probes) {
    const ousq_artifact_t* a = &idx->a;
    if (nq <= 0) return -1;
    const int top_k = std::max(k, 1);
    const int nprobe = std::min(std::max(nprobe_req, 1), a->nlist);
    const int64_t words = (bitset_len + 63) / 64;
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
    {
        std::vector<Cand> cands;
        std::vector<int> probes;
        std::vector<std::pair<uint32_t, int64_t>> order;
#pragma omp for schedule(dynamic, 2)
        for (int64_t qi = 0; qi < nq; ++qi) {
            const uint64_t* bw = nullptr;
            if (filter_mode != OUSQ_FILTER_NONE && bitsets && n_bitsets > 0) {
                const int32_t b = query_bitset ? query_bitset[qi] : 0;
                if (b >= 0 && b < n_bitsets) bw = bitsets + (int64_t)b * words;
            }
            const float* q = queries + qi * a->dim;
            search_single(idx, q, top_k, nprobe, mode, filter_mode == OUSQ_FILTER_FUSED ? bw : nullptr,
                          bitset_len, cands, probes);
            if (out_probes)
                for (int r = 0; r < nprobe; ++r) out_probes[qi * nprobe + r] = probes[r];
            order.resize(cands.size());
            for (size_t i = 0; i < cands.size(); ++i)
                order[i] = {total_order_key(cands[i].dist), (int64_t)i};
            std::stable_sort(order.begin(), order.end(),
                             [](const std::pair<uint32_t, int64_t>& x,
                                const std::pair<uint32_t, int64_t>& y) { return x.first < y.first; });
            int64_t* ids = out_ids + qi * top_k;
            float* ds = out_dists + qi * top_k;
            int64_t n_out = 0;
            const int64_t take = std::min<int64_t>(top_k, (int64_t)order.size());
            for (int64_t j = 0; j < top_k; ++j) {
                int64_t id = -1;
                float dist = std::numeric_limits<float>::infinity();
                if (j < take) {
                    id = cands[order[j].second].id;
                    dist = cands[order[j].second].dist;
                }
                if (filter_mode == OUSQ_FILTER_POST && bw) {
                    if (bit_filtered(bw, bitset_len, id)) continue;
                }
                ids[n_out] = id;
                ds[n_out] = dist;
                ++n_out;
            }
            for (int64_t j = n_out; j < top_k; ++j) {
                ids[j] = -1;
                ds[j] = std::numeric_limits<float>::infinity();
            }
            if (out_counts) out_counts[qi] = n_out;
        }
    }
    return 0;
}

int64_t ousq_candidates(const ousq_index_t* idx, const float* query, int32_t k, int32_t nprobe_req,
                        int32_t mode, int32_t filter_mode, const uint64_t* bitset,
                        int64_t bitset_len, int64_t cap, int32_t* out_list, int64_t* out_local,
                        int32_t* out_fs, int32_t* out_int_ip, float* out_dist) {
    const ousq_artifact_t* a = &idx->a;
    const int top_k = std::max(k, 1);
    const int nprobe = std::min(std::max(nprobe_req, 1), a->nlist);
    std::vector<Cand> cands;
    std::vector<int> probes;
    search_single(idx, query, top_k, nprobe, mode,
                  filter_mode == OUSQ_FILTER_FUSED ? bitset : nullptr, bitset_len, cands, probes);
    const int64_t n = std::min<int64_t>(cap, (int64_t)cands.size());
    for (int64_t i = 0; i < n; ++i) {
        out_list[i] = cands[i].list;
        out_local[i] = cands[i].local;
        out_fs[i] = cands[i].fs;
        out_int_ip[i] = cands[i].iip;
        out_dist[i] = cands[i].dist;
    }
    return (int64_t)cands.size();
}

}  // extern "C"
