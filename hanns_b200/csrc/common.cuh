// common.cuh -- shared device helpers for the IVF-USQ kernels.
//
// All translation units are compiled with --fmad=false: every float operation is
// rounded on its own, as Rust does (no contraction).  Where the reference fuses
// (the AVX-512 rotation's _mm512_fmadd_ps) the kernels call __fmaf_rn explicitly.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hanns {

constexpr int kWarp = 32;

// Rust f32::total_cmp as an unsigned key (negatives reversed, -0.0 < +0.0).
__device__ __forceinline__ uint32_t total_order_key(float f) {
    uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_to_float(uint32_t k) {
    uint32_t b = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
    return __uint_as_float(b);
}

// (v).round().clamp(lo, hi) as iN  -- round half away from zero; NaN -> 0.
__device__ __forceinline__ int round_clamp(float v, float lo, float hi) {
    float r = roundf(v);
    if (r != r) return 0;
    r = fminf(fmaxf(r, lo), hi);
    return (int)r;
}

// dp4a with unsigned a (codes) and signed b (quantised query).
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

__device__ __forceinline__ unsigned lane_id() { return threadIdx.x & 31u; }

// Per-query constants produced by the query-prep kernel.
struct QueryParams {
    float q_scale;         // max(|q_rot|)/127
    float centroid_score;  // <q_rot, rotated global centroid>
    float q_norm_sq;       // ||q||^2 of the raw query
    float lut_scale;
    int32_t q_i8_sum;
    float q_sum;           // sum of q_rot in dimension order from -0.0 (1-bit rerank)
    int32_t pad[2];
};

// score_with_meta + distance, in the reference's operation order
// (src/quantization/usq/quantizer.rs:274-288, src/faiss/ivf_usq.rs:581-593).
__device__ __forceinline__ float rerank_distance(int iip, float4 m, const QueryParams& p, int nbits,
                                                 bool l2) {
    // m = {norm, norm_sq, vmax, quant_quality}
    float score;
    if (m.w <= 1e-12f) {
        score = p.centroid_score;
    } else {
        // (2 vmax) / 2^nbits: dividing by a power of two and multiplying by its exact
        // reciprocal round the same real number, so the product equals the reference's
        // quotient bit for bit
        const float inv_levels = __uint_as_float((uint32_t)(127 - nbits) << 23);
        const float code_scale = __fmul_rn(__fmul_rn(2.0f, m.z), inv_levels);
        const float offset = -m.z;
        const float ip = __fmul_rn(
            p.q_scale, __fadd_rn(__fmul_rn(code_scale, __int2float_rn(iip)),
                                 __fmul_rn(offset, __int2float_rn(p.q_i8_sum))));
        score = __fadd_rn(p.centroid_score, __fdiv_rn(__fmul_rn(m.x, ip), m.w));
    }
    return l2 ? __fsub_rn(__fadd_rn(p.q_norm_sq, m.y), __fmul_rn(2.0f, score)) : -score;
}

// The same distance from an f32 inner product (the reference's non-VNNI paths).
__device__ __forceinline__ float rerank_distance_ip(float ip, float4 m, const QueryParams& p, bool l2) {
    const float score = m.w <= 1e-12f ? p.centroid_score : __fadd_rn(p.centroid_score, __fdiv_rn(__fmul_rn(m.x, ip), m.w));
    return l2 ? __fsub_rn(__fadd_rn(p.q_norm_sq, m.y), __fmul_rn(2.0f, score)) : -score;
}

// compute_ip_scalar (quantizer.rs, nbits other than 1, 4, 8): codes from the LSB-first bit
// stream (packed.rs), each decoded as raw * scale + offset, summed in dimension order from
// +0.0, unfused.
__device__ inline float ip_scalar(const uint8_t* packed, const float* q_rot, int D, int nbits, float vmax,
                                  int code_bytes) {
    const float scale = __fdiv_rn(__fmul_rn(2.0f, vmax), fmaxf((float)(1u << nbits), 1.0f));
    const float offset = -vmax;
    const uint32_t mask = (1u << nbits) - 1u;
    uint32_t buf = 0;
    int bits = 0, byte_idx = 0;
    float ip = 0.0f;
    for (int i = 0; i < D; ++i) {
        while (bits < nbits) {
            const uint32_t next = byte_idx < code_bytes ? (uint32_t)packed[byte_idx] : 0u;
            buf |= next << bits;
            bits += 8;
            ++byte_idx;
        }
        const uint32_t raw = buf & mask;
        buf >>= nbits;
        bits -= nbits;
        const float decoded = __fadd_rn(__fmul_rn((float)raw, scale), offset);
        ip = __fadd_rn(ip, __fmul_rn(q_rot[i], decoded));
    }
    return ip;
}

// compute_ip_1bit (quantizer.rs, AVX-512 path): 16 lanes of the selected q_rot values over
// 16-dimension chunks, the halving tree of _mm512_reduce_add_ps, then vmax * (sum - q_sum).
__device__ inline float ip_1bit(const uint8_t* packed, const float* q_rot, int D, float vmax, float q_sum) {
    float lanes[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) lanes[j] = 0.0f;
    for (int c = 0; c < D / 16; ++c) {
        const uint32_t m = (uint32_t)packed[2 * c] | ((uint32_t)packed[2 * c + 1] << 8);
#pragma unroll
        for (int j = 0; j < 16; ++j) lanes[j] = __fadd_rn(lanes[j], ((m >> j) & 1u) ? q_rot[c * 16 + j] : 0.0f);
    }
    float s8[8], s4[4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s8[i] = __fadd_rn(lanes[i], lanes[i + 8]);
#pragma unroll
    for (int i = 0; i < 4; ++i) s4[i] = __fadd_rn(s8[i], s8[i + 4]);
    const float fs = __fadd_rn(__fadd_rn(s4[0], s4[2]), __fadd_rn(s4[1], s4[3]));
    return __fmul_rn(vmax, __fsub_rn(fs, q_sum));
}

// Packed two-lane fp32 arithmetic of sm_100 (add/sub/mul/fma .rn.f32x2): each lane is
// rounded exactly like the scalar instruction, one instruction serves two lanes.
__device__ __forceinline__ float2 sub2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "sub.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "mul.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
        "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
    return d;
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
    float2 d;
    asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
        "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
        "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
        : "=f"(d.x), "=f"(d.y)
        : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
    return d;
}

}  // namespace hanns

#define HANNS_CUDA_OK(expr)                                                             \
    do {                                                                                \
        cudaError_t _e = (expr);                                                        \
        if (_e != cudaSuccess) throw ::hanns::CudaError(_e, #expr, __FILE__, __LINE__); \
    } while (0)
