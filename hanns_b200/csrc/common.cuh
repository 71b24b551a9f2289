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
    int32_t pad[3];
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
