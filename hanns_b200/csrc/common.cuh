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

}  // namespace hanns

#define HANNS_CUDA_OK(expr)                                                             \
    do {                                                                                \
        cudaError_t _e = (expr);                                                        \
        if (_e != cudaSuccess) throw ::hanns::CudaError(_e, #expr, __FILE__, __LINE__); \
    } while (0)
