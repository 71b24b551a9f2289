// build_kernels.cu -- index construction on the GPU (train / add).
//
// Float arithmetic follows the reference (Rust, no contraction): this file is
// compiled with --fmad=false and IEEE division / square root, so plain C++
// operators round every operation on its own.
//   global mean          src/faiss/ivf_usq.rs:253-263
//   nearest centroid     src/faiss/ivf_usq.rs:611-624 (first strict minimum)
//   encode               src/quantization/usq/quantizer.rs:124-230, 442-541, 652-672
//   FastScan transpose   src/quantization/usq/layout.rs:139-197 (GPU block layout, see below)
//
// GPU FastScan layout: per list, ceil(n/32) blocks of 32 vectors; a block stores,
// for each 64-dim chunk c, the 32 vectors' 8 sign bytes contiguously
// ([block][D/64][32 slots][8 bytes]).  Nibble j of a chunk's 64-bit word is the
// reference's FastScan nibble of group 16c+j (dims 4j..4j+3, LSB = lowest dim).
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace hanns {

__global__ void global_mean_kernel(const float* __restrict__ x, int64_t n, int d,
                                   float* __restrict__ out) {
    const int j = blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= d) return;
    float s = 0.0f;  // vec![0.0f32; dim], then += row by row
#pragma unroll 8
    for (int64_t i = 0; i < n; ++i) s = s + x[i * d + j];
    const float inv_n = 1.0f / (float)n;
    out[j] = s * inv_n;
}

__global__ void row_norm_sq_kernel(const float* __restrict__ x, int64_t n, int d,
                                   float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float* r = x + i * d;
    float s = -0.0f;
    for (int j = 0; j < d; ++j) s = s + r[j] * r[j];
    out[i] = s;
}

__global__ void residual_pad_kernel(const float* __restrict__ x, int64_t n, int d, int D,
                                    const float* __restrict__ c, float* __restrict__ out) {
    const int64_t total = n * D;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / D;
        const int j = (int)(e % D);
        out[e] = j < d ? x[i * d + j] - c[j] : 0.0f;
    }
}

__device__ __forceinline__ int clamp_round(float v, float lo, float hi) {
    float r = roundf(v);
    if (r != r) return 0;
    r = fminf(fmaxf(r, lo), hi);
    return (int)r;
}

__device__ __forceinline__ float objective(float ip, float qed) {
    return qed > 1e-12f ? ip * ip / qed : 0.0f;
}

// One thread per vector.  rotated[i] (D floats) is overwritten with o_hat and
// scratch[i] (D bytes) holds the codes while the greedy refinement runs.
__global__ void encode_rotated_kernel(float* __restrict__ rotated, int64_t n, int D, int nbits,
                                      const float* __restrict__ norm_sq_raw,
                                      uint8_t* __restrict__ scratch, uint8_t* __restrict__ codes,
                                      uint8_t* __restrict__ signs, float4* __restrict__ meta) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    float* o = rotated + i * D;
    uint8_t* cd = scratch + i * D;
    float nsq = -0.0f;
    for (int j = 0; j < D; ++j) nsq = nsq + o[j] * o[j];
    const float norm = sqrtf(nsq);
    if (norm > 1e-12f) {
        const float inv = 1.0f / norm;
        for (int j = 0; j < D; ++j) o[j] = o[j] * inv;
    }
    // greedy_quantize_into (nbits >= 4)
    float max_v = 0.0f;
    for (int j = 0; j < D; ++j) max_v = fmaxf(max_v, fabsf(o[j]));
    max_v = fmaxf(max_v, 1e-6f);
    const float levels = (float)(1u << nbits);
    float scale = (2.0f * max_v) / fmaxf(levels, 1.0f);
    if (fabsf(scale) < 1e-6f) scale = 1e-6f;
    const float offset = -max_v;
    const int max_code = (1 << nbits) - 1;
    for (int j = 0; j < D; ++j)
        cd[j] = (uint8_t)clamp_round((o[j] - offset) / scale, 0.0f, (float)max_code);
    float ip = -0.0f, qed = -0.0f;
    for (int j = 0; j < D; ++j) ip = ip + ((float)cd[j] * scale + offset) * o[j];
    for (int j = 0; j < D; ++j) {
        const float v = (float)cd[j] * scale + offset;
        qed = qed + v * v;
    }
    float obj = objective(ip, qed);
    for (int round = 0; round < 6; ++round) {
        bool improved = false;
        for (int j = 0; j < D; ++j) {
            const float oj = o[j];
            const int current = cd[j];
            const float old_val = (float)current * scale + offset;
            const float target_val = fabsf(ip) > 1e-12f ? oj * qed / ip : oj;
            const int target = clamp_round((target_val - offset) / scale, 0.0f, (float)max_code);
            int cands[5];
            int nc = 0;
            const int tries[5] = {target - 1, target, target + 1, current - 1, current + 1};
#pragma unroll
            for (int t = 0; t < 5; ++t) {
                const int c = tries[t];
                bool ok = c >= 0 && c <= max_code && c != current;
                for (int u = 0; u < nc; ++u) ok = ok && cands[u] != c;
                if (ok) cands[nc++] = c;
            }
            int best_code = current;
            float best_ip = ip, best_qed = qed, best_obj = obj;
            for (int t = 0; t < nc; ++t) {
                const float new_val = (float)cands[t] * scale + offset;
                const float new_ip = ip - oj * old_val + oj * new_val;
                const float new_qed = qed - old_val * old_val + new_val * new_val;
                if (new_qed <= 1e-12f) continue;
                const float new_obj = objective(new_ip, new_qed);
                if (new_obj > best_obj + 1e-10f) {
                    best_code = cands[t];
                    best_ip = new_ip;
                    best_qed = new_qed;
                    best_obj = new_obj;
                }
            }
            if (best_code != current) {
                cd[j] = (uint8_t)best_code;
                ip = best_ip;
                qed = best_qed;
                obj = best_obj;
                improved = true;
            }
        }
        if (!improved) break;
    }
    float vmax = 0.0f;
    for (int j = 0; j < D; ++j) vmax = fmaxf(vmax, fabsf(o[j]));
    vmax = fmaxf(vmax, 1e-6f);
    const float qq = fmaxf(sqrtf(qed), 1e-12f);
    // pack_codes LSB-first (nbits 4 or 8 here) and 1-bit signs (o >= 0)
    const int cb = D * nbits / 8;
    uint8_t* out = codes + i * (int64_t)cb;
    if (nbits == 8) {
        for (int j = 0; j < D; ++j) out[j] = cd[j];
    } else {
        for (int j = 0; j < D / 2; ++j) out[j] = (uint8_t)(cd[2 * j] | (cd[2 * j + 1] << 4));
    }
    uint8_t* sg = signs + i * (int64_t)(D / 8);
    for (int b = 0; b < D / 8; ++b) {
        uint8_t byte = 0;
        for (int t = 0; t < 8; ++t) byte |= (uint8_t)((o[b * 8 + t] >= 0.0f ? 1 : 0) << t);
        sg[b] = byte;
    }
    meta[i] = make_float4(norm, norm_sq_raw[i], vmax, qq);
}

// First strict minimum per row (find_best_centroid).  One warp per row.
__global__ void argmin_rows_kernel(const float* __restrict__ dist, int64_t n, int nlist,
                                   int32_t* __restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (row >= n) return;
    const float* r = dist + row * nlist;
    float best = __int_as_float(0x7f800000);
    int bi = 0x7fffffff;
    for (int c = lane; c < nlist; c += 32) {
        const float v = r[c];
        if (v < best) {
            best = v;
            bi = c;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob < best || (ob == best && oi < bi)) {
            best = ob;
            bi = oi;
        }
    }
    if (lane == 0) out[row] = bi == 0x7fffffff ? 0 : bi;
}

// Deterministic k-means sums: 32.32 fixed point in int64 (order independent).
__global__ void kmeans_accumulate_kernel(const float* __restrict__ x, int64_t n, int d,
                                         const int32_t* __restrict__ assign,
                                         unsigned long long* __restrict__ sums,
                                         int* __restrict__ counts) {
    const int64_t total = n * d;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / d;
        const int j = (int)(e % d);
        const int c = assign[i];
        const long long v = __float2ll_rn(x[e] * 4294967296.0f);
        atomicAdd(&sums[(int64_t)c * d + j], (unsigned long long)v);
        if (j == 0) atomicAdd(&counts[c], 1);
    }
}

// One warp per centroid: new mean of its rows (kept in place when it has none) and the
// L2 shift from the old position (kmeans.rs:246-271), 0 for empty centroids.
__global__ void kmeans_update_kernel(const long long* __restrict__ sums,
                                     const int* __restrict__ counts, int nlist, int d,
                                     float* __restrict__ cent, float* __restrict__ shift) {
    const int c = (int)(((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5);
    const int lane = threadIdx.x & 31;
    if (c >= nlist) return;
    const int cnt = counts[c];
    float ss = 0.0f;
    if (cnt > 0) {
        for (int j = lane; j < d; j += 32) {
            const int64_t e = (int64_t)c * d + j;
            const float nv = (float)((double)sums[e] / 4294967296.0 / (double)cnt);
            const float df = nv - cent[e];
            ss = fmaf(df, df, ss);
            cent[e] = nv;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) shift[c] = sqrtf(ss);
}

// k-means++ seeding (kmeans.rs:138-183), with this library's seeded random stream.
// kpp_dist: min_d[i] = min(min_d[i], ||x_i - c||^2) for the newest centroid c, one warp
// per row; block b covers rows [b*per, (b+1)*per) and writes sum(max(min_d, 0)) of them.
__global__ void kpp_dist_kernel(const float* __restrict__ x, int64_t n, int d,
                                const float* __restrict__ c, int64_t per,
                                float* __restrict__ min_d, double* __restrict__ block_sum) {
    __shared__ double part[8];
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t r0 = (int64_t)blockIdx.x * per;
    const int64_t r1 = min(n, r0 + per);
    double acc = 0.0;
    for (int64_t i = r0 + w; i < r1; i += 8) {
        const float* xi = x + i * d;
        float s = 0.0f;
        for (int j = lane; j < d; j += 32) {
            const float df = xi[j] - c[j];
            s = fmaf(df, df, s);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        float m = min_d[i];
        if (s < m) m = s;
        if (lane == 0) min_d[i] = m;
        acc += (double)fmaxf(m, 0.0f);
    }
    if (lane == 0) part[w] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        double t = 0.0;
        for (int k = 0; k < 8; ++k) t += part[k];
        block_sum[blockIdx.x] = t;
    }
}

// kpp_pick: draw row i with probability max(min_d[i], 0) / total (a uniform row when the
// total is 0) and copy it into centroid slot `slot`.  One thread walks the block sums,
// then the rows of the chosen block, in order.
__global__ void kpp_pick_kernel(const float* __restrict__ x, int64_t n, int d,
                                const float* __restrict__ min_d, const double* __restrict__ block_sum,
                                int nblocks, int64_t per, double u_target, double u_uniform,
                                float* __restrict__ cent, int slot) {
    __shared__ int64_t chosen;
    if (threadIdx.x == 0) {
        double total = 0.0;
        for (int b = 0; b < nblocks; ++b) total += block_sum[b];
        int64_t idx = n - 1;
        if (!(total > 0.0)) {
            idx = min(n - 1, (int64_t)(u_uniform * (double)n));
        } else {
            const double target = u_target * total;
            double cum = 0.0;
            int b = 0;
            for (; b < nblocks - 1; ++b) {
                if (cum + block_sum[b] >= target) break;
                cum += block_sum[b];
            }
            const int64_t r1 = min(n, (int64_t)(b + 1) * per);
            for (int64_t i = (int64_t)b * per; i < r1; ++i) {
                cum += (double)fmaxf(min_d[i], 0.0f);
                if (cum >= target) {
                    idx = i;
                    break;
                }
            }
        }
        chosen = idx;
    }
    __syncthreads();
    const int64_t idx = chosen;
    for (int j = threadIdx.x; j < d; j += blockDim.x) cent[(int64_t)slot * d + j] = x[idx * d + j];
}

__global__ void fill_f32_kernel(float* __restrict__ p, int64_t n, float v) {
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n;
         e += (int64_t)gridDim.x * blockDim.x)
        p[e] = v;
}

// One CTA per list: copy every row's sign bytes into the GPU FastScan blocks.
__global__ void build_fastscan_kernel(const uint8_t* __restrict__ signs,
                                      const int64_t* __restrict__ list_off,
                                      const int64_t* __restrict__ blk_off, int D,
                                      uint2* __restrict__ fs) {
    const int l = blockIdx.x;
    const int64_t beg = list_off[l];
    const int n = (int)(list_off[l + 1] - beg);
    const int nch = D / 64;
    uint2* dst = fs + blk_off[l] * (int64_t)nch * 32;
    for (int e = threadIdx.x; e < n * nch; e += blockDim.x) {
        const int v = e / nch, c = e % nch;
        const uint2 w = *reinterpret_cast<const uint2*>(signs + (beg + v) * (D / 8) + c * 8);
        dst[((int64_t)(v >> 5) * nch + c) * 32 + (v & 31)] = w;
    }
}

__global__ void gather_rows_kernel(const uint8_t* __restrict__ src, const int64_t* __restrict__ perm,
                                   int64_t n, int64_t row_bytes, uint8_t* __restrict__ dst) {
    const int64_t total = n * row_bytes;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t i = e / row_bytes, b = e % row_bytes;
        dst[e] = src[perm[i] * row_bytes + b];
    }
}

static int grid_for(int64_t work, int threads = 256) {
    int64_t b = (work + threads - 1) / threads;
    if (b > 148 * 64) b = 148 * 64;
    return (int)(b < 1 ? 1 : b);
}

void launch_global_mean(const float* x, int64_t n, int d, float* out, cudaStream_t s) {
    global_mean_kernel<<<(d + 127) / 128, 128, 0, s>>>(x, n, d, out);
}
void launch_row_norm_sq(const float* x, int64_t n, int d, float* out, cudaStream_t s) {
    if (n > 0) row_norm_sq_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(x, n, d, out);
}
void launch_residual_pad(const float* x, int64_t n, int d, int D, const float* centroid, float* out,
                         cudaStream_t s) {
    if (n > 0) residual_pad_kernel<<<grid_for(n * D), 256, 0, s>>>(x, n, d, D, centroid, out);
}
void launch_encode_rotated(const float* rotated, int64_t n, int D, int nbits,
                           const float* norm_sq_raw, uint8_t* codes, uint8_t* signs, float4* meta,
                           cudaStream_t s) {
    // `rotated` is used as the o_hat buffer; the caller passes a scratch copy.
    // The byte scratch for codes lives right after the rotated rows (n*D floats).
    if (n <= 0) return;
    uint8_t* scratch = reinterpret_cast<uint8_t*>(const_cast<float*>(rotated) + n * D);
    encode_rotated_kernel<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(
        const_cast<float*>(rotated), n, D, nbits, norm_sq_raw, scratch, codes, signs, meta);
}
void launch_argmin_rows(const float* dist, int64_t n, int nlist, int32_t* out, cudaStream_t s) {
    if (n > 0) argmin_rows_kernel<<<(unsigned)((n * 32 + 255) / 256), 256, 0, s>>>(dist, n, nlist, out);
}
void launch_kmeans_accumulate(const float* x, int64_t n, int d, const int32_t* assign,
                              long long* sums, int* counts, cudaStream_t s) {
    if (n > 0)
        kmeans_accumulate_kernel<<<grid_for(n * d), 256, 0, s>>>(
            x, n, d, assign, reinterpret_cast<unsigned long long*>(sums), counts);
}
void launch_kmeans_update(const long long* sums, const int* counts, int nlist, int d,
                          float* centroids, float* shift, cudaStream_t s) {
    kmeans_update_kernel<<<(unsigned)(((int64_t)nlist * 32 + 255) / 256), 256, 0, s>>>(
        sums, counts, nlist, d, centroids, shift);
}

int kpp_blocks(int64_t n, int64_t* per) {
    const int64_t nb = std::min<int64_t>(1024, std::max<int64_t>(1, (n + 255) / 256));
    *per = (n + nb - 1) / nb;
    return (int)((n + *per - 1) / *per);
}

void launch_kpp_init_min(float* min_d, int64_t n, cudaStream_t s) {
    fill_f32_kernel<<<grid_for(n), 256, 0, s>>>(min_d, n, 3.402823466e38f);
}

void launch_kpp_step(const float* x, int64_t n, int d, float* cent, int slot, float* min_d,
                     double* block_sum, double u_target, double u_uniform, cudaStream_t s) {
    int64_t per = 0;
    const int nb = kpp_blocks(n, &per);
    kpp_dist_kernel<<<nb, 256, 0, s>>>(x, n, d, cent + (int64_t)(slot - 1) * d, per, min_d,
                                       block_sum);
    kpp_pick_kernel<<<1, 256, 0, s>>>(x, n, d, min_d, block_sum, nb, per, u_target, u_uniform,
                                      cent, slot);
}
void launch_build_fastscan(const uint8_t* signs, const int64_t* list_off, const int64_t* blk_off,
                           int nlist, int D, uint2* fs, cudaStream_t s) {
    if (nlist > 0) build_fastscan_kernel<<<nlist, 256, 0, s>>>(signs, list_off, blk_off, D, fs);
}
void launch_gather_rows(const uint8_t* src, const int64_t* perm, int64_t n, int64_t row_bytes,
                        uint8_t* dst, cudaStream_t s) {
    if (n > 0) gather_rows_kernel<<<grid_for(n * row_bytes), 256, 0, s>>>(src, perm, n, row_bytes, dst);
}

}  // namespace hanns
