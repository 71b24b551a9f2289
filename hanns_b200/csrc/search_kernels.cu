// search_kernels.cu -- batched IVF-USQ search on sm_100a.
//
// Pipeline for a batch of nq queries (all device-resident):
//   coarse_l2_kernel      exact sequential L2 of every (query, IVF centroid) pair
//                         (src/faiss/ivf_usq.rs:596-609,627-635)
//   select_probes_kernel  per query the nprobe smallest by (distance, list id),
//                         i.e. the reference's stable sort
//   rotate_kernel         q_rot = P * pad(q) in the AVX-512 order of
//                         src/quantization/usq/rotator.rs:93-120
//   query_state_kernel    q_sum, q_scale, q_i8, sum(q_i8), centroid_score, ||q||^2 and the
//                         FastScan LUT (quantizer.rs:236-270, fastscan.rs:22-66)
//   count/scan/scatter    group the (query, probe) pairs by list so that every list's codes
//                         are read once per batch and shared by all queries that probe it
//   scan_lists_kernel     per (list, query): FastScan scores (i16-wrapped sums of
//                         fastscan.rs:170-227), the exact fastscan_topk kept set
//                         (fastscan.rs:86-146) and integer rerank (quantizer.rs:274-400);
//                         every kept candidate goes to the query's candidate region
//   merge_kernel          per query top-k over its candidates by (distance, probe rank,
//                         FastScan order, list position): the reference's stable sort of
//                         src/faiss/ivf_usq.rs:590-593, padded with (-1, +inf)
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <cstring>

#include "common.cuh"
#include "kernels.h"
#include "warp_select.cuh"

namespace hanns {

__device__ __forceinline__ bool bit_filtered(const uint64_t* words, int64_t len, int64_t id) {
    // Kept iff (id as usize) >= len || bit == 0 (src/faiss/ivf_usq.rs:708-710).
    const uint64_t u = (uint64_t)id;
    if (u >= (uint64_t)len) return false;
    return (words[u >> 6] >> (u & 63)) & 1ull;
}

// ============================================================================
// Coarse: exact L2 (sequential over dims, unfused) for a 64x64 tile per CTA.
// ============================================================================
constexpr int kCT = 64;  // tile edge
constexpr int kCK = 16;  // dims per smem stage

__global__ void __launch_bounds__(256) coarse_l2_kernel(const float* __restrict__ q, int64_t nq,
                                                        const float* __restrict__ cent, int nlist,
                                                        int d, float* __restrict__ dist) {
    __shared__ float qs[kCK][kCT + 4];
    __shared__ float cs[kCK][kCT + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int64_t q0 = (int64_t)blockIdx.y * kCT;
    const int c0 = blockIdx.x * kCT;
    float acc[4][4];
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
        for (int b = 0; b < 4; ++b) acc[a][b] = -0.0f;
    for (int k0 = 0; k0 < d; k0 += kCK) {
        for (int e = threadIdx.x; e < kCT * kCK; e += 256) {
            const int row = e / kCK, kk = e % kCK;
            const int dim = k0 + kk;
            const int64_t qr = q0 + row;
            const int cr = c0 + row;
            qs[kk][row] = (qr < nq && dim < d) ? q[qr * d + dim] : 0.0f;
            cs[kk][row] = (cr < nlist && dim < d) ? cent[(int64_t)cr * d + dim] : 0.0f;
        }
        __syncthreads();
        const int kmax = min(kCK, d - k0);
        for (int kk = 0; kk < kmax; ++kk) {
            float qv[4], cv[4];
#pragma unroll
            for (int a = 0; a < 4; ++a) qv[a] = qs[kk][ty * 4 + a];
#pragma unroll
            for (int b = 0; b < 4; ++b) cv[b] = cs[kk][tx * 4 + b];
#pragma unroll
            for (int a = 0; a < 4; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const float df = __fsub_rn(qv[a], cv[b]);
                    acc[a][b] = __fadd_rn(acc[a][b], __fmul_rn(df, df));
                }
        }
        __syncthreads();
    }
#pragma unroll
    for (int a = 0; a < 4; ++a) {
        const int64_t qr = q0 + ty * 4 + a;
        if (qr >= nq) continue;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const int cr = c0 + tx * 4 + b;
            if (cr < nlist) dist[qr * nlist + cr] = acc[a][b];
        }
    }
}

// Per query (one warp): the nprobe smallest (distance, list) pairs, in order.
__global__ void __launch_bounds__(128) select_probes_kernel(const float* __restrict__ dist,
                                                            int64_t nq, int nlist, int nprobe,
                                                            int32_t* __restrict__ probes,
                                                            uint32_t* __restrict__ sel_scratch) {
    __shared__ uint32_t hist[4][256];
    const int w = threadIdx.x >> 5, lane = (int)lane_id();
    const int64_t qi = (int64_t)blockIdx.x * 4 + w;
    if (qi >= nq) return;
    const float* row = dist + qi * nlist;
    auto key_at = [&](int i, uint32_t& k) {
        k = total_order_key(row[i]);
        return true;
    };
    int less = 0;
    const uint32_t tau = warp_radix_kth(nlist, nprobe, key_at, hist[w], &less);
    // Gather the selected (key, idx): all keys < tau, then the lowest-index ties.
    uint32_t* sk = sel_scratch + qi * 2 * (int64_t)nprobe;
    uint32_t* si = sk + nprobe;
    int cnt = 0, ties_needed = nprobe - less;
    for (int base = 0; base < nlist; base += 32) {
        const int i = base + lane;
        uint32_t k = 0xFFFFFFFFu;
        if (i < nlist) k = total_order_key(row[i]);
        const bool lt = i < nlist && k < tau;
        const bool eq = i < nlist && k == tau;
        const unsigned beq = __ballot_sync(0xffffffffu, eq);
        const int eq_rank = __popc(beq & lanemask_lt());
        const bool take = lt || (eq && eq_rank < ties_needed);
        const unsigned bt = __ballot_sync(0xffffffffu, take);
        if (take) {
            const int pos = cnt + __popc(bt & lanemask_lt());
            sk[pos] = k;
            si[pos] = (uint32_t)i;
        }
        cnt += __popc(bt);
        ties_needed -= min(__popc(beq), max(ties_needed, 0));
    }
    __syncwarp();
    // rank sort by (key, idx)
    for (int a = lane; a < nprobe; a += 32) {
        const uint32_t ka = sk[a], ia = si[a];
        int rank = 0;
        for (int b = 0; b < nprobe; ++b) {
            const uint32_t kb = sk[b], ib = si[b];
            rank += (kb < ka || (kb == ka && ib < ia)) ? 1 : 0;
        }
        probes[qi * nprobe + rank] = (int32_t)ia;
    }
}

// ============================================================================
// Coarse, fast path.  a(q,c) = ||c||^2 - 2 q.c is computed with an FP32 GEMM (FMA,
// sequential over dims inside each thread), then per query every centroid whose a(q,c)
// lies within a rigorous rounding-error bound of the nprobe-th smallest is re-scored
// with the reference's exact sequential L2 and the nprobe best are selected exactly.
// The bound guarantees the exact top-nprobe set is among the re-scored centroids, so
// the probes equal those of coarse_l2_kernel + select_probes_kernel.  A query whose
// candidate set is larger than kCoarseCap (or smaller than nprobe, e.g. NaN inputs)
// takes the exact scan of every centroid instead.
// ============================================================================
constexpr int kGM = 128, kGN = 128, kGK = 16;
constexpr int kCoarseCap = 512;

template <bool kVec>
__global__ void __launch_bounds__(256) coarse_gemm_kernel(const float* __restrict__ q, int64_t nq,
                                                          const float* __restrict__ cent, int nlist,
                                                          int d, const float* __restrict__ cn,
                                                          float* __restrict__ out) {
    __shared__ __align__(16) float As[kGK][kGM + 4];
    __shared__ __align__(16) float Bs[kGK][kGN + 4];
    const int tid = threadIdx.x;
    const int tx = tid & 15, ty = tid >> 4;
    const int64_t q0 = (int64_t)blockIdx.y * kGM;
    const int c0 = blockIdx.x * kGN;
    const int lr = tid >> 2, lk = (tid & 3) * 4;
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
    for (int k0 = 0; k0 < d; k0 += kGK) {
        float ra[2][4], rb[2][4];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int row = lr + 64 * h;
            const int64_t qr = q0 + row;
            const int cr = c0 + row;
            const int kk = k0 + lk;
            if (kVec) {
                float4 va = make_float4(0.f, 0.f, 0.f, 0.f), vb = va;
                if (qr < nq && kk < d) va = __ldg(reinterpret_cast<const float4*>(q + qr * d + kk));
                if (cr < nlist && kk < d)
                    vb = __ldg(reinterpret_cast<const float4*>(cent + (int64_t)cr * d + kk));
                ra[h][0] = va.x; ra[h][1] = va.y; ra[h][2] = va.z; ra[h][3] = va.w;
                rb[h][0] = vb.x; rb[h][1] = vb.y; rb[h][2] = vb.z; rb[h][3] = vb.w;
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    ra[h][j] = (qr < nq && kk + j < d) ? q[qr * d + kk + j] : 0.0f;
                    rb[h][j] = (cr < nlist && kk + j < d) ? cent[(int64_t)cr * d + kk + j] : 0.0f;
                }
            }
        }
        __syncthreads();
#pragma unroll
        for (int h = 0; h < 2; ++h)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                As[lk + j][lr + 64 * h] = ra[h][j];
                Bs[lk + j][lr + 64 * h] = rb[h][j];
            }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < kGK; ++kk) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[kk][ty * 4]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[kk][64 + ty * 4]);
            const float4 b0 = *reinterpret_cast<const float4*>(&Bs[kk][tx * 4]);
            const float4 b1 = *reinterpret_cast<const float4*>(&Bs[kk][64 + tx * 4]);
            const float av[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float bv[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(av[i], bv[j], acc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int64_t qr = q0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + i - 4);
        if (qr >= nq) continue;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int cr = c0 + (j < 4 ? tx * 4 + j : 64 + tx * 4 + j - 4);
            if (cr < nlist) out[qr * nlist + cr] = __fmaf_rn(-2.0f, acc[i][j], cn[cr]);
        }
    }
}

// Exact sequential L2 (the reference's l2_distance) of one query (shared memory, 16-byte
// aligned) to one centroid.  The centroid row comes from L2 in blocks of 16 float4 loads
// issued together, so the dependent add chain waits for one round trip per 64 dims
// instead of one per 4.
__device__ __forceinline__ float exact_l2(const float* qs, const float* __restrict__ c, int d) {
    float s = -0.0f;
    if ((d & 3) == 0) {
        const float4* c4 = reinterpret_cast<const float4*>(c);
        const float4* q4 = reinterpret_cast<const float4*>(qs);
        const int n4 = d / 4;
        int i = 0;
        for (; i + 16 <= n4; i += 16) {
            float4 v[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) v[u] = __ldg(c4 + i + u);
#pragma unroll
            for (int u = 0; u < 16; ++u) {
                const float4 qv = q4[i + u];
                float df = __fsub_rn(qv.x, v[u].x);
                s = __fadd_rn(s, __fmul_rn(df, df));
                df = __fsub_rn(qv.y, v[u].y);
                s = __fadd_rn(s, __fmul_rn(df, df));
                df = __fsub_rn(qv.z, v[u].z);
                s = __fadd_rn(s, __fmul_rn(df, df));
                df = __fsub_rn(qv.w, v[u].w);
                s = __fadd_rn(s, __fmul_rn(df, df));
            }
        }
        for (; i < n4; ++i) {
            const float4 v = __ldg(c4 + i);
            const float4 qv = q4[i];
            float df = __fsub_rn(qv.x, v.x);
            s = __fadd_rn(s, __fmul_rn(df, df));
            df = __fsub_rn(qv.y, v.y);
            s = __fadd_rn(s, __fmul_rn(df, df));
            df = __fsub_rn(qv.z, v.z);
            s = __fadd_rn(s, __fmul_rn(df, df));
            df = __fsub_rn(qv.w, v.w);
            s = __fadd_rn(s, __fmul_rn(df, df));
        }
    } else {
        for (int i = 0; i < d; ++i) {
            const float df = __fsub_rn(qs[i], __ldg(c + i));
            s = __fadd_rn(s, __fmul_rn(df, df));
        }
    }
    return s;
}

// Rounding-error threshold of the approximate coarse step.  For every centroid c of the
// exact top-nprobe set, a(q,c) <= threshold (derivation in the DESIGN notes):
//   |a(q,c) - (||q-c||^2 - ||q||^2)| <= err,  E(c) <= T(c)(1+g),  T(c) <= E(c)/(1-g)
// with g = (d + 8) 2^-24 bounding the relative error of a sequential sum of d terms.
// dot_rel bounds |computed q.c - q.c| / sum|q_i c_i| for the GEMM that produced a(q,c).
struct CoarseErr {
    double gam;  // relative error bound of a sequential sum of d terms
    double Qn;   // computed ||q||^2
    double eQ;   // |Qn - ||q||^2| bound
    double err;  // |a(q,c) - (||q-c||^2 - ||q||^2)| bound, every c
};
__device__ __forceinline__ CoarseErr coarse_err(float qn, float cmax, int d, float dot_rel) {
    CoarseErr e;
    e.gam = (double)(d + 8) * 5.9604644775390625e-8;
    e.Qn = (double)qn;
    e.eQ = 2.0 * e.gam * e.Qn + 1e-30;
    const double qnorm = sqrt(e.Qn) * (1.0 + 2.0 * e.gam);
    const double cm = (double)cmax * (1.0 + 2.0 * e.gam);
    e.err = 4.0 * (double)dot_rel * qnorm * cm + 2.0 * e.gam * cm * cm +
            2.384185791015625e-7 * (cm * cm + 2.0 * qnorm * cm) + 1e-30;
    return e;
}
__device__ __forceinline__ double coarse_threshold(float tau, float qn, float cmax, int d,
                                                   float dot_rel) {
    const CoarseErr e = coarse_err(qn, cmax, d, dot_rel);
    const double e_ub = ((double)tau + e.Qn + e.eQ + e.err) * (1.0 + 2.0 * e.gam);
    return e_ub * (1.0 + 2.0 * e.gam) - e.Qn + e.eQ + e.err;
}

// One warp: the nprobe (<= kCoarseCap) smallest of row[0..nlist) by (total-order key,
// index) -- the stable sort of rank_centroids -- written in order to out[].
__device__ void warp_select_stable(const float* row, int nlist, int nprobe, uint32_t* hist,
                                   uint32_t* sk, int* si, int32_t* out) {
    const int lane = (int)lane_id();
    auto key_at = [&](int i, uint32_t& k) {
        k = total_order_key(row[i]);
        return true;
    };
    int less = 0;
    const uint32_t ktau = warp_radix_kth(nlist, nprobe, key_at, hist, &less);
    int taken = 0, ties_needed = nprobe - less;
    for (int base = 0; base < nlist && taken < nprobe; base += 32) {
        const int i = base + lane;
        uint32_t k = 0xFFFFFFFFu;
        if (i < nlist) k = total_order_key(row[i]);
        const bool lt = i < nlist && k < ktau;
        const bool eq = i < nlist && k == ktau;
        const unsigned beq = __ballot_sync(0xffffffffu, eq);
        const int eq_rank = __popc(beq & lanemask_lt());
        const bool take = lt || (eq && eq_rank < ties_needed);
        const unsigned bt = __ballot_sync(0xffffffffu, take);
        if (take) {
            const int pos = taken + __popc(bt & lanemask_lt());
            if (pos < kCoarseCap) {
                sk[pos] = k;
                si[pos] = i;
            }
        }
        taken += __popc(bt);
        ties_needed -= min(__popc(beq), max(ties_needed, 0));
    }
    __syncwarp();
    const int m = min(taken, min(nprobe, kCoarseCap));
    for (int a = lane; a < m; a += 32) {
        const uint32_t ka = sk[a];
        const int ia = si[a];
        int rank = 0;
        for (int b = 0; b < m; ++b) rank += (sk[b] < ka || (sk[b] == ka && si[b] < ia)) ? 1 : 0;
        out[rank] = ia;
    }
    __syncwarp();
}

// One warp per query, row in global memory (any nlist).  `approx` rows are per-query
// scratch (overwritten with exact distances on fallback).  nprobe <= kCoarseCap / 2.
__global__ void __launch_bounds__(128) coarse_select_exact_kernel(
    float* __restrict__ approx, const float* __restrict__ q, int64_t nq,
    const float* __restrict__ cent, int nlist, int d, int nprobe, float cmax, float dot_rel,
    const int* __restrict__ tc_err, int32_t* __restrict__ probes, int* __restrict__ fallbacks) {
    extern __shared__ __align__(16) float qsm[];  // [4][d]
    __shared__ uint32_t hist[4][256];
    __shared__ uint32_t ckey[4][kCoarseCap];
    __shared__ int cidx[4][kCoarseCap];
    const int w = threadIdx.x >> 5, lane = (int)lane_id();
    const int64_t qi = (int64_t)blockIdx.x * 4 + w;
    if (qi >= nq) return;
    float* qs = qsm + w * d;
    float* row = approx + qi * nlist;
    float qn = 0.0f;
    for (int i = lane; i < d; i += 32) {
        const float v = q[qi * d + i];
        qs[i] = v;
        qn = __fmaf_rn(v, v, qn);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qn = __fadd_rn(qn, __shfl_xor_sync(0xffffffffu, qn, o));
    __syncwarp();
    auto key_at = [&](int i, uint32_t& k) {
        k = total_order_key(row[i]);
        return true;
    };
    int less = 0;
    const float tau = key_to_float(warp_radix_kth(nlist, nprobe, key_at, hist[w], &less));
    const double thr = coarse_threshold(tau, qn, cmax, d, dot_rel);
    const bool approx_ok = !tc_err || *tc_err == 0;
    int cnt = 0;
    for (int base = 0; base < nlist; base += 32) {
        const int c = base + lane;
        const bool in = c < nlist && (double)row[c] <= thr;
        const unsigned b = __ballot_sync(0xffffffffu, in);
        if (in) {
            const int pos = cnt + __popc(b & lanemask_lt());
            if (pos < kCoarseCap) cidx[w][pos] = c;
        }
        cnt += __popc(b);
    }
    __syncwarp();
    if (approx_ok && cnt <= kCoarseCap && cnt >= nprobe) {
        for (int i = lane; i < cnt; i += 32)
            ckey[w][i] = total_order_key(exact_l2(qs, cent + (int64_t)cidx[w][i] * d, d));
        __syncwarp();
        for (int i = lane; i < cnt; i += 32) {
            const uint32_t ki = ckey[w][i];
            const int ii = cidx[w][i];
            int rank = 0;
            for (int j = 0; j < cnt; ++j) {
                const uint32_t kj = ckey[w][j];
                rank += (kj < ki || (kj == ki && cidx[w][j] < ii)) ? 1 : 0;
            }
            if (rank < nprobe) probes[qi * nprobe + rank] = ii;
        }
        return;
    }
    // fallback: exact distance to every centroid, then the stable selection
    if (lane == 0) atomicAdd(fallbacks, 1);
    for (int c = lane; c < nlist; c += 32) row[c] = exact_l2(qs, cent + (int64_t)c * d, d);
    __syncwarp();
    warp_select_stable(row, nlist, nprobe, hist[w], ckey[w], cidx[w], probes + qi * nprobe);
}

// Block-wide k-th smallest total-order key (256 threads).
constexpr int kSelThreads = 256;
constexpr int kSelBins = 4096;  // 12 bits per histogram pass
constexpr int kSelList = 1024;  // shared scratch words (keys of the final bin, block sums)
constexpr int kSelRank = 64;    // a bin this small is ranked exactly

// k-th smallest (1-based) of the keys each thread produces through for_each(f) (f is
// called once per key of the calling thread).  One pass finds the key range; 12-bit
// histogram passes over the bits in which the keys differ, each restricted to the keys
// whose higher bits match the bins chosen so far, narrow the search until the bin of the
// k-th key holds at most kSelRank keys, which are then ranked exactly.  Keys of nearby
// scores share their high bits, so a histogram of fixed high bytes would pile every key
// into one bin.  hist: kSelBins words, list: kSelList words, bcast: 8 ints (shared).
template <class ForEach>
__device__ uint32_t block_select_kth(ForEach for_each, int kth, uint32_t* hist, uint32_t* list,
                                     int* bcast) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
    for_each([&](uint32_t k) {
        kmin = min(kmin, k);
        kmax = max(kmax, k);
    });
    kmin = warp_min_u32(kmin);
    kmax = warp_max_u32(kmax);
    if (lane == 0) {
        list[w] = kmin;
        list[32 + w] = kmax;
    }
    __syncthreads();
    if (tid < 32) {
        uint32_t a = tid < kSelThreads / 32 ? list[tid] : 0xFFFFFFFFu;
        uint32_t b = tid < kSelThreads / 32 ? list[32 + tid] : 0u;
        a = warp_min_u32(a);
        b = warp_max_u32(b);
        if (tid == 0) {
            bcast[6] = (int)a;
            bcast[7] = (int)b;
        }
    }
    __syncthreads();
    kmin = (uint32_t)bcast[6];
    const uint32_t range = (uint32_t)bcast[7] - kmin;
    int res = 32 - __clz(range);  // bits >= res of (key - kmin) are resolved (zero so far)
    uint32_t prefix = 0;
    int r = kth;
    while (res > 0) {
        const int shift = res > 12 ? res - 12 : 0;
        for (int i = tid; i < kSelBins; i += kSelThreads) hist[i] = 0;
        __syncthreads();
        for_each([&](uint32_t k) {
            const uint32_t kp = k - kmin;
            if (res >= 32 || ((kp ^ prefix) >> res) == 0) atomicAdd(&hist[(kp >> shift) & (kSelBins - 1)], 1u);
        });
        __syncthreads();
        // bin of the r-th key: thread t owns bins 16t .. 16t+15
        int s = 0;
#pragma unroll
        for (int b = 0; b < 16; ++b) s += (int)hist[tid * 16 + b];
        const int incl = warp_inclusive_scan(s);
        if (lane == 31) list[64 + w] = (uint32_t)incl;
        __syncthreads();
        int off = 0;
        for (int j = 0; j < w; ++j) off += (int)list[64 + j];
        const int lo = off + incl - s, hi = off + incl;
        if (lo < r && r <= hi) {
            int c = lo, bin = tid * 16;
            for (int b = 0; b < 16; ++b) {
                const int h = (int)hist[tid * 16 + b];
                if (c + h >= r) {
                    bin = tid * 16 + b;
                    break;
                }
                c += h;
            }
            bcast[0] = bin;
            bcast[1] = c;
            bcast[2] = (int)hist[bin];
        }
        __syncthreads();
        const uint32_t bin = (uint32_t)bcast[0];
        r -= bcast[1];
        const int cnt = bcast[2];
        prefix |= (bin << shift) & ~((res >= 32) ? 0u : (0xFFFFFFFFu << res));
        res = shift;
        if (cnt <= kSelRank) break;
        __syncthreads();
    }
    if (res == 0) return kmin + prefix;  // every key of the bin is equal
    // rank the (<= kSelRank) keys of the final bin exactly
    if (tid == 0) bcast[3] = 0;
    __syncthreads();
    for_each([&](uint32_t k) {
        const uint32_t kp = k - kmin;
        if (((kp ^ prefix) >> res) == 0) list[atomicAdd(&bcast[3], 1)] = kp;
    });
    __syncthreads();
    const int cnt = bcast[3];
    for (int t = tid; t < cnt; t += kSelThreads) {
        const uint32_t x = list[t];
        int less = 0, eq_before = 0;
        for (int j = 0; j < cnt; ++j) {
            const uint32_t u = list[j];
            less += u < x ? 1 : 0;
            eq_before += (u == x && j < t) ? 1 : 0;
        }
        if (less + eq_before == r - 1) bcast[4] = (int)x;
    }
    __syncthreads();
    return kmin + (uint32_t)bcast[4];
}

// An upper bound of the k-th smallest value, for a threshold that only has to admit the
// k smallest: one pass bins the values uniformly between their minimum and maximum
// (the binning is monotone in the value), the bin holding the k-th value is found from
// the histogram, and the largest value in that bin is returned.  for_each(f) calls f(v)
// for every value of the calling thread; hist: kSelBins words, list: 64 words, bcast: 8.
template <class ForEach>
__device__ float block_kth_upper(ForEach for_each, int kth, uint32_t* hist, uint32_t* list,
                                 int* bcast) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    float lo = __int_as_float(0x7f800000), hi = -__int_as_float(0x7f800000);
    for_each([&](float v) {
        lo = fminf(lo, v);
        hi = fmaxf(hi, v);
    });
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (lane == 0) {
        list[w] = __float_as_uint(lo);
        list[32 + w] = __float_as_uint(hi);
    }
    for (int i = tid; i < kSelBins; i += kSelThreads) hist[i] = 0;
    __syncthreads();
    if (tid == 0) {
        float a = __uint_as_float(list[0]), b = __uint_as_float(list[32]);
        for (int j = 1; j < kSelThreads / 32; ++j) {
            a = fminf(a, __uint_as_float(list[j]));
            b = fmaxf(b, __uint_as_float(list[32 + j]));
        }
        reinterpret_cast<float*>(bcast)[6] = a;
        reinterpret_cast<float*>(bcast)[7] = b;
    }
    __syncthreads();
    const float vmin = reinterpret_cast<float*>(bcast)[6], vmax = reinterpret_cast<float*>(bcast)[7];
    if (!(vmax > vmin)) return vmax;
    const float scale = __fdiv_rn((float)kSelBins, __fsub_rn(vmax, vmin));
    auto bin_of = [&](float v) {
        const int b = (int)__fmul_rz(__fsub_rn(v, vmin), scale);
        return min(max(b, 0), kSelBins - 1);
    };
    for_each([&](float v) { atomicAdd(&hist[bin_of(v)], 1u); });
    __syncthreads();
    int s = 0;
#pragma unroll
    for (int b = 0; b < 16; ++b) s += (int)hist[tid * 16 + b];
    const int incl = warp_inclusive_scan(s);
    if (lane == 31) list[w] = (uint32_t)incl;
    __syncthreads();
    int off = 0;
    for (int j = 0; j < w; ++j) off += (int)list[j];
    const int lo_c = off + incl - s, hi_c = off + incl;
    if (lo_c < kth && kth <= hi_c) {
        int c = lo_c, bin = tid * 16;
        for (int b = 0; b < 16; ++b) {
            const int h = (int)hist[tid * 16 + b];
            if (c + h >= kth) {
                bin = tid * 16 + b;
                break;
            }
            c += h;
        }
        bcast[0] = bin;
        bcast[1] = 0;  // total-order key of the bin's largest value
    }
    __syncthreads();
    const int bin = bcast[0];
    for_each([&](float v) {
        if (bin_of(v) == bin) atomicMax(reinterpret_cast<unsigned*>(&bcast[1]), total_order_key(v));
    });
    __syncthreads();
    return key_to_float((uint32_t)bcast[1]);
}

// k-th smallest total-order key of row[0..n) (shared or global memory).
__device__ uint32_t block_radix_kth(const float* row, int n, int kth, uint32_t* hist,
                                    uint32_t* list, int* bcast) {
    return block_select_kth(
        [&](auto f) {
            for (int i = threadIdx.x; i < n; i += kSelThreads) f(total_order_key(row[i]));
        },
        kth, hist, list, bcast);
}

// The same over a row left in global memory (n % 4 == 0, 16-byte aligned): four 16-byte
// loads of a thread in flight before any of their values is counted.
__device__ uint32_t block_radix_kth_g4(const float* row, int n, int kth, uint32_t* hist,
                                       uint32_t* list, int* bcast) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int n4 = n >> 2;
    return block_select_kth(
        [&](auto f) {
            for (int b = threadIdx.x; b < n4; b += 4 * kSelThreads) {
                float4 t[4];
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int i = b + j * kSelThreads;
                    if (i < n4) t[j] = __ldcg(r4 + i);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (b + j * kSelThreads < n4) {
                        f(total_order_key(t[j].x));
                        f(total_order_key(t[j].y));
                        f(total_order_key(t[j].z));
                        f(total_order_key(t[j].w));
                    }
                }
            }
        },
        kth, hist, list, bcast);
}

// One 256-thread block per query with the approximate row staged in shared memory
// (nlist small enough); same result as coarse_select_exact_kernel.
__global__ void __launch_bounds__(kSelThreads) coarse_select_block_kernel(
    float* approx, const float* __restrict__ q, int64_t nq,
    const float* __restrict__ cent, int nlist, int d, int nprobe, float cmax, float dot_rel,
    const int* __restrict__ tc_err, int32_t* __restrict__ probes, int* __restrict__ fallbacks,
    int row_in_smem) {
    // row[nlist4] (when row_in_smem; else the row stays in global memory), qs[d4],
    // hist[kSelBins], list[kSelList]
    extern __shared__ __align__(16) float sm[];
    __shared__ int bcast[8];
    __shared__ float red[kSelThreads / 32];
    __shared__ int cidx[kCoarseCap];
    __shared__ uint32_t ckey[kCoarseCap];
    __shared__ int cnt_s;
    __shared__ double thr_s;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int64_t qi = blockIdx.x;
    float* row = row_in_smem ? sm : approx + qi * nlist;
    float* qs = row_in_smem ? sm + ((nlist + 3) & ~3) : sm;
    uint32_t* hist = reinterpret_cast<uint32_t*>(qs + ((d + 3) & ~3));
    uint32_t* list = hist + kSelBins;
    // stage the approximate row and the query: every load of a thread is issued before
    // its first store, so the staging costs one memory round trip per 4 loads
    const float* grow = approx + qi * nlist;
    if (!row_in_smem) {
        // (read in place by the selection passes below)
    } else if ((nlist & 3) == 0) {
        const float4* g4 = reinterpret_cast<const float4*>(grow);
        float4* r4 = reinterpret_cast<float4*>(row);
        const int n4 = nlist >> 2;
        for (int b = 0; b < n4; b += 4 * kSelThreads) {
            float4 t[4];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = b + j * kSelThreads + tid;
                if (i < n4) t[j] = __ldcs(g4 + i);
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = b + j * kSelThreads + tid;
                if (i < n4) r4[i] = t[j];
            }
        }
    } else {
        for (int i = tid; i < nlist; i += kSelThreads) row[i] = grow[i];
    }
    float qn = 0.0f;
    for (int b = 0; b < d; b += 4 * kSelThreads) {
        float v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = b + j * kSelThreads + tid;
            v[j] = i < d ? __ldg(q + qi * d + i) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = b + j * kSelThreads + tid;
            if (i < d) {
                qs[i] = v[j];
                qn = __fmaf_rn(v[j], v[j], qn);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qn = __fadd_rn(qn, __shfl_xor_sync(0xffffffffu, qn, o));
    if (lane == 0) red[w] = qn;
    if (tid == 0) cnt_s = 0;
    __syncthreads();
    qn = 0.0f;
    for (int i = 0; i < kSelThreads / 32; ++i) qn = __fadd_rn(qn, red[i]);
    const bool vec_g = !row_in_smem && (nlist & 3) == 0;
    const float tau = key_to_float(vec_g ? block_radix_kth_g4(row, nlist, nprobe, hist, list, bcast)
                                         : block_radix_kth(row, nlist, nprobe, hist, list, bcast));
    if (tid == 0) thr_s = coarse_threshold(tau, qn, cmax, d, dot_rel);
    __syncthreads();
    const double thr = thr_s;
    auto candidate = [&](int c, float v) {
        if ((double)v <= thr) {
            const int pos = atomicAdd(&cnt_s, 1);
            if (pos < kCoarseCap) cidx[pos] = c;
        }
    };
    if (vec_g) {
        const float4* r4 = reinterpret_cast<const float4*>(row);
        const int n4 = nlist >> 2;
        for (int b = tid; b < n4; b += 4 * kSelThreads) {
            float4 t[4];
#pragma unroll
            for (int j = 0; j < 4; ++j)
                if (b + j * kSelThreads < n4) t[j] = __ldcg(r4 + b + j * kSelThreads);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int i = b + j * kSelThreads;
                if (i < n4) {
                    candidate(4 * i, t[j].x);
                    candidate(4 * i + 1, t[j].y);
                    candidate(4 * i + 2, t[j].z);
                    candidate(4 * i + 3, t[j].w);
                }
            }
        }
    } else {
        for (int c = tid; c < nlist; c += kSelThreads) candidate(c, row[c]);
    }
    __syncthreads();
    const int cnt = cnt_s;
    const bool approx_ok = !tc_err || *tc_err == 0;
    if (approx_ok && cnt <= kCoarseCap && cnt >= nprobe) {
        for (int i = tid; i < cnt; i += kSelThreads)
            ckey[i] = total_order_key(exact_l2(qs, cent + (int64_t)cidx[i] * d, d));
        __syncthreads();
        for (int i = tid; i < cnt; i += kSelThreads) {
            const uint32_t ki = ckey[i];
            const int ii = cidx[i];
            int rank = 0;
            for (int j = 0; j < cnt; ++j) rank += (ckey[j] < ki || (ckey[j] == ki && cidx[j] < ii)) ? 1 : 0;
            if (rank < nprobe) probes[qi * nprobe + rank] = ii;
        }
        return;
    }
    if (tid == 0) atomicAdd(fallbacks, 1);
    for (int c = tid; c < nlist; c += kSelThreads) row[c] = exact_l2(qs, cent + (int64_t)c * d, d);
    __syncthreads();
    if (w == 0) warp_select_stable(row, nlist, nprobe, hist, ckey, cidx, probes + qi * nprobe);
}

// One 256-thread block per query, the approximate row held in registers (NV4 float4 per
// thread, nlist <= 1024 * NV4, nlist % 4 == 0, d % 4 == 0).  Same result as
// coarse_select_block_kernel: k-th approximate key -> rigorous threshold -> exact
// re-score of the candidates (two per thread, packed f32x2) -> stable order.
template <int NV4>
__global__ void __launch_bounds__(kSelThreads) coarse_select_reg_kernel(
    float* __restrict__ approx, const float* __restrict__ q, int64_t nq,
    const float* __restrict__ cent, int nlist, int d, int nprobe, float cmax, float dot_rel,
    const int* __restrict__ tc_err, int32_t* __restrict__ probes, int* __restrict__ fallbacks,
    int* __restrict__ rs) {
    extern __shared__ __align__(16) float sm[];  // qs[d], hist[kSelBins], list[kSelList]
    __shared__ int bcast[8];
    __shared__ float red[kSelThreads / 32];
    __shared__ int cidx[kCoarseCap];
    __shared__ uint32_t ckey[kCoarseCap];
    __shared__ float capx[kCoarseRescoreMax];
    __shared__ int cnt_s;
    __shared__ float thr_s, thr_q;
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int64_t qi = blockIdx.x;
    float* qs = sm;
    uint32_t* hist = reinterpret_cast<uint32_t*>(sm + d);
    uint32_t* list = hist + kSelBins;
    const int n4 = nlist >> 2;
    float* grow = approx + qi * nlist;
    if (rs && tid == 0) rs[qi * kCoarseRsStride] = 0;  // 0: probes written here
    // the row: float4 index tid + 256 j, all loads issued before the first use
    float4 v[NV4];
#pragma unroll
    for (int j = 0; j < NV4; ++j) {
        const int i4 = tid + j * kSelThreads;
        v[j] = i4 < n4 ? __ldcs(reinterpret_cast<const float4*>(grow) + i4)
                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    float qn = 0.0f;
    for (int b = 0; b < d; b += 4 * kSelThreads) {
        float t[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = b + j * kSelThreads + tid;
            t[j] = i < d ? __ldg(q + qi * d + i) : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int i = b + j * kSelThreads + tid;
            if (i < d) {
                qs[i] = t[j];
                qn = __fmaf_rn(t[j], t[j], qn);
            }
        }
    }
    auto val = [&](int j, int e) -> float {
        return e == 0 ? v[j].x : e == 1 ? v[j].y : e == 2 ? v[j].z : v[j].w;
    };
    auto valid = [&](int j) { return tid + j * kSelThreads < n4; };
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) qn = __fadd_rn(qn, __shfl_xor_sync(0xffffffffu, qn, o));
    if (lane == 0) red[w] = qn;
    if (tid == 0) cnt_s = 0;
    // an upper bound of the nprobe-th smallest approximate score is enough: the threshold
    // only has to admit the exact top nprobe
    const float tau_up = block_kth_upper(
        [&](auto f) {
#pragma unroll
            for (int j = 0; j < NV4; ++j)
                if (valid(j))
#pragma unroll
                    for (int e = 0; e < 4; ++e) f(val(j, e));
        },
        nprobe, hist, list, bcast);
    if (tid == 0) {
        float qsum = 0.0f;
        for (int i = 0; i < kSelThreads / 32; ++i) qsum = __fadd_rn(qsum, red[i]);
        // (double)x <= thr  <=>  x <= thr rounded down to a float
        thr_s = __double2float_rd(coarse_threshold(tau_up, qsum, cmax, d, dot_rel));
        thr_q = qsum;
    }
    __syncthreads();
    const float thr = thr_s;
#pragma unroll
    for (int j = 0; j < NV4; ++j)
        if (valid(j))
#pragma unroll
            for (int e = 0; e < 4; ++e)
                if (val(j, e) <= thr) {
                    const int pos = atomicAdd(&cnt_s, 1);
                    if (pos < kCoarseCap) {
                        cidx[pos] = 4 * (tid + j * kSelThreads) + e;
                        if (pos < kCoarseRescoreMax) capx[pos] = val(j, e);
                    }
                }
    __syncthreads();
    const int cnt = cnt_s;
    const bool approx_ok = !tc_err || *tc_err == 0;
    if (approx_ok && cnt <= kCoarseCap && cnt >= nprobe) {
        if (cnt <= kCoarseRescoreMax && rs) {
            // ordering (and the few exact sums it needs) in coarse_rescore_kernel
            int* r = rs + qi * kCoarseRsStride;
            for (int i = tid; i < cnt; i += kSelThreads) {
                r[2 + i] = cidx[i];
                r[2 + kCoarseRescoreMax + i] = __float_as_int(capx[i]);
            }
            if (tid == 0) {
                r[0] = cnt;
                r[1] = __float_as_int(thr_q);
            }
            return;
        }
        for (int i = tid; i < cnt; i += kSelThreads)
            ckey[i] = total_order_key(exact_l2(qs, cent + (int64_t)cidx[i] * d, d));
        __syncthreads();
        for (int i = tid; i < cnt; i += kSelThreads) {
            const uint32_t ki = ckey[i];
            const int ii = cidx[i];
            int rank = 0;
            for (int j = 0; j < cnt; ++j) rank += (ckey[j] < ki || (ckey[j] == ki && cidx[j] < ii)) ? 1 : 0;
            if (rank < nprobe) probes[qi * nprobe + rank] = ii;
        }
        return;
    }
    // fallback: exact distances to every centroid (into the query's scratch row), then the
    // stable selection
    if (tid == 0) atomicAdd(fallbacks, 1);
    for (int c = tid; c < nlist; c += kSelThreads) grow[c] = exact_l2(qs, cent + (int64_t)c * d, d);
    __syncthreads();
    if (w == 0) warp_select_stable(grow, nlist, nprobe, hist, ckey, cidx, probes + qi * nprobe);
}

// coarse_rescore_kernel's staging of the centroid rows (d % 4 == 0 and d > kRsStageMinD;
// shorter rows stream from L2 into each thread's chain, exact_l2): dims per chunk, padded
// row stride (floats; +4 keeps the 16-byte row reads of 8 consecutive lanes on distinct
// banks)
constexpr int kRsStageMinD = 1024;
constexpr int kRsChunk = 64;
constexpr int kRsLd = kRsChunk + 4;
__host__ __device__ inline bool rescore_staged(int d) { return (d & 3) == 0 && d > kRsStageMinD; }
inline size_t coarse_rescore_smem(int d) {
    return ((size_t)((d + 3) & ~3) + (rescore_staged(d) ? 2 * (size_t)kCoarseRescoreMax * kRsLd : 0)) *
           sizeof(float);
}

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
                 "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Order of the candidates coarse_select_reg_kernel left in rs (per query: count, ||q||^2,
// up to kCoarseRescoreMax centroid ids, their approximate scores a).  Each a bounds the
// reference's sequential sum E(c) = exact_l2(q, c):
//   ||q-c||^2 in [a + Qn - eQ - err, a + Qn + eQ + err]   (the coarse threshold's error terms)
//   E(c) in [||q-c||^2 (1 - g), ||q-c||^2 (1 + g)]          (g: sequential-sum bound)
// widened by (1 -/+ 2g).  Two candidates whose intervals are disjoint are ordered by
// them; a candidate whose interval meets another's gets its exact sum (one thread, the
// reference's order), and such pairs are ordered by (exact key, centroid id) -- the stable
// sort.  Typically a handful of the ~nprobe candidates of a query need the exact sum.
template <bool STAGED>
__global__ void __launch_bounds__(kCoarseRescoreMax) coarse_rescore_kernel(const float* __restrict__ q, int64_t nq,
                                                                 const float* __restrict__ cent, int d,
                                                                 int nprobe, float cmax, float dot_rel,
                                                                 const int* __restrict__ rs,
                                                                 int32_t* __restrict__ probes) {
    extern __shared__ __align__(16) float qsm[];  // [d], then the staged rows
    __shared__ double lo_s[kCoarseRescoreMax], hi_s[kCoarseRescoreMax];
    __shared__ uint32_t ckey[kCoarseRescoreMax];
    __shared__ int cidx[kCoarseRescoreMax];
    __shared__ int need_s[kCoarseRescoreMax];
    __shared__ int any_s;
    const int64_t qi = blockIdx.x;
    const int* r = rs + qi * kCoarseRsStride;
    const int cnt = r[0];
    if (cnt == 0) return;  // done by the select kernel
    const int tid = threadIdx.x;
    const CoarseErr e = coarse_err(__int_as_float(r[1]), cmax, d, dot_rel);
    int ci = 0;
    double lo = 0.0, hi = 0.0;
    if (tid < cnt) {
        ci = r[2 + tid];
        const double a = (double)__int_as_float(r[2 + kCoarseRescoreMax + tid]);
        lo = (a + e.Qn - e.eQ - e.err) * (1.0 - 2.0 * e.gam);
        hi = (a + e.Qn + e.eQ + e.err) * (1.0 + 2.0 * e.gam);
        lo_s[tid] = lo;
        hi_s[tid] = hi;
        cidx[tid] = ci;
    }
    if (tid == 0) any_s = 0;
    __syncthreads();
    bool need = false;
    if (tid < cnt)
        for (int j = 0; j < cnt; ++j)
            if (j != tid && !(hi_s[j] < lo || hi < lo_s[j])) need = true;
    need_s[tid] = need ? 1 : 0;
    if (need) any_s = 1;
    __syncthreads();
    if (any_s) {
        for (int i = tid; i < d; i += kCoarseRescoreMax) qsm[i] = q[qi * d + i];
        if (STAGED) {
            // the needed centroid rows, kRsChunk dims at a time, staged in shared memory by
            // all threads with coalesced 16-byte copies (double buffered: the next chunk is
            // in flight while the sums run); each needing thread then continues its row's
            // sequential sum from shared memory
            float* rows = qsm + ((d + 3) & ~3);  // [2][kCoarseRescoreMax][kRsLd]
            int* slot_ci = need_s;  // reused below: slot -> centroid id
            __shared__ int nn_s;
            if (tid == 0) nn_s = 0;
            __syncthreads();
            int slot = -1;
            if (need) {
                slot = atomicAdd(&nn_s, 1);
            }
            __syncthreads();
            const int nn = nn_s;
            if (need) slot_ci[slot] = ci;
            __syncthreads();
            const int nchunk = (d + kRsChunk - 1) / kRsChunk;
            auto stage = [&](int c) {
                float* dst = rows + (c & 1) * (kCoarseRescoreMax * kRsLd);
                const int c0 = c * kRsChunk;
                for (int e = tid; e < nn * (kRsChunk / 4); e += kCoarseRescoreMax) {
                    const int j = e / (kRsChunk / 4), p4 = e - j * (kRsChunk / 4);
                    if (c0 + 4 * p4 < d)
                        cp_async16(dst + j * kRsLd + 4 * p4, cent + (int64_t)slot_ci[j] * d + c0 + 4 * p4);
                }
                cp_async_commit();
            };
            stage(0);
            float acc = -0.0f;
            for (int c = 0; c < nchunk; ++c) {
                if (c + 1 < nchunk) {
                    stage(c + 1);
                    cp_async_wait<1>();
                } else {
                    cp_async_wait<0>();
                }
                __syncthreads();
                if (need) {
                    const float* rj = rows + (c & 1) * (kCoarseRescoreMax * kRsLd) + slot * kRsLd;
                    const int c0 = c * kRsChunk, len = min(kRsChunk, d - c0);
                    for (int i = 0; i < len; i += 4) {
                        const float4 v = *reinterpret_cast<const float4*>(rj + i);
                        const float4 qv = *reinterpret_cast<const float4*>(qsm + c0 + i);
                        float df = __fsub_rn(qv.x, v.x);
                        acc = __fadd_rn(acc, __fmul_rn(df, df));
                        df = __fsub_rn(qv.y, v.y);
                        acc = __fadd_rn(acc, __fmul_rn(df, df));
                        df = __fsub_rn(qv.z, v.z);
                        acc = __fadd_rn(acc, __fmul_rn(df, df));
                        df = __fsub_rn(qv.w, v.w);
                        acc = __fadd_rn(acc, __fmul_rn(df, df));
                    }
                }
                __syncthreads();  // the buffer is restaged two chunks on
            }
            if (need) ckey[tid] = total_order_key(acc);
            // need_s held slot ids; the rank pass reads it as the need flags again
            need_s[tid] = need ? 1 : 0;
            __syncthreads();
        } else {
            __syncthreads();
            if (need) ckey[tid] = total_order_key(exact_l2(qsm, cent + (int64_t)ci * d, d));
            __syncthreads();
        }
    }
    if (tid < cnt) {
        const uint32_t ki = need ? ckey[tid] : 0u;
        int rank = 0;
        for (int j = 0; j < cnt; ++j) {
            if (j == tid) continue;
            if (need && need_s[j])
                rank += (ckey[j] < ki || (ckey[j] == ki && cidx[j] < ci)) ? 1 : 0;
            else
                rank += hi_s[j] < lo ? 1 : 0;
        }
        if (rank < nprobe) probes[qi * nprobe + rank] = ci;
    }
}

__global__ void centroid_norms_kernel(const float* __restrict__ cent, int nlist, int d,
                                      float* __restrict__ cn) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= nlist) return;
    float s = 0.0f;
    for (int i = 0; i < d; ++i) s = __fmaf_rn(cent[(int64_t)c * d + i], cent[(int64_t)c * d + i], s);
    cn[c] = s;
}

// ============================================================================
// Query preparation
// ============================================================================

// P in chain-major order: within each row, Pc[tb*64 + j*4 + k] = P[j + 16*(4*tb + k)]
// (tb < D/64, j < 16, k < 4), so that the four consecutive terms of chain j inside a
// 64-column block are one 16-byte load and a half-warp's loads are 256 contiguous bytes.
__global__ void rotation_chain_major_kernel(const float* __restrict__ P, int D,
                                            float* __restrict__ Pc) {
    const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= (int64_t)D * D) return;
    const int64_t r = e / D;
    const int i = (int)(e - r * D);
    const int tb = i >> 6, j = (i & 63) >> 2, k = i & 3;
    Pc[e] = P[r * D + j + 16 * (4 * tb + k)];
}

// q_rot[q][r] = tree16( lane j: fma chain over c = j, j+16, ... of P[r][c]*x[c] ).
// QT queries per CTA, staged transposed in shared memory ([D][QT+4] floats) so a lane
// reads the QT query values of one column with 16-byte loads.  A half-warp owns R
// consecutive rows (16*R rows per CTA); lane j keeps the chain of column class j for
// R rows x QT queries, so every query value loaded feeds R FMAs and every P value QT.
// Pc is P in chain-major order (rotation_chain_major_kernel): one 16-byte load per row
// brings chain j's next four terms.
template <int QT, int R>
__global__ void __launch_bounds__(256) rotate_kernel(const float* __restrict__ x, int64_t nq,
                                                     int d, int D, const float* __restrict__ Pc,
                                                     float* __restrict__ out) {
    constexpr int LD = QT + 4;
    extern __shared__ __align__(16) float xs[];  // [D][LD]
    const int64_t q0 = (int64_t)blockIdx.y * QT;
    // fill: each thread moves 4 consecutive dims of one query (16-byte loads when d % 4 == 0);
    // consecutive threads take consecutive queries so the transposed stores hit
    // consecutive banks
    const int D4 = D / 4;
#pragma unroll 4
    for (int e = threadIdx.x; e < QT * D4; e += blockDim.x) {
        const int t = e % QT, c = (e / QT) * 4;
        const int64_t qq = q0 + t;
        float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        if (qq < nq) {
            if ((d & 3) == 0) {
                if (c < d) {
                    const float4 f = __ldg(reinterpret_cast<const float4*>(x + qq * d + c));
                    v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
                }
            } else {
#pragma unroll
                for (int k = 0; k < 4; ++k)
                    if (c + k < d) v[k] = x[qq * d + c + k];
            }
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) xs[(c + k) * LD + t] = v[k];
    }
    __syncthreads();
    const int half = threadIdx.x >> 4, j = threadIdx.x & 15;
    const unsigned hmask = 0xFFFFu << (threadIdx.x & 16);
    const int rbase = blockIdx.x * (16 * R) + half * R;
    if (rbase >= D) return;  // D % 64 == 0 and R divides 64: all R rows exist
    const float4* p0 = reinterpret_cast<const float4*>(Pc + (int64_t)rbase * D) + j;
    const int D4r = D / 4;  // float4 per row
    float acc[R][QT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < QT; ++t) acc[r][t] = 0.0f;
    for (int tb = 0; tb < D / 64; ++tb) {
        float4 p4[R];
#pragma unroll
        for (int r = 0; r < R; ++r) p4[r] = __ldg(p0 + (int64_t)r * D4r + tb * 16);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float4* xv = reinterpret_cast<const float4*>(xs + (64 * tb + 16 * k + j) * LD);
#pragma unroll
            for (int t4 = 0; t4 < QT / 4; ++t4) {
                const float4 v = xv[t4];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    const float p = k == 0 ? p4[r].x : k == 1 ? p4[r].y : k == 2 ? p4[r].z : p4[r].w;
                    acc[r][4 * t4 + 0] = __fmaf_rn(p, v.x, acc[r][4 * t4 + 0]);
                    acc[r][4 * t4 + 1] = __fmaf_rn(p, v.y, acc[r][4 * t4 + 1]);
                    acc[r][4 * t4 + 2] = __fmaf_rn(p, v.z, acc[r][4 * t4 + 2]);
                    acc[r][4 * t4 + 3] = __fmaf_rn(p, v.w, acc[r][4 * t4 + 3]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < QT; ++t) {
            float v = acc[r][t];
            v = __fadd_rn(v, __shfl_down_sync(hmask, v, 8, 16));
            v = __fadd_rn(v, __shfl_down_sync(hmask, v, 4, 16));
            v = __fadd_rn(v, __shfl_down_sync(hmask, v, 2, 16));
            v = __fadd_rn(v, __shfl_down_sync(hmask, v, 1, 16));
            acc[r][t] = v;
        }
    if (j == 0) {
#pragma unroll
        for (int t = 0; t < QT; ++t)
            if (q0 + t < nq)
#pragma unroll
                for (int r4 = 0; r4 < R; r4 += 4)
                    *reinterpret_cast<float4*>(out + (q0 + t) * D + rbase + r4) =
                        make_float4(acc[r4][t], acc[r4 + 1][t], acc[r4 + 2][t], acc[r4 + 3][t]);
    }
}

// rotate_kernel for large D: the same chains and tree, with the query tile staged a chunk
// of CW columns at a time ([CW][QT+4] floats, so any D fits in two CTAs per SM).  A
// half-warp owns R consecutive rows; the loads of P's next 64-column block are issued
// before the FMAs of this one, so the L2 round trip hides under them.  Each chain still
// adds its terms in column order: q_rot is bit-identical to rotate_kernel's.
template <int QT, int R>
__global__ void __launch_bounds__(256, 2) rotate_chunked_kernel(const float* __restrict__ x, int64_t nq,
                                                        int d, int D, int CW,
                                                        const float* __restrict__ Pc,
                                                        float* __restrict__ out) {
    constexpr int LD = QT + 4;
    extern __shared__ __align__(16) float xs[];  // [CW][LD]
    const int64_t q0 = (int64_t)blockIdx.y * QT;
    const int half = threadIdx.x >> 4, j = threadIdx.x & 15;
    const unsigned hmask = 0xFFFFu << (threadIdx.x & 16);
    const int rbase = blockIdx.x * (16 * R) + half * R;
    const bool active = rbase < D;  // D % 64 == 0 and R divides 64: all R rows exist
    const float4* p0 = reinterpret_cast<const float4*>(Pc + (int64_t)(active ? rbase : 0) * D) + j;
    const int D4r = D / 4;  // float4 per row
    float acc[R][QT];
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < QT; ++t) acc[r][t] = 0.0f;
    for (int c0 = 0; c0 < D; c0 += CW) {
        const int cw = min(CW, D - c0);
        if (c0 > 0) __syncthreads();  // every lane is done with the previous chunk
        // fill: each thread moves 4 consecutive dims of one query (16-byte loads when
        // d % 4 == 0); consecutive threads take consecutive queries so the transposed
        // stores hit consecutive banks
        const int cw4 = cw / 4;
#pragma unroll 4
        for (int e = threadIdx.x; e < QT * cw4; e += blockDim.x) {
            const int t = e % QT, cl = (e / QT) * 4, c = c0 + cl;
            const int64_t qq = q0 + t;
            float v[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (qq < nq) {
                if ((d & 3) == 0) {
                    if (c < d) {
                        const float4 f = __ldg(reinterpret_cast<const float4*>(x + qq * d + c));
                        v[0] = f.x; v[1] = f.y; v[2] = f.z; v[3] = f.w;
                    }
                } else {
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (c + k < d) v[k] = x[qq * d + c + k];
                }
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) xs[(cl + k) * LD + t] = v[k];
        }
        __syncthreads();
        if (!active) continue;
        const int tb0 = c0 / 64, ntb = cw / 64;
        float4 p4[R], pn[R];
#pragma unroll
        for (int r = 0; r < R; ++r) p4[r] = __ldg(p0 + (int64_t)r * D4r + tb0 * 16);
        for (int u = 0; u < ntb; ++u) {
            if (u + 1 < ntb) {
#pragma unroll
                for (int r = 0; r < R; ++r) pn[r] = __ldg(p0 + (int64_t)r * D4r + (tb0 + u + 1) * 16);
            }
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4* xv = reinterpret_cast<const float4*>(xs + (64 * u + 16 * k + j) * LD);
#pragma unroll
                for (int t4 = 0; t4 < QT / 4; ++t4) {
                    const float4 v = xv[t4];
#pragma unroll
                    for (int r = 0; r < R; ++r) {
                        const float p = k == 0 ? p4[r].x : k == 1 ? p4[r].y : k == 2 ? p4[r].z : p4[r].w;
                        acc[r][4 * t4 + 0] = __fmaf_rn(p, v.x, acc[r][4 * t4 + 0]);
                        acc[r][4 * t4 + 1] = __fmaf_rn(p, v.y, acc[r][4 * t4 + 1]);
                        acc[r][4 * t4 + 2] = __fmaf_rn(p, v.z, acc[r][4 * t4 + 2]);
                        acc[r][4 * t4 + 3] = __fmaf_rn(p, v.w, acc[r][4 * t4 + 3]);
                    }
                }
            }
            if (u + 1 < ntb) {
#pragma unroll
                for (int r = 0; r < R; ++r) p4[r] = pn[r];
            }
        }
    }
    if (!active) return;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
        for (int t = 0; t < QT; ++t) {
            float v = acc[r][t];
            v = __fadd_rn(v, __shfl_down_sync(hmask, v, 8, 16));
            v = __fadd_rn(v, __shfl_down_sync(hmask, v, 4, 16));
            v = __fadd_rn(v, __shfl_down_sync(hmask, v, 2, 16));
            v = __fadd_rn(v, __shfl_down_sync(hmask, v, 1, 16));
            acc[r][t] = v;
        }
    if (j == 0) {
#pragma unroll
        for (int t = 0; t < QT; ++t)
            if (q0 + t < nq)
#pragma unroll
                for (int r4 = 0; r4 < R; r4 += 4)
                    *reinterpret_cast<float4*>(out + (q0 + t) * D + rbase + r4) =
                        make_float4(acc[r4][t], acc[r4 + 1][t], acc[r4 + 2][t], acc[r4 + 3][t]);
    }
}

__device__ __forceinline__ float lut_entry(const float* q4, int nib) {
    float v = 0.0f;
#pragma unroll
    for (int b = 0; b < 4; ++b) v = __fadd_rn(v, ((nib >> b) & 1) ? q4[b] : -q4[b]);
    return v;
}

// One warp per query.
__global__ void __launch_bounds__(128) query_state_kernel(
    const float* __restrict__ x, const float* __restrict__ q_rot, int64_t nq, int d, int D,
    const float* __restrict__ rc, int nbits, QueryParams* __restrict__ qp,
    uint8_t* __restrict__ q_i8p, int8_t* __restrict__ q_i8n, uint8_t* __restrict__ lut) {
    // shared: rc[D], then per warp q_rot[D] and x[d]
    extern __shared__ __align__(16) float qsh[];
    const int w = threadIdx.x >> 5, lane = (int)lane_id();
    float* rc_s = qsh;
    float* r = qsh + D + w * (D + d);
    float* xq = r + D;
    for (int i = threadIdx.x; i < D; i += blockDim.x) rc_s[i] = rc[i];
    const int64_t qi = (int64_t)blockIdx.x * 4 + w;
    const bool valid = qi < nq;
    if (valid) {
        for (int i = lane; i < D; i += 32) r[i] = q_rot[qi * D + i];
        for (int i = lane; i < d; i += 32) xq[i] = x[qi * d + i];
    }
    __syncthreads();
    if (!valid) return;
    // sequential sums (Rust Sum<f32> starts from -0.0), from shared memory, side by side
    // in one loop on lanes 1-3 (no divergent serial passes): lane 1 sum(r * rc), lane 2
    // sum(x * x), lane 3 sum(r), its terms as r * 1.0 (exact)
    float ch = -0.0f;
    if (lane >= 1 && lane <= 3) {
        const float* a = lane == 2 ? xq : r;
        const float* b = lane == 2 ? xq : rc_s;
        const int n = lane == 2 ? d : D;
#pragma unroll 8
        for (int i = 0; i < n; ++i) {
            const float bv = lane == 3 ? 1.0f : b[i];
            ch = __fadd_rn(ch, __fmul_rn(a[i], bv));
        }
    }
    const float cs = __shfl_sync(0xffffffffu, ch, 1);
    const float qn = __shfl_sync(0xffffffffu, ch, 2);
    const float qsum = __shfl_sync(0xffffffffu, ch, 3);
    float m = 0.0f;
    for (int i = lane; i < D; i += 32) m = fmaxf(m, fabsf(r[i]));
    m = fmaxf(warp_max(m), 1e-6f);
    const float q_scale = __fdiv_rn(m, 127.0f);
    int s = 0;
    for (int i = lane; i < D; i += 32) {
        const int v = round_clamp(__fdiv_rn(r[i], q_scale), -127.0f, 127.0f);
        s += v;
        q_i8n[qi * D + i] = (int8_t)v;
        // dp4a layout: 4-bit codes unpack to (even dims, odd dims) per 8 dims.
        int pos = i;
        if (nbits == 4) {
            const int g8 = i >> 3, o = i & 7;
            pos = g8 * 8 + ((o & 1) ? 4 : 0) + (o >> 1);
        }
        q_i8p[qi * D + pos] = (uint8_t)(int8_t)v;
    }
    s = warp_sum(s);
    // FastScan LUT
    const int G = D / 4;
    float lm = 0.0f;
    for (int g = lane; g < G; g += 32) {
        const float* q4 = r + 4 * g;
        for (int nib = 0; nib < 16; ++nib) lm = fmaxf(lm, fabsf(lut_entry(q4, nib)));
    }
    lm = fmaxf(warp_max(lm), 1e-6f);
    const float lut_scale = fmaxf(__fdiv_rn(lm, 127.0f), 1e-6f);
    for (int g = lane; g < G; g += 32) {
        const float* q4 = r + 4 * g;
        uint32_t wv[4] = {0, 0, 0, 0};
        for (int nib = 0; nib < 16; ++nib) {
            const int v = round_clamp(__fdiv_rn(lut_entry(q4, nib), lut_scale), -127.0f, 127.0f);
            wv[nib >> 2] |= (uint32_t)(v + 128) << (8 * (nib & 3));  // offset binary
        }
        *reinterpret_cast<uint4*>(lut + qi * (int64_t)G * 16 + g * 16) =
            make_uint4(wv[0], wv[1], wv[2], wv[3]);
    }
    if (lane == 0) {
        QueryParams p;
        p.q_scale = q_scale;
        p.centroid_score = cs;
        p.q_norm_sq = qn;
        p.lut_scale = lut_scale;
        p.q_i8_sum = s;
        p.q_sum = qsum;
        p.pad[0] = p.pad[1] = 0;
        qp[qi] = p;
    }
}

// ============================================================================
// Group (query, probe) pairs by list
// ============================================================================
__global__ void count_lists_kernel(const int32_t* __restrict__ probes, int64_t n_pairs, int nlist,
                                   const uint8_t* __restrict__ owned, int* __restrict__ cnt) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_pairs;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int l = probes[i];
        if (l < 0 || l >= nlist) continue;
        if (!owned || owned[l]) atomicAdd(&cnt[l], 1);
    }
}

// Queries per item of list l: tensor-core items for lists of at most tc_max_rows rows,
// SIMT items of qpi queries otherwise.
__device__ __forceinline__ int list_item_queries(const int64_t* list_off, int l, int tc_max_rows,
                                                 int n_cand, int qpi, int* kind) {
    const int64_t n = list_off[l + 1] - list_off[l];
    if (tc_max_rows > 0 && n <= tc_max_rows) {
        *kind = 1;
        return tc_queries_per_item(n, n > n_cand);
    }
    *kind = 0;
    return qpi;
}

// Single CTA of 1024 threads: exclusive scans of cnt and of items-per-list, over the lists
// in `order` (null: list order).
__global__ void __launch_bounds__(1024) prefix_lists_kernel(const int* __restrict__ cnt, int nlist,
                                                          const int* __restrict__ order,
                                                          const int64_t* __restrict__ list_off,
                                                          int tc_max_rows, int n_cand, int qpi,
                                                          int* __restrict__ lq_off,
                                                          int* __restrict__ item_off,
                                                          int* __restrict__ n_items) {
    __shared__ int wsum_a[32], wsum_b[32];
    __shared__ int carry_a, carry_b;
    const int lane = (int)lane_id(), w = threadIdx.x >> 5;
    if (threadIdx.x == 0) carry_a = carry_b = 0;
    __syncthreads();
    for (int base = 0; base < nlist; base += 1024) {
        const int i = base + threadIdx.x;
        const int l = i < nlist ? (order ? order[i] : i) : nlist;
        const int a = l < nlist ? cnt[l] : 0;
        int kind = 0;
        const int per = l < nlist ? list_item_queries(list_off, l, tc_max_rows, n_cand, qpi, &kind) : 1;
        const int b = (a + per - 1) / per;
        const int ia = warp_inclusive_scan(a), ib = warp_inclusive_scan(b);
        if (lane == 31) {
            wsum_a[w] = ia;
            wsum_b[w] = ib;
        }
        __syncthreads();
        if (w == 0) {
            const int xa = warp_inclusive_scan(wsum_a[lane]);
            const int xb = warp_inclusive_scan(wsum_b[lane]);
            wsum_a[lane] = xa;
            wsum_b[lane] = xb;
        }
        __syncthreads();
        const int pa = (w ? wsum_a[w - 1] : 0) + ia - a + carry_a;
        const int pb = (w ? wsum_b[w - 1] : 0) + ib - b + carry_b;
        if (l < nlist) {
            lq_off[l] = pa;
            item_off[l] = pb;
        }
        __syncthreads();
        if (threadIdx.x == 1023) {
            carry_a = pa + a;
            carry_b = pb + b;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        lq_off[nlist] = carry_a;
        item_off[nlist] = carry_b;
        *n_items = carry_b;
    }
}

__global__ void scatter_pairs_kernel(const int32_t* __restrict__ probes, int64_t nq, int nprobe,
                                     int nlist, const uint8_t* __restrict__ owned,
                                     const int* __restrict__ lq_off, int* __restrict__ cursor,
                                     int2* __restrict__ lq) {
    const int64_t n_pairs = nq * nprobe;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_pairs;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int l = probes[i];
        if (l < 0 || l >= nlist) continue;
        if (owned && !owned[l]) continue;
        const int pos = lq_off[l] + atomicAdd(&cursor[l], 1);
        lq[pos] = make_int2((int)(i / nprobe), (int)(i % nprobe));
    }
}

__global__ void make_items_kernel(const int* __restrict__ cnt, const int* __restrict__ lq_off,
                                  const int* __restrict__ item_off, int nlist,
                                  const int64_t* __restrict__ list_off, int tc_max_rows, int n_cand,
                                  int qpi, int4* __restrict__ items) {
    for (int l = blockIdx.x * blockDim.x + threadIdx.x; l < nlist; l += gridDim.x * blockDim.x) {
        const int c = cnt[l];
        int kind = 0;
        const int per = list_item_queries(list_off, l, tc_max_rows, n_cand, qpi, &kind);
        int o = item_off[l];
        for (int s = 0; s < c; s += per) items[o++] = make_int4(l, lq_off[l] + s, min(per, c - s), kind);
    }
}

// Candidate region of each (query, probe) pair: min(|list|, n_cand) entries (0 for lists
// this index does not own), laid out in probe order.
__global__ void pair_offsets_kernel(const int32_t* __restrict__ probes, int64_t nq, int nprobe,
                                    const int64_t* __restrict__ list_off, int nlist,
                                    const uint8_t* __restrict__ owned, int n_cand,
                                    int* __restrict__ pair_off, int tc_rows, int* __restrict__ fs_off,
                                    PairTrunc tr) {
    const int lane = (int)lane_id();
    const int64_t q = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (q >= nq) return;
    // the query's FastScan pairs on fs_select's register path (no fused filter, |list| <=
    // kFsRegRows) keep only their top fs_keep entries
    bool trunc = tr.fs_keep > 0 && fs_off;
    if (trunc && tr.fused && tr.bitsets) {
        const int b = tr.query_bitset ? tr.query_bitset[q] : 0;
        if (b >= 0 && b < tr.n_bitsets) trunc = false;
    }
    int carry = 0, fs_carry = 0;
    for (int r0 = 0; r0 < nprobe; r0 += 32) {
        const int r = r0 + lane;
        int cap = 0, fs_n = 0;
        if (r < nprobe) {
            const int l = probes[q * nprobe + r];
            if (l >= 0 && l < nlist && (!owned || owned[l])) {
                const int64_t n = list_off[l + 1] - list_off[l];
                cap = (int)min(n, (int64_t)n_cand);
                // a tensor-core FastScan pair: |list| entries, padded to 8 (16-byte regions)
                if (n > n_cand && n <= tc_rows) {
                    fs_n = (int)((n + 7) & ~7ll);
                    if (trunc && n <= kFsRegRows) cap = min(cap, tr.fs_keep);
                }
            }
        }
        const int inc = warp_inclusive_scan(cap);
        if (r < nprobe) pair_off[q * (nprobe + 1) + r] = carry + inc - cap;
        carry += __shfl_sync(0xffffffffu, inc, 31);
        if (fs_off) {
            const int finc = warp_inclusive_scan(fs_n);
            if (r < nprobe) fs_off[q * nprobe + r] = fs_n > 0 ? fs_carry + finc - fs_n : -1;
            fs_carry += __shfl_sync(0xffffffffu, finc, 31);
        }
    }
    if (lane == 0) pair_off[q * (nprobe + 1) + nprobe] = carry;
}

// ============================================================================
// List scan: FastScan + exact kept set + integer rerank.  Every kept candidate of a
// (query, probe) pair is written with its distance key to the query's candidate
// region; the top-k is taken once per query over all probes by the merge.
// ============================================================================
constexpr int kScanThreads = 256;
constexpr int kScanWarps = kScanThreads / 32;  // queries handled concurrently

constexpr int kScanMaxQ = 32;  // queries per item (the grouping step's limit)
constexpr int kSvMax = 384;    // kept rows per (query, list) held in shared memory

struct ScanSmem {
    uint32_t hist[kScanWarps][256];
    // the item's queries: scalars, candidate region of the (query, probe) pair, query id,
    // probe rank, bitset row (-1: none)
    QueryParams qp[kScanMaxQ];
    int64_t qbase[kScanMaxQ];
    int q[kScanMaxQ], rank[kScanMaxQ], bsi[kScanMaxQ];
    uint16_t sv[kScanWarps][kSvMax];  // kept rows of each warp's (query, list) pair (lists < 64 Ki rows)
    int nc[kScanWarps];               // kept candidates of each warp's pair
    int item;
    int pad[3];  // keeps the dynamic arrays after it 16-byte aligned
};

// ============================================================================
// Top-k of a set of candidate entries (one warp): the k smallest by (distance key, tie)
// among entries whose tie is not ~0, written unsorted to sk/st; returns how many.
// ============================================================================
__device__ int warp_select_topk(const uint32_t* keys, const uint64_t* ties, int total, int k,
                                uint32_t* sk, uint64_t* st, uint32_t* hist) {
    // Unused entries carry key 0xFFFFFFFF and tie ~0 (the scans' fill and compact padding):
    // tau is found on the keys alone (four loads of a lane in flight); ties are read for the
    // entries taken and for those at tau (at tau = 0xFFFFFFFF only valid ties are taken).
    const int lane = (int)lane_id();
    int n_lt = 0;
    for (int b = lane; b < total; b += 128) {
        uint32_t t[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) t[j] = b + 32 * j < total ? keys[b + 32 * j] : 0xFFFFFFFFu;
#pragma unroll
        for (int j = 0; j < 4; ++j) n_lt += t[j] != 0xFFFFFFFFu ? 1 : 0;
    }
    n_lt = warp_sum(n_lt);
    uint32_t tau = 0xFFFFFFFFu;
    if (n_lt >= k) {
        auto key_at = [&](int e, uint32_t& kk) {
            kk = keys[e];
            return kk != 0xFFFFFFFFu;
        };
        int less = 0;
        tau = warp_radix_kth(total, k, key_at, hist, &less);
    }
    int written = 0;
    for (int base = 0; base < total; base += 32) {
        const int e = base + lane;
        const uint32_t kk = e < total ? keys[e] : 0xFFFFFFFFu;
        const bool lt = kk < tau;
        const unsigned bl = __ballot_sync(0xffffffffu, lt);
        if (lt) {
            const int pos = written + __popc(bl & lanemask_lt());
            sk[pos] = kk;
            st[pos] = ties[e];
        }
        written += __popc(bl);
    }
    // entries at tau with a valid tie, in increasing (probe rank, fastscan key, index) order
    uint64_t floor_t = 0;
    bool have_floor = false;
    while (written < k) {
        uint64_t best = ~0ull;
        for (int e = lane; e < total; e += 32) {
            if (keys[e] != tau) continue;
            const uint64_t t = ties[e];
            if (t != ~0ull && (!have_floor || t > floor_t) && t < best) best = t;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t ob = __shfl_xor_sync(0xffffffffu, best, o);
            best = ob < best ? ob : best;
        }
        if (best == ~0ull) break;  // no further valid entry
        if (lane == 0) {
            sk[written] = tau;
            st[written] = best;
        }
        floor_t = best;
        have_floor = true;
        ++written;
    }
    __syncwarp();
    return written;
}

__device__ __forceinline__ int32_t wrap16(int32_t v) { return (int32_t)(int16_t)v; }

// Integer dot of one stored vector with one quantised query (dp4a layout), by the 8
// lanes of a group (lane bits 0-2 = sub); every lane of the warp must call it.  The
// sum is exact, so the split into lanes does not change it.  Groups with active ==
// false contribute nothing and read nothing.
__device__ __forceinline__ int int_ip_group8(const uint8_t* __restrict__ code,
                                             const uint8_t* q, int D, int nbits,
                                             int sub, bool active) {
    int acc0 = 0, acc1 = 0;
    if (active) {
        const uint4* c4 = reinterpret_cast<const uint4*>(code);
        const uint4* q4 = reinterpret_cast<const uint4*>(q);
        if (nbits == 8) {
#pragma unroll 2
            for (int i = sub; i < D / 16; i += 8) {
                const uint4 c = __ldg(c4 + i);
                const uint4 qv = q4[i];  // q: shared or global memory
                acc0 = dp4a_us(c.x, qv.x, acc0);
                acc1 = dp4a_us(c.y, qv.y, acc1);
                acc0 = dp4a_us(c.z, qv.z, acc0);
                acc1 = dp4a_us(c.w, qv.w, acc1);
            }
        } else {  // nbits == 4: 16 code bytes = 32 dims; q layout (even, odd) per 8 dims
#pragma unroll 2
            for (int i = sub; i < D / 32; i += 8) {
                const uint4 c = __ldg(c4 + i);
                const uint4 qa = q4[2 * i], qb = q4[2 * i + 1];
                acc0 = dp4a_us(c.x & 0x0F0F0F0Fu, qa.x, acc0);
                acc1 = dp4a_us(c.x & 0xF0F0F0F0u, qa.y, acc1);
                acc0 = dp4a_us(c.y & 0x0F0F0F0Fu, qa.z, acc0);
                acc1 = dp4a_us(c.y & 0xF0F0F0F0u, qa.w, acc1);
                acc0 = dp4a_us(c.z & 0x0F0F0F0Fu, qb.x, acc0);
                acc1 = dp4a_us(c.z & 0xF0F0F0F0u, qb.y, acc1);
                acc0 = dp4a_us(c.w & 0x0F0F0F0Fu, qb.z, acc0);
                acc1 = dp4a_us(c.w & 0xF0F0F0F0u, qb.w, acc1);
            }
        }
    }
    // 4-bit: acc1 summed the high nibbles in place (16 x their value), an exact multiple of 16
    int acc = acc0 + (nbits == 8 ? acc1 : acc1 >> 4);
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    return acc;
}


// int_ip_group8 with every code load of the lane issued before the first dot product (one
// memory round trip per row); nu_max = NU * 8 code uint4 per row at most.  q is read in
// the dot loop (shared memory or L1-resident rows).
template <int NU>
__device__ __forceinline__ int int_ip_group8_pf(const uint8_t* __restrict__ code, const uint8_t* q,
                                                int D, int nbits, int sub, bool active) {
    int acc0 = 0, acc1 = 0;
    if (active) {
        const uint4* c4 = reinterpret_cast<const uint4*>(code);
        const uint4* q4 = reinterpret_cast<const uint4*>(q);
        const int nu = nbits == 8 ? D / 16 : D / 32;
        uint4 c[NU];
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            const int i = sub + 8 * u;
            c[u] = i < nu ? __ldg(c4 + i) : make_uint4(0u, 0u, 0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < NU; ++u) {
            const int i = sub + 8 * u;
            if (i >= nu) break;
            if (nbits == 8) {
                const uint4 qv = q4[i];
                acc0 = dp4a_us(c[u].x, qv.x, acc0);
                acc1 = dp4a_us(c[u].y, qv.y, acc1);
                acc0 = dp4a_us(c[u].z, qv.z, acc0);
                acc1 = dp4a_us(c[u].w, qv.w, acc1);
            } else {
                const uint4 qa = q4[2 * i], qb = q4[2 * i + 1];
                acc0 = dp4a_us(c[u].x & 0x0F0F0F0Fu, qa.x, acc0);
                acc1 = dp4a_us(c[u].x & 0xF0F0F0F0u, qa.y, acc1);
                acc0 = dp4a_us(c[u].y & 0x0F0F0F0Fu, qa.z, acc0);
                acc1 = dp4a_us(c[u].y & 0xF0F0F0F0u, qa.w, acc1);
                acc0 = dp4a_us(c[u].z & 0x0F0F0F0Fu, qb.x, acc0);
                acc1 = dp4a_us(c[u].z & 0xF0F0F0F0u, qb.y, acc1);
                acc0 = dp4a_us(c[u].w & 0x0F0F0F0Fu, qb.z, acc0);
                acc1 = dp4a_us(c[u].w & 0xF0F0F0F0u, qb.w, acc1);
            }
        }
    }
    // 4-bit: acc1 summed the high nibbles in place (16 x their value), an exact multiple of 16
    int acc = acc0 + (nbits == 8 ? acc1 : acc1 >> 4);
    acc += __shfl_xor_sync(0xffffffffu, acc, 4);
    acc += __shfl_xor_sync(0xffffffffu, acc, 2);
    acc += __shfl_xor_sync(0xffffffffu, acc, 1);
    return acc;
}

// Two rows at once (their code loads all issued before either dot product).
template <int NU>
__device__ __forceinline__ int2 int_ip_group8_pf2(const uint8_t* __restrict__ code_a, const uint8_t* qa_,
                                                  bool act_a, const uint8_t* __restrict__ code_b,
                                                  const uint8_t* qb_, bool act_b, int D, int nbits,
                                                  int sub) {
    const int nu = nbits == 8 ? D / 16 : D / 32;
    uint4 ca[NU], cb[NU];
#pragma unroll
    for (int u = 0; u < NU; ++u) {
        const int i = sub + 8 * u;
        ca[u] = act_a && i < nu ? __ldg(reinterpret_cast<const uint4*>(code_a) + i) : make_uint4(0u, 0u, 0u, 0u);
        cb[u] = act_b && i < nu ? __ldg(reinterpret_cast<const uint4*>(code_b) + i) : make_uint4(0u, 0u, 0u, 0u);
    }
    auto dot = [&](const uint4 (&c)[NU], const uint8_t* q, bool act) {
        int acc0 = 0, acc1 = 0;
        if (act) {
            const uint4* q4 = reinterpret_cast<const uint4*>(q);
#pragma unroll
            for (int u = 0; u < NU; ++u) {
                const int i = sub + 8 * u;
                if (i >= nu) break;
                if (nbits == 8) {
                    const uint4 qv = q4[i];
                    acc0 = dp4a_us(c[u].x, qv.x, acc0);
                    acc1 = dp4a_us(c[u].y, qv.y, acc1);
                    acc0 = dp4a_us(c[u].z, qv.z, acc0);
                    acc1 = dp4a_us(c[u].w, qv.w, acc1);
                } else {
                    const uint4 q0 = q4[2 * i], q1 = q4[2 * i + 1];
                    acc0 = dp4a_us(c[u].x & 0x0F0F0F0Fu, q0.x, acc0);
                    acc1 = dp4a_us(c[u].x & 0xF0F0F0F0u, q0.y, acc1);
                    acc0 = dp4a_us(c[u].y & 0x0F0F0F0Fu, q0.z, acc0);
                    acc1 = dp4a_us(c[u].y & 0xF0F0F0F0u, q0.w, acc1);
                    acc0 = dp4a_us(c[u].z & 0x0F0F0F0Fu, q1.x, acc0);
                    acc1 = dp4a_us(c[u].z & 0xF0F0F0F0u, q1.y, acc1);
                    acc0 = dp4a_us(c[u].w & 0x0F0F0F0Fu, q1.z, acc0);
                    acc1 = dp4a_us(c[u].w & 0xF0F0F0F0u, q1.w, acc1);
                }
            }
        }
        return acc0 + (nbits == 8 ? acc1 : acc1 >> 4);  // 4-bit: high nibbles in place
    };
    int x = dot(ca, qa_, act_a), y = dot(cb, qb_, act_b);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {
        x += __shfl_xor_sync(0xffffffffu, x, o);
        y += __shfl_xor_sync(0xffffffffu, y, o);
    }
    return make_int2(x, y);
}

constexpr int kPfUnits = 3;  // rows of up to 24 code uint4 (4-bit D <= 768, 8-bit D <= 384)

__global__ void __launch_bounds__(kScanThreads, 4) scan_lists_kernel(ScanArgs a) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    ScanSmem& sm = *reinterpret_cast<ScanSmem*>(smem_raw);
    // FastScan LUT of the current 8 queries: word pair (g*16 + nib) = (queries 0-3, 4-7),
    // one offset-binary byte per query
    // (128-byte aligned, so a LUT row base OR a nibble's byte offset is its address)
    const uint32_t smem_base = (uint32_t)__cvta_generic_to_shared(smem_raw);
    const uint32_t lut_pad = (128u - ((smem_base + (uint32_t)sizeof(ScanSmem)) & 127u)) & 127u;
    uint2* lut8 = reinterpret_cast<uint2*>(smem_raw + sizeof(ScanSmem) + lut_pad);  // [G*16]
    const uint32_t lut8_s = smem_base + (uint32_t)sizeof(ScanSmem) + lut_pad;
    const bool use_sv = a.n_cand <= kSvMax && a.max_len <= 65536;
    // q_i8 (dp4a layout) of the current FastScan query group, rows padded by 16 bytes
    uint8_t* qsm = reinterpret_cast<uint8_t*>(lut8 + a.G * 16);  // [kScanWarps][D + 16]
    const int qld = a.D + 16;
    const int tid = threadIdx.x, w = tid >> 5, lane = (int)lane_id();
    const int grp = lane >> 3, sub = lane & 7;  // 4 groups of 8 lanes per warp
    const bool pf = (a.nbits == 8 ? a.D / 16 : a.D / 32) <= 8 * kPfUnits;
    int16_t* my_scores_base = a.scores + (int64_t)blockIdx.x * kScanWarps * a.max_len;
    const bool l2 = a.metric_l2 != 0;
    const int pstride = a.nprobe + 1;

    for (;;) {
        if (tid == 0) sm.item = atomicAdd(a.item_counter, 1);
        __syncthreads();
        const int item = sm.item;
        __syncthreads();
        if (item >= *a.n_items) break;
        const int4 it = a.items[item];
        const int l = it.x;
        const int64_t beg = a.list_off[l];
        const int n = (int)(a.list_off[l + 1] - beg);
        if (it.w != 0) continue;  // a tensor-core item (scan_tc_kernel)
        // the item's queries, staged once (no dependent global loads in the rerank loops)
        if (tid < it.z) {
            const int2 pr = a.lq[it.y + tid];
            sm.q[tid] = pr.x;
            sm.rank[tid] = pr.y;
            sm.qbase[tid] = (int64_t)pr.x * a.q_stride + a.pair_off[(int64_t)pr.x * pstride + pr.y];
            sm.qp[tid] = a.qp[pr.x];
            int b = -1;
            if (a.fused && a.bitsets) {
                b = a.query_bitset ? a.query_bitset[pr.x] : 0;
                if (b < 0 || b >= a.n_bitsets) b = -1;
            }
            sm.bsi[tid] = b;
        }
        __syncthreads();
        if (n <= a.n_cand) {
            // no FastScan: every live row is a candidate of every query of the item; blocks
            // of 8 rows of one query spread over the warps (groups of 8 lanes take rows
            // j0 + grp and j0 + 4 + grp), then lanes 0-7 finish the 8 rows in parallel
            const int nbq = (n + 7) >> 3;  // row blocks per query
            const int total = it.z * nbq;
            for (int blk = w; blk < total; blk += kScanWarps) {
                const int i = blk / nbq;
                const int j0 = (blk - i * nbq) * 8;
                const int ja = j0 + grp, jb = j0 + 4 + grp;
                const uint8_t* qrow = a.q_i8p + (int64_t)sm.q[i] * a.D;
                const uint8_t* ca = a.codes + (beg + min(ja, n - 1)) * a.code_bytes;
                const uint8_t* cb = a.codes + (beg + min(jb, n - 1)) * a.code_bytes;
                int2 ip;
                if (pf) {
                    ip = int_ip_group8_pf2<kPfUnits>(ca, qrow, ja < n, cb, qrow, jb < n, a.D, a.nbits, sub);
                } else {
                    ip.x = int_ip_group8(ca, qrow, a.D, a.nbits, sub, ja < n);
                    ip.y = int_ip_group8(cb, qrow, a.D, a.nbits, sub, jb < n);
                }
                const int src = (lane & 3) * 8;
                const int ipx = __shfl_sync(0xffffffffu, ip.x, src);
                const int ipy = __shfl_sync(0xffffffffu, ip.y, src);
                const int v = j0 + lane;
                if (lane < 8 && v < n) {
                    const int64_t row = beg + v;
                    const int b = sm.bsi[i];
                    const bool dead =
                        b >= 0 && bit_filtered(a.bitsets + (int64_t)b * a.bitset_words, a.bitset_len, a.ids[row]);
                    const int64_t dst = sm.qbase[i] + v;
                    if (dead) {
                        a.cand_key[dst] = 0xFFFFFFFFu;
                        a.cand_tie[dst] = ~0ull;
                    } else {
                        const float4 m = __ldg(a.meta + row);
                        const int ipv = lane < 4 ? ipx : ipy;
                        a.cand_key[dst] = total_order_key(rerank_distance(ipv, m, sm.qp[i], a.nbits, l2));
                        a.cand_tie[dst] = ((uint64_t)sm.rank[i] << 48) | (uint32_t)v;
                        if (a.cand_dbg) a.cand_dbg[dst] = make_int2(ipv, INT32_MIN);
                    }
                }
            }
            continue;
        }
        const uint2* fsb = a.fs + a.fs_blk_off[l] * (int64_t)a.nchunks * 32;
        for (int qg = 0; qg < it.z; qg += kScanWarps) {
            const int nq_here = min(kScanWarps, it.z - qg);
            // the group's q_i8 rows into shared memory (read by the rerank, behind the barriers
            // of the FastScan phases; the previous group's rerank ended with a barrier)
            for (int e = tid; e < nq_here * (a.D / 16); e += kScanThreads) {
                const int i = e / (a.D / 16), c = e - i * (a.D / 16);
                *reinterpret_cast<uint4*>(qsm + i * qld + 16 * c) =
                    __ldg(reinterpret_cast<const uint4*>(a.q_i8p + (int64_t)sm.q[qg + i] * a.D) + c);
            }
            {
                // interleave the 8 queries' offset-binary LUTs: word g*16+nib of quad h =
                // q(4h)|q(4h+1)<<8|q(4h+2)<<16|q(4h+3)<<24 (16 LUT bytes of each query per
                // thread, 4x4 byte transposes with PRMT); absent queries read 0x80 (zero)
                for (int m = tid; m < a.G; m += kScanThreads) {
                    uint4 L[8];
#pragma unroll
                    for (int t = 0; t < 8; ++t) {
                        const int qq = qg + t;
                        L[t] = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);
                        if (qq < it.z)
                            L[t] = __ldg(reinterpret_cast<const uint4*>(a.lut + (int64_t)sm.q[qq] * a.G * 16) + m);
                    }
                    uint32_t out[2][16];
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t w0[4] = {L[4 * h].x, L[4 * h].y, L[4 * h].z, L[4 * h].w};
                        const uint32_t w1[4] = {L[4 * h + 1].x, L[4 * h + 1].y, L[4 * h + 1].z, L[4 * h + 1].w};
                        const uint32_t w2[4] = {L[4 * h + 2].x, L[4 * h + 2].y, L[4 * h + 2].z, L[4 * h + 2].w};
                        const uint32_t w3[4] = {L[4 * h + 3].x, L[4 * h + 3].y, L[4 * h + 3].z, L[4 * h + 3].w};
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const uint32_t t0 = __byte_perm(w0[i], w1[i], 0x5140);
                            const uint32_t t1 = __byte_perm(w2[i], w3[i], 0x5140);
                            const uint32_t t2 = __byte_perm(w0[i], w1[i], 0x7362);
                            const uint32_t t3 = __byte_perm(w2[i], w3[i], 0x7362);
                            out[h][4 * i + 0] = __byte_perm(t0, t1, 0x5410);
                            out[h][4 * i + 1] = __byte_perm(t0, t1, 0x7632);
                            out[h][4 * i + 2] = __byte_perm(t2, t3, 0x5410);
                            out[h][4 * i + 3] = __byte_perm(t2, t3, 0x7632);
                        }
                    }
                    uint4* dst = reinterpret_cast<uint4*>(lut8 + m * 16);
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        dst[i] = make_uint4(out[0][2 * i], out[1][2 * i], out[0][2 * i + 1], out[1][2 * i + 1]);
                }
                __syncthreads();
                // FastScan scores of 8 queries per row: one 8-byte LUT load per nibble
                for (int v = tid; v < n; v += kScanThreads) {
                    const int blk = v >> 5, slot = v & 31;
                    const uint2* src = fsb + (int64_t)blk * a.nchunks * 32 + slot;
                    uint32_t a02 = 0, a13 = 0, b02 = 0, b13 = 0;
                    int tot[8] = {0, 0, 0, 0, 0, 0, 0, 0};
                    for (int c0 = 0; c0 < a.nchunks; c0 += 4) {
                        uint2 wds[4];
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            wds[u] = c0 + u < a.nchunks ? __ldg(src + (c0 + u) * 32) : make_uint2(0u, 0u);
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int c = c0 + u;
                            if (c >= a.nchunks) break;
                            const uint2 wd = wds[u];
                            const uint32_t lrow_s = lut8_s + (uint32_t)c * 2048u;  // 128-aligned
                            // nibble J: shared address = row base | nibble * 8, plus the entry
                            // block J * 128 as the load's immediate; bytes 0, 2 and bytes 1, 3
                            // of each word go into 16-bit lanes (one PRMT with a zero source)
#define HANNS_FS_NIBBLE(J)                                                                     \
    {                                                                                          \
        const uint32_t word_ = (J) < 8 ? wd.x : wd.y;                                          \
        const int sh_ = 4 * ((J) & 7);                                                         \
        const uint32_t addr_ = ((sh_ == 0 ? word_ << 3 : word_ >> (sh_ - 3)) & 0x78u) | lrow_s; \
        uint32_t ex_, ey_;                                                                     \
        asm volatile("ld.shared.v2.u32 {%0, %1}, [%2+%3];"                                     \
                     : "=r"(ex_), "=r"(ey_)                                                    \
                     : "r"(addr_), "n"((J) * 128));                                            \
        a02 += ex_ & 0x00FF00FFu;                                                              \
        a13 += __byte_perm(ex_, 0u, 0x4341);                                                   \
        b02 += ey_ & 0x00FF00FFu;                                                              \
        b13 += __byte_perm(ey_, 0u, 0x4341);                                                   \
    }
                            HANNS_FS_NIBBLE(0) HANNS_FS_NIBBLE(1) HANNS_FS_NIBBLE(2) HANNS_FS_NIBBLE(3)
                            HANNS_FS_NIBBLE(4) HANNS_FS_NIBBLE(5) HANNS_FS_NIBBLE(6) HANNS_FS_NIBBLE(7)
                            HANNS_FS_NIBBLE(8) HANNS_FS_NIBBLE(9) HANNS_FS_NIBBLE(10) HANNS_FS_NIBBLE(11)
                            HANNS_FS_NIBBLE(12) HANNS_FS_NIBBLE(13) HANNS_FS_NIBBLE(14) HANNS_FS_NIBBLE(15)
#undef HANNS_FS_NIBBLE
                            if ((c & 15) == 15) {
                                tot[0] += (int)(a02 & 0xFFFFu);
                                tot[2] += (int)(a02 >> 16);
                                tot[1] += (int)(a13 & 0xFFFFu);
                                tot[3] += (int)(a13 >> 16);
                                tot[4] += (int)(b02 & 0xFFFFu);
                                tot[6] += (int)(b02 >> 16);
                                tot[5] += (int)(b13 & 0xFFFFu);
                                tot[7] += (int)(b13 >> 16);
                                a02 = a13 = b02 = b13 = 0;
                            }
                        }
                    }
                    tot[0] += (int)(a02 & 0xFFFFu);
                    tot[2] += (int)(a02 >> 16);
                    tot[1] += (int)(a13 & 0xFFFFu);
                    tot[3] += (int)(a13 >> 16);
                    tot[4] += (int)(b02 & 0xFFFFu);
                    tot[6] += (int)(b02 >> 16);
                    tot[5] += (int)(b13 & 0xFFFFu);
                    tot[7] += (int)(b13 >> 16);
                    const int bias = 128 * a.G;
#pragma unroll
                    for (int t = 0; t < 8; ++t)
                        if (t < nq_here)
                            my_scores_base[(int64_t)t * a.max_len + v] = (int16_t)wrap16(tot[t] - bias);
                }
                __syncthreads();
            }
            if (w < nq_here) {
                const int qs_ = qg + w;
                const int rank = sm.rank[qs_];
                const uint64_t* bw = sm.bsi[qs_] >= 0 ? a.bitsets + (int64_t)sm.bsi[qs_] * a.bitset_words : nullptr;
                auto live = [&](int v) {
                    return !bw || !bit_filtered(bw, a.bitset_len, a.ids[beg + v]);
                };
                int n_live = n;
                if (bw) {
                    int c = 0;
                    for (int v = lane; v < n; v += 32) c += live(v) ? 1 : 0;
                    n_live = warp_sum(c);
                }
                const int16_t* sc = my_scores_base + (int64_t)w * a.max_len;
                const int64_t rbase = sm.qbase[qs_];
                uint64_t* my_tie = a.cand_tie + rbase;
                uint16_t* my_sv = use_sv ? sm.sv[w] : nullptr;
                const uint64_t rank_bits = (uint64_t)rank << 48;
                int n_c = 0;  // kept candidates written to my_tie
                if (n_live > a.n_cand) {
                    // s* = n_cand-th largest score among live rows (key = 32767 - score)
                    auto key_at = [&](int v, uint32_t& k) {
                        if (!live(v)) return false;
                        k = (uint32_t)(32767 - (int)sc[v]);
                        return true;
                    };
                    int c_gt = 0, c_eq = 0;
                    const uint32_t tau =
                        warp_radix_kth16(n, a.n_cand, key_at, sm.hist[w], &c_gt, &c_eq);
                    // F = first n_cand rows (in list order) with score >= s*; gt_F = rows > s* in F.
                    // When exactly n_cand rows score >= s*, F is all of them (no pass needed).
                    int cnt_ge = 0, cnt_gt = 0, p_end = n, gt_f = c_gt;
                    for (int base = 0; c_gt + c_eq != a.n_cand && base < n; base += 32) {
                        const int v = base + lane;
                        uint32_t k = 0xFFFFFFFFu;
                        const bool valid = v < n && key_at(v, k);
                        const bool ge = valid && k <= tau, gt = valid && k < tau;
                        const unsigned bge = __ballot_sync(0xffffffffu, ge);
                        const unsigned bgt = __ballot_sync(0xffffffffu, gt);
                        const int c = __popc(bge);
                        if (cnt_ge + c >= a.n_cand) {
                            const int need = a.n_cand - cnt_ge;
                            const bool here = ge && __popc(bge & lanemask_le()) == need;
                            const int pos = __ffs(__ballot_sync(0xffffffffu, here)) - 1;
                            p_end = base + pos;
                            gt_f = cnt_gt + __popc(bgt & (pos == 31 ? 0xffffffffu : ((2u << pos) - 1u)));
                            break;
                        }
                        cnt_ge += c;
                        cnt_gt += __popc(bgt);
                    }
                    const int m_drop = c_gt - gt_f;  // lowest-index ties evicted by later rows
                    int eq_seen = 0;
                    for (int base = 0; base < n; base += 32) {
                        const int v = base + lane;
                        uint32_t k = 0xFFFFFFFFu;
                        const bool valid = v < n && key_at(v, k);
                        const bool gt = valid && k < tau;
                        const bool eq = valid && k == tau && v <= p_end;
                        const unsigned beq = __ballot_sync(0xffffffffu, eq);
                        const int eq_rank = eq_seen + __popc(beq & lanemask_le());
                        const bool keep = gt || (eq && eq_rank > m_drop);
                        const unsigned bk = __ballot_sync(0xffffffffu, keep);
                        if (keep) {
                            const int pos = n_c + __popc(bk & lanemask_lt());
                            if (pos < a.n_cand) {
                                my_tie[pos] = rank_bits | ((uint64_t)k << 32) | (uint32_t)v;
                                if (my_sv) my_sv[pos] = (uint16_t)v;
                                if (a.cand_dbg) a.cand_dbg[rbase + pos].y = 32767 - (int)k;
                            }
                        }
                        n_c += __popc(bk);
                        eq_seen += __popc(beq);
                    }
                } else {
                    for (int base = 0; base < n; base += 32) {
                        const int v = base + lane;
                        const bool keep = v < n && live(v);
                        const unsigned bk = __ballot_sync(0xffffffffu, keep);
                        if (keep) {
                            const int pos = n_c + __popc(bk & lanemask_lt());
                            my_tie[pos] = rank_bits | (uint32_t)v;
                            if (my_sv) my_sv[pos] = (uint16_t)v;
                            if (a.cand_dbg) a.cand_dbg[rbase + pos].y = INT32_MIN;
                        }
                        n_c += __popc(bk);
                    }
                }
                n_c = min(n_c, a.n_cand);  // the kept set has exactly n_cand rows
                // unused entries of the pair's region (rows removed by the filter)
                for (int j = n_c + lane; j < a.n_cand; j += 32) {
                    my_tie[j] = ~0ull;
                    a.cand_key[rbase + j] = 0xFFFFFFFFu;
                }
                if (lane == 0) sm.nc[w] = n_c;
            }
            // a full group reranks warp by warp the query each warp just selected (its own
            // sm.nc / sv / ties): the warp only waits for itself.  This holds because a full
            // group has one warp per query (wpq = kScanWarps / nq_here = 1, so iq == w
            // below); a different warp-to-query mapping needs the block barrier back.
            if (nq_here == kScanWarps)
                __syncwarp();
            else
                __syncthreads();
            // integer rerank of the group's kept candidates, 8 per warp at a time (two per
            // group of 8 lanes, their loads issued together)
            // warps per query: wpq = 8 / nq_here; warp w reranks query w / wpq, candidates
            // j = part*8 + 0..7, part = w % wpq, stepping by wpq*8: groups of 8 lanes take
            // j0 + grp and j0 + 4 + grp (their code loads issued together), then lanes 0-7
            // each finish one of the 8 (distance, key store) in parallel
            const int wpq = kScanWarps / nq_here;  // 1 for a full group: iq == w
            const int iq = w / wpq, part = w - iq * wpq;
            if (iq < nq_here && a.nbits != 4 && a.nbits != 8) {
                // f32 rerank (1-bit chains, or the scalar dequantised sum): a lane per kept
                // candidate; the query's q_rot values are the same address in every lane
                const int nc_i = sm.nc[iq];
                const uint16_t* svi = sm.sv[iq];
                const int64_t rb = sm.qbase[qg + iq];
                const QueryParams& qpi = sm.qp[qg + iq];
                const float* qr = a.q_rot + (int64_t)sm.q[qg + iq] * a.D;
                for (int j0 = part * 32; j0 < nc_i; j0 += wpq * 32) {
                    const int j = j0 + lane;
                    if (j >= nc_i) continue;
                    const uint32_t v = use_sv ? (uint32_t)svi[j] : (uint32_t)a.cand_tie[rb + j];
                    const float4 m = __ldg(a.meta + beg + v);
                    const uint8_t* cr = a.codes + (beg + v) * a.code_bytes;
                    float ip = 0.0f;
                    if (m.w > 1e-12f)
                        ip = a.nbits == 1 ? ip_1bit(cr, qr, a.D, m.z, qpi.q_sum)
                                          : ip_scalar(cr, qr, a.D, a.nbits, m.z, a.code_bytes);
                    a.cand_key[rb + j] = total_order_key(rerank_distance_ip(ip, m, qpi, l2));
                    if (a.cand_dbg) a.cand_dbg[rb + j].x = INT32_MIN;
                }
            } else if (iq < nq_here) {
                const int nc_i = sm.nc[iq];
                const uint8_t* qrow = qsm + iq * qld;
                const uint16_t* svi = sm.sv[iq];
                const int64_t rb = sm.qbase[qg + iq];
                const QueryParams& qpi = sm.qp[qg + iq];
                auto row_of = [&](int j) -> uint32_t {
                    // kept rows: shared memory, or the ties this CTA wrote (coherent load)
                    return use_sv ? (uint32_t)svi[j] : (uint32_t)a.cand_tie[rb + j];
                };
                for (int j0 = part * 8; j0 < nc_i; j0 += wpq * 8) {
                    const int ja = j0 + grp, jb = j0 + 4 + grp;
                    const bool acta = ja < nc_i, actb = jb < nc_i;
                    const uint32_t va = acta ? row_of(ja) : 0u;
                    const uint32_t vb = actb ? row_of(jb) : 0u;
                    const uint8_t* ca = a.codes + (beg + va) * a.code_bytes;
                    const uint8_t* cb = a.codes + (beg + vb) * a.code_bytes;
                    int2 ip;
                    if (pf) {
                        ip = int_ip_group8_pf2<kPfUnits>(ca, qrow, acta, cb, qrow, actb, a.D, a.nbits, sub);
                    } else {
                        ip.x = int_ip_group8(ca, qrow, a.D, a.nbits, sub, acta);
                        ip.y = int_ip_group8(cb, qrow, a.D, a.nbits, sub, actb);
                    }
                    // lane L < 8 finishes candidate j0 + L (group L & 3, slot L >> 2)
                    const int src = (lane & 3) * 8;
                    const int ipx = __shfl_sync(0xffffffffu, ip.x, src);
                    const int ipy = __shfl_sync(0xffffffffu, ip.y, src);
                    const int jl = j0 + lane;
                    if (lane < 8 && jl < nc_i) {
                        const float4 m = __ldg(a.meta + beg + row_of(jl));
                        const int ipv = lane < 4 ? ipx : ipy;
                        a.cand_key[rb + jl] = total_order_key(rerank_distance(ipv, m, qpi, a.nbits, l2));
                        if (a.cand_dbg) a.cand_dbg[rb + jl].x = ipv;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// warp_select_topk for at most 32 * S entries: the keys are read once into registers and
// the radix passes run on them (same result and contract).
template <int S>
__device__ int warp_select_topk_small(const uint32_t* keys, const uint64_t* ties, int total, int k,
                                      uint32_t* sk, uint64_t* st, uint32_t* hist) {
    const int lane = (int)lane_id();
    uint32_t kk[S];
    bool ok[S];
    int cnt = 0;
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
#pragma unroll
    for (int j = 0; j < S; ++j) {
        const int e = lane + 32 * j;
        ok[j] = e < total && ties[e] != ~0ull;
        kk[j] = ok[j] ? keys[e] : 0xFFFFFFFFu;
        if (ok[j]) {
            ++cnt;
            kmin = min(kmin, kk[j]);
            kmax = max(kmax, kk[j]);
        }
    }
    const int n_valid = warp_sum(cnt);
    const int take = min(k, n_valid);
    if (take == 0) return 0;
    uint32_t tau = 0xFFFFFFFFu;
    if (n_valid > k) {
        kmin = warp_min_u32(kmin);
        kmax = warp_max_u32(kmax);
        const uint32_t range = kmax - kmin;
        uint32_t prefix = 0;
        int remaining = k;
        for (int hi = 32 - __clz(range); hi > 0; hi -= 8) {
            const int shift = hi > 8 ? hi - 8 : 0;
#pragma unroll
            for (int b = 0; b < 8; ++b) hist[lane * 8 + b] = 0;
            __syncwarp();
#pragma unroll
            for (int j = 0; j < S; ++j)
                if (ok[j]) {
                    const uint32_t kp = kk[j] - kmin;
                    if (hi >= 32 || ((kp ^ prefix) >> hi) == 0) atomicAdd(&hist[(kp >> shift) & 255u], 1u);
                }
            __syncwarp();
            int sum = 0;
#pragma unroll
            for (int b = 0; b < 8; ++b) sum += (int)hist[lane * 8 + b];
            const int incl = warp_inclusive_scan(sum);
            const unsigned hit = __ballot_sync(0xffffffffu, incl >= remaining);
            const int src = __ffs(hit) - 1;
            int bin = 0, before = 0;
            if (lane == src) {
                int c = incl - sum;
                for (int b = 0; b < 8; ++b) {
                    const int h = (int)hist[lane * 8 + b];
                    if (c + h >= remaining) {
                        bin = lane * 8 + b;
                        break;
                    }
                    c += h;
                }
                before = c;
            }
            bin = __shfl_sync(0xffffffffu, bin, src);
            before = __shfl_sync(0xffffffffu, before, src);
            remaining -= before;
            prefix |= (uint32_t)bin << shift;
            __syncwarp();
        }
        tau = kmin + prefix;
    }
    int written = 0;
#pragma unroll
    for (int j = 0; j < S; ++j) {
        const bool lt = ok[j] && (n_valid <= k || kk[j] < tau);
        const unsigned bl = __ballot_sync(0xffffffffu, lt);
        if (lt) {
            const int pos = written + __popc(bl & lanemask_lt());
            sk[pos] = kk[j];
            st[pos] = ties[lane + 32 * j];
        }
        written += __popc(bl);
    }
    // ties at tau: chosen in increasing (probe rank, fastscan key, index) order
    uint64_t floor_t = 0;
    bool have_floor = false;
    while (written < take) {
        uint64_t best = ~0ull;
#pragma unroll
        for (int j = 0; j < S; ++j)
            if (ok[j] && kk[j] == tau) {
                const uint64_t t = ties[lane + 32 * j];
                if ((!have_floor || t > floor_t) && t < best) best = t;
            }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t ob = __shfl_xor_sync(0xffffffffu, best, o);
            best = ob < best ? ob : best;
        }
        if (lane == 0) {
            sk[written] = tau;
            st[written] = best;
        }
        floor_t = best;
        have_floor = true;
        ++written;
    }
    __syncwarp();
    return take;
}

// USQ rerank of caller-chosen stored rows (the reference's score_with_meta + distance,
// quantizer.rs:274-288,382-400, ivf_usq.rs:581-586): pair p = (query p / m, row
// rows[p]) per group of 8 lanes; rows outside [0, ntotal) give +inf.
__global__ void __launch_bounds__(256) rerank_rows_kernel(RerankRowsArgs a) {
    const int lane = (int)lane_id(), grp = lane >> 3, sub = lane & 7;
    const int64_t total = a.nq * a.m;
    const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
    for (int64_t p0 = ((int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * 4; p0 < total;
         p0 += warps * 4) {
        const int64_t p = p0 + grp;
        int64_t row = -1;
        int64_t q = 0;
        if (p < total) {
            q = p / a.m;
            row = a.rows[p];
        }
        const bool act = row >= 0 && row < a.ntotal;
        const uint8_t* code = a.codes + (act ? row : 0) * a.code_bytes;
        const int iip = int_ip_group8(code, a.q_i8p + q * a.D, a.D, a.nbits, sub, act);
        if (p < total && sub == 0)
            a.out[p] = act ? rerank_distance(iip, a.meta[row], a.qp[q], a.nbits, a.metric_l2 != 0)
                           : __int_as_float(0x7f800000);
    }
}

// Per (query, probe) pair (one warp): the k best of the pair's kept candidates, into a
// fixed slot of k entries (rank * k) of the query's compact region; unused entries get
// key ~0u and tie ~0ull.  The top-k of a query over the union of its pairs' top-k equals
// its top-k over all candidates.
__global__ void __launch_bounds__(128) compact_pairs_kernel(CompactArgs a) {
    __shared__ uint32_t hist[4][256];
    const int w = threadIdx.x >> 5, lane = (int)lane_id();
    const int64_t pr = (int64_t)blockIdx.x * 4 + w;
    if (pr >= a.nq * a.nprobe) return;
    const int64_t q = pr / a.nprobe;
    const int r = (int)(pr - q * a.nprobe);
    const int* po = a.pair_off + q * (a.nprobe + 1);
    const int64_t base = q * a.q_stride + po[r];
    const int total = po[r + 1] - po[r];
    uint32_t* ok = a.out_key + pr * a.k;
    uint64_t* ot = a.out_tie + pr * a.k;
    int take = 0;
    if (total > 0 && total <= 32 * 8)
        take = warp_select_topk_small<8>(a.cand_key + base, a.cand_tie + base, total, a.k, ok, ot,
                                         hist[w]);
    else if (total > 0)
        take = warp_select_topk(a.cand_key + base, a.cand_tie + base, total, a.k, ok, ot, hist[w]);
    for (int i = take + lane; i < a.k; i += 32) {
        ok[i] = 0xFFFFFFFFu;
        ot[i] = ~0ull;
    }
}

// ============================================================================
// Final merge: per query (one warp) top-k over all kept candidates of its probes,
// ordered by (distance key, probe rank, FastScan key, list position).
// ============================================================================
// One query by one warp (sel_key / sel_tie: its [k] scratch).
__device__ void merge_query_warp(const MergeArgs& a, int64_t q, uint32_t* hist_w) {
    const int lane = (int)lane_id();
    const int total = a.fixed_total > 0 ? a.fixed_total : a.pair_off[q * (a.nprobe + 1) + a.nprobe];
    uint32_t* sk = a.sel_key + q * a.k;
    uint64_t* st = a.sel_tie + q * a.k;  // probe rank << 48 | fastscan key << 32 | index
    const int take = total <= 32 * 8
                         ? warp_select_topk_small<8>(a.cand_key + q * a.q_stride, a.cand_tie + q * a.q_stride,
                                                     total, a.k, sk, st, hist_w)
                         : warp_select_topk(a.cand_key + q * a.q_stride, a.cand_tie + q * a.q_stride,
                                            total, a.k, sk, st, hist_w);
    // sort the selected entries by (key, tie) and write the row
    for (int i = lane; i < a.k; i += 32) {
        if (i >= take) {
            if (!a.shard_mode) {
                a.out_ids[q * a.k + i] = -1;
                a.out_dists[q * a.k + i] = __int_as_float(0x7f800000);
            } else {
                a.out_ids[q * a.k + i] = -1;
                a.out_dists[q * a.k + i] = __int_as_float(0x7f800000);
                a.out_keys[q * a.k + i] = ~0ull;
            }
            continue;
        }
        const uint32_t ki = sk[i];
        const uint64_t ti = st[i];
        int rank = 0;
        for (int j = 0; j < take; ++j) {
            const uint32_t kj = sk[j];
            const uint64_t tj = st[j];
            rank += (kj < ki || (kj == ki && tj < ti)) ? 1 : 0;
        }
        const int r = (int)(ti >> 48);
        const uint32_t idx = (uint32_t)(ti & 0xFFFFFFFFull);
        int64_t id = -1;
        if (r < a.nprobe) {
            const int l = a.probes[q * a.nprobe + r];
            if (l >= 0 && l < a.nlist && idx < (uint32_t)(a.list_off[l + 1] - a.list_off[l]))
                id = a.ids[a.list_off[l] + idx];
        }
        a.out_ids[q * a.k + rank] = id;
        a.out_dists[q * a.k + rank] = key_to_float(ki);
        if (a.shard_mode) a.out_keys[q * a.k + rank] = ti;
    }
    __syncwarp();
    if (a.post_bitsets) {  // reference post-filter: drop filtered ids, keep order
        const uint64_t* bw = nullptr;
        const int b = a.query_bitset ? a.query_bitset[q] : 0;
        if (b >= 0 && b < a.n_bitsets) bw = a.post_bitsets + (int64_t)b * a.bitset_words;
        int n_out = 0;
        for (int base = 0; base < a.k; base += 32) {
            const int i = base + lane;
            int64_t id = 0;
            float dd = 0;
            bool keep = false;
            if (i < a.k) {
                id = a.out_ids[q * a.k + i];
                dd = a.out_dists[q * a.k + i];
                keep = !bw || !bit_filtered(bw, a.bitset_len, id);
            }
            const unsigned bk = __ballot_sync(0xffffffffu, keep);
            __syncwarp();
            if (keep) {
                const int pos = n_out + __popc(bk & lanemask_lt());
                a.out_ids[q * a.k + pos] = id;
                a.out_dists[q * a.k + pos] = dd;
            }
            n_out += __popc(bk);
            __syncwarp();
        }
        for (int i = n_out + lane; i < a.k; i += 32) {
            a.out_ids[q * a.k + i] = -1;
            a.out_dists[q * a.k + i] = __int_as_float(0x7f800000);
        }
        if (lane == 0 && a.out_counts) a.out_counts[q] = n_out;
    } else if (lane == 0 && a.out_counts) {
        a.out_counts[q] = a.k;
    }
}

// ============================================================================
// Kept sets of the tensor-core FastScan pairs (n_cand < |list| <= the tensor-core row limit):
// the tensor-core scan wrote every row's 16-bit FastScan score and int_ip of the pair to the
// FastScan scratch; a warp per pair takes the reference heap's kept set with the closed form
// of scan_lists_kernel (src/quantization/usq/fastscan.rs:86-146) and writes each kept row's
// distance key (src/quantization/usq/quantizer.rs:274-288) and tie to the pair's region.
// ============================================================================
// Packed halfword compare result (0xFFFF per true half) -> 2 bits, low half first.
__device__ __forceinline__ uint32_t half_bits(uint32_t m) { return (m & 1u) | ((m >> 15) & 2u); }

// Position of the k-th (1-based) set bit of x (x has at least k).
__device__ __forceinline__ int nth_set_bit64(uint64_t x, int k) {
    for (int i = 1; i < k; ++i) x &= x - 1ull;
    return __ffsll((long long)x) - 1;
}

// Kept set and distances of one unfiltered tensor-core FastScan pair (n_cand < n <= 64 PW
// rows), a warp with the pair's scores in registers: lane l holds rows l * 2 PW .. + 2 PW
// (list order is lane-major) as packed halfwords.  s* = the n_cand-th largest score by
// binary search on the score (packed compares, one warp reduction per probe); the heap
// boundary and the evicted ties at s* from per-lane row masks and warp prefix sums; the
// kept rows' int_ip and metadata are loaded four rows at a time before their distances.
template <int PW>
__device__ void fs_select_regs(const FsSelectArgs& a, int64_t q, int r, int64_t beg, int n,
                               const int16_t* gsc, const int32_t* gip, int lane, uint32_t* kept,
                               uint32_t* hist) {
    constexpr int RPL = 2 * PW;  // rows per lane
    const int row0 = lane * RPL;
    const int npad = (n + 7) & ~7;  // the pair's scratch region
    uint32_t sw[PW];
#pragma unroll
    for (int k = 0; k < PW / 4; ++k) {
        const int rr = row0 + 8 * k;
        const uint4 x = rr < npad ? __ldg(reinterpret_cast<const uint4*>(gsc + rr))
                                  : make_uint4(0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u);
        sw[4 * k] = x.x;
        sw[4 * k + 1] = x.y;
        sw[4 * k + 2] = x.z;
        sw[4 * k + 3] = x.w;
    }
    const uint64_t valid = row0 >= n ? 0ull
                                     : (n - row0 >= RPL ? (RPL == 64 ? ~0ull : (1ull << RPL) - 1ull)
                                                        : (1ull << (n - row0)) - 1ull);
    // rows >= n read as -32768: never counted by the search (its probes are > the minimum)
    uint32_t mx = 0x80008000u, mn = 0x7FFF7FFFu;
#pragma unroll
    for (int wi = 0; wi < PW; ++wi) {
        const uint32_t hm = ((valid >> (2 * wi)) & 1ull ? 0x0000FFFFu : 0u) | ((valid >> (2 * wi + 1)) & 1ull ? 0xFFFF0000u : 0u);
        sw[wi] = (sw[wi] & hm) | (0x80008000u & ~hm);
        mx = __vmaxs2(mx, sw[wi]);
        mn = __vmins2(mn, (sw[wi] & hm) | (0x7FFF7FFFu & ~hm));
    }
    const int smax = __reduce_max_sync(0xffffffffu, max((int)(int16_t)(mx & 0xFFFFu), (int)(int16_t)(mx >> 16)));
    const int smin = __reduce_min_sync(0xffffffffu, min((int)(int16_t)(mn & 0xFFFFu), (int)(int16_t)(mn >> 16)));
    // s* = the largest y with (rows scoring >= y) >= n_cand: that count is n > n_cand at
    // smin and 0 at smax + 1; c_hi ends as the rows above s*
    int lo = smin, hi = smax + 1, c_hi = 0;
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        const uint32_t yy = (uint32_t)(uint16_t)mid * 0x10001u;
        uint32_t cp = 0u;  // per-half counts (each at most PW)
#pragma unroll
        for (int wi = 0; wi < PW; ++wi) cp += __vsetges2(sw[wi], yy);
        const int c = (int)__reduce_add_sync(0xffffffffu, (cp & 0xFFFFu) + (cp >> 16));
        if (c >= a.n_cand) {
            lo = mid;
        } else {
            hi = mid;
            c_hi = c;
        }
    }
    const int s_star = lo, c_gt = c_hi;
    const uint32_t ss = (uint32_t)(uint16_t)s_star * 0x10001u;
    uint64_t ge = 0ull, gt = 0ull;
#pragma unroll
    for (int wi = 0; wi < PW; ++wi) {
        ge |= (uint64_t)half_bits(__vcmpges2(sw[wi], ss)) << (2 * wi);
        gt |= (uint64_t)half_bits(__vcmpgts2(sw[wi], ss)) << (2 * wi);
    }
    ge &= valid;
    gt &= valid;
    // boundary: p_end = the n_cand-th row with score >= s*, gt_f = rows above s* up to it
    const int cge = __popcll(ge), cgt = __popcll(gt);
    const int pge = warp_inclusive_scan(cge) - cge, pgt = warp_inclusive_scan(cgt) - cgt;
    const bool here = pge < a.n_cand && pge + cge >= a.n_cand;
    int pe = 0, gf = 0;
    if (here) {
        const int idx = nth_set_bit64(ge, a.n_cand - pge);
        pe = row0 + idx;
        gf = pgt + __popcll(gt & (idx == 63 ? ~0ull : ((2ull << idx) - 1ull)));
    }
    const int src = __ffs(__ballot_sync(0xffffffffu, here)) - 1;
    const int p_end = __shfl_sync(0xffffffffu, pe, src);
    const int m_drop = c_gt - __shfl_sync(0xffffffffu, gf, src);  // lowest-index ties evicted
    // rows at s* up to p_end, without the first m_drop of them in list order
    const uint64_t le_p = row0 > p_end ? 0ull : (p_end - row0 >= RPL - 1 ? ~0ull : (2ull << (p_end - row0)) - 1ull);
    uint64_t eqm = ge & ~gt & le_p;
    const int ceq = __popcll(eqm), peq = warp_inclusive_scan(ceq) - ceq;
    for (int d = min(max(m_drop - peq, 0), ceq); d > 0; --d) eqm &= eqm - 1ull;
    const uint64_t keep = gt | eqm;
    const int ck = __popcll(keep), pk = warp_inclusive_scan(ck) - ck;
    // the kept rows (row, score) in list order to the warp's list, then their distance keys
    // and ties with every lane busy
#pragma unroll
    for (int j = 0; j < RPL; ++j) {
        if (!((keep >> j) & 1ull)) continue;
        const int pos = pk + __popcll(keep & ((1ull << j) - 1ull));
        const uint32_t sv = (j & 1) ? (sw[j >> 1] >> 16) : (sw[j >> 1] & 0xFFFFu);
        if (pos < a.n_cand) kept[pos] = ((uint32_t)(row0 + j) << 16) | sv;
    }
    __syncwarp();
    const int n_kept = min(__shfl_sync(0xffffffffu, pk + ck, 31), a.n_cand);
    const QueryParams qp = a.qp[q];
    const bool l2 = a.metric_l2 != 0;
    const int* po = a.pair_off + q * (a.nprobe + 1) + r;
    const int64_t rbase = q * a.q_stride + po[0];
    const uint64_t rank_bits = (uint64_t)r << 48;
    // a region of cap < n_kept entries (the pair offsets kept room for the pair's top k
    // only): the distance keys go to kk first, then the cap smallest by (key, tie)
    const int cap = po[1] - po[0];
    const bool trunc = cap < n_kept;
    uint32_t* kk = kept + kFsRegRows / 2;  // (trunc only when n_cand <= kFsRegRows / 2)
    for (int e0 = 0; e0 < n_kept; e0 += 64) {
        // two entries per lane, their loads issued together
        int ipv[2];
        float4 mv[2];
        uint32_t ent[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int e = e0 + 32 * h + lane;
            ent[h] = e < n_kept ? kept[e] : 0u;
            const int v = (int)(ent[h] >> 16);
            ipv[h] = e < n_kept ? __ldg(gip + v) : 0;
            mv[h] = e < n_kept ? __ldg(a.meta + beg + v) : make_float4(0.f, 0.f, 0.f, 0.f);
        }
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int e = e0 + 32 * h + lane;
            if (e >= n_kept) continue;
            const int v = (int)(ent[h] >> 16), sv = (int)(int16_t)(ent[h] & 0xFFFFu);
            const float dist = rerank_distance(ipv[h], mv[h], qp, a.nbits, l2);
            if (trunc) {
                kk[e] = total_order_key(dist);
                continue;
            }
            a.cand_key[rbase + e] = total_order_key(dist);
            a.cand_tie[rbase + e] = rank_bits | ((uint64_t)(uint32_t)(32767 - sv) << 32) | (uint32_t)v;
            if (a.cand_dbg) a.cand_dbg[rbase + e] = make_int2(ipv[h], sv);
        }
    }
    __syncwarp();
    if (!trunc) return;
    // the pair's top cap by (key, FastScan key, row) -- the merge's order inside one pair, so
    // the query's top k over all pairs is unchanged.
    auto tie_of = [&](int e) {
        const uint32_t en = kept[e];
        return rank_bits | ((uint64_t)(uint32_t)(32767 - (int)(int16_t)(en & 0xFFFFu)) << 32) | (en >> 16);
    };
    // Fast path: the cap-th smallest of the 32 lane minima bounds the cap-th smallest key
    // from above (those cap lanes hold cap entries at or below it; at least cap lanes hold
    // entries because n_kept > cap and cap <= 32).  The entries at or below the bound --
    // usually little more than cap -- take one lane each and are ranked by (key, tie),
    // which is unique, with a shuffle loop; ranks < cap are written in order.
    if (cap <= 32) {
        uint32_t lm = 0xFFFFFFFFu;
        for (int e = lane; e < n_kept; e += 32) lm = min(lm, kk[e]);
        uint32_t bound = 0;
        for (int i = 0; i < cap; ++i) {
            bound = __reduce_min_sync(0xffffffffu, lm);
            const unsigned b = __ballot_sync(0xffffffffu, lm == bound);
            if (lane == __ffs(b) - 1) lm = 0xFFFFFFFFu;
        }
        int nc = 0;
        for (int e0 = 0; e0 < n_kept; e0 += 32) {
            const int e = e0 + lane;
            const bool in = e < n_kept && kk[e] <= bound;
            const unsigned b = __ballot_sync(0xffffffffu, in);
            if (in && nc + __popc(b & lanemask_lt()) < 32) hist[nc + __popc(b & lanemask_lt())] = (uint32_t)e;
            nc += __popc(b);
        }
        __syncwarp();
        if (nc <= 32) {
            const int e = lane < nc ? (int)hist[lane] : 0;
            const uint32_t key = lane < nc ? kk[e] : 0xFFFFFFFFu;
            const uint64_t tie = lane < nc ? tie_of(e) : ~0ull;
            int rk = 0;
            for (int j = 0; j < nc; ++j) {
                const uint32_t kj = __shfl_sync(0xffffffffu, key, j);
                const uint64_t tj = __shfl_sync(0xffffffffu, tie, j);
                rk += (kj < key || (kj == key && tj < tie)) ? 1 : 0;
            }
            if (lane < nc && rk < cap) {
                a.cand_key[rbase + rk] = key;
                a.cand_tie[rbase + rk] = tie;
            }
            __syncwarp();
            return;
        }
        __syncwarp();
    }
    // general path: tau = the cap-th smallest key, every entry below it, then the smallest
    // (FastScan key, row) among the entries at tau
    int n_less = 0;
    const uint32_t tau = warp_radix_kth(
        n_kept, cap,
        [&](int i, uint32_t& key) {
            key = kk[i];
            return true;
        },
        hist, &n_less);
    int n_w = 0;
    for (int b = 0; b < n_kept; b += 32) {
        const int e = b + lane;
        const bool take = e < n_kept && kk[e] < tau;
        const unsigned bt = __ballot_sync(0xffffffffu, take);
        if (take) {
            const int pos = n_w + __popc(bt & lanemask_lt());
            a.cand_key[rbase + pos] = kk[e];
            a.cand_tie[rbase + pos] = tie_of(e);
        }
        n_w += __popc(bt);
    }
    // ties at tau (rare: equal distances): the smallest remaining tie, one at a time
    uint64_t floor_t = 0;
    for (bool first = true; n_w < cap; ++n_w, first = false) {
        uint64_t best = ~0ull;
        for (int e = lane; e < n_kept; e += 32) {
            if (kk[e] != tau) continue;
            const uint64_t t = tie_of(e);
            if ((first || t > floor_t) && t < best) best = t;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint64_t ob = __shfl_xor_sync(0xffffffffu, best, o);
            best = ob < best ? ob : best;
        }
        floor_t = best;
        if (lane == 0) {
            a.cand_key[rbase + n_w] = tau;
            a.cand_tie[rbase + n_w] = best;
        }
    }
    __syncwarp();
}

// One (query, probe) pair of the FastScan selection, by one warp.
__device__ void fs_select_pair(const FsSelectArgs& a, int64_t q, int r, int lane, uint32_t* hist_w,
                               uint32_t* kept_w) {
    const int64_t pr = q * a.nprobe + r;
    const int fo = a.fs_off[pr];
    if (fo < 0) return;
    const int l = a.probes[pr];
    const int64_t beg = a.list_off[l];
    const int n = (int)(a.list_off[l + 1] - beg);
    const int16_t* sc = a.fs_sc + q * a.fs_stride + fo;
    const int32_t* ip = a.fs_ip + q * a.fs_stride + fo;
    const QueryParams qp = a.qp[q];
    const bool l2 = a.metric_l2 != 0;
    const int64_t rbase = q * a.q_stride + a.pair_off[q * (a.nprobe + 1) + r];
    const uint64_t* bw = nullptr;
    if (a.fused && a.bitsets) {
        const int b = a.query_bitset ? a.query_bitset[q] : 0;
        if (b >= 0 && b < a.n_bitsets) bw = a.bitsets + (int64_t)b * a.bitset_words;
    }
    if (!bw && n <= kFsRegRows) {
        // unfiltered (every row live, n > n_cand): the pair's scores in registers
        if (n <= kFsRegRows / 2)
            fs_select_regs<8>(a, q, r, beg, n, sc, ip, lane, kept_w, hist_w);
        else
            fs_select_regs<16>(a, q, r, beg, n, sc, ip, lane, kept_w, hist_w);
        return;
    }
    auto live = [&](int v) { return !bw || !bit_filtered(bw, a.bitset_len, a.ids[beg + v]); };
    int n_live = n;
    if (bw) {
        int c = 0;
        for (int v = lane; v < n; v += 32) c += live(v) ? 1 : 0;
        n_live = warp_sum(c);
    }
    const uint64_t rank_bits = (uint64_t)r << 48;
    // kept row v at position pos: its distance and tie (fs_key ~0: no FastScan key)
    auto emit = [&](int v, int pos, uint32_t fs_key) {
        const float dist = rerank_distance(ip[v], __ldg(a.meta + beg + v), qp, a.nbits, l2);
        a.cand_key[rbase + pos] = total_order_key(dist);
        a.cand_tie[rbase + pos] = rank_bits | (fs_key != 0xFFFFFFFFu ? (uint64_t)fs_key << 32 : 0ull) | (uint32_t)v;
        if (a.cand_dbg)
            a.cand_dbg[rbase + pos] = make_int2(ip[v], fs_key != 0xFFFFFFFFu ? 32767 - (int)fs_key : INT32_MIN);
    };
    int n_c = 0;
    if (n_live > a.n_cand) {
        // s* = n_cand-th largest score among live rows (key = 32767 - score)
        auto key_at = [&](int v, uint32_t& k) {
            if (!live(v)) return false;
            k = (uint32_t)(32767 - (int)sc[v]);
            return true;
        };
        int c_gt = 0, c_eq = 0;
        const uint32_t tau = warp_radix_kth16(n, a.n_cand, key_at, hist_w, &c_gt, &c_eq);
        // F = first n_cand rows (in list order) with score >= s*; gt_F = rows > s* in F.
        // When exactly n_cand rows score >= s*, F is all of them (no pass needed).
        int cnt_ge = 0, cnt_gt = 0, p_end = n, gt_f = c_gt;
        for (int base = 0; c_gt + c_eq != a.n_cand && base < n; base += 32) {
            const int v = base + lane;
            uint32_t k = 0xFFFFFFFFu;
            const bool valid = v < n && key_at(v, k);
            const bool ge = valid && k <= tau, gt = valid && k < tau;
            const unsigned bge = __ballot_sync(0xffffffffu, ge);
            const unsigned bgt = __ballot_sync(0xffffffffu, gt);
            const int c = __popc(bge);
            if (cnt_ge + c >= a.n_cand) {
                const int need = a.n_cand - cnt_ge;
                const bool here = ge && __popc(bge & lanemask_le()) == need;
                const int pos = __ffs(__ballot_sync(0xffffffffu, here)) - 1;
                p_end = base + pos;
                gt_f = cnt_gt + __popc(bgt & (pos == 31 ? 0xffffffffu : ((2u << pos) - 1u)));
                break;
            }
            cnt_ge += c;
            cnt_gt += __popc(bgt);
        }
        const int m_drop = c_gt - gt_f;  // lowest-index ties evicted by later rows
        int eq_seen = 0;
        for (int base = 0; base < n; base += 32) {
            const int v = base + lane;
            uint32_t k = 0xFFFFFFFFu;
            const bool valid = v < n && key_at(v, k);
            const bool gt = valid && k < tau;
            const bool eq = valid && k == tau && v <= p_end;
            const unsigned beq = __ballot_sync(0xffffffffu, eq);
            const int eq_rank = eq_seen + __popc(beq & lanemask_le());
            const bool keep = gt || (eq && eq_rank > m_drop);
            const unsigned bk = __ballot_sync(0xffffffffu, keep);
            if (keep) {
                const int pos = n_c + __popc(bk & lanemask_lt());
                if (pos < a.n_cand) emit(v, pos, k);
            }
            n_c += __popc(bk);
            eq_seen += __popc(beq);
        }
    } else {
        // every live row is kept, in list order
        for (int base = 0; base < n; base += 32) {
            const int v = base + lane;
            const bool keep = v < n && live(v);
            const unsigned bk = __ballot_sync(0xffffffffu, keep);
            if (keep) emit(v, n_c + __popc(bk & lanemask_lt()), 0xFFFFFFFFu);
            n_c += __popc(bk);
        }
    }
    n_c = min(n_c, a.n_cand);
    // unused entries of the pair's region of n_cand entries (rows removed by the filter)
    for (int j = n_c + lane; j < a.n_cand; j += 32) {
        a.cand_tie[rbase + j] = ~0ull;
        a.cand_key[rbase + j] = 0xFFFFFFFFu;
    }
}

// Persistent warps over the grouping step's pairs (this rank's, grouped by list), round
// robin: the pairs of one list (same cost) go to different warps.
__global__ void __launch_bounds__(256, 4) fs_select_kernel(FsSelectArgs a) {
    __shared__ uint32_t hist[8][256];
    __shared__ uint32_t kept_rows[8][kFsRegRows];  // register path: each warp's kept (row, score)
    const int w = threadIdx.x >> 5, lane = (int)lane_id();
    const int total = *a.n_lq;
    const int n_warps = gridDim.x * 8;
    for (int u = blockIdx.x * 8 + w; u < total; u += n_warps) {
        const int2 pr = a.lq[u];
        fs_select_pair(a, pr.x, pr.y, lane, hist[w], kept_rows[w]);
    }
}

// ============================================================================
// Final merge, one 256-thread block per query (k <= kMergeMaxK): the top k of all kept
// candidates of the query's probes by (distance key, tie = probe rank << 48 | FastScan key
// << 32 | position), sorted -- the same result as compact_pairs_kernel + merge_kernel.
// The query's keys are read once (into shared memory when they fit); a block radix
// select finds the k-th smallest key tau; ties are read only for the entries taken and
// for those at tau.  Unused entries carry key 0xFFFFFFFF and tie ~0 (the scans' fill):
// they sort after every valid entry, and at tau = 0xFFFFFFFF only valid ties are taken.
// ============================================================================
constexpr int kMergeKeyCap = 8192;  // keys of one query held in shared memory
constexpr int kMergeEqCap = 256;    // ties at tau ranked at once

struct MergeSmem {
    uint32_t hist[kSelBins];
    uint32_t list[kSelList];
    int bcast[8];
    int cnt[4];
    unsigned long long best;
    uint64_t eq[kMergeEqCap];
};

// One query by the whole block (mdyn: sel ties [k], sel keys [k], keys [kMergeKeyCap]).
__device__ void merge_query_block(const MergeArgs& a, int64_t q, MergeSmem& ms, uint8_t* mdyn) {
    const int tid = threadIdx.x, lane = tid & 31;
    const int k = a.k;
    uint64_t* st = reinterpret_cast<uint64_t*>(mdyn);
    uint32_t* sk = reinterpret_cast<uint32_t*>(st + k);
    uint32_t* ks = sk + k;
    const int total = a.pair_off[q * (a.nprobe + 1) + a.nprobe];
    const uint32_t* gk = a.cand_key + q * a.q_stride;
    const uint64_t* gt = a.cand_tie + q * a.q_stride;
    const bool in_smem = total <= kMergeKeyCap;
    if (tid < 4) ms.cnt[tid] = 0;
    int n_lt = 0;  // entries below 0xFFFFFFFF (all valid)
    for (int e = tid; e < total; e += kSelThreads) {
        const uint32_t kk = gk[e];
        if (in_smem) ks[e] = kk;
        n_lt += kk != 0xFFFFFFFFu ? 1 : 0;
    }
    const uint32_t* keys = in_smem ? ks : gk;
    n_lt = warp_sum(n_lt);
    __syncthreads();
    if (lane == 0) atomicAdd(&ms.cnt[0], n_lt);
    __syncthreads();
    n_lt = ms.cnt[0];
    uint32_t tau = 0xFFFFFFFFu;
    // (four keys of a thread loaded before any is counted: the keys may be in global memory)
    if (n_lt >= k)
        tau = block_select_kth(
            [&](auto f) {
                for (int b = threadIdx.x; b < total; b += 4 * kSelThreads) {
                    uint32_t t[4];
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int e = b + j * kSelThreads;
                        t[j] = e < total ? keys[e] : 0xFFFFFFFFu;
                    }
#pragma unroll
                    for (int j = 0; j < 4; ++j)
                        if (t[j] != 0xFFFFFFFFu) f(t[j]);
                }
            },
            k, ms.hist, ms.list, ms.bcast);
    // the entries below tau (any order) and the valid ties at tau
    for (int b = tid; b < total; b += 4 * kSelThreads) {
        uint32_t t[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = b + j * kSelThreads;
            t[j] = e < total ? keys[e] : 0xFFFFFFFFu;
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int e = b + j * kSelThreads;
            if (e >= total) continue;
            const uint32_t kk = t[j];
            if (kk < tau) {
                const int p = atomicAdd(&ms.cnt[1], 1);
                sk[p] = kk;
                st[p] = gt[e];
            } else if (kk == tau) {
                const uint64_t tt = gt[e];
                if (tt != ~0ull) {
                    const int p = atomicAdd(&ms.cnt[2], 1);
                    if (p < kMergeEqCap) ms.eq[p] = tt;
                }
            }
        }
    }
    __syncthreads();
    const int less = ms.cnt[1], n_eq = ms.cnt[2];
    const int need = min(k - less, n_eq);
    const int take = less + need;
    if (n_eq <= kMergeEqCap) {
        // the `need` smallest ties at tau (a query's ties are distinct): rank among them
        for (int j = tid; j < n_eq; j += kSelThreads) {
            const uint64_t t = ms.eq[j];
            int r = 0;
            for (int i = 0; i < n_eq; ++i) r += ms.eq[i] < t ? 1 : 0;
            if (r < need) {
                sk[less + r] = tau;
                st[less + r] = t;
            }
        }
    } else {
        // many entries at tau: the smallest remaining tie, need times
        uint64_t floor_t = 0;
        for (int r = 0; r < need; ++r) {
            if (tid == 0) ms.best = ~0ull;
            __syncthreads();
            uint64_t best = ~0ull;
            for (int e = tid; e < total; e += kSelThreads) {
                if (keys[e] != tau) continue;
                const uint64_t t = gt[e];
                if (t != ~0ull && (r == 0 || t > floor_t) && t < best) best = t;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                const uint64_t ob = __shfl_xor_sync(0xffffffffu, best, o);
                best = ob < best ? ob : best;
            }
            if (lane == 0) atomicMin(&ms.best, (unsigned long long)best);
            __syncthreads();
            floor_t = ms.best;
            if (tid == 0) {
                sk[less + r] = tau;
                st[less + r] = floor_t;
            }
        }
    }
    __syncthreads();
    // sorted row: each taken entry's rank by (key, tie)
    for (int i = tid; i < k; i += kSelThreads) {
        if (i >= take) {
            a.out_ids[q * k + i] = -1;
            a.out_dists[q * k + i] = __int_as_float(0x7f800000);
            if (a.shard_mode) a.out_keys[q * k + i] = ~0ull;
            continue;
        }
        const uint32_t ki = sk[i];
        const uint64_t ti = st[i];
        int rank = 0;
        for (int j = 0; j < take; ++j) {
            const uint32_t kj = sk[j];
            rank += (kj < ki || (kj == ki && st[j] < ti)) ? 1 : 0;
        }
        const int r = (int)(ti >> 48);
        const uint32_t idx = (uint32_t)(ti & 0xFFFFFFFFull);
        int64_t id = -1;
        if (r < a.nprobe) {
            const int l = a.probes[q * a.nprobe + r];
            if (l >= 0 && l < a.nlist && idx < (uint32_t)(a.list_off[l + 1] - a.list_off[l]))
                id = a.ids[a.list_off[l] + idx];
        }
        a.out_ids[q * k + rank] = id;
        a.out_dists[q * k + rank] = key_to_float(ki);
        if (a.shard_mode) a.out_keys[q * k + rank] = ti;
    }
    __syncthreads();
    if (threadIdx.x < 32 && a.post_bitsets) {  // reference post-filter: drop filtered ids, keep order
        const uint64_t* bw = nullptr;
        const int b = a.query_bitset ? a.query_bitset[q] : 0;
        if (b >= 0 && b < a.n_bitsets) bw = a.post_bitsets + (int64_t)b * a.bitset_words;
        int n_out = 0;
        for (int base = 0; base < k; base += 32) {
            const int i = base + lane;
            int64_t id = 0;
            float dd = 0;
            bool keep = false;
            if (i < k) {
                id = a.out_ids[q * k + i];
                dd = a.out_dists[q * k + i];
                keep = !bw || !bit_filtered(bw, a.bitset_len, id);
            }
            const unsigned bk = __ballot_sync(0xffffffffu, keep);
            __syncwarp();
            if (keep) {
                const int pos = n_out + __popc(bk & lanemask_lt());
                a.out_ids[q * k + pos] = id;
                a.out_dists[q * k + pos] = dd;
            }
            n_out += __popc(bk);
            __syncwarp();
        }
        for (int i = n_out + lane; i < k; i += 32) {
            a.out_ids[q * k + i] = -1;
            a.out_dists[q * k + i] = __int_as_float(0x7f800000);
        }
        if (lane == 0 && a.out_counts) a.out_counts[q] = n_out;
    } else if (threadIdx.x == 0 && a.out_counts) {
        a.out_counts[q] = k;
    }
    __syncthreads();  // (the next query reuses the shared memory)
}

// Eight queries per block: each by a warp when every one has at most kMergeWarpMax
// candidates (many small regions, e.g. a list shard's), else one after another by the
// whole block.
constexpr int kMergeWarpMax = 2048;
__global__ void __launch_bounds__(kSelThreads) merge_direct_kernel(MergeArgs a) {
    __shared__ MergeSmem ms;
    __shared__ int small_s;
    extern __shared__ __align__(16) uint8_t mdyn[];
    const int64_t q0 = (int64_t)blockIdx.x * 8;
    const int nq_b = (int)(a.nq - q0 < 8 ? a.nq - q0 : 8);
    if (threadIdx.x == 0) {
        int mx = 0;
        for (int i = 0; i < nq_b; ++i) mx = max(mx, a.pair_off[(q0 + i) * (a.nprobe + 1) + a.nprobe]);
        small_s = mx <= kMergeWarpMax ? 1 : 0;
    }
    __syncthreads();
    if (small_s) {
        const int w = threadIdx.x >> 5;
        if (w < nq_b) merge_query_warp(a, q0 + w, ms.hist + 256 * w);
        return;
    }
    for (int i = 0; i < nq_b; ++i) merge_query_block(a, q0 + i, ms, mdyn);
}

__global__ void __launch_bounds__(128) merge_kernel(MergeArgs a) {
    __shared__ uint32_t hist[4][256];
    const int w = threadIdx.x >> 5;
    const int64_t q = (int64_t)blockIdx.x * 4 + w;
    if (q >= a.nq) return;
    merge_query_warp(a, q, hist[w]);
}

}  // namespace hanns

namespace hanns {

// Cross-shard merge: per query (one warp) the k best of world sorted shard rows by
// (distance, merge key).  Keys are unique per query, so the result equals the
// single-GPU order.
__global__ void __launch_bounds__(128) merge_shards_kernel(const float* __restrict__ dists,
                                                           const uint64_t* __restrict__ keys,
                                                           const int64_t* __restrict__ ids,
                                                           int world, int64_t nq, int k,
                                                           int64_t* __restrict__ out_ids,
                                                           float* __restrict__ out_dists) {
    const int w = threadIdx.x >> 5, lane = (int)lane_id();
    const int64_t q = (int64_t)blockIdx.x * 4 + w;
    if (q >= nq) return;
    // k-way merge by repeated warp argmin over the shard heads (world <= 32).
    int head = 0;  // lane s < world owns shard s's cursor
    for (int out = 0; out < k; ++out) {
        uint32_t dk = 0xFFFFFFFFu;
        uint64_t mk = ~0ull;
        if (lane < world && head < k) {
            const int64_t e = ((int64_t)lane * nq + q) * k + head;
            if (keys[e] != ~0ull) {
                dk = total_order_key(dists[e]);
                mk = keys[e];
            }
        }
        uint32_t bdk = dk;
        uint64_t bmk = mk;
        int bl = lane;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const uint32_t odk = __shfl_xor_sync(0xffffffffu, bdk, o);
            const uint64_t omk = __shfl_xor_sync(0xffffffffu, bmk, o);
            const int ol = __shfl_xor_sync(0xffffffffu, bl, o);
            if (odk < bdk || (odk == bdk && (omk < bmk || (omk == bmk && ol < bl)))) {
                bdk = odk;
                bmk = omk;
                bl = ol;
            }
        }
        if (bmk == ~0ull) {
            if (lane == 0) {
                for (int j = out; j < k; ++j) {
                    out_ids[q * k + j] = -1;
                    out_dists[q * k + j] = __int_as_float(0x7f800000);
                }
            }
            return;
        }
        if (lane == bl) {
            const int64_t e = ((int64_t)lane * nq + q) * k + head;
            out_ids[q * k + out] = ids[e];
            out_dists[q * k + out] = dists[e];
            ++head;
        }
    }
}

void launch_coarse_l2(const float* q, int64_t nq, const float* cent, int nlist, int d, float* dist,
                      cudaStream_t s) {
    if (nq <= 0) return;
    dim3 grid((nlist + kCT - 1) / kCT, (unsigned)((nq + kCT - 1) / kCT));
    coarse_l2_kernel<<<grid, 256, 0, s>>>(q, nq, cent, nlist, d, dist);
}

void launch_select_probes(const float* dist, int64_t nq, int nlist, int nprobe, int32_t* probes,
                          uint32_t* scratch, cudaStream_t s) {
    if (nq <= 0) return;
    select_probes_kernel<<<(unsigned)((nq + 3) / 4), 128, 0, s>>>(dist, nq, nlist, nprobe, probes,
                                                                  scratch);
}

void launch_coarse_gemm(const float* q, int64_t nq, const float* cent, const float* cn, int nlist,
                        int d, float* approx, cudaStream_t s) {
    if (nq <= 0) return;
    dim3 grid((nlist + kGN - 1) / kGN, (unsigned)((nq + kGM - 1) / kGM));
    if ((d & 3) == 0)
        coarse_gemm_kernel<true><<<grid, 256, 0, s>>>(q, nq, cent, nlist, d, cn, approx);
    else
        coarse_gemm_kernel<false><<<grid, 256, 0, s>>>(q, nq, cent, nlist, d, cn, approx);
}

int launch_coarse_select(float* approx, const float* q, int64_t nq, const float* cent, int nlist,
                          int d, int nprobe, float cmax, float dot_rel, const int* tc_err,
                          int32_t* probes, int* fallbacks, int* rs, cudaStream_t s) {
    if (nq <= 0) return 0;
    const size_t reg_bytes = ((size_t)d + kSelBins + kSelList) * sizeof(float);
    if ((nlist & 3) == 0 && (d & 3) == 0 && nlist <= 16 * kSelThreads &&
        reg_bytes <= 112 * 1024) {
        const int nv4 = (nlist / 4 + kSelThreads - 1) / kSelThreads;  // float4 per thread
        auto go = [&](auto kern) {
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 112 * 1024);
            kern<<<(unsigned)nq, kSelThreads, reg_bytes, s>>>(approx, q, nq, cent, nlist, d, nprobe,
                                                               cmax, dot_rel, tc_err, probes, fallbacks, rs);
        };
        if (nv4 <= 1) go(coarse_select_reg_kernel<1>);
        else if (nv4 == 2) go(coarse_select_reg_kernel<2>);
        else if (nv4 == 3) go(coarse_select_reg_kernel<3>);
        else go(coarse_select_reg_kernel<4>);
        if (rs) {
            const size_t rs_bytes = coarse_rescore_smem(d);
            if (rescore_staged(d)) {
                cudaFuncSetAttribute(coarse_rescore_kernel<true>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize, (int)rs_bytes);
                coarse_rescore_kernel<true><<<(unsigned)nq, kCoarseRescoreMax, rs_bytes, s>>>(
                    q, nq, cent, d, nprobe, cmax, dot_rel, rs, probes);
            } else {
                coarse_rescore_kernel<false><<<(unsigned)nq, kCoarseRescoreMax, rs_bytes, s>>>(
                    q, nq, cent, d, nprobe, cmax, dot_rel, rs, probes);
            }
        }
        return rs ? 2 : 1;
    }
    const size_t blk_bytes =
        ((size_t)((nlist + 3) & ~3) + ((d + 3) & ~3) + kSelBins + kSelList) * sizeof(float);
    // (the row in global memory: many lists -- each pass reads it from there)
    const size_t blk_bytes_g = ((size_t)((d + 3) & ~3) + kSelBins + kSelList) * sizeof(float);
    if (blk_bytes <= 112 * 1024 || blk_bytes_g <= 112 * 1024) {
        const bool in_smem = blk_bytes <= 112 * 1024;
        cudaFuncSetAttribute(coarse_select_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             112 * 1024);
        coarse_select_block_kernel<<<(unsigned)nq, kSelThreads, in_smem ? blk_bytes : blk_bytes_g, s>>>(
            approx, q, nq, cent, nlist, d, nprobe, cmax, dot_rel, tc_err, probes, fallbacks, in_smem ? 1 : 0);
    } else {
        const size_t qbytes = (size_t)4 * d * sizeof(float);
        cudaFuncSetAttribute(coarse_select_exact_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             180 * 1024);
        coarse_select_exact_kernel<<<(unsigned)((nq + 3) / 4), 128, qbytes, s>>>(
            approx, q, nq, cent, nlist, d, nprobe, cmax, dot_rel, tc_err, probes, fallbacks);
    }
    return 1;
}

void launch_centroid_norms(const float* cent, int nlist, int d, float* cn, cudaStream_t s) {
    centroid_norms_kernel<<<(nlist + 127) / 128, 128, 0, s>>>(cent, nlist, d, cn);
}

void launch_rotation_chain_major(const float* P, int D, float* Pc, cudaStream_t s) {
    const int64_t n = (int64_t)D * D;
    rotation_chain_major_kernel<<<(unsigned)((n + 255) / 256), 256, 0, s>>>(P, D, Pc);
}

void launch_rotate(const float* x, int64_t nq, int d, int D, const float* Pc, float* out,
                   cudaStream_t s) {
    if (nq <= 0) return;
    if (D <= 1024) {
        // the whole query tile in shared memory (at most 48 KB: two CTAs per SM)
        constexpr int QT = 8, R = 8;
        const size_t smem = (size_t)D * (QT + 4) * sizeof(float);
        cudaFuncSetAttribute(rotate_kernel<QT, R>, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        dim3 grid((D + 16 * R - 1) / (16 * R), (unsigned)((nq + QT - 1) / QT));
        rotate_kernel<QT, R><<<grid, 256, smem, s>>>(x, nq, d, D, Pc, out);
        return;
    }
    // larger D: 768-column chunks of the query tile (61 KB: still two CTAs per SM, where
    // the whole tile would allow one), 16 queries x 4 rows per thread with the next block
    // of P prefetched (P crosses L2 once per 16 queries; it no longer fits the L1s)
    constexpr int QT = 16, R = 4;
    const int CW = 768;
    const size_t smem = (size_t)CW * (QT + 4) * sizeof(float);
    cudaFuncSetAttribute(rotate_chunked_kernel<QT, R>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
    dim3 grid((D + 16 * R - 1) / (16 * R), (unsigned)((nq + QT - 1) / QT));
    rotate_chunked_kernel<QT, R><<<grid, 256, smem, s>>>(x, nq, d, D, CW, Pc, out);
}

void launch_query_state(const float* x, const float* q_rot, int64_t nq, int d, int D,
                        const float* rc, int nbits, QueryParams* qp, uint8_t* q_i8p,
                        int8_t* q_i8n, uint8_t* lut, cudaStream_t s) {
    if (nq <= 0) return;
    const size_t smem = (size_t)(D + 4 * (D + d)) * sizeof(float);
    cudaFuncSetAttribute(query_state_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    query_state_kernel<<<(unsigned)((nq + 3) / 4), 128, smem, s>>>(x, q_rot, nq, d, D, rc, nbits, qp,
                                                                q_i8p, q_i8n, lut);
}

void launch_group_pairs(const int32_t* probes, int64_t nq, int nprobe, int nlist,
                        const uint8_t* owned, const int64_t* list_off, const int* order,
                        int tc_max_rows, int n_cand,
                        int qpi, int* cnt, int* cursor, int* lq_off, int* item_off, int* n_items,
                        int2* lq, int4* items, cudaStream_t s) {
    cudaMemsetAsync(cnt, 0, sizeof(int) * nlist, s);
    cudaMemsetAsync(cursor, 0, sizeof(int) * nlist, s);
    const int64_t pairs = nq * nprobe;
    const int blocks = (int)std::min<int64_t>((pairs + 255) / 256, 4096);
    count_lists_kernel<<<blocks, 256, 0, s>>>(probes, pairs, nlist, owned, cnt);
    prefix_lists_kernel<<<1, 1024, 0, s>>>(cnt, nlist, order, list_off, tc_max_rows, n_cand, qpi, lq_off,
                                           item_off, n_items);
    scatter_pairs_kernel<<<blocks, 256, 0, s>>>(probes, nq, nprobe, nlist, owned, lq_off, cursor, lq);
    make_items_kernel<<<(nlist + 255) / 256, 256, 0, s>>>(cnt, lq_off, item_off, nlist, list_off,
                                                          tc_max_rows, n_cand, qpi, items);
}

size_t scan_smem_bytes(int D) {
    return sizeof(ScanSmem) + 128 + (size_t)(D / 4) * 16 * sizeof(uint2) + (size_t)kScanWarps * (D + 16);
}

int scan_grid_size(int D) {
    int dev = 0, sms = 0, per_sm = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaFuncSetAttribute(scan_lists_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, scan_lists_kernel, kScanThreads,
                                                      scan_smem_bytes(D)) != cudaSuccess ||
        per_sm < 1)
        per_sm = 1;
    return sms * per_sm;
}

void launch_pair_offsets(const int32_t* probes, int64_t nq, int nprobe, const int64_t* list_off,
                         int nlist, const uint8_t* owned, int n_cand, int* pair_off, int tc_rows,
                         int* fs_off, const PairTrunc& tr, cudaStream_t s) {
    if (nq <= 0) return;
    pair_offsets_kernel<<<(unsigned)((nq + 7) / 8), 256, 0, s>>>(probes, nq, nprobe, list_off, nlist,
                                                                owned, n_cand, pair_off, tc_rows, fs_off, tr);
}

void launch_scan(const ScanArgs& a, int grid, cudaStream_t s) {
    const size_t smem = scan_smem_bytes(a.D);
    cudaFuncSetAttribute(scan_lists_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    scan_lists_kernel<<<grid, kScanThreads, smem, s>>>(a);
}

void launch_rerank_rows(const RerankRowsArgs& a, cudaStream_t s) {
    const int64_t groups = a.nq * a.m;
    if (groups <= 0) return;
    const int64_t blocks = std::min<int64_t>((groups + 31) / 32, 148 * 16);
    rerank_rows_kernel<<<(unsigned)blocks, 256, 0, s>>>(a);
}

void launch_compact_pairs(const CompactArgs& a, cudaStream_t s) {
    const int64_t pairs = a.nq * a.nprobe;
    if (pairs > 0) compact_pairs_kernel<<<(unsigned)((pairs + 3) / 4), 128, 0, s>>>(a);
}

void launch_merge(const MergeArgs& a, cudaStream_t s) {
    if (a.nq <= 0) return;
    merge_kernel<<<(unsigned)((a.nq + 3) / 4), 128, 0, s>>>(a);
}

void launch_fs_select(const FsSelectArgs& a, int grid, cudaStream_t s) {
    if (a.nq * a.nprobe > 0) fs_select_kernel<<<grid, 256, 0, s>>>(a);
}

void launch_merge_direct(const MergeArgs& a, cudaStream_t s) {
    if (a.nq <= 0) return;
    const size_t smem = (size_t)a.k * 12 + (size_t)kMergeKeyCap * 4;
    HANNS_CUDA_OK(cudaFuncSetAttribute(merge_direct_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    merge_direct_kernel<<<(unsigned)((a.nq + 7) / 8), kSelThreads, smem, s>>>(a);
}

void launch_merge_shards(const float* dists, const uint64_t* keys, const int64_t* ids, int world,
                         int64_t nq, int k, int64_t* out_ids, float* out_dists, cudaStream_t s) {
    if (nq <= 0) return;
    merge_shards_kernel<<<(unsigned)((nq + 3) / 4), 128, 0, s>>>(dists, keys, ids, world, nq, k,
                                                                 out_ids, out_dists);
}

}  // namespace hanns
