// coarse_tc.cu -- approximate coarse scores a(q,c) = ||c||^2 - 2 q.c on the sm_100a
// tensor cores (tcgen05.mma kind::f16, bf16 operands, fp32 accumulation in TMEM).
//
// Both operands are split into bf16 hi/lo parts (x = hi + lo + r, |r| <= 2^-16 |x|) and
// q.c is accumulated as hi.hi + hi.lo + lo.hi, so the product error stays near 2^-14
// relative; the exact re-score in coarse_select_* (search_kernels.cu) turns this
// approximation into the reference's exact probe set, with an error bound that covers
// the bf16 representation and the tensor-core accumulation.
//
// One CTA computes one 128 (queries) x 256 (centroids) tile.  Warp roles:
//   warp 0  TMA producer: 2-stage ring of {A hi, A lo 128x64; B hi, B lo 256x64} bf16
//           tiles (one 64-wide K block of both splits, so every tile crosses L2 once),
//           128-byte swizzle, one mbarrier per stage with the transaction byte count
//   warp 1  TMEM allocation (256 fp32 columns) and the single-thread MMA issuer:
//           4 x 3 (hi.hi, hi.lo, lo.hi) M128 N256 K16 per stage, tcgen05.commit releases
//           the stage
//   warps 2-5  epilogue: tcgen05.ld of the 128x256 accumulator (32 rows per warp),
//           out = fma(-2, acc, ||c||^2) stored row-major [nq][nlist]
// Every mbarrier wait is bounded; on expiry the kernel records an error code and
// every role leaves its loop, so the CTA always reaches the TMEM deallocation.
#include <cuda.h>
#include <cuda_bf16.h>

#include <cstdint>
#include <cstdio>

#include "common.cuh"
#include "kernels.h"

namespace hanns {
namespace {

constexpr int kTM = 128, kTN = 256, kTK = 64;  // tile; kTK bf16 = 128 bytes (one swizzle row)
constexpr int kStagesTC = 2;
constexpr int kABytes = kTM * kTK * 2;  // 16 KiB
constexpr int kBBytes = kTN * kTK * 2;  // 32 KiB
// stage layout: A hi | A lo | B hi | B lo (each 1024-byte aligned)
constexpr int kStageBytes = 2 * kABytes + 2 * kBBytes;
constexpr int kTcThreads = 192;
constexpr uint32_t kWaitLimit = 1u << 26;  // bounded spins (seconds), then error

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for the phase with the given parity: gives up after kWaitLimit polls or
// 2 seconds, whichever comes first; false on expiry.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t addr = smem_u32(bar);
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0; it < kWaitLimit; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        if (done) return true;
        if ((it & 255) == 255 && global_ns() - t0 > 2000000000ull) return false;
    }
    return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar,
                                            int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
        "{%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

// K-major operand, 128-byte swizzle: rows of 128 B, 8-row (1024 B) swizzle atoms.
// start >> 4 in [0,14), LBO=1 (16 B units) in [16,30), SBO=1024 B in [32,46),
// version 1 in [46,48), layout type 2 (SWIZZLE_128B) in [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D f32 (bit 4), A bf16 (bits 7-9 = 1), B bf16
// (bits 10-12 = 1), both K-major, N>>3 at bit 17, M>>4 at bit 24.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTN >> 3) << 17) |
                            ((uint32_t)(kTM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
        "%28, %29, %30, %31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
          "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
          "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

struct TcMaps {
    CUtensorMap qh, ql, ch, cl;
};

__global__ void __launch_bounds__(kTcThreads, 1) coarse_tc_kernel(
    const __grid_constant__ TcMaps maps, int64_t nq, int nlist, int kblocks /* K / 64 */,
    const float* __restrict__ cn, float* __restrict__ out, int* __restrict__ err_flag) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStagesTC * kStageBytes);
    uint64_t* empty = full + kStagesTC;
    uint64_t* acc_full = empty + kStagesTC;
    uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(acc_full + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * kTN;
    const int64_t m0 = (int64_t)blockIdx.y * kTM;
    const int total_kb = kblocks;

    if (threadIdx.x == 0) {
        for (int s = 0; s < kStagesTC; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(acc_full, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(tmem_holder)),
                     "r"(kTN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = *tmem_holder;

    if (warp == 0) {
        if (lane == 0) {
            for (int kb = 0; kb < total_kb && !*abort_flag; ++kb) {
                const int s = kb % kStagesTC;
                const int round = kb / kStagesTC;
                if (round > 0 && !mbar_wait(&empty[s], (round - 1) & 1)) {
                    *abort_flag = 1;
                    atomicExch(err_flag, 1);
                    break;
                }
                const int kk = kb * kTK;
                uint8_t* dst = smem + s * kStageBytes;
                mbar_expect_tx(&full[s], kStageBytes);
                tma_load_2d(dst, &maps.qh, &full[s], kk, (int)m0);
                tma_load_2d(dst + kABytes, &maps.ql, &full[s], kk, (int)m0);
                tma_load_2d(dst + 2 * kABytes, &maps.ch, &full[s], kk, n0);
                tma_load_2d(dst + 2 * kABytes + kBBytes, &maps.cl, &full[s], kk, n0);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            for (int kb = 0; kb < total_kb && !*abort_flag; ++kb) {
                const int s = kb % kStagesTC;
                if (!mbar_wait(&full[s], (kb / kStagesTC) & 1)) {
                    *abort_flag = 1;
                    atomicExch(err_flag, 2);
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                const uint32_t ah = smem_u32(smem + s * kStageBytes);
                const uint32_t al = ah + kABytes;
                const uint32_t bh = ah + 2 * kABytes;
                const uint32_t bl = bh + kBBytes;
#pragma unroll
                for (int k = 0; k < kTK / 16; ++k) {  // K16 steps = 32 bytes inside the swizzle row
                    umma_f16(tmem, sw128_desc(ah + k * 32), sw128_desc(bh + k * 32),
                             (kb > 0 || k > 0) ? 1u : 0u);
                    umma_f16(tmem, sw128_desc(ah + k * 32), sw128_desc(bl + k * 32), 1u);
                    umma_f16(tmem, sw128_desc(al + k * 32), sw128_desc(bh + k * 32), 1u);
                }
                umma_commit(&empty[s]);
            }
            umma_commit(acc_full);
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32*(w%4) .. +31 = tile rows
        const int quad = warp & 3;
        const bool ok = mbar_wait(acc_full, 0);
        if (!ok) {
            *abort_flag = 1;
            atomicExch(err_flag, 3);
        } else {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const int row = quad * 32 + lane;
            const int64_t qrow = m0 + row;
            const bool vec = (nlist & 3) == 0;
#pragma unroll 1
            for (int c0 = 0; c0 < kTN; c0 += 32) {
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)c0, v);
                if (qrow < nq) {
                    float* orow = out + qrow * (int64_t)nlist;
                    const int cbase = n0 + c0;
                    if (vec && cbase + 32 <= nlist) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) {
                            const float4 c4 = __ldg(reinterpret_cast<const float4*>(cn + cbase + j));
                            float4 o;
                            o.x = __fmaf_rn(-2.0f, __uint_as_float(v[j + 0]), c4.x);
                            o.y = __fmaf_rn(-2.0f, __uint_as_float(v[j + 1]), c4.y);
                            o.z = __fmaf_rn(-2.0f, __uint_as_float(v[j + 2]), c4.z);
                            o.w = __fmaf_rn(-2.0f, __uint_as_float(v[j + 3]), c4.w);
                            *reinterpret_cast<float4*>(orow + cbase + j) = o;
                        }
                    } else {
                        for (int j = 0; j < 32; ++j)
                            if (cbase + j < nlist)
                                orow[cbase + j] =
                                    __fmaf_rn(-2.0f, __uint_as_float(v[j]), cn[cbase + j]);
                    }
                }
            }
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 1) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTN)
                     : "memory");
    }
}

// x [rows][d] f32 -> hi, lo [rows][K] bf16 (zero padded), x = hi + lo + r.
__global__ void split_bf16_kernel(const float* __restrict__ x, int64_t rows, int d, int K,
                                  __nv_bfloat16* __restrict__ hi, __nv_bfloat16* __restrict__ lo) {
    const int64_t total = rows * K;
    for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
         e += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = e / K;
        const int k = (int)(e % K);
        const float v = k < d ? x[r * d + k] : 0.0f;
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        hi[e] = h;
        lo[e] = __float2bfloat16_rn(__fsub_rn(v, __bfloat162float(h)));
    }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    }
    return fn;
}

bool make_map(CUtensorMap* m, const void* base, int64_t rows, int K, int box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTK, (cuuint32_t)box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
              estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

int coarse_tc_k(int d) { return (d + kTK - 1) / kTK * kTK; }

void launch_split_bf16(const float* x, int64_t rows, int d, int K, void* hi, void* lo,
                       cudaStream_t s) {
    if (rows <= 0) return;
    int64_t blocks = (rows * K + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    split_bf16_kernel<<<(unsigned)blocks, 256, 0, s>>>(x, rows, d, K,
                                                       static_cast<__nv_bfloat16*>(hi),
                                                       static_cast<__nv_bfloat16*>(lo));
}

// Returns false (nothing launched) when the tensor maps cannot be encoded.
bool launch_coarse_tc(const void* qh, const void* ql, int64_t nq, const void* ch, const void* cl,
                      int nlist, int K, const float* cn, float* out, int* err_flag,
                      cudaStream_t s) {
    if (nq <= 0) return true;
    TcMaps maps;
    if (!make_map(&maps.qh, qh, nq, K, kTM) || !make_map(&maps.ql, ql, nq, K, kTM) ||
        !make_map(&maps.ch, ch, nlist, K, kTN) || !make_map(&maps.cl, cl, nlist, K, kTN))
        return false;
    const size_t smem = (size_t)kStagesTC * kStageBytes + 1024 + 256;
    cudaFuncSetAttribute(coarse_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    dim3 grid((nlist + kTN - 1) / kTN, (unsigned)((nq + kTM - 1) / kTM));
    coarse_tc_kernel<<<grid, kTcThreads, smem, s>>>(maps, nq, nlist, K / kTK, cn, out, err_flag);
    return true;
}

}  // namespace hanns
