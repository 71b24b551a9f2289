// scan_tc.cu -- list scan of the FastScan-sized lists on the sm_100a tensor cores.
//
// One persistent CTA per SM takes whole (list, <= 32 queries) items whose list is longer
// than the candidate count n_cand (so the reference runs FastScan on it) and at most
// kMaxTiles * 128 rows.  Both integer stages are int8 GEMMs (tcgen05.mma kind::i8, int32
// accumulation in TMEM, exact):
//
//   FastScan   raw[v][i] = sum_g LUT_i[g][nib_g(v)]
//              = onehot(v) . LUT_i  over K = 16 * G bytes, A = one-hot rows (u8 0/1,
//              built in shared memory from the sign bits), B = the queries' LUTs (s8).
//              The int32 sum wrapped to 16 bits equals the reference's i16 wraparound
//              accumulation (fastscan.rs:170-227).
//   rerank     int_ip[v][i] = sum_d code_u8[v][d] * q_i8[i][d] over K = D bytes, A = the
//              list's codes unpacked to one byte per dimension, B = the queries' q_i8
//              (quantizer.rs:382-400).
//
// The kept set of each (query, list) pair is the reference's FastScan heap result, found
// with the same closed form as the SIMT scan (search_kernels.cu) on the 16-bit scores;
// the rerank epilogue writes (distance key, rank << 48 | FastScan key << 32 | position)
// of every kept row to the query's candidate region, exactly like the SIMT scan.
//
// Warp roles (17 warps):
//   warps 0-7   builders: fetch items, write each 256-byte K step of the A (rows) and B
//               (queries) operands into a 3-stage ring (128-byte swizzle, K-major), the
//               global loads of step s+1 issued before the stores of step s
//   warps 8-15  epilogue: FastScan scores TMEM -> shared memory, the kept set of each
//               query, then per rerank tile the distances of the kept rows
//   warp 16     TMEM allocation and the single-thread MMA issuer
// Hand-offs are mbarriers: stage full (8 builder arrivals) / empty (tcgen05.commit),
// item slot full / empty, FastScan accumulators full / copied out, and two rerank
// accumulators full / free, so building, MMAs, selection and epilogues of consecutive
// tiles and items overlap.  Every wait is bounded (2 s); on expiry the kernel records an
// error code, every role leaves its loop, and the TMEM is freed.
#include <cstdint>

#include "common.cuh"
#include "kernels.h"
#include "warp_select.cuh"

namespace hanns {
namespace {

constexpr int kBuildWarps = 8, kEpiWarps = 8;
constexpr int kCtrlWarp = kBuildWarps + kEpiWarps;  // 16
constexpr int kThreads = (kCtrlWarp + 1) * 32;      // 544
constexpr int kRows = 128;                          // MMA M: list rows per tile
constexpr int kQ = 32;                              // MMA N: queries per item
constexpr int kSlab = 128;                          // K bytes per swizzle slab
constexpr int kStepSlabs = 2;                       // K bytes per pipeline step: 256
constexpr int kASlab = kRows * kSlab;               // 16 KiB
constexpr int kBSlab = kQ * kSlab;                  // 4 KiB
constexpr int kAStage = kASlab * kStepSlabs;        // 32 KiB
constexpr int kStageBytes = kAStage + kBSlab * kStepSlabs;  // 40 KiB
constexpr int kNS = 3;                              // stages
constexpr int kMaxTiles = 8;                        // FastScan accumulators resident in TMEM
constexpr int kMaxRows = kMaxTiles * kRows;         // 1024
constexpr int kTmemCols = 512;
constexpr int kIpCol0 = kMaxTiles * kQ;             // 256 and 288: rerank accumulators
constexpr int kMaxWords = kMaxRows / 32;            // kept-bitmap words per query
constexpr int kSlots = 4;                           // item slots in flight
constexpr uint32_t kWaitLimit = 1u << 26;

// kind::i8 instruction descriptor: D s32 (bits 4-5 = 2), A u8 (bits 7-9 = 0), B s8
// (bits 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdescI8 =
    (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(kQ >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

struct ItemSlot {
    int item, n, nq, pad;
    int64_t beg;
    int q[kQ], rank[kQ];
    int64_t base[kQ];  // candidate region of each query's (query, probe) pair
    QueryParams qp[kQ];
};

struct TcSmem {
    int16_t sc[kQ][kMaxRows];        // FastScan scores of the current item
    uint32_t bitmap[kQ][kMaxWords];  // kept rows per query
    int prefix[kQ][kMaxWords];       // kept rows before each bitmap word
    int used_fs[kQ];
    uint32_t hist[kEpiWarps][256];
    ItemSlot slot[kSlots];
    uint64_t full[kNS], empty[kNS];
    uint64_t item_full[kSlots], item_empty[kSlots];
    uint64_t fs_full, fs_free;
    uint64_t ip_full[2], ip_free[2];
    uint32_t tmem;
    volatile int abort;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait for the phase with the given parity (2 s or kWaitLimit polls, or until
// another role raised the abort flag).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
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
        if ((it & 255) == 255 && (*abort || global_ns() - t0 > 2000000000ull)) return false;
    }
    return false;
}

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(kIdescI8), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
        "%11, %12, %13, %14, %15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
          "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Barrier of the 8 epilogue warps that also ORs a flag over them, so that every warp
// takes the same branch after it (a failed wait never leaves a warp behind a barrier).
__device__ __forceinline__ bool epi_sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, %2, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"((uint32_t)v), "n"(kEpiWarps * 32)
        : "memory");
    return r != 0;
}

// Byte offset of the 16-byte chunk c (0..7) of row r inside one 128-byte-swizzled slab.
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
    return (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
}

__device__ __forceinline__ bool filtered(const uint64_t* words, int64_t len, int64_t id) {
    const uint64_t u = (uint64_t)id;
    if (u >= (uint64_t)len) return false;
    return (words[u >> 6] >> (u & 63)) & 1ull;
}

// Global loads of one builder thread for one pipeline step.
struct StepLoad {
    uint32_t sign;  // FastScan: 8 groups of sign nibbles
    uint4 a[8];     // rerank: the row's codes for this step
    uint4 b[2];     // the queries' LUT / q_i8 chunks
};

__global__ void __launch_bounds__(kThreads, 1) scan_tc_kernel(TcScanArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                 ~(uintptr_t)1023);
    TcSmem& sm = *reinterpret_cast<TcSmem*>(stages + kNS * kStageBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool l2 = a.metric_l2 != 0;
    const int sign_bytes = a.D / 8;
    const int nkc_fs = a.D / 64;                       // K = 16 G = 4 D bytes, 256 per step
    const int Dp = (a.D + kSlab - 1) / kSlab * kSlab;  // rerank K, zero padded
    const int slabs_rr = Dp / kSlab;
    const int nkc_rr = (slabs_rr + kStepSlabs - 1) / kStepSlabs;

    if (tid == 0) {
        for (int s = 0; s < kNS; ++s) {
            mbar_init(&sm.full[s], kBuildWarps);
            mbar_init(&sm.empty[s], 1);
        }
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&sm.item_full[s], 1);
            mbar_init(&sm.item_empty[s], 1 + kEpiWarps);
        }
        mbar_init(&sm.fs_full, 1);
        mbar_init(&sm.fs_free, kEpiWarps);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&sm.ip_full[b], 1);
            mbar_init(&sm.ip_free[b], kEpiWarps);
        }
        sm.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kCtrlWarp) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&sm.tmem)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const uint32_t tmem = sm.tmem;
    auto fail = [&](int code) {
        if (!sm.abort) atomicExch(a.err_flag, code);
        sm.abort = 1;
    };

    if (warp < kBuildWarps) {
        // ------------------------------------------------------------ builders
        const int bt = tid;                            // 0..255
        const int r = bt & (kRows - 1), h = bt >> 7;   // row, slab of the step
        uint32_t gstep = 0;
        for (int j = 0;; ++j) {
            const int si = j % kSlots;
            ItemSlot& S = sm.slot[si];
            if (warp == 0) {
                // publish the next item once every consumer released the slot
                bool free_ok = j < kSlots || mbar_wait(&sm.item_empty[si], ((j / kSlots) - 1) & 1, &sm.abort);
                free_ok = __all_sync(0xffffffffu, free_ok);
                if (!free_ok) {
                    fail(5);
                    break;
                }
                int it = 0;
                if (lane == 0) {
                    for (;;) {
                        it = atomicAdd(a.item_counter, 1);
                        if (it >= *a.n_items) break;
                        const int l = a.items[it].x;
                        const int64_t n = a.list_off[l + 1] - a.list_off[l];
                        if (n > a.n_cand && n <= kMaxRows) break;
                    }
                }
                it = __shfl_sync(0xffffffffu, it, 0);
                if (it >= *a.n_items) {
                    if (lane == 0) S.item = -1;
                } else {
                    const int4 rec = a.items[it];
                    const int64_t beg = a.list_off[rec.x];
                    if (lane == 0) {
                        S.item = it;
                        S.beg = beg;
                        S.n = (int)(a.list_off[rec.x + 1] - beg);
                        S.nq = rec.z;
                    }
                    if (lane < rec.z) {
                        const int2 pr = a.lq[rec.y + lane];
                        S.q[lane] = pr.x;
                        S.rank[lane] = pr.y;
                        S.base[lane] = (int64_t)pr.x * a.q_stride +
                                       a.pair_off[(int64_t)pr.x * (a.nprobe + 1) + pr.y];
                        S.qp[lane] = a.qp[pr.x];
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.item_full[si]);
            }
            const bool got = __all_sync(0xffffffffu, mbar_wait(&sm.item_full[si], (j / kSlots) & 1, &sm.abort));
            if (!got) {
                fail(5);
                break;
            }
            if (S.item < 0) break;
            const int n = S.n, nq = S.nq;
            const int64_t beg = S.beg;
            const int ntiles = (n + kRows - 1) / kRows;
            const int nfs = ntiles * nkc_fs, nsteps = nfs + ntiles * nkc_rr;
            auto load = [&](int st, StepLoad& L) {
                if (st < nfs) {
                    const int t = st / nkc_fs, kc = st % nkc_fs;
                    const int v = t * kRows + r;
                    L.sign = v < n ? *reinterpret_cast<const uint32_t*>(
                                         a.signs + (beg + v) * (int64_t)sign_bytes + kc * 8 + h * 4)
                                   : 0u;
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        const int idx = bt + m * 256, i = idx >> 4, cc = idx & 15;
                        L.b[m] = i < nq ? *reinterpret_cast<const uint4*>(
                                              a.lut + ((int64_t)S.q[i] * a.G + kc * 16 + cc) * 16)
                                        : make_uint4(0u, 0u, 0u, 0u);
                    }
                } else {
                    const int s2 = st - nfs, t = s2 / nkc_rr, kc = s2 % nkc_rr;
                    const int v = t * kRows + r;
                    const int d0 = kc * 256 + h * 128;  // this thread's 128 dimensions
                    const uint8_t* crow = a.codes + (beg + v) * (int64_t)a.code_bytes;
                    if (a.nbits == 8) {
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            L.a[u] = (v < n && d0 + 16 * u < a.D)
                                         ? *reinterpret_cast<const uint4*>(crow + d0 + 16 * u)
                                         : make_uint4(0u, 0u, 0u, 0u);
                    } else {
#pragma unroll
                        for (int u = 0; u < 4; ++u)
                            L.a[u] = (v < n && d0 + 32 * u < a.D)
                                         ? *reinterpret_cast<const uint4*>(crow + d0 / 2 + 16 * u)
                                         : make_uint4(0u, 0u, 0u, 0u);
                    }
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        const int idx = bt + m * 256, i = idx >> 4, cc = idx & 15;
                        const int dq = kc * 256 + cc * 16;
                        L.b[m] = (i < nq && dq < a.D)
                                     ? *reinterpret_cast<const uint4*>(a.q_i8 + (int64_t)S.q[i] * a.D + dq)
                                     : make_uint4(0u, 0u, 0u, 0u);
                    }
                }
            };
            auto build = [&](int st, const StepLoad& L, uint8_t* A) {
                uint8_t* B = A + kAStage;
                if (st < nfs) {
                    // one-hot rows: the 8 groups of this thread's slab, 16 bytes each
#pragma unroll
                    for (int jg = 0; jg < 8; ++jg) {
                        const uint32_t nib = (L.sign >> (4 * jg)) & 15u;
                        const uint32_t bit = 1u << (8 * (nib & 3u));
                        uint4 o;
                        o.x = (nib >> 2) == 0 ? bit : 0u;
                        o.y = (nib >> 2) == 1 ? bit : 0u;
                        o.z = (nib >> 2) == 2 ? bit : 0u;
                        o.w = (nib >> 2) == 3 ? bit : 0u;
                        *reinterpret_cast<uint4*>(A + h * kASlab + sw_off(r, jg)) = o;
                    }
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        const int idx = bt + m * 256, i = idx >> 4, cc = idx & 15;
                        uint4 w = L.b[m];
                        w.x ^= 0x80808080u;  // offset-binary LUT byte -> s8
                        w.y ^= 0x80808080u;
                        w.z ^= 0x80808080u;
                        w.w ^= 0x80808080u;
                        *reinterpret_cast<uint4*>(B + (cc >> 3) * kBSlab + sw_off(i, cc & 7)) = w;
                    }
                } else {
                    if (a.nbits == 8) {
#pragma unroll
                        for (int u = 0; u < 8; ++u)
                            *reinterpret_cast<uint4*>(A + h * kASlab + sw_off(r, u)) = L.a[u];
                    } else {  // 4-bit, low nibble = even dimension: 16 code bytes -> 32 dims
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const uint4 c = L.a[u];
                            const uint32_t lo0 = c.x & 0x0F0F0F0Fu, hi0 = (c.x >> 4) & 0x0F0F0F0Fu;
                            const uint32_t lo1 = c.y & 0x0F0F0F0Fu, hi1 = (c.y >> 4) & 0x0F0F0F0Fu;
                            const uint32_t lo2 = c.z & 0x0F0F0F0Fu, hi2 = (c.z >> 4) & 0x0F0F0F0Fu;
                            const uint32_t lo3 = c.w & 0x0F0F0F0Fu, hi3 = (c.w >> 4) & 0x0F0F0F0Fu;
                            *reinterpret_cast<uint4*>(A + h * kASlab + sw_off(r, 2 * u)) =
                                make_uint4(__byte_perm(lo0, hi0, 0x5140), __byte_perm(lo0, hi0, 0x7362),
                                           __byte_perm(lo1, hi1, 0x5140), __byte_perm(lo1, hi1, 0x7362));
                            *reinterpret_cast<uint4*>(A + h * kASlab + sw_off(r, 2 * u + 1)) =
                                make_uint4(__byte_perm(lo2, hi2, 0x5140), __byte_perm(lo2, hi2, 0x7362),
                                           __byte_perm(lo3, hi3, 0x5140), __byte_perm(lo3, hi3, 0x7362));
                        }
                    }
#pragma unroll
                    for (int m = 0; m < 2; ++m) {
                        const int idx = bt + m * 256, i = idx >> 4, cc = idx & 15;
                        *reinterpret_cast<uint4*>(B + (cc >> 3) * kBSlab + sw_off(i, cc & 7)) = L.b[m];
                    }
                }
            };
            StepLoad cur, nxt;
            load(0, cur);
            bool ok = true;
            for (int st = 0; st < nsteps; ++st, ++gstep) {
                if (st + 1 < nsteps) load(st + 1, nxt);
                const uint32_t s = gstep % kNS, use = gstep / kNS;
                const bool freed = use == 0 || mbar_wait(&sm.empty[s], (use - 1) & 1, &sm.abort);
                if (!__all_sync(0xffffffffu, freed)) {
                    ok = false;
                    break;
                }
                build(st, cur, stages + s * kStageBytes);
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.full[s]);
                cur = nxt;
            }
            if (!ok) {
                fail(6);
                break;
            }
        }
    } else if (warp == kCtrlWarp) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t gstep = 0, gtile = 0;
            for (int j = 0;; ++j) {
                const int si = j % kSlots;
                const ItemSlot& S = sm.slot[si];
                if (!mbar_wait(&sm.item_full[si], (j / kSlots) & 1, &sm.abort)) {
                    fail(7);
                    break;
                }
                if (S.item < 0) break;
                const int ntiles = (S.n + kRows - 1) / kRows;
                bool ok = true;
                // FastScan accumulators are free once the epilogue copied the previous item's
                if (j >= 1 && !mbar_wait(&sm.fs_free, (j - 1) & 1, &sm.abort)) ok = false;
                for (int t = 0; t < ntiles && ok; ++t)
                    for (int kc = 0; kc < nkc_fs; ++kc, ++gstep) {
                        const uint32_t s = gstep % kNS;
                        if (!mbar_wait(&sm.full[s], (gstep / kNS) & 1, &sm.abort)) {
                            ok = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const uint32_t abase = smem_u32(stages + s * kStageBytes), bbase = abase + kAStage;
                        for (int sl = 0; sl < kStepSlabs; ++sl)
#pragma unroll
                            for (int k4 = 0; k4 < kSlab / 32; ++k4)
                                umma_i8(tmem + (uint32_t)(t * kQ), sw128_desc(abase + sl * kASlab + k4 * 32),
                                        sw128_desc(bbase + sl * kBSlab + k4 * 32),
                                        (kc > 0 || sl > 0 || k4 > 0) ? 1u : 0u);
                        umma_commit(&sm.empty[s]);
                    }
                if (ok) umma_commit(&sm.fs_full);
                for (int t = 0; t < ntiles && ok; ++t, ++gtile) {
                    const uint32_t b = gtile & 1u, use = gtile >> 1;
                    if (use >= 1 && !mbar_wait(&sm.ip_free[b], (use - 1) & 1, &sm.abort)) {
                        ok = false;
                        break;
                    }
                    const uint32_t dcol = tmem + (uint32_t)(kIpCol0 + b * kQ);
                    for (int kc = 0; kc < nkc_rr; ++kc, ++gstep) {
                        const uint32_t s = gstep % kNS;
                        if (!mbar_wait(&sm.full[s], (gstep / kNS) & 1, &sm.abort)) {
                            ok = false;
                            break;
                        }
                        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                        const uint32_t abase = smem_u32(stages + s * kStageBytes), bbase = abase + kAStage;
                        const int nsl = min(kStepSlabs, slabs_rr - kc * kStepSlabs);
                        for (int sl = 0; sl < nsl; ++sl)
#pragma unroll
                            for (int k4 = 0; k4 < kSlab / 32; ++k4)
                                umma_i8(dcol, sw128_desc(abase + sl * kASlab + k4 * 32),
                                        sw128_desc(bbase + sl * kBSlab + k4 * 32),
                                        (kc > 0 || sl > 0 || k4 > 0) ? 1u : 0u);
                        umma_commit(&sm.empty[s]);
                    }
                    if (ok) umma_commit(&sm.ip_full[b]);
                }
                if (!ok) {
                    fail(7);
                    break;
                }
                mbar_arrive(&sm.item_empty[si]);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        // Every failed wait turns into `bad`, which is ORed over the epilogue warps at the
        // next barrier; all of them leave the loop together.
        const int e = warp - kBuildWarps;             // 0..7
        const int quarter = warp & 3, half = e >> 2;  // TMEM lanes 32*quarter.., queries 16*half..
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        uint32_t gtile = 0;
        for (int j = 0;; ++j) {
            const int si = j % kSlots;
            const ItemSlot& S = sm.slot[si];
            bool bad = !__all_sync(0xffffffffu, mbar_wait(&sm.item_full[si], (j / kSlots) & 1, &sm.abort));
            if (epi_sync_or(bad)) {
                fail(8);
                break;
            }
            if (S.item < 0) break;
            const int n = S.n, nq = S.nq;
            const int64_t beg = S.beg;
            const int ntiles = (n + kRows - 1) / kRows;
            // FastScan scores: TMEM -> shared memory (16-bit wrap)
            bad = !__all_sync(0xffffffffu, mbar_wait(&sm.fs_full, j & 1, &sm.abort));
            if (!bad) {
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                for (int t = 0; t < ntiles; ++t) {
                    uint32_t v16[16];
                    tmem_ld16(tmem + lane_base + (uint32_t)(t * kQ + half * 16), v16);
                    const int v = t * kRows + quarter * 32 + lane;
#pragma unroll
                    for (int jj = 0; jj < 16; ++jj) sm.sc[half * 16 + jj][v] = (int16_t)v16[jj];
                }
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.fs_free);
            }
            if (epi_sync_or(bad)) {
                fail(8);
                break;
            }
            // the kept set of each query (warp per query)
            for (int i = e; i < nq; i += kEpiWarps) {
                const int q = S.q[i];
                const uint64_t* bw = nullptr;
                if (a.fused && a.bitsets) {
                    const int b = a.query_bitset ? a.query_bitset[q] : 0;
                    if (b >= 0 && b < a.n_bitsets) bw = a.bitsets + (int64_t)b * a.bitset_words;
                }
                auto live = [&](int v) { return !bw || !filtered(bw, a.bitset_len, a.ids[beg + v]); };
                int n_live = n;
                if (bw) {
                    int c = 0;
                    for (int v = lane; v < n; v += 32) c += live(v) ? 1 : 0;
                    n_live = warp_sum(c);
                }
                const int16_t* s = sm.sc[i];
                const int npad = ntiles * kRows;
                int n_c = 0;
                if (n_live > a.n_cand) {
                    // s* = n_cand-th largest score among live rows (key = 32767 - score); the
                    // kept set is every row above s* plus the s*-rows the reference's heap keeps
                    auto key_at = [&](int v, uint32_t& k) {
                        if (!live(v)) return false;
                        k = (uint32_t)(32767 - (int)s[v]);
                        return true;
                    };
                    int c_gt = 0;
                    const uint32_t tau = warp_radix_kth(n, a.n_cand, key_at, sm.hist[e], &c_gt);
                    int cnt_ge = 0, cnt_gt = 0, p_end = n, gt_f = 0;
                    for (int base = 0; base < n; base += 32) {
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
                    const int m_drop = c_gt - gt_f;
                    int eq_seen = 0;
                    for (int base = 0; base < npad; base += 32) {
                        const int v = base + lane;
                        uint32_t k = 0xFFFFFFFFu;
                        const bool valid = v < n && key_at(v, k);
                        const bool gt = valid && k < tau;
                        const bool eq = valid && k == tau && v <= p_end;
                        const unsigned beq = __ballot_sync(0xffffffffu, eq);
                        const int eq_rank = eq_seen + __popc(beq & lanemask_le());
                        const bool keep = gt || (eq && eq_rank > m_drop);
                        const unsigned bk = __ballot_sync(0xffffffffu, keep);
                        if (lane == 0) {
                            sm.bitmap[i][base >> 5] = bk;
                            sm.prefix[i][base >> 5] = n_c;
                        }
                        n_c += __popc(bk);
                        eq_seen += __popc(beq);
                    }
                    if (lane == 0) sm.used_fs[i] = 1;
                } else {
                    for (int base = 0; base < npad; base += 32) {
                        const int v = base + lane;
                        const unsigned bk = __ballot_sync(0xffffffffu, v < n && live(v));
                        if (lane == 0) {
                            sm.bitmap[i][base >> 5] = bk;
                            sm.prefix[i][base >> 5] = n_c;
                        }
                        n_c += __popc(bk);
                    }
                    if (lane == 0) sm.used_fs[i] = 0;
                }
                n_c = min(n_c, a.n_cand);
                // unused entries of the pair's region (rows removed by the filter)
                const int64_t rb = S.base[i];
                for (int jj = n_c + lane; jj < a.n_cand; jj += 32) {
                    a.cand_tie[rb + jj] = ~0ull;
                    a.cand_key[rb + jj] = 0xFFFFFFFFu;
                }
            }
            if (epi_sync_or(false)) break;
            // rerank epilogue per tile: distances of the kept rows
            for (int t = 0; t < ntiles && !bad; ++t, ++gtile) {
                const uint32_t b = gtile & 1u, use = gtile >> 1;
                if (!__all_sync(0xffffffffu, mbar_wait(&sm.ip_full[b], use & 1, &sm.abort))) {
                    bad = true;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                uint32_t ip[16];
                tmem_ld16(tmem + lane_base + (uint32_t)(kIpCol0 + b * kQ + half * 16), ip);
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.ip_free[b]);
                const int v = t * kRows + quarter * 32 + lane;
                if (v < n) {
                    const float4 m = __ldg(a.meta + beg + v);
                    const int wi = v >> 5;
                    const uint32_t below = (1u << (v & 31)) - 1u;
#pragma unroll 4
                    for (int jj = 0; jj < 16; ++jj) {
                        const int i = half * 16 + jj;
                        if (i >= nq) break;
                        const uint32_t word = sm.bitmap[i][wi];
                        if (!((word >> (v & 31)) & 1u)) continue;
                        const int pos = sm.prefix[i][wi] + __popc(word & below);
                        if (pos >= a.n_cand) continue;
                        const uint32_t fkey = sm.used_fs[i] ? (uint32_t)(32767 - (int)sm.sc[i][v]) : 0u;
                        const float dist = rerank_distance((int)ip[jj], m, S.qp[i], a.nbits, l2);
                        const int64_t dst = S.base[i] + pos;
                        a.cand_key[dst] = total_order_key(dist);
                        a.cand_tie[dst] = ((uint64_t)S.rank[i] << 48) | ((uint64_t)fkey << 32) | (uint32_t)v;
                    }
                }
            }
            // the next item rewrites the scores and bitmaps
            if (epi_sync_or(bad)) {
                fail(9);
                break;
            }
            if (lane == 0) mbar_arrive(&sm.item_empty[si]);
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == kCtrlWarp) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

}  // namespace

int scan_tc_max_rows() { return kMaxRows; }

size_t scan_tc_smem_bytes() { return (size_t)kNS * kStageBytes + sizeof(TcSmem) + 1024; }

void launch_scan_tc(const TcScanArgs& a, int grid, cudaStream_t s) {
    const size_t smem = scan_tc_smem_bytes();
    cudaFuncSetAttribute(scan_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    scan_tc_kernel<<<grid, kThreads, smem, s>>>(a);
}

}  // namespace hanns
