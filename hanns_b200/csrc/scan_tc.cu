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
// Operands are K-major with the 128-byte swizzle (8-row, 1024-byte atoms), written by the
// CTA's threads (generic proxy) and published to the tensor core with
// fence.proxy.async.  A two-stage ring of 512-byte K chunks overlaps building chunk s+1
// with the MMAs of chunk s; tcgen05.commit on a per-stage mbarrier releases a stage.
// Every mbarrier wait is bounded (2 s); on expiry the kernel records an error code,
// leaves its item loop and frees its TMEM.
#include <cstdint>

#include "common.cuh"
#include "kernels.h"
#include "warp_select.cuh"

namespace hanns {
namespace {

constexpr int kThreads = 256;                      // 8 warps
constexpr int kRows = 128;                         // MMA M: list rows per tile
constexpr int kQ = 32;                             // MMA N: queries per item
constexpr int kSlab = 128;                         // K bytes per swizzle slab
constexpr int kChunkSlabs = 4;                     // K bytes per pipeline step: 512
constexpr int kASlab = kRows * kSlab;              // 16 KiB
constexpr int kBSlab = kQ * kSlab;                 // 4 KiB
constexpr int kAStage = kASlab * kChunkSlabs;      // 64 KiB
constexpr int kStageBytes = kAStage + kBSlab * kChunkSlabs;  // 80 KiB
constexpr int kNStages = 2;
constexpr int kMaxTiles = 14;                      // FastScan accumulators resident in TMEM
constexpr int kTmemCols = 512;
constexpr int kIpCol0 = kMaxTiles * kQ;            // 448 and 480: rerank accumulators
constexpr int kMaxWords = kMaxTiles * kRows / 32;  // kept-bitmap words per query
constexpr uint32_t kWaitLimit = 1u << 26;

// kind::i8 instruction descriptor: D s32 (bits 4-5 = 2), A u8 (bits 7-9 = 0), B s8
// (bits 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
constexpr uint32_t kIdescI8 =
    (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(kQ >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);

struct TcSmem {
    uint32_t bitmap[kQ][kMaxWords];  // kept rows per query
    int prefix[kQ][kMaxWords];       // kept rows before each bitmap word
    uint32_t hist[kThreads / 32][256];
    QueryParams qp[kQ];
    int64_t base[kQ];  // candidate region of each query's (query, probe) pair
    int q[kQ], rank[kQ], used_fs[kQ];
    uint64_t mbar[kNStages];
    uint32_t tmem;
    int item;
    int fail;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

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

// Byte offset of the 16-byte chunk c (0..7) of row r inside one 128-byte-swizzled slab.
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
    return (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
}

__device__ __forceinline__ bool filtered(const uint64_t* words, int64_t len, int64_t id) {
    const uint64_t u = (uint64_t)id;
    if (u >= (uint64_t)len) return false;
    return (words[u >> 6] >> (u & 63)) & 1ull;
}

__global__ void __launch_bounds__(kThreads, 1) scan_tc_kernel(TcScanArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* stages = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                 ~(uintptr_t)1023);
    TcSmem& sm = *reinterpret_cast<TcSmem*>(stages + kNStages * kStageBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool l2 = a.metric_l2 != 0;
    const int pstride = a.nprobe + 1;
    const int sign_bytes = a.D / 8;
    const int slabs_fs = a.D / 32;               // K = 16 G = 4 D bytes
    const int nkc_fs = (slabs_fs + kChunkSlabs - 1) / kChunkSlabs;
    const int Dp = (a.D + kSlab - 1) / kSlab * kSlab;  // rerank K, zero padded
    const int slabs_rr = Dp / kSlab;
    const int nkc_rr = (slabs_rr + kChunkSlabs - 1) / kChunkSlabs;
    const int max_rows = kMaxTiles * kRows;

    if (tid == 0) {
        for (int s = 0; s < kNStages; ++s)
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_u32(&sm.mbar[s])));
        sm.fail = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0) {
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
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;  // this warp's TMEM lanes
    const int half = warp >> 2;                                    // queries 16*half .. +15

    uint32_t step = 0;  // pipeline steps issued by this CTA (stage = step & 1)
    bool ok = true;

    // Waits until stage s may be rebuilt (its previous MMAs are complete).
    auto acquire = [&](uint32_t st) {
        const uint32_t s = st & 1u, use = st >> 1;
        bool good = true;
        if (use >= 1) good = mbar_wait(&sm.mbar[s], (use - 1) & 1u);
        return good;
    };
    // Publishes the stage written by the threads and issues its MMAs (one thread).
    auto issue = [&](uint32_t st, uint32_t tmem_d, int nslabs, bool first_chunk) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        __syncthreads();
        if (tid == 0) {
            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
            const uint32_t abase = smem_u32(stages + (st & 1u) * kStageBytes);
            const uint32_t bbase = abase + kAStage;
            for (int sl = 0; sl < nslabs; ++sl)
#pragma unroll
                for (int k4 = 0; k4 < kSlab / 32; ++k4)
                    umma_i8(tmem_d, sw128_desc(abase + sl * kASlab + k4 * 32),
                            sw128_desc(bbase + sl * kBSlab + k4 * 32),
                            (!first_chunk || sl > 0 || k4 > 0) ? 1u : 0u);
            umma_commit(&sm.mbar[st & 1u]);
        }
    };
    // Waits for the MMAs of step st (and, by commit order, every earlier one).
    auto finish = [&](uint32_t st) {
        const bool good = mbar_wait(&sm.mbar[st & 1u], (st >> 1) & 1u);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        return good;
    };

    for (;;) {
        if (tid == 0) {
            int it;
            for (;;) {
                it = atomicAdd(a.item_counter, 1);
                if (it >= *a.n_items) break;
                const int l = a.items[it].x;
                const int64_t n = a.list_off[l + 1] - a.list_off[l];
                if (n > a.n_cand && n <= max_rows) break;
            }
            sm.item = it;
        }
        __syncthreads();
        const int item = sm.item;
        if (item >= *a.n_items || !ok) break;
        const int4 it = a.items[item];
        const int l = it.x, nq_i = it.z;
        const int64_t beg = a.list_off[l];
        const int n = (int)(a.list_off[l + 1] - beg);
        const int ntiles = (n + kRows - 1) / kRows;
        if (tid < nq_i) {
            const int2 pr = a.lq[it.y + tid];
            sm.q[tid] = pr.x;
            sm.rank[tid] = pr.y;
            sm.base[tid] = (int64_t)pr.x * a.q_stride + a.pair_off[(int64_t)pr.x * pstride + pr.y];
            sm.qp[tid] = a.qp[pr.x];
        }
        // (the first issue() barrier orders these writes before their readers)

        // ---- phase 1: FastScan scores, one 32-column accumulator per 128-row tile
        for (int t = 0; t < ntiles && ok; ++t) {
            for (int kc = 0; kc < nkc_fs && ok; ++kc) {
                ok = __syncthreads_and(acquire(step));
                if (!ok) break;
                uint8_t* A = stages + (step & 1u) * kStageBytes;
                uint8_t* B = A + kAStage;
                const int nslabs = min(kChunkSlabs, slabs_fs - kc * kChunkSlabs);
                // A: one-hot rows; thread = (row, 16 groups)
                {
                    const int r = tid & (kRows - 1), hg = tid >> 7;  // hg: groups 16*hg .. +15
                    const int v = t * kRows + r;
                    const int g0 = kc * kChunkSlabs * 8 + hg * 16;     // absolute group
                    if (v < n && hg * 2 < nslabs) {
                        const uint2 sb = *reinterpret_cast<const uint2*>(
                            a.signs + (beg + v) * (int64_t)sign_bytes + g0 / 2);
#pragma unroll
                        for (int j = 0; j < 16; ++j) {
                            const uint32_t word = j < 8 ? sb.x : sb.y;
                            const uint32_t nib = (word >> (4 * (j & 7))) & 15u;
                            const int gl = hg * 16 + j;
                            uint4 o = make_uint4(0u, 0u, 0u, 0u);
                            const uint32_t bit = 1u << (8 * (nib & 3u));
                            o.x = (nib >> 2) == 0 ? bit : 0u;
                            o.y = (nib >> 2) == 1 ? bit : 0u;
                            o.z = (nib >> 2) == 2 ? bit : 0u;
                            o.w = (nib >> 2) == 3 ? bit : 0u;
                            *reinterpret_cast<uint4*>(A + (gl >> 3) * kASlab + sw_off(r, gl & 7)) = o;
                        }
                    }
                }
                // B: the queries' LUTs as s8 (offset-binary byte ^ 0x80)
                for (int idx = tid; idx < kQ * nslabs * 8; idx += kThreads) {
                    const int i = idx / (nslabs * 8), gl = idx % (nslabs * 8);
                    if (i >= nq_i) continue;
                    const int g = kc * kChunkSlabs * 8 + gl;
                    uint4 w = *reinterpret_cast<const uint4*>(a.lut + ((int64_t)sm.q[i] * a.G + g) * 16);
                    w.x ^= 0x80808080u;
                    w.y ^= 0x80808080u;
                    w.z ^= 0x80808080u;
                    w.w ^= 0x80808080u;
                    *reinterpret_cast<uint4*>(B + (gl >> 3) * kBSlab + sw_off(i, gl & 7)) = w;
                }
                issue(step, tmem + (uint32_t)(t * kQ), nslabs, kc == 0);
                ++step;
            }
        }
        if (!ok) break;
        ok = __syncthreads_and(finish(step - 1));
        if (!ok) break;

        // ---- phase 2: 16-bit scores to shared memory, then the kept set of each query
        const int npad = ntiles * kRows;
        int16_t* sc = reinterpret_cast<int16_t*>(stages);  // [kQ][npad]
        for (int t = 0; t < ntiles; ++t) {
            uint32_t v16[16];
            tmem_ld16(tmem + lane_base + (uint32_t)(t * kQ + half * 16), v16);
            const int v = t * kRows + (warp & 3) * 32 + lane;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int i = half * 16 + j;
                if (i < nq_i) sc[i * npad + v] = (int16_t)v16[j];
            }
        }
        __syncthreads();
        for (int i = warp; i < nq_i; i += kThreads / 32) {
            const int q = sm.q[i];
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
            const int16_t* s = sc + i * npad;
            int n_c = 0;
            if (n_live > a.n_cand) {
                // s* = n_cand-th largest score among live rows (key = 32767 - score); the kept
                // set is every row above s* plus the s*-rows the reference's heap retains
                auto key_at = [&](int v, uint32_t& k) {
                    if (!live(v)) return false;
                    k = (uint32_t)(32767 - (int)s[v]);
                    return true;
                };
                int c_gt = 0;
                const uint32_t tau = warp_radix_kth(n, a.n_cand, key_at, sm.hist[warp], &c_gt);
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
            const int64_t rb = sm.base[i];
            for (int j = n_c + lane; j < a.n_cand; j += 32) {
                a.cand_tie[rb + j] = ~0ull;
                a.cand_key[rb + j] = 0xFFFFFFFFu;
            }
        }
        __syncthreads();  // scores region is free again; bitmaps are complete

        // ---- phase 3: integer rerank of every tile, distances of the kept rows
        for (int t = 0; t < ntiles && ok; ++t) {
            const uint32_t ipcol = (uint32_t)(kIpCol0 + (t & 1) * kQ);
            for (int kc = 0; kc < nkc_rr && ok; ++kc) {
                ok = __syncthreads_and(acquire(step));
                if (!ok) break;
                uint8_t* A = stages + (step & 1u) * kStageBytes;
                uint8_t* B = A + kAStage;
                const int nslabs = min(kChunkSlabs, slabs_rr - kc * kChunkSlabs);
                // A: codes, one byte per dimension; thread = (row, 16 chunks of 16 dims)
                {
                    const int r = tid & (kRows - 1), hc = tid >> 7;
                    const int v = t * kRows + r;
                    if (v < n && hc * 2 < nslabs) {
                        const uint8_t* crow = a.codes + (beg + v) * (int64_t)a.code_bytes;
                        for (int j = 0; j < 16; ++j) {
                            const int cl = hc * 16 + j;                    // chunk in the step
                            const int d0 = (kc * kChunkSlabs * 8 + cl) * 16;  // first dimension
                            uint4 o = make_uint4(0u, 0u, 0u, 0u);
                            if (d0 < a.D) {
                                if (a.nbits == 8) {
                                    o = *reinterpret_cast<const uint4*>(crow + d0);
                                } else {  // 4-bit, low nibble = even dimension
                                    const uint2 c = *reinterpret_cast<const uint2*>(crow + d0 / 2);
                                    const uint32_t lo0 = c.x & 0x0F0F0F0Fu, hi0 = (c.x >> 4) & 0x0F0F0F0Fu;
                                    const uint32_t lo1 = c.y & 0x0F0F0F0Fu, hi1 = (c.y >> 4) & 0x0F0F0F0Fu;
                                    o.x = __byte_perm(lo0, hi0, 0x5140);
                                    o.y = __byte_perm(lo0, hi0, 0x7362);
                                    o.z = __byte_perm(lo1, hi1, 0x5140);
                                    o.w = __byte_perm(lo1, hi1, 0x7362);
                                }
                            }
                            *reinterpret_cast<uint4*>(A + (cl >> 3) * kASlab + sw_off(r, cl & 7)) = o;
                        }
                    }
                }
                // B: the queries' q_i8 (natural order), zero past D
                for (int idx = tid; idx < kQ * nslabs * 8; idx += kThreads) {
                    const int i = idx / (nslabs * 8), cl = idx % (nslabs * 8);
                    if (i >= nq_i) continue;
                    const int d0 = (kc * kChunkSlabs * 8 + cl) * 16;
                    uint4 w = make_uint4(0u, 0u, 0u, 0u);
                    if (d0 < a.D) w = *reinterpret_cast<const uint4*>(a.q_i8 + (int64_t)sm.q[i] * a.D + d0);
                    *reinterpret_cast<uint4*>(B + (cl >> 3) * kBSlab + sw_off(i, cl & 7)) = w;
                }
                issue(step, tmem + ipcol, nslabs, kc == 0);
                ++step;
            }
            if (!ok) break;
            ok = __syncthreads_and(finish(step - 1));
            if (!ok) break;
            // epilogue: warp = (32 rows, 16 queries)
            uint32_t ip[16], fs[16];
            tmem_ld16(tmem + lane_base + ipcol + (uint32_t)(half * 16), ip);
            tmem_ld16(tmem + lane_base + (uint32_t)(t * kQ + half * 16), fs);
            const int v = t * kRows + (warp & 3) * 32 + lane;
            if (v < n) {
                const float4 m = __ldg(a.meta + beg + v);
                const int wi = v >> 5;
                const uint32_t below = (1u << (v & 31)) - 1u;
#pragma unroll 4
                for (int j = 0; j < 16; ++j) {
                    const int i = half * 16 + j;
                    if (i >= nq_i) break;
                    const uint32_t word = sm.bitmap[i][wi];
                    if (!((word >> (v & 31)) & 1u)) continue;
                    const int pos = sm.prefix[i][wi] + __popc(word & below);
                    if (pos >= a.n_cand) continue;
                    const uint32_t fkey =
                        sm.used_fs[i] ? (uint32_t)(32767 - (int)(int16_t)fs[j]) : 0u;
                    const float dist = rerank_distance((int)ip[j], m, sm.qp[i], a.nbits, l2);
                    const int64_t dst = sm.base[i] + pos;
                    a.cand_key[dst] = total_order_key(dist);
                    a.cand_tie[dst] = ((uint64_t)sm.rank[i] << 48) | ((uint64_t)fkey << 32) | (uint32_t)v;
                }
            }
            asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
        }
        if (!ok) break;
        __syncthreads();  // per-item shared state is rewritten by the next item
    }
    if (!ok && tid == 0) atomicExch(a.err_flag, 4);
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == 0) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

}  // namespace

int scan_tc_max_rows() { return kMaxTiles * kRows; }

size_t scan_tc_smem_bytes() { return (size_t)kNStages * kStageBytes + sizeof(TcSmem) + 1024; }

void launch_scan_tc(const TcScanArgs& a, int grid, cudaStream_t s) {
    const size_t smem = scan_tc_smem_bytes();
    cudaFuncSetAttribute(scan_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    scan_tc_kernel<<<grid, kThreads, smem, s>>>(a);
}

}  // namespace hanns
