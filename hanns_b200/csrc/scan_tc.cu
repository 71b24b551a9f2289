// scan_tc.cu -- list scan on the sm_100a tensor cores.
//
// One persistent CTA per SM takes items: one list of at most kTcMaxRows rows and the
// queries that probe it (tc_queries_per_item: up to 128 for a FastScan list, kTcItemCols /
// T for a rerank-only one).  The list's rows are the MMA's M side, in T tiles of 128; the
// item's queries are its N side (N = queries rounded up to 16).  The GEMMs run over groups
// of G = min(T, 256 / N) row tiles, so one group's accumulators fill at most one TMEM half.
// Both integer stages of the reference's search are int8 GEMMs (tcgen05.mma kind::i8, int32
// accumulation in TMEM, exact):
//
//   FastScan   raw[v][i] = sum_g LUT_i[g][nib_g(v)]                    (fastscan.rs:170-227)
//              = onehot(v) . LUT_i over K = 16 G bytes: A = one-hot rows (u8 0/1, one
//              16-byte group per 4 dimensions, built in shared memory from the sign bits),
//              B = the queries' LUTs as stored (offset-binary u8: every row has exactly
//              one 1 per group, so the sum exceeds the signed-LUT sum by 128 G, which the
//              epilogue subtracts).  The int32 sum wrapped to 16 bits equals the reference's
//              i16 wraparound accumulation.  Only lists longer than n_cand.
//   rerank     int_ip[v][i] = sum_d code_u8[v][d] * q_i8[i][d] over K = D bytes
//              (quantizer.rs:382-400): A = the codes unpacked to one byte per dimension
//              in q_i8p's order (4-bit codes: per 8 dimensions the 4 even, then the 4
//              odd ones -- the low and the high nibbles of a 32-bit code word), B = q_i8p.
//
// Per group, the FastScan GEMM (G x N accumulator columns <= 256) fills one half of the
// 512 TMEM columns and the rerank GEMM the other half; consecutive GEMMs alternate halves,
// so one GEMM overlaps the epilogue of the one before.  A list's one-hot rows and codes are
// built once for up to 128 queries (the B stages -- the queries' operands -- are reloaded
// per group instead).  A FastScan item's epilogue streams
// every (row, query) score and int_ip to the FastScan scratch, from which fs_select_kernel
// (search_kernels.cu, a warp per pair at full occupancy) takes the reference's heap kept set
// (fastscan.rs:86-146) and the kept rows' distances.  A rerank-only item keeps every live
// row: its epilogue writes each kept row's distance key and tie key (rank << 48 | position)
// to the query's candidate region.
//
// Operands stream through two rings of 32 KiB stages (128 rows x 256 K bytes: two 128-byte
// swizzle atoms, K-major): A (kNA slots, the row tiles) and B (kNB slots, the queries).  Per
// GEMM and K slab the MMA consumes one B stage and then the group's A stages.  Each A slot
// has two builder warps (64 rows each) and each B slot one; a builder fills its slot's
// positions in ring order, so every wait of a builder on its slot's empty barrier is for
// the phase right after the last one it saw.
//
// Warp roles (19 warps, 96 registers each):
//   warps 0-5   A builders, two per slot.  One-hot rows (sign bytes loaded into registers
//               before the slot is free, then expanded), 4-bit codes (the warp's first
//               round of raw bytes loaded, the other prefetched into L1, unpacked), 8-bit
//               codes (cp.async straight into their swizzled places)
//   warp 6      TMEM allocation and the MMA issuer (the whole warp runs the loop with
//               warp-uniform descriptors; one elected lane issues the MMAs and commits)
//   warp 7      item scheduler: takes items, fills the item slots, prefetches the next
//               item's list into L2
//   warps 8-15  epilogue (thread per row, warp w on TMEM lanes 32 (w % 4) .., warps w and
//               w + 4 on the two halves of the item's query columns): FastScan items'
//               scores and int_ip TMEM -> the FastScan scratch; rerank-only items' kept
//               rows (bitmaps) and their distances and ties
//   warps 16-18 B builders: the queries' LUT or q_i8p slab rows, cp.async
//               Copies complete on the slot's full barrier (cp.async.mbarrier.arrive): a
//               builder never waits for them.
// Every wait is bounded (wait_ns, 2 s by default): on expiry the kernel records an error
// code, every role leaves its loop, the MMAs already issued complete, and the TMEM is
// freed.
#include <cstdint>

#include "common.cuh"
#include "kernels.h"

namespace hanns {
namespace {

constexpr int kNA = 3, kNB = 3;                   // ring slots
constexpr int kAW = 2;                            // builder warps per A slot (64 rows each)
constexpr int kAWarps = kNA * kAW;                // warps 0-5: A builders
constexpr int kMmaWarp = kAWarps;                 // 6
constexpr int kSchedWarp = kMmaWarp + 1;          // 7
constexpr int kEpiWarp0 = kSchedWarp + 1;         // 8-15: epilogue, two per TMEM lane quarter
constexpr int kEpiWarps = 8;
constexpr int kBWarp0 = kEpiWarp0 + kEpiWarps;    // 16-18: B builders, one per B slot
constexpr int kBuildWarps = kAWarps + kNB;        // 9
constexpr int kRB = 128 / 32 / kAW;               // 32-row blocks per A builder warp
constexpr int kThreads = (kBWarp0 + kNB) * 32;    // 608
static_assert(kEpiWarp0 % 4 == 0, "epilogue warp w reads TMEM lanes 32 (w % 4) ..");
constexpr int kRows = 128;                        // MMA M: list rows per tile
constexpr int kMaxQ = 128;                        // queries per item
constexpr int kHalfCols = 256;                    // TMEM columns of one GEMM
constexpr int kTmemCols = 2 * kHalfCols;
constexpr int kAtom = 128;                        // K bytes of one 128-byte swizzle atom
constexpr int kAtomBytes = kRows * kAtom;         // 16 KiB: 128 rows of one atom
constexpr int kSlab = 2 * kAtom;                  // K bytes per stage (two atoms)
constexpr int kStageBytes = 2 * kAtomBytes;       // 32 KiB
constexpr int kWordCap = kTcItemCols * 4;         // kept-row bitmap words (rerank-only items): N * T * 4
constexpr int kSlots = 2;                         // items in flight
constexpr uint32_t kWaitLimit = 1u << 24;
static_assert(kTcItemCols <= kHalfCols, "one GEMM's accumulators fill at most one TMEM half");
static_assert(kTcMaxRows / kRows * 16 <= kTcItemCols, "an item holds at least 16 queries");

// kind::i8 instruction descriptor: D s32 (bits 4-5 = 2), A u8 (bits 7-9 = 0), B u8 (0) or
// s8 (1) at bits 10-12, both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__device__ __forceinline__ uint32_t idesc_i8(int n, bool b_signed) {
    return (2u << 4) | (0u << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(kRows >> 4) << 24);
}

struct ItemSlot {
    int item, n, nq, T;  // item < 0: no more work
    int N, fs, list, pad;
    int64_t beg;
    int q[kMaxQ], rank[kMaxQ], bsi[kMaxQ];
    int64_t base[kMaxQ];  // candidate region of each query's (query, probe) pair
    int64_t fsb[kMaxQ];   // FastScan items: the pair's place in the FastScan scratch
    // the query constants of the rerank distance (QueryParams fields)
    float q_scale[kMaxQ], centroid_score[kMaxQ], q_norm_sq[kMaxQ];
    int q_i8_sum[kMaxQ];
};

struct TcSmem {
    uint32_t bitmap[kWordCap];  // kept rows of rerank-only items [query][word], word stride T * 4
    int prefix[kWordCap];       // kept rows before each bitmap word
    ItemSlot slot[kSlots];
    uint64_t a_full[kNA], a_empty[kNA], b_full[kNB], b_empty[kNB];
    uint64_t item_full[kSlots], item_empty[kSlots];
    uint64_t acc_full[2], acc_free[2];  // per TMEM half: a GEMM done / read out
    uint64_t drain;  // the MMA issuer's last commit: every MMA it issued has completed
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

// Arrives on the barrier once this thread's cp.async copies issued so far have landed.
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait for the phase with the given parity: try_wait suspends the thread in
// hardware between checks; gives up after limit_ns, kWaitLimit tries, or once another role
// raised the abort flag.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t limit_ns) {
    const uint32_t addr = smem_u32(bar);
    auto try_wait = [&]() {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(addr), "r"(parity)
            : "memory");
        return done != 0;
    };
    if (try_wait()) return true;  // (most waits: no timer read)
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0; it < kWaitLimit; ++it) {
        if (try_wait()) return true;
        if (*abort || global_ns() - t0 > limit_ns) return false;
    }
    return false;
}

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// The descriptor of K step k4 (32 bytes) of a stage whose descriptor is d: atom k4 / 4
// (kAtomBytes further), 32 (k4 % 4) bytes into it; the start address field counts
// 16-byte units.
__device__ __forceinline__ uint64_t desc_k(uint64_t d, int k4) {
    return d + (uint64_t)((k4 >> 2) * (kAtomBytes >> 4) + 2 * (k4 & 3));
}

// D (+)= A B^T, kind::i8 (u8 A; u8 or s8 B by idesc), issued by the one lane elect.sync
// picks (the lowest active lane) while the whole warp executes the instruction with
// warp-uniform operands.
__device__ __forceinline__ void umma_i8_elect(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p, e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// tcgen05.commit by the elected lane: the barrier's phase completes once every MMA that
// lane issued so far has completed.
__device__ __forceinline__ void umma_commit_elect(uint64_t* bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7])
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

// Byte offset of the 16-byte K chunk c (0..15) of row r inside a stage: chunks 0-7 in the
// first 128-byte-swizzled atom (128 rows x 128 bytes), chunks 8-15 in the second.
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
    return (uint32_t)(c >> 3) * (uint32_t)kAtomBytes + (uint32_t)r * 128u + ((uint32_t)((c & 7) ^ (r & 7)) << 4);
}

__device__ __forceinline__ bool filtered(const uint64_t* words, int64_t len, int64_t id) {
    const uint64_t u = (uint64_t)id;
    if (u >= (uint64_t)len) return false;
    return (words[u >> 6] >> (u & 63)) & 1ull;
}

// One-hot row chunk of a 4-bit FastScan nibble: byte `nib` of the 16 is 1.
__device__ __forceinline__ uint4 onehot16(uint32_t nib) {
    const uint32_t bit = 1u << (8 * (nib & 3u));
    const uint32_t w = nib >> 2;
    return make_uint4(w == 0 ? bit : 0u, w == 1 ? bit : 0u, w == 2 ? bit : 0u, w == 3 ? bit : 0u);
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

// Hint: the byte range [p, p + bytes) into L2 (p and bytes multiples of 16, bytes > 0).
__device__ __forceinline__ void l2_prefetch(const void* p, uint64_t bytes) {
    const uint64_t cap = 1ull << 20;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p),
                 "r"((uint32_t)(bytes < cap ? bytes : cap))
                 : "memory");
}

// Time-breakdown counters (a.prof, per CTA; ns of the globaltimer, one lane per role):
//   0 builder item loop (warp 0)  1 its empty-slot waits  2 its item waits
//   3 MMA full-stage waits  4 MMA accumulator-free waits  5 MMA item loop
//   6 epilogue accumulator waits  7 FastScan copy-out  8 selection  9 rerank epilogue
//   10 epilogue item waits  11 epilogue item loop  12 items  13 stages  14 the part of 3
//   spent on B stages
enum ProfSlot { kPBuild, kPBuildWaitSlot, kPBuildWaitItem, kPMmaWaitFull, kPMmaWaitFree, kPMma,
                kPEpiWaitAcc, kPEpiCopy, kPEpiSelect, kPEpiRerank, kPEpiWaitItem, kPEpi, kPItems,
                kPStages, kPMmaWaitB };

__global__ void __launch_bounds__(kThreads, 1) scan_tc_kernel(TcScanArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // (pointer arithmetic on the shared array: the compiler keeps every access below in the
    // shared state space)
    uint8_t* const ring_a = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* const ring_b = ring_a + kNA * kStageBytes;
    TcSmem& sm = *reinterpret_cast<TcSmem*>(ring_b + kNB * kStageBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool l2 = a.metric_l2 != 0;
    const int fs_slabs = a.D / 64;                   // K = 16 G = 4 D bytes
    const int rr_slabs = (a.D + kSlab - 1) / kSlab;  // K = D bytes

    if (tid == 0) {
        for (int s = 0; s < kNA; ++s) {
            mbar_init(&sm.a_full[s], 32 * kAW);  // the builder warps' lanes
            mbar_init(&sm.a_empty[s], 1);
        }
        for (int s = 0; s < kNB; ++s) {
            mbar_init(&sm.b_full[s], 32);
            mbar_init(&sm.b_empty[s], 1);
        }
        for (int s = 0; s < kSlots; ++s) {
            mbar_init(&sm.item_full[s], 1);
            mbar_init(&sm.item_empty[s], kBuildWarps + 1 + kEpiWarps);
        }
        for (int h = 0; h < 2; ++h) {
            mbar_init(&sm.acc_full[h], 1);
            mbar_init(&sm.acc_free[h], kEpiWarps);
        }
        mbar_init(&sm.drain, 1);
        sm.abort = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kMmaWarp) {
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
    const uint64_t wl = a.wait_ns;
    unsigned long long* const prof = a.prof ? a.prof + (int64_t)blockIdx.x * kTcProfSlots : nullptr;
    // a profiling lane adds the time since t to a counter of its role (kept in a register;
    // each role's profiling lane stores its counters once, after its loop)
    auto padd = [&](bool mine, uint64_t& acc, uint64_t t) {
        if (prof && mine) acc += global_ns() - t;
    };
    auto fail = [&](int code) {
        if (!sm.abort) atomicExch(a.err_flag, code);
        sm.abort = 1;
    };

    if (warp < kAWarps || warp >= kBWarp0) {
        // ------------------------------------------------------------ builders
        const bool is_b = warp >= kBWarp0;
        const int my = is_b ? warp - kBWarp0 : warp / kAW;  // the ring slot this warp fills
        const int part = is_b ? 0 : warp % kAW;              // A: rows 64 part .. + 63
        const int ns = is_b ? kNB : kNA;
        uint64_t* const full = is_b ? &sm.b_full[my] : &sm.a_full[my];
        uint64_t* const empty = is_b ? &sm.b_empty[my] : &sm.a_empty[my];
        uint8_t* const X = (is_b ? ring_b : ring_a) + my * kStageBytes;
        const uint32_t xs = smem_u32(X);
        const bool pl = warp == 0 && lane == 0;  // the builders' profiling lane
        uint64_t p_loop = 0, p_wslot = 0, p_witem = 0, p_items = 0, p_stages = 0;
        uint32_t gpos = 0;  // ring position of the item's first stage in this warp's ring
        for (int j = 0;; ++j) {
            const int si = j % kSlots;
            const ItemSlot& S = sm.slot[si];
            const uint64_t t_item = prof ? global_ns() : 0;
            const bool got = __all_sync(0xffffffffu, mbar_wait(&sm.item_full[si], (j / kSlots) & 1, &sm.abort, wl));
            padd(pl, p_witem, t_item);
            if (!got) {
                fail(5);
                break;
            }
            if (S.item < 0) break;
            const int n = S.n, nq = S.nq, N = S.N, T = S.T;
            const int64_t beg = S.beg;
            const int fss = S.fs ? fs_slabs : 0;
            // this ring's stages of the item, group by group (G row tiles per GEMM): B per
            // slab, A per slab and row tile of the group
            const int G = min(T, kHalfCols / N), ngr = (T + G - 1) / G, nsl = fss + rr_slabs;
            const int nst = is_b ? nsl * ngr : nsl * T;
            const uint8_t* const fsl =
                reinterpret_cast<const uint8_t*>(a.fs + a.fs_blk_off[S.list] * (int64_t)a.nchunks * 32);
            bool ok = true;
            for (int idx = (int)(((uint32_t)my + (uint32_t)ns - gpos % (uint32_t)ns) % (uint32_t)ns); idx < nst;
                 idx += ns) {
                const uint32_t use = (gpos + (uint32_t)idx) / (uint32_t)ns;
                int sl, t = 0;
                if (is_b) {
                    sl = idx % nsl;
                } else {
                    const int g = min(idx / (nsl * G), ngr - 1);
                    const int t0 = g * G, Tg = min(G, T - t0), r = idx - g * nsl * G;
                    sl = r / Tg;
                    t = t0 + (r - sl * Tg);
                }
                const bool fsp = sl < fss;
                const int s = fsp ? sl : sl - fss;
                // the A stage's raw words, loaded before the slot is free (this warp's rows:
                // 32 k + lane for k = kRB * part .. + kRB - 1)
                uint2 wv[kRB];  // one-hot: the 8 sign bytes (64 dimensions) of each row
                uint4 c4[8];    // 4-bit codes: the first of this warp's rounds of raw bytes
                const int nj = min(8, (a.D - s * kSlab) / 32);  // 32-dimension quarters of the slab
                // 4-bit raw quarter of round rd, step m (rows r = 32 rd + 8 (m / 2) + lane / 4;
                // quarter jj = lane % 4 + 4 (m % 2)): its address and whether it exists
                auto q4src = [&](int rd, int m, bool& has) {
                    const int r = 32 * rd + 8 * (m >> 1) + (lane >> 2), jj = (lane & 3) + 4 * (m & 1);
                    const int v = t * kRows + r;
                    has = v < n && jj < nj;
                    return a.codes + (beg + v) * (int64_t)a.code_bytes + s * (kSlab / 2) + 16 * jj;
                };
                if (!is_b && fsp) {
                    // sign bytes of row v for slab s (64 dimensions): the row's 8-byte chunk s
                    // (layout [block of 32 rows][chunk][row in block])
#pragma unroll
                    for (int kk = 0; kk < kRB; ++kk) {
                        const int k = kRB * part + kk;
                        const int v = t * kRows + 32 * k + lane;
                        wv[kk] = v < n ? __ldg(reinterpret_cast<const uint2*>(
                                             fsl + ((((int64_t)(t * 4 + k) * a.nchunks + s) * 32 + lane) * 8)))
                                       : make_uint2(0u, 0u);
                    }
                } else if (!is_b && a.nbits == 4) {
                    // the warp's first round into registers, the others into L1 (loaded after
                    // the stores before)
#pragma unroll
                    for (int rr = 0; rr < kRB; ++rr)
#pragma unroll
                        for (int m = 0; m < 8; ++m) {
                            bool has;
                            const uint8_t* src = q4src(kRB * part + rr, m, has);
                            if (rr == 0)
                                c4[m] = has ? __ldg(reinterpret_cast<const uint4*>(src)) : make_uint4(0u, 0u, 0u, 0u);
                            else if (has)
                                asm volatile("prefetch.global.L1 [%0];" ::"l"(src));
                        }
                }
                const uint64_t t_w = prof ? global_ns() : 0;
                const bool freed = use == 0 || mbar_wait(empty, (use - 1) & 1, &sm.abort, wl);
                padd(pl, p_wslot, t_w);
                if (!__all_sync(0xffffffffu, freed)) {
                    ok = false;
                    break;
                }
                if (is_b) {
                    // queries' LUT (FastScan) or q_i8p (rerank) slab: lane l copies chunk
                    // c = l % 16 of queries i = l / 16, + 2, ... (padding queries: their
                    // columns are never read)
                    const int c = lane & 15;
                    const uint8_t* const src = (fsp ? a.lut : a.q_i8p) + s * kSlab + c * 16;
                    const int64_t row = fsp ? (int64_t)a.G * 16 : (int64_t)a.D;
                    const uint32_t dst = xs + (uint32_t)(c >> 3) * (uint32_t)kAtomBytes;
                    const uint32_t cx = (uint32_t)(c & 7);
                    if (fsp || s * kSlab + c * 16 < a.D) {
#pragma unroll 4
                        for (int i = lane >> 4; i < nq; i += 2)
                            cp_async16(dst + (uint32_t)i * 128u + ((cx ^ (uint32_t)(i & 7)) << 4),
                                       src + (int64_t)S.q[i] * row);
                    }
                    cp_async_arrive(full);
                } else if (fsp) {
#pragma unroll
                    for (int kk = 0; kk < kRB; ++kk) {
                        const int r = 32 * (kRB * part + kk) + lane;
                        if (t * kRows + r < n) {
#pragma unroll
                            for (int c = 0; c < 16; ++c)
                                *reinterpret_cast<uint4*>(X + sw_off(r, c)) =
                                    onehot16(((c < 8 ? wv[kk].x : wv[kk].y) >> (4 * (c & 7))) & 15u);
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive(full);
                } else if (a.nbits == 8) {
                    // 8-bit codes are the operand: straight into their swizzled places
                    for (int e = part * (kRows / kAW) * 16 + lane; e < (part + 1) * (kRows / kAW) * 16; e += 32) {
                        const int r = e >> 4, c = e & 15;
                        const int v = t * kRows + r, d = s * kSlab + c * 16;
                        if (v < n && d < a.D)
                            cp_async16(xs + sw_off(r, c), a.codes + (beg + v) * (int64_t)a.code_bytes + d);
                    }
                    cp_async_arrive(full);
                } else {
                    // 4-bit codes: a 16-byte quarter jj (32 dimensions, 4 code words of 8) becomes
                    // chunks 2 jj and 2 jj + 1: per word its low nibbles, then its high ones
#pragma unroll 1
                    for (int rd = kRB * part; rd < kRB * (part + 1); ++rd) {
                        if (rd > kRB * part) {
#pragma unroll
                            for (int m = 0; m < 8; ++m) {
                                bool has;
                                const uint8_t* src = q4src(rd, m, has);
                                c4[m] = has ? __ldg(reinterpret_cast<const uint4*>(src)) : make_uint4(0u, 0u, 0u, 0u);
                            }
                        }
#pragma unroll
                        for (int m = 0; m < 8; ++m) {
                            const int r = 32 * rd + 8 * (m >> 1) + (lane >> 2), jj = (lane & 3) + 4 * (m & 1);
                            if (t * kRows + r < n && jj < nj) {
                                const uint4 c = c4[m];
                                const uint32_t M = 0x0F0F0F0Fu;
                                *reinterpret_cast<uint4*>(X + sw_off(r, 2 * jj)) =
                                    make_uint4(c.x & M, (c.x >> 4) & M, c.y & M, (c.y >> 4) & M);
                                *reinterpret_cast<uint4*>(X + sw_off(r, 2 * jj + 1)) =
                                    make_uint4(c.z & M, (c.z >> 4) & M, c.w & M, (c.w >> 4) & M);
                            }
                        }
                    }
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    mbar_arrive(full);
                }
            }
            if (!ok) {
                fail(6);
                break;
            }
            gpos += (uint32_t)nst;
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.item_empty[si]);
            padd(pl, p_loop, t_item);
            p_items += 1;
            p_stages += (uint64_t)(nsl * (T + ngr));
        }
        if (prof && pl) {
            prof[kPBuild] = p_loop;
            prof[kPBuildWaitSlot] = p_wslot;
            prof[kPBuildWaitItem] = p_witem;
            prof[kPItems] = p_items;
            prof[kPStages] = p_stages;
        }
    } else if (warp == kMmaWarp) {
        // ------------------------------------------------------------ MMA issuer
        // The whole warp runs the loop, so the ring positions and descriptors are
        // warp-uniform values; every lane waits on the barriers (the warp proceeds only if
        // all of them saw the phase complete), and one elected lane -- the same one each
        // time -- issues the tcgen05.mma and tcgen05.commit instructions.
        {
            uint32_t ga = 0, gb = 0, uc = 0;  // ring positions, GEMMs so far
            uint64_t p_wfull = 0, p_wfree = 0, p_loop = 0, p_wb = 0;
            const bool pl = lane == 0;  // the MMA warp's profiling lane
            auto wait_all = [&](uint64_t* bar, uint32_t parity) {
                return __all_sync(0xffffffffu, mbar_wait(bar, parity, &sm.abort, wl)) != 0;
            };
            for (int j = 0;; ++j) {
                const int si = j % kSlots;
                const ItemSlot& S = sm.slot[si];
                if (!wait_all(&sm.item_full[si], (j / kSlots) & 1)) {
                    if (lane == 0) fail(7);
                    break;
                }
                if (S.item < 0) break;
                const uint64_t t_item = prof ? global_ns() : 0;
                const int N = S.N, T = S.T;
                const int G = min(T, kHalfCols / N), ngr = (T + G - 1) / G;
                bool ok = true;
                // one GEMM over a group of Tg row tiles: per slab the B stage, then the Tg A
                // stages (nk K steps of 32) into half uc & 1, once the epilogue read out the
                // GEMM two before
                auto gemm = [&](int slabs, int k_bytes, uint32_t idesc, int Tg) {
                    const uint32_t h = uc & 1, use = uc >> 1;
                    const uint32_t dcol = tmem + h * kHalfCols;
                    const uint64_t t_f = prof ? global_ns() : 0;
                    if (use >= 1 && !wait_all(&sm.acc_free[h], (use - 1) & 1)) {
                        ok = false;
                        return;
                    }
                    padd(pl, p_wfree, t_f);
                    for (int s = 0; s < slabs && ok; ++s) {
                        const uint32_t bs = gb % kNB;
                        uint64_t t_w = prof ? global_ns() : 0;
                        if (!wait_all(&sm.b_full[bs], (gb / kNB) & 1)) {
                            ok = false;
                            break;
                        }
                        padd(pl, p_wfull, t_w);
                        padd(pl, p_wb, t_w);
                        const int nk = min(kSlab, k_bytes - s * kSlab) / 32;
                        const uint64_t bd = sw128_desc(smem_u32(ring_b + bs * kStageBytes));
                        for (int t = 0; t < Tg; ++t) {
                            const uint32_t as = ga % kNA;
                            t_w = prof ? global_ns() : 0;
                            if (!wait_all(&sm.a_full[as], (ga / kNA) & 1)) {
                                ok = false;
                                break;
                            }
                            padd(pl, p_wfull, t_w);
                            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                            const uint64_t ad = sw128_desc(smem_u32(ring_a + as * kStageBytes));
                            for (int k4 = 0; k4 < nk; ++k4)
                                umma_i8_elect(dcol + (uint32_t)(t * N), desc_k(ad, k4), desc_k(bd, k4),
                                              idesc, (s > 0 || k4 > 0) ? 1u : 0u);
                            umma_commit_elect(&sm.a_empty[as]);
                            ++ga;
                        }
                        if (!ok) break;
                        umma_commit_elect(&sm.b_empty[bs]);
                        ++gb;
                    }
                    if (ok) umma_commit_elect(&sm.acc_full[h]);
                    ++uc;
                };
                for (int g = 0; g < ngr && ok; ++g) {
                    const int Tg = min(G, T - g * G);
                    if (S.fs) gemm(fs_slabs, 4 * a.D, idesc_i8(N, false), Tg);
                    if (ok) gemm(rr_slabs, a.D, idesc_i8(N, true), Tg);
                }
                if (!ok) {
                    if (lane == 0) fail(7);
                    break;
                }
                if (lane == 0) mbar_arrive(&sm.item_empty[si]);
                padd(pl, p_loop, t_item);
            }
            if (prof && pl) {
                prof[kPMmaWaitFull] = p_wfull;
                prof[kPMmaWaitFree] = p_wfree;
                prof[kPMma] = p_loop;
                prof[kPMmaWaitB] = p_wb;
            }
            // before the TMEM is freed, every MMA issued (also after an abort) completes;
            // this wait ignores the abort flag and gives up after 0.5 s
            umma_commit_elect(&sm.drain);
            int no_abort = 0;
            const bool drained = __all_sync(0xffffffffu, mbar_wait(&sm.drain, 0, &no_abort, 500000000ull)) != 0;
            if (!drained && lane == 0) fail(10);
        }
        __syncwarp();
    } else if (warp == kSchedWarp) {
        // ------------------------------------------------------------ item scheduler
        int next_it = -1;  // lane 0: the item fetched ahead
        auto fetch_item = [&]() -> int {
            for (;;) {
                const int it = atomicAdd(a.item_counter, 1);
                if (it >= *a.n_items) return it;
                // tensor-core items of non-empty lists (an empty list has no candidates)
                const int4 rec = a.items[it];
                if (rec.w == 1 && a.list_off[rec.x + 1] > a.list_off[rec.x]) return it;
            }
        };
        for (int j = 0;; ++j) {
            const int si = j % kSlots;
            ItemSlot& S = sm.slot[si];
            // publish the next item once every role released the slot
            const bool free_ok = __all_sync(
                0xffffffffu, j < kSlots || mbar_wait(&sm.item_empty[si], ((j / kSlots) - 1) & 1, &sm.abort, wl));
            if (!free_ok) {
                fail(5);
                break;
            }
            int it = 0;
            if (lane == 0) {
                it = next_it >= 0 ? next_it : fetch_item();
                next_it = it < *a.n_items ? fetch_item() : it;
                if (next_it < *a.n_items) {  // (a non-empty list)
                    // the following item's list into L2 while this one is scanned
                    const int l = a.items[next_it].x;
                    const int64_t b0 = a.list_off[l], n = a.list_off[l + 1] - b0;
                    l2_prefetch(a.codes + b0 * a.code_bytes, (uint64_t)n * a.code_bytes);
                    l2_prefetch(a.fs + a.fs_blk_off[l] * (int64_t)a.nchunks * 32,
                                (uint64_t)((n + 31) / 32) * a.nchunks * 256);
                    l2_prefetch(a.meta + b0, (uint64_t)n * 16);
                }
            }
            it = __shfl_sync(0xffffffffu, it, 0);
            const bool last = it >= *a.n_items;
            if (last) {
                if (lane == 0) S.item = -1;
            } else {
                const int4 rec = a.items[it];
                const int64_t beg = a.list_off[rec.x];
                const int n = (int)(a.list_off[rec.x + 1] - beg);
                if (lane == 0) {
                    S.item = it;
                    S.beg = beg;
                    S.n = n;
                    S.nq = rec.z;
                    S.T = (n + kRows - 1) / kRows;
                    S.N = (rec.z + 15) & ~15;
                    S.fs = n > a.n_cand ? 1 : 0;
                    S.list = rec.x;
                }
                for (int i = lane; i < rec.z; i += 32) {
                    const int2 pr = a.lq[rec.y + i];
                    S.q[i] = pr.x;
                    S.rank[i] = pr.y;
                    S.base[i] = (int64_t)pr.x * a.q_stride + a.pair_off[(int64_t)pr.x * (a.nprobe + 1) + pr.y];
                    S.fsb[i] = n > a.n_cand ? (int64_t)pr.x * a.fs_stride + a.fs_off[(int64_t)pr.x * a.nprobe + pr.y] : 0;
                    const QueryParams qp = a.qp[pr.x];
                    S.q_scale[i] = qp.q_scale;
                    S.centroid_score[i] = qp.centroid_score;
                    S.q_norm_sq[i] = qp.q_norm_sq;
                    S.q_i8_sum[i] = qp.q_i8_sum;
                    int b = -1;
                    if (a.fused && a.bitsets) {
                        b = a.query_bitset ? a.query_bitset[pr.x] : 0;
                        if (b < 0 || b >= a.n_bitsets) b = -1;
                    }
                    S.bsi[i] = b;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&sm.item_full[si]);
            if (last) break;
        }
    } else {
        // ------------------------------------------------------------ epilogue
        // Every failed wait turns into `bad`, which is ORed over the epilogue warps at the
        // next barrier; all of them leave the loop together.
        const int e = warp - kEpiWarp0;               // 0..kEpiWarps-1
        const int quarter = warp & 3, half = e >> 2;  // TMEM lanes 32*quarter.., column half
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        uint32_t uc = 0;  // GEMMs so far (the MMA issuer's count)
        const bool pl = e == 0 && lane == 0;  // the epilogue's profiling lane
        uint64_t p_wacc = 0, p_copy = 0, p_sel = 0, p_rr = 0, p_witem = 0, p_loop = 0;
        const int lut_bias = 128 * a.G;       // offset-binary LUT: the u8 sum's excess
        for (int j = 0;; ++j) {
            const int si = j % kSlots;
            const ItemSlot& S = sm.slot[si];
            const uint64_t t_item = prof ? global_ns() : 0;
            bool bad = !__all_sync(0xffffffffu, mbar_wait(&sm.item_full[si], (j / kSlots) & 1, &sm.abort, wl));
            padd(pl, p_witem, t_item);
            const uint64_t t_body = prof ? global_ns() : 0;
            if (epi_sync_or(bad)) {
                fail(8);
                break;
            }
            if (S.item < 0) break;
            const int n = S.n, nq = S.nq, N = S.N, T = S.T;
            const int64_t beg = S.beg;
            const int NP = T * kRows, W = T * 4;  // rows incl. padding, bitmap words per query
            constexpr int kEpiHalves = kEpiWarps / 4;  // warps per TMEM lane quarter
            const int c_lo = half * (N / kEpiHalves), c_hi = c_lo + N / kEpiHalves;
            // waits for the next GEMM's accumulators; false on a failed wait
            auto gemm_begin = [&](uint32_t& dcol) -> bool {
                const uint32_t h = uc & 1, use = uc >> 1;
                dcol = tmem + h * kHalfCols + lane_base;
                const uint64_t t_w = prof ? global_ns() : 0;
                const bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.acc_full[h], use & 1, &sm.abort, wl));
                padd(pl, p_wacc, t_w);
                if (ok) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                return ok;
            };
            auto gemm_end = [&]() {
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.acc_free[uc & 1]);
                ++uc;
            };
            const uint64_t t_copy = prof ? global_ns() : 0;
            if (S.fs) {
                // FastScan item, group by group of G row tiles: every row's score (16-bit wrap
                // of the signed-LUT sum) and then its int_ip to the FastScan scratch;
                // fs_select_kernel takes the kept sets
                const int G = min(T, kHalfCols / N), ngr = (T + G - 1) / G;
                for (int gg = 0; gg < 2 * ngr && !bad; ++gg) {
                    const int g = gg & 1, t0 = (gg >> 1) * G, Tg = min(G, T - t0);
                    const uint64_t t_g = prof ? global_ns() : 0;
                    uint32_t dcol;
                    if (!gemm_begin(dcol)) {
                        bad = true;
                        break;
                    }
                    for (int t = 0; t < Tg; ++t) {
                        const int v = (t0 + t) * kRows + quarter * 32 + lane;
                        for (int c = c_lo; c < c_hi && c < nq; c += 8) {
                            uint32_t x[8];
                            tmem_ld8(dcol + (uint32_t)(t * N + c), x);
                            if (v >= n) continue;
#pragma unroll
                            for (int jj = 0; jj < 8; ++jj) {
                                if (c + jj >= nq) break;
                                const int64_t o = S.fsb[c + jj] + v;
                                if (g == 0)
                                    a.fs_sc[o] = (int16_t)((int)x[jj] - lut_bias);
                                else
                                    a.fs_ip[o] = (int32_t)x[jj];
                            }
                        }
                    }
                    gemm_end();
                    padd(pl, g == 0 ? p_copy : p_rr, t_g);
                }
                if (epi_sync_or(bad)) {
                    fail(8);
                    break;
                }
                padd(pl, p_loop, t_body);
                if (lane == 0) mbar_arrive(&sm.item_empty[si]);
                continue;
            }
            const uint64_t t_sel = prof ? global_ns() : 0;
            // rerank-only item (|list| <= n_cand): every live row is kept.  The kept rows as
            // bitmap words (row v is bit v % 32 of word v / 32) with the kept rows before each
            // word: without a filter in closed form (thread per query), else a warp per query.
            {
                const int qpw = (nq + kEpiWarps - 1) / kEpiWarps;
                const int i = e * qpw + lane;
                if (lane < qpw && i < nq && S.bsi[i] < 0) {
                    for (int w = 0; w < W; ++w) {
                        const int lo = 32 * w;
                        sm.bitmap[i * W + w] = lo >= n ? 0u : (n - lo >= 32 ? 0xFFFFFFFFu : (1u << (n - lo)) - 1u);
                        sm.prefix[i * W + w] = min(lo, n);
                    }
                }
            }
            for (int i = e; i < nq; i += kEpiWarps) {
                const int bsi = S.bsi[i];
                if (bsi < 0) continue;
                const uint64_t* bw = a.bitsets + (int64_t)bsi * a.bitset_words;
                int n_c = 0;
                for (int base = 0; base < NP; base += 32) {
                    const int v = base + lane;
                    const unsigned bk =
                        __ballot_sync(0xffffffffu, v < n && !filtered(bw, a.bitset_len, a.ids[beg + v]));
                    if (lane == 0) {
                        sm.bitmap[i * W + (base >> 5)] = bk;
                        sm.prefix[i * W + (base >> 5)] = n_c;
                    }
                    n_c += __popc(bk);
                }
                // unused entries of the pair's region of |list| entries (rows removed by the filter)
                const int64_t rb = S.base[i];
                for (int jj = n_c + lane; jj < n; jj += 32) {
                    a.cand_tie[rb + jj] = ~0ull;
                    a.cand_key[rb + jj] = 0xFFFFFFFFu;
                }
            }
            bad = epi_sync_or(false);  // (every bitmap is visible after it)
            padd(pl, p_sel, t_sel);
            const uint64_t t_rr = prof ? global_ns() : 0;
            // rerank: thread per row, the distance and tie keys of the kept (query, row) pairs
            uint32_t dcol;
            if (!bad && !gemm_begin(dcol)) bad = true;
            if (!bad) {
                for (int t = 0; t < T; ++t) {
                    const int v = t * kRows + quarter * 32 + lane;
                    const bool row_ok = v < n;
                    const float4 m = row_ok ? __ldg(a.meta + beg + v) : make_float4(0.f, 0.f, 0.f, 0.f);
                    const int wi = t * 4 + quarter;
                    const uint32_t below = (1u << lane) - 1u;
                    for (int c = c_lo; c < c_hi && c < nq; c += 8) {
                        uint32_t ip[8];
                        tmem_ld8(dcol + (uint32_t)(t * N + c), ip);
                        // the 8 queries are independent: every load is unconditional (query
                        // index clamped), only the distance and its stores are predicated
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) {
                            const int i = min(c + jj, nq - 1);
                            const uint32_t word = sm.bitmap[i * W + wi];
                            const int pos = sm.prefix[i * W + wi] + __popc(word & below);
                            QueryParams qp;
                            qp.q_scale = S.q_scale[i];
                            qp.centroid_score = S.centroid_score[i];
                            qp.q_norm_sq = S.q_norm_sq[i];
                            qp.q_i8_sum = S.q_i8_sum[i];
                            const int64_t dst = S.base[i] + pos;
                            const uint64_t rank_bits = (uint64_t)S.rank[i] << 48;
                            if (row_ok && c + jj < nq && ((word >> lane) & 1u)) {
                                const float dist = rerank_distance((int)ip[jj], m, qp, a.nbits, l2);
                                a.cand_key[dst] = total_order_key(dist);
                                a.cand_tie[dst] = rank_bits | (uint32_t)v;  // (no FastScan key)
                                if (a.cand_dbg) a.cand_dbg[dst] = make_int2((int)ip[jj], INT32_MIN);
                            }
                        }
                    }
                }
                gemm_end();
            }
            // the next item rewrites the scores and bitmaps
            if (epi_sync_or(bad)) {
                fail(9);
                break;
            }
            padd(pl, p_rr, t_rr);
            padd(pl, p_loop, t_body);
            if (lane == 0) mbar_arrive(&sm.item_empty[si]);
        }
        if (prof && pl) {
            prof[kPEpiWaitAcc] = p_wacc;
            prof[kPEpiCopy] = p_copy;
            prof[kPEpiSelect] = p_sel;
            prof[kPEpiRerank] = p_rr;
            prof[kPEpiWaitItem] = p_witem;
            prof[kPEpi] = p_loop;
        }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
    __syncthreads();
    if (warp == kMmaWarp) {
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                     "r"(kTmemCols)
                     : "memory");
    }
}

}  // namespace

size_t scan_tc_smem_bytes() { return (size_t)(kNA + kNB) * kStageBytes + sizeof(TcSmem) + 1024; }

void launch_scan_tc(const TcScanArgs& a, int grid, cudaStream_t s) {
    const size_t smem = scan_tc_smem_bytes();
    HANNS_CUDA_OK(cudaFuncSetAttribute(scan_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    scan_tc_kernel<<<grid, kThreads, smem, s>>>(a);
    HANNS_CUDA_OK(cudaGetLastError());  // a launch the resources refuse fails here, not silently
}

}  // namespace hanns
