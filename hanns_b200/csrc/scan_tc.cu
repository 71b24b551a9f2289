// scan_tc.cu -- list scan on the sm_100a tensor cores.
//
// One persistent CTA per SM takes items: one list of at most kTcMaxRows rows and up to 128
// of the queries that probe it.  The list's rows are the MMA's M side, in T tiles of 128;
// the item's queries are its N side (N = queries rounded up to 16).  Both integer stages of
// the reference's search are int8 GEMMs (tcgen05.mma kind::i8, int32 accumulation in TMEM,
// exact):
//
//   FastScan   raw[v][i] = sum_g LUT_i[g][nib_g(v)]                    (fastscan.rs:170-227)
//              = onehot(v) . LUT_i over K = 16 G bytes: A = one-hot rows (u8 0/1, one
//              16-byte group per 4 dimensions, built in shared memory from the sign bits),
//              B = the queries' LUTs (s8).  The int32 sum wrapped to 16 bits equals the
//              reference's i16 wraparound accumulation.  Only lists longer than n_cand.
//   rerank     int_ip[v][i] = sum_d code_u8[v][d] * q_i8[i][d] over K = D bytes
//              (quantizer.rs:382-400): A = the codes unpacked to one byte per dimension,
//              B = the queries' q_i8 in dimension order.
//
// An item's row tiles are processed in groups of Tg = 256 / N tiles ("units"): a unit's
// accumulators (Tg x N columns) fill one half of the 512 TMEM columns, and consecutive
// units alternate halves, so the GEMMs of one unit overlap the epilogue of the previous
// one.  Each one-hot / code row is built once per item; the queries' slab is built once
// per unit.  An item runs its FastScan units, then (after the kept sets are known) its
// rerank units.  The kept set of each (query, list) pair is the reference's FastScan heap
// result (fastscan.rs:86-146), found with the same closed form as the SIMT scan
// (search_kernels.cu) on the 16-bit scores; as in the SIMT scan, the selection writes each
// kept row's tie key (rank << 48 | FastScan key << 32 | position) and the rerank epilogue
// its distance key to the query's candidate region.
//
// Warp roles (17 warps):
//   warps 0-7   builders: fetch items (warp 0), then write the operand stages of the item --
//               per unit and K slab of 128 bytes one B stage (the queries) and the unit's A
//               stages (its row tiles) -- into two rings (A: kNA x 16 KiB, B: kNB x 16 KiB;
//               128-byte swizzle, K-major); a warp builds a whole stage (round robin over
//               the warps) from bytes it copies in with cp.async
//   warps 8-15  epilogue: FastScan scores TMEM -> the CTA's global scratch (L2), the kept
//               set of each query (warp per query, its score row staged in shared memory)
//               with the candidates' tie keys, the distances of the kept rows (thread per
//               row)
//   warp 16     TMEM allocation and the single-thread MMA issuer
// Hand-offs are mbarriers, waited on with try_wait (the hardware suspends the waiting
// threads); every wait is bounded (wait_ns, 2 s by default): on expiry the kernel records
// an error code, every role leaves its loop, the MMAs already issued complete, and the
// TMEM is freed.
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
constexpr int kMaxQ = 128;                          // MMA N limit: queries per item
constexpr int kHalfCols = 256;                      // TMEM columns of one unit
constexpr int kTmemCols = 2 * kHalfCols;
constexpr int kSlab = 128;                          // K bytes per stage (one swizzle atom)
constexpr int kStageBytes = kRows * kSlab;          // 16 KiB
constexpr int kNA = 4, kNB = 2;                     // ring stages
constexpr int kWordCap = 4096;                      // kept-row bitmap words: N * T * 4
constexpr int kSlots = 2;                           // items in flight
constexpr uint32_t kWaitLimit = 1u << 24;
static_assert(kTcScoreScratch >= (int64_t)kMaxQ * kTcMaxRows, "score scratch of one item");
static_assert(kWordCap * 32 >= 1024 * kRows, "N * T <= 1024 (tc_queries_per_item)");

// kind::i8 instruction descriptor: D s32 (bits 4-5 = 2), A u8 (bits 7-9 = 0), B s8
// (bits 10-12 = 1), both K-major, N >> 3 at bit 17, M >> 4 at bit 24.
__device__ __forceinline__ uint32_t idesc_i8(int n) {
    return (2u << 4) | (0u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kRows >> 4) << 24);
}

struct ItemSlot {
    int item, n, nq, T;   // item < 0: no more work
    int N, fs, list, Tg;  // Tg: row tiles per unit
    int64_t beg;
    int q[kMaxQ], rank[kMaxQ], bsi[kMaxQ];
    int64_t base[kMaxQ];  // candidate region of each query's (query, probe) pair
    QueryParams qp[kMaxQ];
};

struct TcSmem {
    // one query's FastScan scores at a time per epilogue warp, double-buffered (the next
    // query's row is copied in while the current one is selected)
    int16_t stage[kEpiWarps][2][kTcMaxRows];
    uint32_t bitmap[kWordCap];  // kept rows [query][word], word stride T * 4
    int prefix[kWordCap];       // kept rows before each bitmap word
    uint32_t hist[kEpiWarps][256];
    ItemSlot slot[kSlots];
    uint64_t a_full[kNA], a_empty[kNA], b_full[kNB], b_empty[kNB];
    uint64_t item_full[kSlots], item_empty[kSlots];
    uint64_t acc_full[2], acc_free[2];  // per TMEM half: a unit's GEMMs done / read out
    uint64_t drain;  // the MMA issuer's last commit: every MMA it issued has completed
    // per ring slot: how many of its positions had their builder pass the empty wait
    uint32_t a_tick[kNA], b_tick[kNB];
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

// Bounded wait until a ring slot's ticket reaches `use`: the builder of the slot's previous
// position has passed its own empty wait.  Stages are built by several warps out of order,
// and a parity wait cannot tell the phase it waits for from the one two phases older; with
// the ticket the empty barrier has always completed the phase before the awaited one.
__device__ __forceinline__ bool ticket_wait(const volatile uint32_t* tk, uint32_t use,
                                            volatile int* abort, uint64_t limit_ns) {
    if (*tk == use) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0; it < kWaitLimit; ++it) {
        if (*tk == use) return true;
        if (*abort || global_ns() - t0 > limit_ns) return false;
        __nanosleep(20);
    }
    return false;
}

__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
    return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// The descriptor of saddr + 32 k bytes (a K step of 32 bytes inside the swizzle atom):
// the start address field counts 16-byte units.
__device__ __forceinline__ uint64_t desc_k(uint64_t d, int k4) { return d + (uint64_t)(2 * k4); }

__device__ __forceinline__ void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
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

// Byte offset of the 16-byte chunk c (0..7) of row r inside one 128-byte-swizzled slab.
__device__ __forceinline__ uint32_t sw_off(int r, int c) {
    return (uint32_t)r * 128u + ((uint32_t)(c ^ (r & 7)) << 4);
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

// dp4a-layout q_i8 (per 8 dimensions: the 4 even ones, then the 4 odd ones) to dimension
// order, 16 dimensions.
__device__ __forceinline__ uint4 q_natural(uint4 v) {
    return make_uint4(__byte_perm(v.x, v.y, 0x5140), __byte_perm(v.x, v.y, 0x7362),
                      __byte_perm(v.z, v.w, 0x5140), __byte_perm(v.z, v.w, 0x7362));
}

// The units of an item: ng groups of Tg row tiles (the last one has last_nt), first the
// FastScan units (when FastScan runs), then the rerank units.  Per unit and K slab the MMA
// consumes one B stage (the queries) and then the unit's A stages (its row tiles).
struct ItemGeo {
    int Tg, ng, last_nt, fs_slabs, rr_slabs, fs_stages;  // fs_stages: stages of all FS units
    __device__ int unit_tiles(int g) const { return g == ng - 1 ? last_nt : Tg; }
};

__device__ __forceinline__ ItemGeo item_geo(int T, int N, bool fs, int fs_slabs, int rr_slabs) {
    ItemGeo g;
    g.Tg = min(T, max(1, kHalfCols / N));
    g.ng = (T + g.Tg - 1) / g.Tg;
    g.last_nt = T - (g.ng - 1) * g.Tg;
    g.fs_slabs = fs ? fs_slabs : 0;
    g.rr_slabs = rr_slabs;
    g.fs_stages = g.fs_slabs * (g.ng + T);
    return g;
}

// Stage g of an item: kind 0 FastScan B (LUTs), 1 FastScan A (one-hot rows), 2 rerank B
// (q_i8), 3 rerank A (codes); s = K slab, t = row tile; idx = its place among the item's B
// stages (kinds 0, 2) or A stages (kinds 1, 3), i.e. its ring position after the item's first.
struct StageInfo {
    int kind, s, t, idx;
};

__device__ __forceinline__ StageInfo stage_info(int g, const ItemGeo& geo, int T) {
    const bool fs = g < geo.fs_stages;
    const int gg = fs ? g : g - geo.fs_stages;
    const int S = fs ? geo.fs_slabs : geo.rr_slabs;
    const int per_full = S * (1 + geo.Tg);
    const int grp = min(gg / per_full, geo.ng - 1);
    const int rem = gg - grp * per_full;
    const int nt = geo.unit_tiles(grp);
    StageInfo r;
    r.s = rem / (1 + nt);
    const int u = rem - r.s * (1 + nt);
    if (u == 0) {
        r.kind = fs ? 0 : 2;
        r.t = -1;
        r.idx = (fs ? 0 : geo.fs_slabs * geo.ng) + grp * S + r.s;
    } else {
        r.kind = fs ? 1 : 3;
        r.t = grp * geo.Tg + u - 1;
        r.idx = (fs ? 0 : geo.fs_slabs * T) + grp * S * geo.Tg + r.s * nt + (u - 1);
    }
    return r;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
// This lane's copies so far have landed in shared memory.
__device__ __forceinline__ void cp_async_drain() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Copies the first n scores of a score row (global, 256-byte aligned) into a staging buffer
// (shared, 16-byte aligned) with 16-byte cp.async by the 32 lanes of a warp, as one group.
__device__ __forceinline__ void stage_row(int16_t* dst, const int16_t* src, int n, int lane) {
    const uint32_t d = smem_u32(dst);
    for (int c = lane; c * 8 < n; c += 32) cp_async16(d + c * 16, src + c * 8);
    asm volatile("cp.async.commit_group;" ::: "memory");
}

// Hint: the byte range [p, p + bytes) into L2 (p and bytes multiples of 16, bytes > 0).
__device__ __forceinline__ void l2_prefetch(const void* p, uint64_t bytes) {
    const uint64_t cap = 1ull << 20;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p),
                 "r"((uint32_t)(bytes < cap ? bytes : cap))
                 : "memory");
}

// Time-breakdown counters (a.prof, per CTA; ns of the globaltimer, one lane per role):
//   0 builder item loop  1 builder empty-slot waits  2 builder item waits
//   3 MMA full-stage waits  4 MMA accumulator-free waits  5 MMA item loop
//   6 epilogue accumulator waits  7 FastScan copy-out  8 selection  9 rerank epilogue
//   10 epilogue item waits  11 epilogue item loop  12 items  13 stages
enum ProfSlot { kPBuild, kPBuildWaitSlot, kPBuildWaitItem, kPMmaWaitFull, kPMmaWaitFree, kPMma,
                kPEpiWaitAcc, kPEpiCopy, kPEpiSelect, kPEpiRerank, kPEpiWaitItem, kPEpi, kPItems,
                kPStages };

__global__ void __launch_bounds__(kThreads, 1) scan_tc_kernel(TcScanArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* ring_a = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                 ~(uintptr_t)1023);
    uint8_t* ring_b = ring_a + kNA * kStageBytes;
    TcSmem& sm = *reinterpret_cast<TcSmem*>(ring_b + kNB * kStageBytes);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const bool l2 = a.metric_l2 != 0;
    const int fs_slabs = a.D / 32;                   // K = 16 G = 4 D bytes
    const int rr_slabs = (a.D + kSlab - 1) / kSlab;  // K = D bytes
    int16_t* const sc_global = a.scores + (int64_t)blockIdx.x * kTcScoreScratch;

    if (tid == 0) {
        for (int s = 0; s < kNA; ++s) {
            mbar_init(&sm.a_full[s], 1);
            mbar_init(&sm.a_empty[s], 1);
            sm.a_tick[s] = 0;
        }
        for (int s = 0; s < kNB; ++s) {
            mbar_init(&sm.b_full[s], 1);
            mbar_init(&sm.b_empty[s], 1);
            sm.b_tick[s] = 0;
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
    const uint64_t wl = a.wait_ns;
    unsigned long long* const prof = a.prof ? a.prof + (int64_t)blockIdx.x * kTcProfSlots : nullptr;
    // a profiling lane adds the time since t to slot k
    auto padd = [&](bool mine, int k, uint64_t t) {
        if (prof && mine) prof[k] += global_ns() - t;
    };
    auto fail = [&](int code) {
        if (!sm.abort) atomicExch(a.err_flag, code);
        sm.abort = 1;
    };

    if (warp < kBuildWarps) {
        // ------------------------------------------------------------ builders
        // Warp w builds the item's stages w, w + 8, w + 16, ... whole: the raw bytes arrive
        // by cp.async in the stage's ring slot and are transformed there by the lane that
        // copied them (LUT sign flip, q_i8 to dimension order) or expanded row by row in
        // ascending rounds of 32 rows (one-hot rows from the sign words, 4-bit codes unpacked)
        // from raw bytes parked at the slot's end, which no round overwrites before reading.
        uint32_t ga = 0, gb = 0;  // ring positions of the item's first A / B stage
        int next_it = -1;         // warp 0 lane 0: the item fetched ahead
        auto fetch_item = [&]() -> int {
            for (;;) {
                const int it = atomicAdd(a.item_counter, 1);
                if (it >= *a.n_items) return it;
                // tensor-core items of non-empty lists (an empty list has no candidates)
                const int4 rec = a.items[it];
                if (rec.w == 1 && a.list_off[rec.x + 1] > a.list_off[rec.x]) return it;
            }
        };
        const bool pl = warp == 0 && lane == 0;  // the builders' profiling lane
        for (int j = 0;; ++j) {
            const int si = j % kSlots;
            ItemSlot& S = sm.slot[si];
            const uint64_t t_item = prof ? global_ns() : 0;
            if (warp == 0) {
                // publish the next item once every role released the slot
                bool free_ok = j < kSlots || mbar_wait(&sm.item_empty[si], ((j / kSlots) - 1) & 1, &sm.abort, wl);
                padd(pl, kPBuildWaitItem, t_item);
                free_ok = __all_sync(0xffffffffu, free_ok);
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
                if (it >= *a.n_items) {
                    if (lane == 0) S.item = -1;
                } else {
                    const int4 rec = a.items[it];
                    const int64_t beg = a.list_off[rec.x];
                    const int n = (int)(a.list_off[rec.x + 1] - beg);
                    if (lane == 0) {
                        const int T = (n + kRows - 1) / kRows, N = (rec.z + 15) & ~15;
                        S.item = it;
                        S.beg = beg;
                        S.n = n;
                        S.nq = rec.z;
                        S.T = T;
                        S.N = N;
                        S.fs = n > a.n_cand ? 1 : 0;
                        S.list = rec.x;
                        S.Tg = min(T, max(1, kHalfCols / N));
                    }
                    for (int i = lane; i < rec.z; i += 32) {
                        const int2 pr = a.lq[rec.y + i];
                        S.q[i] = pr.x;
                        S.rank[i] = pr.y;
                        S.base[i] = (int64_t)pr.x * a.q_stride + a.pair_off[(int64_t)pr.x * (a.nprobe + 1) + pr.y];
                        S.qp[i] = a.qp[pr.x];
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
            }
            const bool got = __all_sync(0xffffffffu, mbar_wait(&sm.item_full[si], (j / kSlots) & 1, &sm.abort, wl));
            if (!got) {
                fail(5);
                break;
            }
            if (S.item < 0) break;
            const int n = S.n, nq = S.nq, N = S.N, T = S.T;
            const int64_t beg = S.beg;
            const ItemGeo geo = item_geo(T, N, S.fs != 0, fs_slabs, rr_slabs);
            const int nb_st = (geo.fs_slabs + geo.rr_slabs) * geo.ng;  // B stages of the item
            const int na_st = (geo.fs_slabs + geo.rr_slabs) * T;       // A stages
            const int nst = na_st + nb_st;
            const uint2* fsl = a.fs + a.fs_blk_off[S.list] * (int64_t)a.nchunks * 32;
            bool ok = true;
            for (int g = warp; g < nst; g += kBuildWarps) {
                const StageInfo st = stage_info(g, geo, T);
                const bool is_b = (st.kind & 1) == 0;
                const uint32_t pos = (is_b ? gb : ga) + (uint32_t)st.idx;
                const int ns = is_b ? kNB : kNA;
                const uint32_t slot = pos % ns, use = pos / ns;
                const uint64_t t_w = prof ? global_ns() : 0;
                volatile uint32_t* tk = is_b ? &sm.b_tick[slot] : &sm.a_tick[slot];
                const bool freed = ticket_wait(tk, use, &sm.abort, wl) &&
                                   (use == 0 || mbar_wait(is_b ? &sm.b_empty[slot] : &sm.a_empty[slot],
                                                          (use - 1) & 1, &sm.abort, wl));
                padd(pl, kPBuildWaitSlot, t_w);
                if (!__all_sync(0xffffffffu, freed)) {
                    ok = false;
                    break;
                }
                if (lane == 0) {
                    __threadfence_block();
                    *tk = use + 1;  // the slot's next position may wait for this one's use
                }
                uint8_t* X = (is_b ? ring_b : ring_a) + slot * kStageBytes;
                const uint32_t xs = smem_u32(X);
                if (is_b) {
                    // queries' LUT (kind 0) or q_i8 (kind 2) slab: chunk c of query i
                    const int nch = N * 8;
                    for (int idx = lane; idx < nch; idx += 32) {
                        const int i = idx >> 3, c = idx & 7;
                        if (i >= nq) continue;  // padding query: its columns are never read
                        const int q = S.q[i];
                        if (st.kind == 0)
                            cp_async16(xs + sw_off(i, c), a.lut + ((int64_t)q * a.G * 16 + st.s * kSlab + c * 16));
                        else if (st.s * kSlab + c * 16 < a.D)
                            cp_async16(xs + sw_off(i, c), a.q_i8p + ((int64_t)q * a.D + st.s * kSlab + c * 16));
                    }
                    cp_async_drain();
                    if (st.kind == 0 || a.nbits == 4) {
                        for (int idx = lane; idx < nch; idx += 32) {
                            const int i = idx >> 3, c = idx & 7;
                            if (i >= nq || (st.kind == 2 && st.s * kSlab + c * 16 >= a.D)) continue;
                            uint4* w = reinterpret_cast<uint4*>(X + sw_off(i, c));
                            uint4 v = *w;
                            if (st.kind == 0) {  // offset-binary LUT byte -> s8
                                v.x ^= 0x80808080u;
                                v.y ^= 0x80808080u;
                                v.z ^= 0x80808080u;
                                v.w ^= 0x80808080u;
                            } else {
                                v = q_natural(v);
                            }
                            *w = v;
                        }
                    }
                } else if (st.kind == 1) {
                    // one-hot rows: the slab's sign word of each row (4 bytes) at the slot's end
                    const uint32_t raw = xs + kStageBytes - 4 * kRows;
                    for (int r = lane; r < kRows; r += 32) {
                        const int v = st.t * kRows + r;
                        if (v < n)
                            cp_async4(raw + 4 * r, reinterpret_cast<const uint8_t*>(
                                                        fsl + ((int64_t)(v >> 5) * a.nchunks + (st.s >> 1)) * 32 + (v & 31)) +
                                                        4 * (st.s & 1));
                    }
                    cp_async_drain();
                    __syncwarp();
#pragma unroll 1
                    for (int r = lane; r < kRows; r += 32) {
                        const int v = st.t * kRows + r;
                        const uint32_t word = v < n ? *reinterpret_cast<const uint32_t*>(X + kStageBytes - 4 * kRows + 4 * r) : 0u;
                        __syncwarp();  // the round's raw words are read before its rows overwrite them
                        if (v < n) {
#pragma unroll
                            for (int c = 0; c < 8; ++c)
                                *reinterpret_cast<uint4*>(X + sw_off(r, c)) = onehot16((word >> (4 * c)) & 15u);
                        }
                        __syncwarp();
                    }
                } else if (a.nbits == 8) {
                    // 8-bit codes are the operand: straight into their swizzled places
                    for (int idx = lane; idx < kRows * 8; idx += 32) {
                        const int r = idx >> 3, c = idx & 7;
                        const int v = st.t * kRows + r, d = st.s * kSlab + c * 16;
                        if (v < n && d < a.D)
                            cp_async16(xs + sw_off(r, c), a.codes + (beg + v) * (int64_t)a.code_bytes + d);
                    }
                    cp_async_drain();
                } else {
                    // 4-bit codes: the slab's 64 packed bytes of each row at the slot's second half
                    const uint32_t raw = xs + kStageBytes / 2;
                    for (int idx = lane; idx < kRows * 4; idx += 32) {
                        const int r = idx >> 2, jj = idx & 3;
                        const int v = st.t * kRows + r;
                        if (v < n && st.s * kSlab + 32 * jj < a.D)
                            cp_async16(raw + 64 * r + 16 * jj,
                                       a.codes + (beg + v) * (int64_t)a.code_bytes + st.s * (kSlab / 2) + 16 * jj);
                    }
                    cp_async_drain();
                    __syncwarp();
                    const int nj = min(4, (a.D - st.s * kSlab) / 32);  // 32-dimension quarters
#pragma unroll 1
                    for (int r = lane; r < kRows; r += 32) {
                        const int v = st.t * kRows + r;
                        uint4 c4[4];
#pragma unroll
                        for (int jj = 0; jj < 4; ++jj)
                            c4[jj] = (v < n && jj < nj) ? *reinterpret_cast<const uint4*>(X + kStageBytes / 2 + 64 * r + 16 * jj)
                                                        : make_uint4(0u, 0u, 0u, 0u);
                        __syncwarp();  // the round's raw rows are read before its rows overwrite them
                        if (v < n) {
#pragma unroll
                            for (int jj = 0; jj < 4; ++jj) {
                                if (jj >= nj) break;
                                // low nibble = even dimension: 16 code bytes -> 32 dimensions
                                const uint4 c = c4[jj];
                                const uint32_t lo0 = c.x & 0x0F0F0F0Fu, hi0 = (c.x >> 4) & 0x0F0F0F0Fu;
                                const uint32_t lo1 = c.y & 0x0F0F0F0Fu, hi1 = (c.y >> 4) & 0x0F0F0F0Fu;
                                const uint32_t lo2 = c.z & 0x0F0F0F0Fu, hi2 = (c.z >> 4) & 0x0F0F0F0Fu;
                                const uint32_t lo3 = c.w & 0x0F0F0F0Fu, hi3 = (c.w >> 4) & 0x0F0F0F0Fu;
                                *reinterpret_cast<uint4*>(X + sw_off(r, 2 * jj)) =
                                    make_uint4(__byte_perm(lo0, hi0, 0x5140), __byte_perm(lo0, hi0, 0x7362),
                                               __byte_perm(lo1, hi1, 0x5140), __byte_perm(lo1, hi1, 0x7362));
                                *reinterpret_cast<uint4*>(X + sw_off(r, 2 * jj + 1)) =
                                    make_uint4(__byte_perm(lo2, hi2, 0x5140), __byte_perm(lo2, hi2, 0x7362),
                                               __byte_perm(lo3, hi3, 0x5140), __byte_perm(lo3, hi3, 0x7362));
                            }
                        }
                        __syncwarp();
                    }
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(is_b ? &sm.b_full[slot] : &sm.a_full[slot]);
            }
            if (!ok) {
                fail(6);
                break;
            }
            ga += (uint32_t)na_st;
            gb += (uint32_t)nb_st;
            if (lane == 0) mbar_arrive(&sm.item_empty[si]);
            padd(pl, kPBuild, t_item);
            if (prof && pl) {
                prof[kPItems] += 1;
                prof[kPStages] += (unsigned long long)nst;
            }
        }
    } else if (warp == kCtrlWarp) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t ga = 0, gb = 0, uc = 0;  // ring positions, units so far
            for (int j = 0;; ++j) {
                const int si = j % kSlots;
                const ItemSlot& S = sm.slot[si];
                if (!mbar_wait(&sm.item_full[si], (j / kSlots) & 1, &sm.abort, wl)) {
                    fail(7);
                    break;
                }
                if (S.item < 0) break;
                const uint64_t t_item = prof ? global_ns() : 0;
                const int N = S.N;
                const uint32_t idesc = idesc_i8(N);
                const ItemGeo geo = item_geo(S.T, N, S.fs != 0, fs_slabs, rr_slabs);
                bool ok = true;
                // one unit: per slab the B stage then the unit's A stages (nk K-steps of 32)
                // into half uc & 1, once the epilogue read out the unit two before
                auto unit = [&](int slabs, int k_bytes, int nt) {
                    const uint32_t h = uc & 1, use = uc >> 1;
                    const uint32_t dcol = tmem + h * kHalfCols;
                    const uint64_t t_f = prof ? global_ns() : 0;
                    if (use >= 1 && !mbar_wait(&sm.acc_free[h], (use - 1) & 1, &sm.abort, wl)) {
                        ok = false;
                        return;
                    }
                    padd(true, kPMmaWaitFree, t_f);
                    for (int s = 0; s < slabs && ok; ++s) {
                        const uint32_t bs = gb % kNB;
                        uint64_t t_w = prof ? global_ns() : 0;
                        if (!mbar_wait(&sm.b_full[bs], (gb / kNB) & 1, &sm.abort, wl)) {
                            ok = false;
                            break;
                        }
                        padd(true, kPMmaWaitFull, t_w);
                        const int nk = min(kSlab, k_bytes - s * kSlab) / 32;
                        const uint64_t bd = sw128_desc(smem_u32(ring_b + bs * kStageBytes));
                        for (int t = 0; t < nt; ++t) {
                            const uint32_t as = ga % kNA;
                            t_w = prof ? global_ns() : 0;
                            if (!mbar_wait(&sm.a_full[as], (ga / kNA) & 1, &sm.abort, wl)) {
                                ok = false;
                                break;
                            }
                            padd(true, kPMmaWaitFull, t_w);
                            asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                            const uint64_t ad = sw128_desc(smem_u32(ring_a + as * kStageBytes));
                            for (int k4 = 0; k4 < nk; ++k4)
                                umma_i8(dcol + (uint32_t)(t * N), desc_k(ad, k4), desc_k(bd, k4), idesc,
                                        (s > 0 || k4 > 0) ? 1u : 0u);
                            umma_commit(&sm.a_empty[as]);
                            ++ga;
                        }
                        if (!ok) break;
                        umma_commit(&sm.b_empty[bs]);
                        ++gb;
                    }
                    if (ok) umma_commit(&sm.acc_full[h]);
                    ++uc;
                };
                for (int g = 0; g < geo.ng && ok && geo.fs_slabs > 0; ++g)
                    unit(geo.fs_slabs, 4 * a.D, geo.unit_tiles(g));
                for (int g = 0; g < geo.ng && ok; ++g) unit(geo.rr_slabs, a.D, geo.unit_tiles(g));
                if (!ok) {
                    fail(7);
                    break;
                }
                mbar_arrive(&sm.item_empty[si]);
                padd(true, kPMma, t_item);
            }
            // before the TMEM is freed, every MMA issued (also after an abort) completes;
            // this wait ignores the abort flag and gives up after 0.5 s
            umma_commit(&sm.drain);
            int no_abort = 0;
            if (!mbar_wait(&sm.drain, 0, &no_abort, 500000000ull)) fail(10);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        // Every failed wait turns into `bad`, which is ORed over the epilogue warps at the
        // next barrier; all of them leave the loop together.
        const int e = warp - kBuildWarps;             // 0..7
        const int quarter = warp & 3, half = e >> 2;  // TMEM lanes 32*quarter.., column half
        const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
        uint32_t uc = 0;  // units so far (the MMA issuer's count)
        const bool pl = e == 0 && lane == 0;  // the epilogue's profiling lane
        for (int j = 0;; ++j) {
            const int si = j % kSlots;
            const ItemSlot& S = sm.slot[si];
            const uint64_t t_item = prof ? global_ns() : 0;
            bool bad = !__all_sync(0xffffffffu, mbar_wait(&sm.item_full[si], (j / kSlots) & 1, &sm.abort, wl));
            padd(pl, kPEpiWaitItem, t_item);
            const uint64_t t_body = prof ? global_ns() : 0;
            if (epi_sync_or(bad)) {
                fail(8);
                break;
            }
            if (S.item < 0) break;
            const int n = S.n, nq = S.nq, N = S.N;
            const int64_t beg = S.beg;
            const ItemGeo geo = item_geo(S.T, N, S.fs != 0, fs_slabs, rr_slabs);
            const int NP = S.T * kRows, W = S.T * 4;  // score row stride, bitmap words per query
            int16_t* const scp = sc_global;
            const int c_lo = half * (N >> 1), c_hi = c_lo + (N >> 1);
            // waits for the next unit's accumulators; false on a failed wait
            auto unit_begin = [&](uint32_t& dcol) -> bool {
                const uint32_t h = uc & 1, use = uc >> 1;
                dcol = tmem + h * kHalfCols + lane_base;
                const uint64_t t_w = prof ? global_ns() : 0;
                const bool ok = __all_sync(0xffffffffu, mbar_wait(&sm.acc_full[h], use & 1, &sm.abort, wl));
                padd(pl, kPEpiWaitAcc, t_w);
                if (ok) asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
                return ok;
            };
            auto unit_end = [&]() {
                asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&sm.acc_free[uc & 1]);
                ++uc;
            };
            // FastScan units: scores TMEM -> the scratch (16-bit wrap)
            const uint64_t t_copy = prof ? global_ns() : 0;
            for (int g = 0; g < geo.ng && geo.fs_slabs > 0 && !bad; ++g) {
                uint32_t dcol;
                if (!unit_begin(dcol)) {
                    bad = true;
                    break;
                }
                const int t0 = g * geo.Tg, nt = geo.unit_tiles(g);
                for (int t = 0; t < nt; ++t) {
                    const int v = (t0 + t) * kRows + quarter * 32 + lane;
                    for (int c = c_lo; c < c_hi; c += 8) {
                        uint32_t v8[8];
                        tmem_ld8(dcol + (uint32_t)(t * N + c), v8);
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) scp[(c + jj) * NP + v] = (int16_t)v8[jj];
                    }
                }
                unit_end();
            }
            __threadfence();  // the scores are read back (through L2) by other warps' copies
            if (epi_sync_or(bad)) {
                fail(8);
                break;
            }
            padd(pl, kPEpiCopy, t_copy);
            const uint64_t t_sel = prof ? global_ns() : 0;
            // the kept set of each query (warp per query) and its candidates' tie keys
            int sb = 0;  // staging buffer of the current query
            if (S.fs && e < nq) stage_row(sm.stage[e][0], scp + e * NP, n, lane);
            for (int i = e; i < nq; i += kEpiWarps, sb ^= 1) {
                if (S.fs) {
                    // the next query's row into the other buffer, then wait for this one's
                    if (i + kEpiWarps < nq) {
                        stage_row(sm.stage[e][sb ^ 1], scp + (i + kEpiWarps) * NP, n, lane);
                        asm volatile("cp.async.wait_group 1;" ::: "memory");
                    } else {
                        asm volatile("cp.async.wait_group 0;" ::: "memory");
                    }
                    __syncwarp();
                }
                const int bsi = S.bsi[i];
                const uint64_t* bw = bsi >= 0 ? a.bitsets + (int64_t)bsi * a.bitset_words : nullptr;
                // the live rows, as this lane's bits: row v = lane + 32 j is bit j of lm0 (j < 32)
                // or of lm1 (j >= 32); n <= kTcMaxRows = 2048 rows
                uint32_t lm0 = 0u, lm1 = 0u;
                for (int v = lane, j = 0; v < n; v += 32, ++j)
                    if (!bw || !filtered(bw, a.bitset_len, a.ids[beg + v])) {
                        if (j < 32)
                            lm0 |= 1u << j;
                        else
                            lm1 |= 1u << (j - 32);
                    }
                auto live = [&](int v) {
                    const int j = v >> 5;
                    return (((j < 32 ? lm0 : lm1) >> (j & 31)) & 1u) != 0u;
                };
                const int n_live = __reduce_add_sync(0xffffffffu, __popc(lm0) + __popc(lm1));
                const int16_t* sv = sm.stage[e][sb];
                uint32_t* bm = sm.bitmap + i * W;
                int* px = sm.prefix + i * W;
                const int64_t rb = S.base[i];
                const uint64_t rank_bits = (uint64_t)S.rank[i] << 48;
                int n_c = 0;
                if (S.fs && n_live > a.n_cand) {
                    // s* = n_cand-th largest score among live rows (key = 32767 - score); the
                    // kept set is every row above s* plus the s*-rows the reference's heap keeps
                    auto key_at = [&](int v, uint32_t& k) {
                        if (!live(v)) return false;
                        k = (uint32_t)(32767 - (int)sv[v]);
                        return true;
                    };
                    // range-adaptive radix passes (a query's scores cluster: bins spread over
                    // the range it spans collide far less than fixed high-byte bins)
                    int c_gt = 0;
                    const uint32_t tau = warp_radix_kth(n, a.n_cand, key_at, sm.hist[e], &c_gt);
                    const int c_eq = -1;  // not counted: the boundary pass below always runs
                    // F = first n_cand rows (in list order) with score >= s*; gt_F = rows > s* in F.
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
                    for (int base = 0; base < NP; base += 32) {
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
                            bm[base >> 5] = bk;
                            px[base >> 5] = n_c;
                        }
                        if (keep) {
                            const int pos = n_c + __popc(bk & lanemask_lt());
                            if (pos < a.n_cand) {
                                a.cand_tie[rb + pos] = rank_bits | ((uint64_t)k << 32) | (uint32_t)v;
                                if (a.cand_dbg) a.cand_dbg[rb + pos].y = 32767 - (int)k;
                            }
                        }
                        n_c += __popc(bk);
                        eq_seen += __popc(beq);
                    }
                } else {
                    // every live row is kept, in list order
                    for (int base = 0; base < NP; base += 32) {
                        const int v = base + lane;
                        const bool keep = v < n && live(v);
                        const unsigned bk = __ballot_sync(0xffffffffu, keep);
                        if (lane == 0) {
                            bm[base >> 5] = bk;
                            px[base >> 5] = n_c;
                        }
                        if (keep) {
                            const int pos = n_c + __popc(bk & lanemask_lt());
                            if (pos < a.n_cand) {
                                a.cand_tie[rb + pos] = rank_bits | (uint32_t)v;
                                if (a.cand_dbg) a.cand_dbg[rb + pos].y = INT32_MIN;
                            }
                        }
                        n_c += __popc(bk);
                    }
                }
                __syncwarp();  // the staging buffer is rewritten two queries later
                n_c = min(n_c, a.n_cand);
                // unused entries of the pair's region of min(|list|, n_cand) entries (rows
                // removed by the filter)
                const int cap = min(n, a.n_cand);
                for (int jj = n_c + lane; jj < cap; jj += 32) {
                    a.cand_tie[rb + jj] = ~0ull;
                    a.cand_key[rb + jj] = 0xFFFFFFFFu;
                }
            }
            bad = epi_sync_or(false);
            padd(pl, kPEpiSelect, t_sel);
            const uint64_t t_rr = prof ? global_ns() : 0;
            // rerank units: thread per row, the distances of the kept (query, row) pairs
            for (int g = 0; g < geo.ng && !bad; ++g) {
                uint32_t dcol;
                if (!unit_begin(dcol)) {
                    bad = true;
                    break;
                }
                const int t0 = g * geo.Tg, nt = geo.unit_tiles(g);
                for (int t = 0; t < nt; ++t) {
                    const int v = (t0 + t) * kRows + quarter * 32 + lane;
                    const bool row_ok = v < n;
                    const float4 m = row_ok ? __ldg(a.meta + beg + v) : make_float4(0.f, 0.f, 0.f, 0.f);
                    const int wi = (t0 + t) * 4 + quarter;
                    const uint32_t below = (1u << lane) - 1u;
                    for (int c = c_lo; c < c_hi; c += 8) {
                        uint32_t ip[8];
                        tmem_ld8(dcol + (uint32_t)(t * N + c), ip);
                        if (!row_ok) continue;
#pragma unroll
                        for (int jj = 0; jj < 8; ++jj) {
                            const int i = c + jj;
                            if (i >= nq) break;
                            const uint32_t word = sm.bitmap[i * W + wi];
                            if (!((word >> lane) & 1u)) continue;
                            const int pos = sm.prefix[i * W + wi] + __popc(word & below);
                            if (pos >= a.n_cand) continue;
                            const float dist = rerank_distance((int)ip[jj], m, S.qp[i], a.nbits, l2);
                            const int64_t dst = S.base[i] + pos;
                            a.cand_key[dst] = total_order_key(dist);  // (its tie: the selection)
                            if (a.cand_dbg) a.cand_dbg[dst].x = (int)ip[jj];
                        }
                    }
                }
                unit_end();
            }
            // the next item rewrites the scores and bitmaps
            if (epi_sync_or(bad)) {
                fail(9);
                break;
            }
            padd(pl, kPEpiRerank, t_rr);
            padd(pl, kPEpi, t_body);
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

size_t scan_tc_smem_bytes() { return (size_t)(kNA + kNB) * kStageBytes + sizeof(TcSmem) + 1024; }

void launch_scan_tc(const TcScanArgs& a, int grid, cudaStream_t s) {
    const size_t smem = scan_tc_smem_bytes();
    cudaFuncSetAttribute(scan_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    scan_tc_kernel<<<grid, kThreads, smem, s>>>(a);
}

}  // namespace hanns
