// warp_select.cuh -- warp-level helpers shared by the search kernels: lane masks, scans,
// reductions and the radix k-th-key selection.
#pragma once

#include "common.cuh"

namespace hanns {

__device__ __forceinline__ unsigned lanemask_le() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_le;" : "=r"(m));
    return m;
}
__device__ __forceinline__ unsigned lanemask_lt() {
    unsigned m;
    asm("mov.u32 %0, %%lanemask_lt;" : "=r"(m));
    return m;
}

__device__ __forceinline__ int warp_inclusive_scan(int v) {
    const int lane = (int)lane_id();
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        int t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

__device__ __forceinline__ int warp_sum(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ uint32_t warp_min_u32(uint32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = min(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Finds the `kth` smallest key (1-based) among the valid keys produced by key_at(i) for
// i in [0, n) (at least kth of them must be valid).  Returns the key; *n_less = number of
// valid keys strictly smaller.  One pass finds the key range; the radix passes then
// resolve only the bits in which the keys differ, 8 at a time (keys of nearby scores
// share their high bytes, and a pass over equal digits would serialise every atomic on
// one bin).  hist: 256 words of shared memory owned by this warp.
template <class KeyAt>
__device__ uint32_t warp_radix_kth(int n, int kth, KeyAt key_at, uint32_t* hist, int* n_less) {
    const int lane = (int)lane_id();
    uint32_t kmin = 0xFFFFFFFFu, kmax = 0u;
    for (int i = lane; i < n; i += 32) {
        uint32_t key;
        if (key_at(i, key)) {
            kmin = min(kmin, key);
            kmax = max(kmax, key);
        }
    }
    kmin = warp_min_u32(kmin);
    kmax = warp_max_u32(kmax);
    const uint32_t range = kmax - kmin;
    uint32_t prefix = 0;  // resolved high bits of key - kmin
    int remaining = kth, less = 0;
    for (int hi = 32 - __clz(range); hi > 0; hi -= 8) {
        const int shift = hi > 8 ? hi - 8 : 0;
#pragma unroll
        for (int b = 0; b < 8; ++b) hist[lane * 8 + b] = 0;
        __syncwarp();
        for (int i = lane; i < n; i += 32) {
            uint32_t key;
            if (key_at(i, key)) {
                const uint32_t kp = key - kmin;
                if (hi >= 32 || ((kp ^ prefix) >> hi) == 0) atomicAdd(&hist[(kp >> shift) & 255u], 1u);
            }
        }
        __syncwarp();
        // this lane's 8 bins, in registers: the bin search below needs no further loads
        int hv[8], s = 0;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            hv[b] = (int)hist[lane * 8 + b];
            s += hv[b];
        }
        const int incl = warp_inclusive_scan(s);
        const unsigned hit = __ballot_sync(0xffffffffu, incl >= remaining);
        const int src = __ffs(hit) - 1;  // hit != 0 because remaining <= total
        // every lane finds the first of its bins that reaches `remaining` (the answer is src's)
        int c = incl - s, bin = 7, before = 0;
        bool found = false;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            if (!found && c + hv[b] >= remaining) {
                found = true;
                bin = b;
                before = c;
            }
            c += hv[b];
        }
        bin = __shfl_sync(0xffffffffu, lane * 8 + bin, src);
        before = __shfl_sync(0xffffffffu, before, src);
        less += before;
        remaining -= before;
        prefix |= (uint32_t)bin << shift;
        __syncwarp();
    }
    *n_less = less;
    return kmin + prefix;
}

// warp_radix_kth for keys known to lie in [0, 65535] (16-bit FastScan keys): two 8-bit
// passes, no range pass.  Same contract as warp_radix_kth; *n_equal = keys equal to the
// returned one.
template <typename KeyAt>
__device__ uint32_t warp_radix_kth16(int n, int kth, KeyAt key_at, uint32_t* hist, int* n_less,
                                     int* n_equal) {
    const int lane = (int)lane_id();
    uint32_t prefix = 0;
    int remaining = kth, less = 0;
    for (int shift = 8; shift >= 0; shift -= 8) {
#pragma unroll
        for (int b = 0; b < 8; ++b) hist[lane * 8 + b] = 0;
        __syncwarp();
        for (int i = lane; i < n; i += 32) {
            uint32_t key;
            if (key_at(i, key) && (shift == 8 || (key >> 8) == (prefix >> 8)))
                atomicAdd(&hist[(key >> shift) & 255u], 1u);
        }
        __syncwarp();
        int s = 0;
#pragma unroll
        for (int b = 0; b < 8; ++b) s += (int)hist[lane * 8 + b];
        const int incl = warp_inclusive_scan(s);
        const unsigned hit = __ballot_sync(0xffffffffu, incl >= remaining);
        const int src = __ffs(hit) - 1;  // hit != 0 because remaining <= total
        int bin = 0, before = 0;
        if (lane == src) {
            int c = incl - s;
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
        less += before;
        remaining -= before;
        prefix |= (uint32_t)bin << shift;
        __syncwarp();
    }
    *n_less = less;
    *n_equal = (int)hist[prefix & 255u];  // the last pass counted keys by their low byte
    __syncwarp();
    return prefix;
}

}  // namespace hanns
