// coarse_static.cu -- the coarse-probe step (exact L2 to every IVF centroid, then the
// nprobe nearest lists per query) for callers that cannot allocate device memory.
//
// Who needs this: a host process that hands all of its GPU memory to its own pool at
// start-up (a database or serving engine with a fixed HBM budget) must not call
// cudaMalloc behind the pool's back, and a latency-critical caller cannot afford
// cudaMalloc/cudaFree, which may synchronise the device.  The regular search path keeps
// a per-index workspace that it grows with cudaMalloc; this entry point instead uses one
// fixed scratch array that lives in the library's own device image.
//
// The scratch is a file-scope __device__ array of kStaticScratchBytes (16 MiB).  Every
// GPU that loads the library holds it until the process exits.  In host code the
// array's name is only a stand-in for the device symbol, so its device address is
// looked up with cudaGetSymbolAddress, once per device, with that device current, the
// first time the entry point runs on it; that first call should therefore happen before
// any stream capture begins.
//
// All calls share the one array and nothing in it needs to start at zero: the distance
// kernel writes every distance it later reads and the selection writes its own scratch
// before reading it.  Calls that overlap on the GPU (different streams, or different
// host threads without ordering) race on the array; order them on one stream.
#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"
#include "hanns_gpu.h"
#include "kernels.h"

namespace {

constexpr size_t kStaticScratchBytes = 16u << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

}  // namespace

// Declared in include/hanns_gpu.h.
extern "C" int32_t hanns_gpu_coarse_probes_static(const float* d_queries, int64_t nq,
                                                  const float* d_centroids, int32_t nlist,
                                                  int32_t dim, int32_t nprobe, int32_t* d_probes,
                                                  void* stream) {
    if (!d_queries || !d_centroids || !d_probes || nq <= 0 || nlist <= 0 || dim <= 0 ||
        nprobe < 1 || nprobe > nlist) {
        hanns::set_last_error("invalid argument");
        return HANNS_INVALID_ARG;
    }
    // distances [nq][nlist] f32, then selection scratch [nq][2*nprobe] u32 (256-B aligned)
    const size_t dist_bytes = ((size_t)nq * (size_t)nlist * sizeof(float) + 255) & ~(size_t)255;
    const size_t sel_bytes = (size_t)nq * 2 * (size_t)nprobe * sizeof(uint32_t);
    if (dist_bytes + sel_bytes > kStaticScratchBytes) {
        hanns::set_last_error(
            "hanns_gpu_coarse_probes_static needs " + std::to_string(dist_bytes + sel_bytes) +
            " bytes of scratch; its fixed scratch holds " + std::to_string(kStaticScratchBytes) +
            " (nq*nlist must stay below about 4 million): split the batch");
        return HANNS_INVALID_ARG;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        hanns::set_last_error("no current CUDA device");
        return HANNS_INTERNAL;
    }
    void* base = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        if (!g_scratch_ptr[dev]) {
            void* p = nullptr;
            const cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
            if (e != cudaSuccess || !p) {
                hanns::set_last_error(std::string("cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
                return HANNS_INTERNAL;
            }
            g_scratch_ptr[dev] = p;
        }
        base = g_scratch_ptr[dev];
    }
    float* dist = static_cast<float*>(base);
    uint32_t* sel = reinterpret_cast<uint32_t*>(static_cast<unsigned char*>(base) + dist_bytes);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    hanns::launch_coarse_l2(d_queries, nq, d_centroids, nlist, dim, dist, s);
    hanns::launch_select_probes(dist, nq, nlist, nprobe, d_probes, sel, s);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        hanns::set_last_error(std::string("launch failed: ") + cudaGetErrorString(e));
        return HANNS_INTERNAL;
    }
    return HANNS_OK;
}
