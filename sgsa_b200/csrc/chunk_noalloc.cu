// sgsa_chunk_fwd_noalloc: the chunked SGSA forward for callers that cannot
// allocate device memory at call time -- code that runs while the process is
// not allowed to grow its device footprint (a serving runtime with a fixed
// memory plan, a host framework whose allocator is locked, plugin code that
// is handed only its inputs and outputs).  Instead of a caller-provided
// workspace it uses one fixed scratch array compiled into this library.
//
// The scratch lives in a file-scope __device__ array, so every GPU that loads
// the library holds kNoAllocScratchBytes of device memory until the process
// exits.  Host code cannot use the array's name as a device address; the
// address is looked up with cudaGetSymbolAddress once per device, on the
// first call made with that device current (so that first call should come
// before any stream capture).  All calls share the array: calls that overlap
// on the GPU (different streams, or different host threads, same device)
// race on it and must be serialised by the caller.  Nothing in the array
// needs to start at zero: every scratch word the kernels read is written
// earlier in the same call, so what a previous call left behind is never seen.
// That is why SGSA_FLAG_REUSE_PREP is refused here: it would make the scan read
// per-chunk operands that some earlier call -- possibly another caller's
// problem -- left in the shared array.
// The device address is cached per device number for the life of the process;
// a cudaDeviceReset (or anything else that tears down the primary context and
// reloads the module) invalidates it, so this entry point must not be used
// after such a reset.
#include <mutex>
#include <stdio.h>

#include "common.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = (size_t)64 << 20;  // 64 MiB

static __device__ __align__(256) unsigned char g_chunk_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_ptr[kMaxDevices] = {};

}  // namespace

extern "C" int sgsa_chunk_fwd_noalloc(const void *q, const void *k, const void *v,
                                      const void *beta, const void *gamma, const void *sparse_k,
                                      const void *sparse_v, const void *alpha,
                                      const float *initial_state, void *o, float *final_state,
                                      int B, int T, int H, int D, int dtype, int chunk_size,
                                      int flags, void *stream) {
    if (B <= 0 || T <= 0 || H <= 0)
        return sgsa_chunk_fwd(q, k, v, beta, gamma, sparse_k, sparse_v, alpha, initial_state, o,
                              final_state, B, T, H, D, dtype, chunk_size, flags, nullptr, 0,
                              stream);
    if (flags & SGSA_FLAG_REUSE_PREP) return SGSA_ERR_UNSUPPORTED;
    const size_t need = sgsa_chunk_fwd_workspace_size(B, T, H, D, flags);
    if (need == 0) return SGSA_ERR_SHAPE;
    if (need > kNoAllocScratchBytes) return SGSA_ERR_WORKSPACE;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return SGSA_ERR_DEVICE;
    void *ptr = nullptr;
    {
        std::lock_guard<std::mutex> lock(g_mu);
        if (!g_scratch_ptr[dev]) {
            void *p = nullptr;
            if (cudaGetSymbolAddress(&p, g_chunk_scratch) != cudaSuccess || !p) {
                cudaGetLastError();
                return SGSA_ERR_LAUNCH;
            }
            g_scratch_ptr[dev] = p;
        }
        ptr = g_scratch_ptr[dev];
    }
    return sgsa_chunk_fwd(q, k, v, beta, gamma, sparse_k, sparse_v, alpha, initial_state, o,
                          final_state, B, T, H, D, dtype, chunk_size, flags, ptr,
                          kNoAllocScratchBytes, stream);
}
