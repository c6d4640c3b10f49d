// k_noalloc.cu -- greedy argmax for callers that cannot allocate device memory.
//
// aexis_cuda_argmax keeps its per-row 64-bit keys in the context's scratch
// buffer, which the context allocates with cudaMalloc on first use. Some
// callers of this library cannot do that: a host engine that owns every byte
// of device memory through its own allocator (a game engine's graphics
// interop path, for instance), or a per-frame callback that must never block,
// where cudaMalloc / cudaFree may synchronise the whole device. For them,
// aexis_cuda_argmax_static runs the same two-pass argmax with its keys in a
// fixed array compiled into this library, needs no context, and allocates
// nothing.
#include <atomic>
#include <mutex>

#include "aexis_internal.h"

#define AEXIS_API extern "C" __attribute__((visibility("default")))

namespace {

// The keys live here. Every GPU that loads the library holds this array
// (AEXIS_ARGMAX_STATIC_MAX_ROWS * 8 bytes) until the process exits.
__device__ __align__(256) unsigned long long g_static_keys[AEXIS_ARGMAX_STATIC_MAX_ROWS];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
std::atomic<void*> g_keys_addr[kMaxDevices] = {};
int g_sm_count[kMaxDevices] = {};

// Per-device set-up, once, with that device current: the device address of
// the key array (host code may not use g_static_keys itself; its host name
// is only a stand-in) and the SM count used to size the grid.
int setup_device(int dev) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_keys_addr[dev].load()) return AEXIS_OK;
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_static_keys) != cudaSuccess || !p) return AEXIS_E_CUDA;
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
        return AEXIS_E_CUDA;
    g_sm_count[dev] = sms;
    g_keys_addr[dev].store(p);
    return AEXIS_OK;
}

}  // namespace

AEXIS_API int aexis_cuda_argmax_static(const float* logits, int rows, int width, int ld, int32_t* out_idx,
                                       void* cuda_stream) {
    if (!logits || !out_idx) return AEXIS_E_NULL;
    if (width <= 0 || rows <= 0) return AEXIS_E_RANGE;
    if (rows > AEXIS_ARGMAX_STATIC_MAX_ROWS) return AEXIS_E_RANGE;
    if (ld < width) return AEXIS_E_SHAPE;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return AEXIS_E_CUDA;
    void* keys = g_keys_addr[dev].load();
    if (!keys) {
        const int rc = setup_device(dev);
        if (rc) return rc;
        keys = g_keys_addr[dev].load();
    }
    // The same kernels as aexis_cuda_argmax: the keys are cleared on the
    // stream (cudaMemsetAsync allocates nothing), then max-reduced, decoded.
    const cudaError_t e = launch_argmax(logits, rows, width, ld, out_idx,
                                        static_cast<unsigned long long*>(keys), g_sm_count[dev],
                                        static_cast<cudaStream_t>(cuda_stream));
    return e == cudaSuccess ? AEXIS_OK : AEXIS_E_CUDA;
}
