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
#include <cuda.h>

#include <mutex>

#include "aexis_internal.h"

#define AEXIS_API extern "C" __attribute__((visibility("default")))

namespace {

// The keys live here. Every GPU that loads the library holds this array
// (AEXIS_ARGMAX_STATIC_MAX_ROWS * 8 bytes) until the process exits.
__device__ __align__(256) unsigned long long g_static_keys[AEXIS_ARGMAX_STATIC_MAX_ROWS];

// The array's device address belongs to one CUDA context: a host that makes
// its own context current (cuCtxCreate) or resets the device gets a new copy
// of the array at another address. The set-up below is therefore keyed by
// the current context's ID (cuCtxGetId: unique over the process lifetime,
// never reused), looked up through the runtime's driver entry point so the
// library needs no link against the driver library.
constexpr int kMaxDevices = 64;
struct DeviceSetup {
    unsigned long long ctx_id = 0;  // 0: not set up
    void* keys = nullptr;
    int sms = 0;
};
std::mutex g_setup_mutex;
DeviceSetup g_setup[kMaxDevices];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
CtxGetIdFn g_ctx_get_id = nullptr;

// ID of the calling thread's current context, or 0 on failure. With no
// context current yet (a caller that never used the runtime on this thread),
// cudaSetDevice makes the device's primary context current first.
unsigned long long current_context_id(int dev) {
    if (!g_ctx_get_current || !g_ctx_get_id) {
        void* f1 = nullptr;
        void* f2 = nullptr;
        cudaDriverEntryPointQueryResult q1 = cudaDriverEntryPointSymbolNotFound, q2 = q1;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f1, cudaEnableDefault, &q1) != cudaSuccess ||
            cudaGetDriverEntryPoint("cuCtxGetId", &f2, cudaEnableDefault, &q2) != cudaSuccess ||
            q1 != cudaDriverEntryPointSuccess || q2 != cudaDriverEntryPointSuccess || !f1 || !f2)
            return 0;
        g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(f1);
        g_ctx_get_id = reinterpret_cast<CtxGetIdFn>(f2);
    }
    CUcontext c = nullptr;
    unsigned long long id = 0;
    if (g_ctx_get_current(&c) != CUDA_SUCCESS) return 0;
    if (!c && (cudaSetDevice(dev) != cudaSuccess || g_ctx_get_current(&c) != CUDA_SUCCESS || !c)) return 0;
    if (g_ctx_get_id(c, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Set-up for the current device and context, with that device current: the
// device address of the key array (host code may not pass g_static_keys
// itself to a kernel; its host name is only a stand-in) and the SM count used
// to size the grid. Runs on the first call in each context.
int setup_device(int dev, DeviceSetup* out) {
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    const unsigned long long id = current_context_id(dev);
    if (!id) return AEXIS_E_CUDA;
    DeviceSetup& st = g_setup[dev];
    if (st.ctx_id != id) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_static_keys) != cudaSuccess || !p) return AEXIS_E_CUDA;
        int sms = 0;
        if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
            return AEXIS_E_CUDA;
        st.keys = p;
        st.sms = sms;
        st.ctx_id = id;
    }
    *out = st;
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
    DeviceSetup st;
    const int rc = setup_device(dev, &st);
    if (rc) return rc;
    // The same kernels as aexis_cuda_argmax: the keys are cleared on the
    // stream (cudaMemsetAsync allocates nothing), then max-reduced, decoded.
    const cudaError_t e = launch_argmax(logits, rows, width, ld, out_idx, static_cast<unsigned long long*>(st.keys),
                                        st.sms, static_cast<cudaStream_t>(cuda_stream));
    return e == cudaSuccess ? AEXIS_OK : AEXIS_E_CUDA;
}
