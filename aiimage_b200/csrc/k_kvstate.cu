// k_kvstate.cu -- conversion of the decoders' KV caches to and from the
// reference's Pack4 CDHW layout.
//
// The reference keeps each attention layer's K and V cache in a texture
// ("cache_k<i>" / "cache_v<i>" of Qwen35DecoderState, Qwen35DecoderSession.cs:
// 48-100, handed from step to step at :550-568) of logical shape
// [w = head_dim, h = positions, c = kv_heads], stored as Pack4 CDHW: element
// (x, y, c) at ((c/4 * rows + y) * head_dim + x) * 4 + (c & 3), fp32 (the
// layout AppendSequencePack4Cdhw writes, HLSL Pack4Elementwise:84-98, and
// SdpaAttentionPack4Cdhw reads). The decoders here keep one layer's cache as
// fp16 [kv_heads][cap][head_dim], optionally with each 128-byte half row's
// 16-byte chunks XOR-swizzled by position & 7 (the batched tensor-core
// attention). These kernels move one layer of one sequence between the two.
#include "decoder_internal.h"

namespace {

// Offset of dim d in a cache row of position p (see cache_dim in k_batch.cu).
__device__ __forceinline__ int kv_row_dim(int p, int d, int swz) {
    if (!swz) return d;
    const int ch = d >> 3;
    return (((ch & 8) | ((ch & 7) ^ (p & 7))) << 3) | (d & 7);
}

// out[((c/4 * rows + y) * D + x) * 4 + (c & 3)] for every x < D, y < rows,
// c < 4 * ceil(kvh / 4): the cache value for c < kvh and y < len, else 0.
// One thread per output float4 (one texel: four heads of one (x, y)).
__global__ void kv_export_kernel(const __half* __restrict__ kc, const __half* __restrict__ vc, int kvh, int cap,
                                 int D, int swz, int len, int rows, float* __restrict__ k_out,
                                 float* __restrict__ v_out) {
    const int slices = (kvh + 3) / 4;
    const long long texels = (long long)slices * rows * D;
    for (long long t = blockIdx.x * (long long)blockDim.x + threadIdx.x; t < texels;
         t += (long long)gridDim.x * blockDim.x) {
        const int x = (int)(t % D);
        const int y = (int)((t / D) % rows);
        const int sl = (int)(t / ((long long)D * rows));
        float4 kv4 = make_float4(0.f, 0.f, 0.f, 0.f), vv4 = kv4;
        float* kp = &kv4.x;
        float* vp = &vv4.x;
        if (y < len) {
#pragma unroll
            for (int lane = 0; lane < 4; ++lane) {
                const int c = sl * 4 + lane;
                if (c < kvh) {
                    const size_t off = ((size_t)c * cap + y) * D + kv_row_dim(y, x, swz);
                    kp[lane] = __half2float(kc[off]);
                    vp[lane] = __half2float(vc[off]);
                }
            }
        }
        reinterpret_cast<float4*>(k_out)[t] = kv4;
        reinterpret_cast<float4*>(v_out)[t] = vv4;
    }
}

// The inverse for positions y < len: cache = fp16 (round to nearest even) of
// the Pack4 value. Positions at and past len are left as they are.
__global__ void kv_import_kernel(const float* __restrict__ k_in, const float* __restrict__ v_in, int kvh, int cap,
                                 int D, int swz, int len, int rows, __half* __restrict__ kc, __half* __restrict__ vc) {
    const long long total = (long long)kvh * len * D;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int x = (int)(i % D);
        const int y = (int)((i / D) % len);
        const int c = (int)(i / ((long long)D * len));
        const size_t src = (((size_t)(c >> 2) * rows + y) * D + x) * 4 + (c & 3);
        const size_t dst = ((size_t)c * cap + y) * D + kv_row_dim(y, x, swz);
        kc[dst] = __float2half_rn(k_in[src]);
        vc[dst] = __float2half_rn(v_in[src]);
    }
}

int kv_grid(long long work) {
    long long b = (work + 255) / 256;
    if (b > 148LL * 16) b = 148LL * 16;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace

cudaError_t launch_kv_export(const __half* kc, const __half* vc, int kvh, int cap, int D, int swz, int len, int rows,
                             float* k_out, float* v_out, cudaStream_t s) {
    const long long texels = (long long)((kvh + 3) / 4) * rows * D;
    kv_export_kernel<<<kv_grid(texels), 256, 0, s>>>(kc, vc, kvh, cap, D, swz, len, rows, k_out, v_out);
    return cudaGetLastError();
}

cudaError_t launch_kv_import(const float* k_in, const float* v_in, int kvh, int cap, int D, int swz, int len, int rows,
                             __half* kc, __half* vc, cudaStream_t s) {
    if (len <= 0) return cudaSuccess;
    kv_import_kernel<<<kv_grid((long long)kvh * len * D), 256, 0, s>>>(k_in, v_in, kvh, cap, D, swz, len, rows, kc,
                                                                       vc);
    return cudaGetLastError();
}
