// k_topk.cu -- per-row top-k of a logit matrix in one pass over the row.
//
// Order: larger value first; equal values by ascending index (the argmax tie
// rule of AexisArgMaxPack4LinearMat, HLSL Pack4Matmul:645-686, extended to k
// entries); NaN never selected; -0 counts as +0. Every element has a unique
// 64-bit key (orderable value << 32 | ~index), so "the k largest keys" is the
// exact answer; rows with fewer than k selectable values are padded with
// (-inf, -1).
//
// One CTA of 16 warps per row. Each warp streams its share of the row with
// 128-bit loads and keeps a shared-memory buffer of candidate keys: an
// element enters only when its key beats the warp's threshold (one compare and
// one ballot per element). When the buffer nears full, the warp sorts it
// (bitonic, in shared memory), keeps its k largest and raises the threshold to
// the k-th key, so on typical rows a warp compacts a handful of times. At the
// end the warps' survivors (at most 16 k keys) are sorted together and the k
// largest written out. The row is read from memory once.
#include "aexis_internal.h"

namespace {

constexpr int kTkWarps = 16;
constexpr int kTkThreads = kTkWarps * 32;
constexpr int kTkBuf = 256;                 // candidate keys per warp
constexpr int kTkMaxK = 64;

__device__ __forceinline__ unsigned long long tk_key(float v, int i) {
    if (v != v) return 0ull;  // NaN: never selected
    const unsigned int o = aexis_orderable(v == 0.0f ? 0.0f : v);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned int)i);
}

// Warp-wide bitonic sort, descending, of buf[0, n) padded with zero keys to
// the next power of two (n <= kTkBuf).
__device__ void warp_sort_desc(unsigned long long* buf, int n, int lane) {
    int np = 32;
    while (np < n) np <<= 1;
    for (int i = n + lane; i < np; i += 32) buf[i] = 0ull;
    __syncwarp();
    for (int size = 2; size <= np; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = lane; i < np; i += 32) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long a = buf[i], b = buf[j];
                    if (desc ? (a < b) : (a > b)) {
                        buf[i] = b;
                        buf[j] = a;
                    }
                }
            }
            __syncwarp();
        }
    }
}

__global__ void __launch_bounds__(kTkThreads) topk_stream_kernel(const float* logits, int width, int ld, int k,
                                                                  float* vals, int32_t* idx) {
    __shared__ unsigned long long buf[kTkWarps][kTkBuf];
    __shared__ unsigned long long merged[kTkWarps * kTkMaxK];
    const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* x = logits + (long long)row * ld;
    unsigned long long* wb = buf[warp];
    unsigned long long thr = 0ull;  // admit keys > thr
    int cnt = 0;                    // warp-uniform
    const unsigned int lt = (1u << lane) - 1u;

    auto offer = [&](unsigned long long key) {
        const bool cand = key > thr;
        const unsigned int m = __ballot_sync(0xffffffffu, cand);
        if (m) {
            if (cand) wb[cnt + __popc(m & lt)] = key;
            cnt += __popc(m);
            if (cnt > kTkBuf - 32) {
                __syncwarp();
                warp_sort_desc(wb, cnt, lane);
                cnt = k;
                thr = wb[k - 1];
            }
        }
    };

    // Vector part: every warp takes 32 consecutive float4 per round (16-byte
    // aligned rows only); the tail and unaligned rows go element by element.
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    const int nvec = vec ? width / 4 : 0;
    for (int base = warp * 32; base < nvec; base += kTkThreads) {
        const int q = base + lane;
        float4 v = make_float4(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000), __int_as_float(0x7fc00000),
                               __int_as_float(0x7fc00000));
        if (q < nvec) v = reinterpret_cast<const float4*>(x)[q];
        offer(tk_key(v.x, 4 * q));
        offer(tk_key(v.y, 4 * q + 1));
        offer(tk_key(v.z, 4 * q + 2));
        offer(tk_key(v.w, 4 * q + 3));
    }
    for (int base = 4 * nvec + warp * 32; base < width; base += kTkThreads) {
        const int i = base + lane;
        offer(i < width ? tk_key(x[i], i) : 0ull);
    }
    // Each warp keeps its k largest.
    __syncwarp();
    if (cnt > k) {
        warp_sort_desc(wb, cnt, lane);
        cnt = k;
    }
    for (int i = lane; i < k; i += 32) merged[warp * k + i] = i < cnt ? wb[i] : 0ull;
    __syncthreads();
    // Block-wide bitonic sort of the 16 k survivors, descending.
    const int total = kTkWarps * k;
    int np = 1;
    while (np < total) np <<= 1;
    unsigned long long* all = &buf[0][0];  // reuse: np <= kTkWarps * kTkBuf
    for (int i = tid; i < np; i += kTkThreads) all[i] = i < total ? merged[i] : 0ull;
    __syncthreads();
    for (int size = 2; size <= np; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < np; i += kTkThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long a = all[i], b = all[j];
                    if (desc ? (a < b) : (a > b)) {
                        all[i] = b;
                        all[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int j = tid; j < k; j += kTkThreads) {
        const unsigned long long key = all[j];
        float* vo = vals + (long long)row * k + j;
        int32_t* io = idx + (long long)row * k + j;
        if (key != 0ull) {
            const unsigned int hi = (unsigned int)(key >> 32);
            const unsigned int bits = (hi & 0x80000000u) ? (hi & 0x7FFFFFFFu) : ~hi;
            *vo = __uint_as_float(bits);
            *io = (int32_t)(0xFFFFFFFFu - (unsigned int)(key & 0xFFFFFFFFull));
        } else {
            *vo = -INFINITY;
            *io = -1;
        }
    }
}

}  // namespace

cudaError_t launch_topk(const float* logits, int rows, int width, int ld, int k, float* vals, int32_t* idx,
                        cudaStream_t s) {
    if (k < 1 || k > kTkMaxK) return cudaErrorInvalidValue;
    topk_stream_kernel<<<rows, kTkThreads, 0, s>>>(logits, width, ld, k, vals, idx);
    return cudaGetLastError();
}
