// k_topk.cu -- per-row top-k of a logit matrix.
//
// Order: larger value first; equal values by ascending index (the argmax tie
// rule of AexisArgMaxPack4LinearMat, HLSL Pack4Matmul:645-686, extended to k
// entries); NaN never selected; -0 counts as +0. Every element has a unique
// 64-bit key (orderable value << 32 | ~index), so "the k largest keys" is the
// exact answer; rows with fewer than k selectable values are padded with
// (-inf, -1).
//
// Two kernels. topk_partial_kernel: each row is cut into S slices, one CTA of
// 8 warps per slice (so rows x S CTAs keep every SM busy). A sorted sample of
// 256 evenly spaced elements of the slice gives a starting threshold with about
// 3k elements above it; each warp streams its share with 128-bit loads, four
// values compared against the threshold's value per warp vote (about two
// instructions per element); groups holding a candidate get buffer slots from
// one warp scan, and only candidate lanes build keys. A buffer past half full
// is sorted (bitonic) down to its k largest, raising the threshold. If fewer than k elements of the slice pass
// the sampled threshold, the slice is streamed again without it, so the
// result is exact. The CTA writes its k largest keys. topk_merge_kernel sorts
// a row's S x k keys and writes the k largest.
#include "aexis_internal.h"

namespace {

constexpr int kTkWarps = 8;
constexpr int kTkThreads = kTkWarps * 32;
constexpr int kTkBuf = 256;       // candidate keys per warp
constexpr int kTkMaxK = 64;
constexpr int kTkSamples = 256;
constexpr int kTkMaxSplits = 16;

__device__ __forceinline__ unsigned long long tk_key(float v, int i) {
    if (v != v) return 0ull;  // NaN: never selected
    const unsigned int o = aexis_orderable(v == 0.0f ? 0.0f : v);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned int)i);
}

__device__ __forceinline__ float tk_value(unsigned long long key) {
    const unsigned int hi = (unsigned int)(key >> 32);
    return __uint_as_float((hi & 0x80000000u) ? (hi & 0x7FFFFFFFu) : ~hi);
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

// Block-wide bitonic sort, descending, of a[0, np) (np a power of two).
__device__ void block_sort_desc(unsigned long long* a, int np, int tid, int nthreads) {
    for (int size = 2; size <= np; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < np; i += nthreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long x = a[i], y = a[j];
                    if (desc ? (x < y) : (x > y)) {
                        a[i] = y;
                        a[j] = x;
                    }
                }
            }
            __syncthreads();
        }
    }
}

// Slice `blockIdx.x` of row `blockIdx.y`: its k largest keys (descending,
// zero-padded) -> part[(row * S + slice) * k ..].
__global__ void __launch_bounds__(kTkThreads) topk_partial_kernel(const float* logits, int width, int ld, int k,
                                                                   int S, unsigned long long* part) {
    __shared__ unsigned long long buf[kTkWarps][kTkBuf];
    __shared__ unsigned long long merged[kTkWarps * kTkMaxK];
    __shared__ int warp_cnt[kTkWarps];
    const int slice = blockIdx.x, row = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const float* x = logits + (long long)row * ld;
    // Slice bounds on 4-element boundaries (the last slice takes the tail).
    const int quads = width / 4;
    const int q0 = (int)((long long)slice * quads / S), q1 = (int)((long long)(slice + 1) * quads / S);
    const int e0 = 4 * q0, e1 = slice == S - 1 ? width : 4 * q1;
    const int len = e1 - e0;
    unsigned long long* wb = buf[warp];
    const unsigned int lt = (1u << lane) - 1u;

    // Starting threshold: key of rank r in a sorted sample, about 3k elements
    // of the slice above it when the values have no order along the index.
    unsigned long long thr0 = 0ull;
    if (len >= 8 * kTkSamples) {
        unsigned long long* smp = &buf[0][0];
        for (int i = tid; i < kTkSamples; i += kTkThreads) {
            const int e = e0 + (int)(((long long)i * len) / kTkSamples);
            smp[i] = tk_key(x[e], e);
        }
        __syncthreads();
        block_sort_desc(smp, kTkSamples, tid, kTkThreads);
        int r = (int)((3LL * k * kTkSamples + len - 1) / len);
        r = r < 2 ? 2 : r;
        thr0 = r < kTkSamples ? smp[r] : 0ull;
        __syncthreads();
    }

    unsigned long long thr = 0ull;  // admit keys > thr
    float thr_v = -INFINITY;        // only values >= thr_v can beat thr
    int cnt = 0;                    // warp-uniform
    auto set_thr = [&](unsigned long long t) {
        thr = t;
        thr_v = t == 0ull ? -INFINITY : tk_value(t);
    };
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
                set_thr(wb[k - 1]);
            }
        }
    };

    // Append every value of v that reaches the threshold's value: a warp scan
    // of the per-lane counts gives each candidate its buffer slot. Values
    // equal to the threshold's may carry keys below it; they are harmless
    // (every value left out is strictly smaller than every value appended).
    auto append4 = [&](const float4 v, int e) {
        const bool c0 = v.x >= thr_v, c1 = v.y >= thr_v, c2 = v.z >= thr_v, c3 = v.w >= thr_v;
        const int nc = (int)c0 + (int)c1 + (int)c2 + (int)c3;
        int incl = nc;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += t;
        }
        const int added = __shfl_sync(0xffffffffu, incl, 31);
        int pos = cnt + incl - nc;
        if (c0) wb[pos++] = tk_key(v.x, e);
        if (c1) wb[pos++] = tk_key(v.y, e + 1);
        if (c2) wb[pos++] = tk_key(v.z, e + 2);
        if (c3) wb[pos++] = tk_key(v.w, e + 3);
        cnt += added;
        if (cnt > kTkBuf - 128) {  // room for the next 128 values
            __syncwarp();
            warp_sort_desc(wb, cnt, lane);
            cnt = cnt < k ? cnt : k;
            if (cnt == k) set_thr(wb[k - 1]);
        }
    };

    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    const float nan = __int_as_float(0x7fc00000);
    constexpr int kUnroll = 4;
    for (int pass = 0; pass < 2; ++pass) {
        cnt = 0;
        set_thr(pass == 0 ? thr0 : 0ull);
        int done = e0;  // elements of [e0, e1) covered by the vector loop
        if (vec) {
            const float4* x4 = reinterpret_cast<const float4*>(x);
            for (int base = q0 + warp * 32; base < q1; base += kUnroll * kTkThreads) {
                float4 v[kUnroll];
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int q = base + u * kTkThreads + lane;
                    v[u] = q < q1 ? x4[q] : make_float4(nan, nan, nan, nan);
                }
#pragma unroll
                for (int u = 0; u < kUnroll; ++u) {
                    const int q = base + u * kTkThreads + lane;
                    // NaN and everything below the threshold's value fail this
                    // compare (fmaxf drops NaN; -0 >= +0 holds; the key
                    // comparison settles ties).
                    const float m4 = fmaxf(fmaxf(v[u].x, v[u].y), fmaxf(v[u].z, v[u].w));
                    if (!__any_sync(0xffffffffu, m4 >= thr_v)) continue;
                    append4(v[u], 4 * q);
                }
            }
            done = 4 * q1;
        }
        for (int base = done + warp * 32; base < e1; base += kTkThreads) {
            const int i = base + lane;
            offer(i < e1 ? tk_key(x[i], i) : 0ull);
        }
        if (lane == 0) warp_cnt[warp] = cnt;
        __syncthreads();
        int total = 0;
#pragma unroll
        for (int w = 0; w < kTkWarps; ++w) total += warp_cnt[w];
        __syncthreads();
        if (pass == 1 || thr0 == 0ull || total >= k) break;
    }
    // Each warp keeps its k largest; then the CTA's k largest.
    __syncwarp();
    if (cnt > k) {
        warp_sort_desc(wb, cnt, lane);
        cnt = k;
    }
    for (int i = lane; i < k; i += 32) merged[warp * k + i] = i < cnt ? wb[i] : 0ull;
    __syncthreads();
    const int nm = kTkWarps * k;
    int np = 1;
    while (np < nm) np <<= 1;
    unsigned long long* all = &buf[0][0];  // np <= kTkWarps * kTkBuf
    for (int i = tid; i < np; i += kTkThreads) all[i] = i < nm ? merged[i] : 0ull;
    __syncthreads();
    block_sort_desc(all, np, tid, kTkThreads);
    unsigned long long* out = part + ((long long)row * S + slice) * k;
    for (int j = tid; j < k; j += kTkThreads) out[j] = all[j];
}

// Row `blockIdx.x`: the k largest of its S x k slice keys.
__global__ void __launch_bounds__(kTkThreads) topk_merge_kernel(const unsigned long long* part, int S, int k,
                                                                 float* vals, int32_t* idx) {
    __shared__ unsigned long long all[kTkMaxSplits * kTkMaxK];
    const int row = blockIdx.x, tid = threadIdx.x;
    const int n = S * k;
    int np = 1;
    while (np < n) np <<= 1;
    const unsigned long long* src = part + (long long)row * n;
    for (int i = tid; i < np; i += kTkThreads) all[i] = i < n ? src[i] : 0ull;
    __syncthreads();
    block_sort_desc(all, np, tid, kTkThreads);
    for (int j = tid; j < k; j += kTkThreads) {
        const unsigned long long key = all[j];
        float* vo = vals + (long long)row * k + j;
        int32_t* io = idx + (long long)row * k + j;
        if (key != 0ull) {
            *vo = tk_value(key);
            *io = (int32_t)(0xFFFFFFFFu - (unsigned int)(key & 0xFFFFFFFFull));
        } else {
            *vo = -INFINITY;
            *io = -1;
        }
    }
}

int topk_splits(int rows, int width, int sm_count) {
    int S = (4 * sm_count + rows - 1) / rows;
    const int by_len = width / 4096;  // slices of at least ~4K elements
    S = S > by_len ? by_len : S;
    S = S > kTkMaxSplits ? kTkMaxSplits : S;
    return S < 1 ? 1 : S;
}

}  // namespace

size_t topk_scratch_bytes(int rows, int width, int k, int sm_count) {
    return (size_t)rows * topk_splits(rows, width, sm_count) * k * sizeof(unsigned long long);
}

cudaError_t launch_topk(const float* logits, int rows, int width, int ld, int k, float* vals, int32_t* idx,
                        void* scratch, int sm_count, cudaStream_t s) {
    if (k < 1 || k > kTkMaxK) return cudaErrorInvalidValue;
    const int S = topk_splits(rows, width, sm_count);
    unsigned long long* part = reinterpret_cast<unsigned long long*>(scratch);
    topk_partial_kernel<<<dim3(S, rows), kTkThreads, 0, s>>>(logits, width, ld, k, S, part);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    topk_merge_kernel<<<rows, kTkThreads, 0, s>>>(part, S, k, vals, idx);
    return cudaGetLastError();
}
