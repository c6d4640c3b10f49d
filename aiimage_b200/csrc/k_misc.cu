// k_misc.cu -- the pointwise / reduction kernels of the decoder hot path, in
// the reference's logical Pack4 layouts (used by the per-op C ABI; the fused
// decoder in k_decoder.cu uses its own layouts).
#include "aexis_internal.h"

namespace {

constexpr int kT = 256;

// ------------------------------------------------------------------ dequant
// One AexisGemm2DReadB (HLSL Pack4Matmul:707-734) per element: (float)q * s,
// a single fp32 multiply, so the result is bit-identical to the reference.
template <typename ST>
__global__ void dequant_kernel(const uint32_t* P, const ST* S, int kind, int group, int n, int k,
                               float* out) {
    const long long total = (long long)n * k;
    for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (long long)gridDim.x * blockDim.x) {
        const long long row = idx / k;
        float s, q;
        if (kind == WK_Q4) {
            const uint32_t raw = (P[idx >> 3] >> ((idx & 7) * 4)) & 0xFu;
            q = (float)(raw >= 8u ? (int)raw - 16 : (int)raw);
            const long long si = group > 0 ? idx / group : row;
            if constexpr (sizeof(ST) == 2) s = __half2float(S[si]); else s = S[si];
        } else {
            const uint32_t raw = (P[idx >> 2] >> ((idx & 3) * 8)) & 0xFFu;
            q = (float)(raw >= 128u ? (int)raw - 256 : (int)raw);
            if constexpr (sizeof(ST) == 2) s = __half2float(S[row]); else s = S[row];
        }
        out[idx] = __fmul_rn(q, s);
    }
}

__global__ void dense_to_f32_kernel(const void* data, int dtype, long long total, float* out) {
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x)
        out[i] = aexis_load_act(data, dtype, i);
}

// ------------------------------------------------------------------ rmsnorm
// AexisRmsNormPack4LinearMat (COMMON:4531-4563): one CTA per row; the sum of
// squares is a fixed-order tree (deterministic), the rest is elementwise.
__global__ void rmsnorm_kernel(const void* x, int x_dtype, int width, int ld, const float* gamma,
                               int affine_size, float eps, void* y, int y_dtype) {
    __shared__ float red[kT / 32];
    const long long base = (long long)blockIdx.x * ld;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < width; i += kT) {
        const float v = aexis_load_act(x, x_dtype, base + i);
        ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kT / 32; ++w) tot += red[w];
    const float inv = 1.0f / sqrtf(fmaxf(tot / (float)width + eps, 1e-20f));
    for (int i = threadIdx.x; i < width; i += kT) {
        float v = aexis_load_act(x, x_dtype, base + i) * inv;
        if (gamma && affine_size > 0) v = v * gamma[min(max(i, 0), affine_size - 1)];
        aexis_store_out(y, y_dtype, base + i, v);
    }
}

__device__ __forceinline__ long long p4(int W, int H, int x, int y, int c) {
    return (((long long)(c >> 2) * H + y) * W + x) * 4 + (c & 3);
}

// --------------------------------------------------------------------- rope
// AexisRotaryEmbedPack4_Impl (HLSL Pack4PointwiseNorm:414-473), one thread per
// element of the Pack4 CDHW [embed, seq, 1, heads] tensor.
__global__ void rope_kernel(const float* src, int E, int L, int NH, const float* cosv,
                            const float* sinv, int interleaved, float* out) {
    const long long total = (long long)NH * L * E;
    const int half = max(1, E / 2);
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int e = (int)(t % E);
        const int seq = (int)((t / E) % L);
        const int head = (int)(t / ((long long)E * L));
        int pair0, pair1, ci;
        bool first;
        if (interleaved) {
            const int j = e / 2;
            pair0 = j * 2; pair1 = pair0 + 1; ci = seq * half + j; first = (e & 1) == 0;
        } else {
            const int j2 = e < half ? e : e - half;
            pair0 = j2; pair1 = half + j2; ci = seq * half + j2; first = e < half;
        }
        const long long o = p4(E, L, e, seq, head);
        if (pair1 >= E) { out[o] = src[o]; continue; }
        const float c = cosv[ci], s = sinv[ci];
        const float x0 = src[p4(E, L, pair0, seq, head)], x1 = src[p4(E, L, pair1, seq, head)];
        out[o] = first ? __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s))
                       : __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
    }
}

// ---------------------------------------------------------------- kv append
// AexisAppendSequencePack4CDHW_Impl (HLSL Pack4Elementwise:84-98).
__global__ void kv_append_kernel(const float4* cur, int W, int rows, int slices, int offset,
                                 float4* cache, int cache_rows) {
    const long long total = (long long)W * rows * slices;
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int x = (int)(t % W);
        const int y = (int)((t / W) % rows);
        const int z = (int)(t / ((long long)W * rows));
        const int dy = offset + y;
        if (dy < 0 || dy >= cache_rows) continue;
        cache[((long long)z * cache_rows + dy) * W + x] = cur[t];
    }
}

// AexisConcatSequencePack4CDHW_Impl (HLSL Pack4Elementwise:64-81).
__global__ void kv_concat_kernel(const float4* a, int ah, const float4* b, int bh, int W, int slices,
                                 float4* out, int oh) {
    const long long total = (long long)W * oh * slices;
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int x = (int)(t % W);
        const int y = (int)((t / W) % oh);
        const int z = (int)(t / ((long long)W * oh));
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (y < ah) v = a[((long long)z * ah + y) * W + x];
        else if (y < ah + bh) v = b[((long long)z * bh + (y - ah)) * W + x];
        out[t] = v;
    }
}

// --------------------------------------------------------------------- sdpa
// AexisSdpaAttentionPack4CDHW_Impl (HLSL Pack4Matmul:420-557): one CTA per
// (query row, head); scores live in dynamic shared memory (any dst_len that
// fits, no 4096 cap). Each score and each output element is a sequential fp32
// sum in the reference's order.
__global__ void sdpa_kernel(const float* q, const float* k, const float* v, int src_len, int dst_len,
                            int E, int OE, int NH, int NG, float scale, const float* mask, int mask_w,
                            int mask_h, int causal, int causal_offset, float* out) {
    extern __shared__ float sc[];
    __shared__ float red[kT / 32];
    const int row = blockIdx.x, head = blockIdx.y;
    const int hpg = max(1, NH / NG);
    const int kh = min(max(0, NG - 1), head / hpg);
    const int off = max(0, causal_offset);
    for (int col = threadIdx.x; col < dst_len; col += kT) {
        float s = 0.0f;
        for (int i = 0; i < E; ++i)
            s = __fadd_rn(s, __fmul_rn(q[p4(E, src_len, i, row, head)], k[p4(E, dst_len, i, col, kh)]));
        s = __fmul_rn(s, scale);
        if (causal && col > row + off) s = -1.0e20f;
        else if (mask && col < mask_w && row < mask_h) s = __fadd_rn(s, mask[((long long)row * mask_w + col) * 4]);
        sc[col] = s;
    }
    __syncthreads();
    float mx = -3.402823466e+38f;
    for (int col = threadIdx.x; col < dst_len; col += kT) mx = fmaxf(mx, sc[col]);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int w = 1; w < kT / 32; ++w) mx = fmaxf(mx, red[w]);
    __syncthreads();
    float sum = 0.0f;
    for (int col = threadIdx.x; col < dst_len; col += kT) {
        const float e = expf(sc[col] - mx);
        sc[col] = e;
        sum += e;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sum;
    __syncthreads();
    float tot = 0.0f;
#pragma unroll
    for (int w = 0; w < kT / 32; ++w) tot += red[w];
    const float inv = 1.0f / fmaxf(tot, 1e-20f);
    for (int col = threadIdx.x; col < dst_len; col += kT) sc[col] = sc[col] * inv;
    __syncthreads();
    for (int ox = threadIdx.x; ox < OE; ox += kT) {
        float acc = 0.0f;
        for (int col = 0; col < dst_len; ++col)
            acc = __fadd_rn(acc, __fmul_rn(sc[col], v[p4(OE, dst_len, ox, col, kh)]));
        out[p4(OE, src_len, ox, row, head)] = acc;
    }
}

// ------------------------------------------------------------------- argmax
// Two passes over 64-bit keys (aexis_argmax_key): per-block maxima are
// max-reduced with atomicMax, then decoded.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) { return aexis_argmax_key(v, idx); }

__global__ void argmax_partial_kernel(const float* logits, int width, int ld, unsigned long long* keys,
                                      long long offset = 0) {
    const int row = blockIdx.y;
    const float* x = logits + (long long)row * ld;
    // Each thread scans its elements in ascending index order keeping the
    // first strict maximum (NaN never compares greater), then builds one key;
    // the key order settles ties across threads (lower index wins, -0 == +0).
    // A NaN at global index 0 wins, as in the reference's scan that starts
    // from element 0.
    float bv = -INFINITY;
    int bi = -1;
    const int tid = blockIdx.x * blockDim.x + threadIdx.x, nth = gridDim.x * blockDim.x;
    auto take = [&](float v, int i) {
        if (v > bv || (bi < 0 && v == v)) {
            bv = v;
            bi = i;
        }
    };
    int start = 0;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const int nvec = width / 4;
        const float4* x4 = reinterpret_cast<const float4*>(x);
#pragma unroll 4
        for (int q = tid; q < nvec; q += nth) {
            const float4 v = x4[q];
            take(v.x, 4 * q);
            take(v.y, 4 * q + 1);
            take(v.z, 4 * q + 2);
            take(v.w, 4 * q + 3);
        }
        start = 4 * nvec;
    }
    for (int i = start + tid; i < width; i += nth) take(x[i], i);
    unsigned long long best = bi >= 0 ? argmax_key(bv, (int)(offset + bi)) : 0ull;
    if (tid == 0 && offset == 0 && width > 0) {
        const unsigned long long k0 = argmax_key(x[0], 0);
        best = k0 > best ? k0 : best;
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0 && best != 0ull) atomicMax(keys + row, best);
}

__global__ void argmax_finish_kernel(const unsigned long long* keys, int rows, int32_t* out) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r < rows) {
        out[r] = aexis_argmax_index(keys[r]);
    }
}

// -------------------------------------------------------------------- embed
// AexisEmbedValue (HLSL BufferTensor:37-62) for every (word, p).
template <typename ST>
__global__ void embed_kernel(const int32_t* words, int count, const void* data, const ST* S, int kind,
                             int group, int vocab, int dim, const float* bias, float* out) {
    const long long total = (long long)count * dim;
    for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total;
         t += (long long)gridDim.x * blockDim.x) {
        const int q = (int)(t / dim), p = (int)(t % dim);
        const int w = min(max(words[q], 0), vocab - 1);
        const long long wi = (long long)w * dim + p;
        float v;
        if (kind == WK_Q4) {
            const uint32_t raw = (((const uint32_t*)data)[wi >> 3] >> ((wi & 7) * 4)) & 0xFu;
            float s;
            if constexpr (sizeof(ST) == 2) s = __half2float(S[wi / group]); else s = S[wi / group];
            v = __fmul_rn((float)(raw >= 8u ? (int)raw - 16 : (int)raw), s);
        } else if (kind == WK_Q8) {
            const uint32_t raw = (((const uint32_t*)data)[wi >> 2] >> ((wi & 3) * 8)) & 0xFFu;
            float s;
            if constexpr (sizeof(ST) == 2) s = __half2float(S[w]); else s = S[w];
            v = __fmul_rn((float)(raw >= 128u ? (int)raw - 256 : (int)raw), s);
        } else if (kind == WK_F16) {
            v = __half2float(((const __half*)data)[wi]);
        } else {
            v = ((const float*)data)[wi];
        }
        if (bias) v = __fadd_rn(v, bias[p]);
        out[t] = v;
    }
}

__global__ void swish_kernel(const float* x, int n, float* y) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        y[i] = x[i] / (1.0f + expf(-x[i]));
}

__global__ void swiglu_kernel(const float* g, const float* u, int n, float* y) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x)
        y[i] = __fmul_rn(g[i] / (1.0f + expf(-g[i])), u[i]);
}

// W8A8 activation codes (AexisQuantizeGemmActivationForInt8, HLSL
// Pack4Matmul:792-800): q = clamp(round(v / scale) + zp) over [-128, 127]
// (signed) or [0, 255] (unsigned), rounding half to even. The GEMM consumes
// the integer q - zp, exact in fp16 for |zp| <= 1024, and applies `scale` in
// its epilogue, so each product (q - zp) * w is exact.
__global__ void act_quant_i8_kernel(const void* a, int a_dtype, int lda, int m, int k, float scale, int zp,
                                    int is_unsigned, __half* out) {
    const long long total = (long long)m * k;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long r = i / k, c = i - r * k;
        out[i] = __float2half_rn(aexis_act_code(aexis_load_act(a, a_dtype, r * lda + c), scale, zp, is_unsigned));
    }
}

// A Pack4 texture-array activation (the inputPacked A of
// AexisGemm2DPack4LinearTextureAFromPack4, HLSL Pack4Matmul:880-891,
// 1106-1190) gathered into row-major [m][k] of the same dtype. Element
// (row, kk) is lane kk & 3 of texel (x, row, slice) with pack = kk >> 2,
// x = pack % width, slice = pack / width; the texel sits at
// ((slice * height + row) * width + x) * 4. Packs past the last slice read 0
// (the reference's loop stops there).
template <typename T>
__global__ void gather_pack4a_kernel(const T* a, int width, int height, int slices, int m, int k, T* out) {
    const long long total = (long long)m * k;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i / k), kk = (int)(i - (long long)r * k);
        const int pack = kk >> 2, x = pack % width, sl = pack / width;
        T v = T(0.0f);
        if (sl < slices) v = a[(((long long)sl * height + r) * width + x) * 4 + (kk & 3)];
        out[i] = v;
    }
}

// Bounded wait on a flag nothing sets: one thread polls it until
// limit_cycles of SM clock pass, then records AEXIS_E_TIMEOUT in the status
// word and returns (the path every bounded barrier wait takes when it gives up).
__global__ void selftest_wait_kernel(const volatile int* flag, long long limit_cycles, int* status) {
    if (threadIdx.x != 0) return;
    const long long t0 = clock64();
    while (*flag == 0) {
        if (clock64() - t0 > limit_cycles) {
            atomicCAS(status, 0, (int)AEXIS_E_TIMEOUT);
            return;
        }
    }
}

inline int grid_for(long long total, int threads = kT) {
    long long b = (total + threads - 1) / threads;
    if (b > 148LL * 32) b = 148LL * 32;
    return (int)(b < 1 ? 1 : b);
}

}  // namespace

cudaError_t launch_dequant(const aexis_weights* w, float* out, cudaStream_t s) {
    const long long total = (long long)w->n * w->k;
    if (w->kind == WK_F16 || w->kind == WK_F32) {
        dense_to_f32_kernel<<<grid_for(total), kT, 0, s>>>(w->data, w->kind == WK_F16 ? AEXIS_F16 : AEXIS_F32,
                                                           total, out);
    } else if (w->scale_dtype == AEXIS_F16) {
        dequant_kernel<__half><<<grid_for(total), kT, 0, s>>>((const uint32_t*)w->data, (const __half*)w->scales,
                                                              w->kind, w->group, w->n, w->k, out);
    } else {
        dequant_kernel<float><<<grid_for(total), kT, 0, s>>>((const uint32_t*)w->data, (const float*)w->scales,
                                                             w->kind, w->group, w->n, w->k, out);
    }
    return cudaGetLastError();
}

cudaError_t launch_rmsnorm(const void* x, int x_dtype, int rows, int width, int ld, const float* gamma,
                           int affine_size, float eps, void* y, int y_dtype, cudaStream_t s) {
    rmsnorm_kernel<<<rows, kT, 0, s>>>(x, x_dtype, width, ld, gamma, affine_size, eps, y, y_dtype);
    return cudaGetLastError();
}

cudaError_t launch_rope(const float* src, int E, int L, int NH, const float* cosv, const float* sinv,
                        int interleaved, float* out, cudaStream_t s) {
    rope_kernel<<<grid_for((long long)E * L * NH), kT, 0, s>>>(src, E, L, NH, cosv, sinv, interleaved, out);
    return cudaGetLastError();
}

cudaError_t launch_kv_append(const float* cur, int W, int rows, int slices, int offset, float* cache,
                             int cache_rows, cudaStream_t s) {
    kv_append_kernel<<<grid_for((long long)W * rows * slices), kT, 0, s>>>(
        (const float4*)cur, W, rows, slices, offset, (float4*)cache, cache_rows);
    return cudaGetLastError();
}

cudaError_t launch_kv_concat(const float* a, int ah, const float* b, int bh, int W, int slices, float* out,
                             int oh, cudaStream_t s) {
    kv_concat_kernel<<<grid_for((long long)W * oh * slices), kT, 0, s>>>(
        (const float4*)a, ah, (const float4*)b, bh, W, slices, (float4*)out, oh);
    return cudaGetLastError();
}

size_t sdpa_smem_bytes(int dst_len) { return (size_t)dst_len * sizeof(float); }

cudaError_t launch_sdpa(const float* q, const float* k, const float* v, int src_len, int dst_len, int E,
                        int OE, int NH, int NG, float scale, const float* mask, int mask_w, int mask_h,
                        int causal, int causal_offset, float* out, cudaStream_t s) {
    const size_t smem = sdpa_smem_bytes(dst_len);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(sdpa_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    sdpa_kernel<<<dim3(src_len, NH), kT, smem, s>>>(q, k, v, src_len, dst_len, E, OE, NH, NG, scale, mask,
                                                    mask_w, mask_h, causal, causal_offset, out);
    return cudaGetLastError();
}

cudaError_t launch_argmax(const float* logits, int rows, int width, int ld, int32_t* out,
                          unsigned long long* keys, int sm_count, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(keys, 0, sizeof(unsigned long long) * rows, s);
    if (e != cudaSuccess) return e;
    int bx = (width + kT * 8 - 1) / (kT * 8);
    const int cap = (sm_count * 8 + rows - 1) / rows;
    if (bx > cap) bx = cap;
    if (bx < 1) bx = 1;
    argmax_partial_kernel<<<dim3(bx, rows), kT, 0, s>>>(logits, width, ld, keys);
    argmax_finish_kernel<<<(rows + kT - 1) / kT, kT, 0, s>>>(keys, rows, out);
    return cudaGetLastError();
}

cudaError_t launch_argmax_keys(const float* logits, int rows, int width, int ld, long long offset,
                               unsigned long long* keys, int sm_count, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(keys, 0, sizeof(unsigned long long) * rows, s);
    if (e != cudaSuccess) return e;
    int bx = (width + kT * 8 - 1) / (kT * 8);
    const int cap = (sm_count * 8 + rows - 1) / rows;
    if (bx > cap) bx = cap;
    if (bx < 1) bx = 1;
    argmax_partial_kernel<<<dim3(bx, rows), kT, 0, s>>>(logits, width, ld, keys, offset);
    return cudaGetLastError();
}

cudaError_t launch_embed(const int32_t* words, int count, const aexis_weights* t, const float* bias, float* out,
                         cudaStream_t s) {
    const long long total = (long long)count * t->k;
    if (t->scale_dtype == AEXIS_F16)
        embed_kernel<__half><<<grid_for(total), kT, 0, s>>>(words, count, t->data, (const __half*)t->scales,
                                                            t->kind, t->group, t->n, t->k, bias, out);
    else
        embed_kernel<float><<<grid_for(total), kT, 0, s>>>(words, count, t->data, (const float*)t->scales,
                                                           t->kind, t->group, t->n, t->k, bias, out);
    return cudaGetLastError();
}

cudaError_t launch_swish(const float* x, int n, float* y, cudaStream_t s) {
    swish_kernel<<<grid_for(n), kT, 0, s>>>(x, n, y);
    return cudaGetLastError();
}

cudaError_t launch_swiglu(const float* g, const float* u, int n, float* y, cudaStream_t s) {
    swiglu_kernel<<<grid_for(n), kT, 0, s>>>(g, u, n, y);
    return cudaGetLastError();
}

cudaError_t launch_act_quant_i8(const void* a, int a_dtype, int lda, int m, int k, float scale, int zero_point,
                                int is_unsigned, __half* out, cudaStream_t s) {
    act_quant_i8_kernel<<<grid_for((long long)m * k), kT, 0, s>>>(a, a_dtype, lda, m, k, scale, zero_point,
                                                                   is_unsigned, out);
    return cudaGetLastError();
}

cudaError_t launch_gather_pack4a(const void* a, int a_dtype, int width, int height, int slices, int m, int k,
                                 void* out, cudaStream_t s) {
    const int g = grid_for((long long)m * k);
    if (a_dtype == AEXIS_F16)
        gather_pack4a_kernel<__half><<<g, kT, 0, s>>>((const __half*)a, width, height, slices, m, k, (__half*)out);
    else
        gather_pack4a_kernel<float><<<g, kT, 0, s>>>((const float*)a, width, height, slices, m, k, (float*)out);
    return cudaGetLastError();
}

cudaError_t launch_selftest_wait(int* flag, long long limit_cycles, int* status, cudaStream_t s) {
    cudaError_t e = cudaMemsetAsync(flag, 0, sizeof(int), s);
    if (e != cudaSuccess) return e;
    selftest_wait_kernel<<<1, 32, 0, s>>>(flag, limit_cycles, status);
    return cudaGetLastError();
}
