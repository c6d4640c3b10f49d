// k_batch.cu -- batched greedy decoding: B independent sequences with ragged
// contexts share one decoder's Q8 weights (the BASELINE config-4 workload,
// Qwen35DecoderSession.DecodeCore + SelectNextToken run for B sequences at
// once, Qwen35DecoderSession.cs:469-585, 734-809).
//
// One step for all B sequences, captured once into a CUDA graph with
// programmatic dependent launch on every edge:
//   embed       h[b] = E[token[b]]
//   per layer   prep  RMSNorm(h) -> fp16 hi/lo activations, zero qkv
//               gemm  qkv += x Wqkv^T          (tensor cores, split K)
//               rope  RoPE of q and k, fp16 K/V appended at pos[b]
//               attn  split attention over each sequence's own context
//               prep  attn -> activations
//               gemm  h += attn Wo^T           (residual through the atomics)
//               prep  RMSNorm(h), zero gate/up
//               gemm  gu += x Wgu^T
//               prep  silu(g) * u
//               gemm  h += act Wdown^T
//   lm_head     prep RMSNorm(h); gemm logits = x Wlm^T; per-row argmax keys
//   finish      token[b] = argmax, out[step][b] = token, pos[b] += 1
// The linears run on gemm_q8_tc_kernel: the weight matrix is read once per
// step for all B rows (the weight-only GEMM of Pack4Matmul:1038-1104 batched).
#include <cmath>
#include <cstring>
#include <new>

#include "decoder_internal.h"
#include "gemv_dev.cuh"

#define AEXIS_API extern "C" __attribute__((visibility("default")))

namespace {

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

constexpr int kBatThreads = 256;
constexpr int kBatChunk = 128;        // context positions per attention CTA
constexpr int kBatMaxGroup = 8;       // query heads per KV head
constexpr int kBatMaxHeadDim = 256;
constexpr int kBatMaxCap = 8192;      // positions per sequence

// splitmix64 finaliser (Steele, Lea and Flood, "Fast splittable pseudorandom
// number generators", OOPSLA 2014).
__host__ __device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// Synthetic context value of (sequence, layer, K/V, head, position, dim): a
// 24-bit uniform in [-0.5, 0.5), exact in fp32, then rounded to fp16. The
// oracle's decoder fills its cache with the same function.
__device__ __forceinline__ __half ctx_value(unsigned long long seq_key, int layer, int kind, int head, int pos,
                                            int dim) {
    const unsigned long long idx =
        ((((unsigned long long)layer * 2 + kind) * 256 + head) * 65536 + (unsigned long long)pos) * 256 + dim;
    const unsigned long long r = mix64(seq_key ^ idx);
    const float u = (float)(r >> 40) * (1.0f / 16777216.0f) - 0.5f;
    return __float2half_rn(u);
}

// Element offset of dim d inside a cache row of position p. swz = 0: plain;
// swz = 1 (D = 128, the tensor-core attention): the 16-byte chunks of each
// 128-byte half row XOR-swizzled by p & 7, so a bulk copy of consecutive rows
// lands in shared memory ready for conflict-free ldmatrix.
__device__ __forceinline__ int cache_dim(int p, int d, int swz) {
    if (!swz) return d;
    const int ch = d >> 3;
    return (((ch & 8) | ((ch & 7) ^ (p & 7))) << 3) | (d & 7);
}

// Fills positions [0, ctx[b]) of every layer's K and V cache of sequence b
// with ctx_value and sets pos[b] = ctx[b]. Caches [layers][B][kvh][cap][D].
__global__ void bat_fill_kernel(__half* kc, __half* vc, int layers, int B, int kvh, int cap, int D, const int* ctx,
                                const unsigned long long* seq_keys, int* pos, int swz) {
    const int b = blockIdx.y;
    const int n = ctx[b];
    const long long per_layer = (long long)kvh * n * D;
    const long long total = (long long)layers * per_layer;
    const unsigned long long key = seq_keys[b];
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int l = (int)(i / per_layer);
        const long long r = i % per_layer;
        const int g = (int)(r / ((long long)n * D));
        const int p = (int)((r / D) % n);
        const int d = (int)(r % D);
        const size_t off = ((((size_t)l * B + b) * kvh + g) * cap + p) * D + cache_dim(p, d, swz);
        kc[off] = ctx_value(key, l, 0, g, p, d);
        vc[off] = ctx_value(key, l, 1, g, p, d);
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) pos[b] = n;
}

// h[b] = E[clamp(token[b])] (fp16 table -> fp32).
__global__ void bat_embed_kernel(const __half* table, int vocab, int hidden, const int* token, float* h) {
    griddep_wait();
    griddep_launch();
    const int b = blockIdx.y;
    int t = token[b];
    t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
    const __half* row = table + (long long)t * hidden;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
        h[(long long)b * hidden + i] = __half2float(row[i]);
}

// RoPE (rotate-half, HLSL Pack4PointwiseNorm:414-473) of the q and k rows of
// qkv[b] (the decoder's internal row order: rotate-half pairs adjacent, see
// rope_map), q -> q[b][n_heads * D] fp32, k and v -> fp16 caches at pos[b].
// Grid (row blocks, B): one row per thread.
__global__ void bat_rope_kernel(const float* qkv, int rows, const int* rope_map, const float* cosv,
                                const float* sinv, const int* pos, int D, int rot, int n_heads, int kvh, int cap, int B,
                                float* q, __half* kc, __half* vc, int swz) {
    griddep_wait();
    griddep_launch();
    const int b = blockIdx.y;
    const int p = pos[b];
    const int half = rot >> 1;
    const float* src = qkv + (long long)b * rows;
    for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
        const int desc = rope_map[r];
        const int kind = desc >> 24, head = (desc >> 12) & 0xFFF, dim = desc & 0xFFF;
        const float val = src[r];
        float out = val;
        if (kind != 2 && dim < rot) {
            const float partner = src[r ^ 1];
            const bool first = dim < half;
            const int j = first ? dim : dim - half;
            const float c = cosv[(long long)p * half + j];
            const float s = sinv[(long long)p * half + j];
            const float x0 = first ? val : partner, x1 = first ? partner : val;
            out = first ? x0 * c - x1 * s : x0 * s + x1 * c;
        }
        if (kind == 0) {
            q[((long long)b * n_heads + head) * D + dim] = out;
        } else {
            __half* cache = kind == 1 ? kc : vc;
            cache[(((size_t)b * kvh + head) * cap + p) * D + cache_dim(p, dim, swz)] = __float2half_rn(out);
        }
    }
}

// Split attention for sequence b, KV head g, context positions
// [split * kBatChunk, ...) of ctx = pos[b] + 1, for the HPG query heads of
// that KV head: K and V of the chunk arrive by two bulk copies; scores
// (q . k) * scale, per-split max m, sum l and o = sum e * v; the last CTA of
// (b, g) merges the splits with weights e^(m_s - M) / sum_s l_s e^(m_s - M).
// Mathematically the reference's two-pass softmax (HLSL Pack4Matmul:485-547)
// with GQA kv = h / (H / Hkv).
//   scores: TPP = D / DPT threads per position, DPT = 64 / HPG dims each
//           (16-byte chunks interleaved so a position's threads read one
//           contiguous run), the HPG x DPT query values held in registers,
//           partial dots added by shuffles within the TPP lanes;
//   values: each thread owns two dims of every head over every VG-th
//           position; the VG partial sums are added through shared memory.
// Dynamic shared memory: K and V chunks (2 x kBatChunk x D fp16).
template <int HPG, int PC>
__global__ void __launch_bounds__(kBatThreads, 3) bat_attn_kernel(const float* q, const __half* kc, const __half* vc,
                                                               int cap, int D, int n_heads, int kvh, float scale,
                                                               const int* pos, float* part, unsigned int* counters,
                                                               float* out, int* status) {
    constexpr int MS = kBatMaxCap / PC;  // most splits of a sequence
    constexpr int DPT = 64 / HPG;
    constexpr int KC = DPT / 8;  // 16-byte K chunks per thread and position
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(16) float sc[PC][HPG];  // scores, then e = exp(s - m), [p][h]
    __shared__ float stat[HPG][2];
    __shared__ float wsm[HPG][MS];
    __shared__ __align__(8) uint64_t bar;
    __shared__ bool last, ok;
    griddep_wait();
    griddep_launch();
    const int split = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
    const int ctx = pos[b] + 1;
    const int active = (ctx + PC - 1) / PC;
    if (split >= active) return;
    const int p0 = split * PC, p1 = min(ctx, p0 + PC), np = p1 - p0;
    const int tid = threadIdx.x, warp = tid >> 5;
    __half* ks = reinterpret_cast<__half*>(smem);
    __half* vs = ks + (size_t)PC * D;
    const size_t head_off = ((size_t)b * kvh + g) * cap;
    if (tid == 0) {
        aexis_dev::mbar_init(&bar, 1);
        aexis_dev::fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        const uint32_t bytes = (uint32_t)np * D * 2;
        aexis_dev::mbar_arrive_expect_tx(&bar, 2 * bytes);
        aexis_dev::bulk_g2s_plain(ks, kc + (head_off + p0) * D, bytes, &bar);
        aexis_dev::bulk_g2s_plain(vs, vc + (head_off + p0) * D, bytes, &bar);
    }
    // This thread's query slice: chunks s, s + TPP, ... (8 dims each) of every head.
    const int tpp = D / DPT;
    const int slot = tid % tpp;
    const float* qb = q + ((long long)b * n_heads + g * HPG) * D;
    float qr[HPG][DPT];
#pragma unroll
    for (int h = 0; h < HPG; ++h)
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            const float4 a0 = *reinterpret_cast<const float4*>(qb + h * D + (slot + j * tpp) * 8);
            const float4 a1 = *reinterpret_cast<const float4*>(qb + h * D + (slot + j * tpp) * 8 + 4);
            qr[h][j * 8 + 0] = a0.x; qr[h][j * 8 + 1] = a0.y; qr[h][j * 8 + 2] = a0.z; qr[h][j * 8 + 3] = a0.w;
            qr[h][j * 8 + 4] = a1.x; qr[h][j * 8 + 5] = a1.y; qr[h][j * 8 + 6] = a1.z; qr[h][j * 8 + 7] = a1.w;
        }
    if (tid == 0) {
        ok = aexis_dev::mbar_wait(&bar, 0);
        if (!ok) aexis_dev::report_timeout(status);  // the copies never completed: nothing is merged
    }
    __syncthreads();
    if (!ok) return;
    aexis_dev::mbar_try_wait(&bar, 0);  // completed phase: acquire the copied bytes in every thread
    // Scores. Every lane runs every pass (the shuffles need the whole warp).
    const int ppp = kBatThreads / tpp;
    for (int base = 0; base < np; base += ppp) {
        const int pp = base + tid / tpp;
        const bool valid = pp < np;
        float acc[HPG];
#pragma unroll
        for (int h = 0; h < HPG; ++h) acc[h] = 0.0f;
#pragma unroll
        for (int j = 0; j < KC; ++j) {
            uint4 raw = make_uint4(0u, 0u, 0u, 0u);
            if (valid) raw = *reinterpret_cast<const uint4*>(ks + (size_t)pp * D + (slot + j * tpp) * 8);
            const __half2* k2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 kf = __half22float2(k2[e]);
#pragma unroll
                for (int h = 0; h < HPG; ++h)
                    acc[h] = fmaf(qr[h][j * 8 + 2 * e + 1], kf.y, fmaf(qr[h][j * 8 + 2 * e], kf.x, acc[h]));
            }
        }
#pragma unroll
        for (int h = 0; h < HPG; ++h)
            for (int o = tpp >> 1; o >= 1; o >>= 1) acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], o);
        if (valid && slot == 0) {
#pragma unroll
            for (int h = 0; h < HPG; ++h) sc[pp][h] = acc[h] * scale;
        }
    }
    __syncthreads();
    for (int h = warp; h < HPG; h += kBatThreads / 32) {
        const int lane = tid & 31;
        float m = -INFINITY;
        for (int i = lane; i < np; i += 32) m = fmaxf(m, sc[i][h]);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int i = lane; i < np; i += 32) {
            const float e = expf(sc[i][h] - m);
            sc[i][h] = e;
            l += e;
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) {
            stat[h][0] = m;
            stat[h][1] = l;
        }
    }
    __syncthreads();
    // Values.
    const int dpairs = D >> 1;
    const int VG = kBatThreads / dpairs;
    const int dt = tid % dpairs, vg = tid / dpairs;
    float o0[HPG], o1[HPG];
#pragma unroll
    for (int h = 0; h < HPG; ++h) o0[h] = o1[h] = 0.0f;
    for (int p = vg; p < np; p += VG) {
        const float2 v = __half22float2(*reinterpret_cast<const __half2*>(vs + (size_t)p * D + 2 * dt));
        float pr[HPG];
        if constexpr (HPG % 4 == 0) {
#pragma unroll
            for (int h = 0; h < HPG; h += 4) {
                const float4 t = *reinterpret_cast<const float4*>(&sc[p][h]);
                pr[h] = t.x; pr[h + 1] = t.y; pr[h + 2] = t.z; pr[h + 3] = t.w;
            }
        } else {
#pragma unroll
            for (int h = 0; h < HPG; ++h) pr[h] = sc[p][h];
        }
#pragma unroll
        for (int h = 0; h < HPG; ++h) {
            o0[h] = fmaf(pr[h], v.x, o0[h]);
            o1[h] = fmaf(pr[h], v.y, o1[h]);
        }
    }
    float* red = reinterpret_cast<float*>(smem);  // [VG][HPG][D] over the K chunk, free now
#pragma unroll
    for (int h = 0; h < HPG; ++h)
        *reinterpret_cast<float2*>(red + ((size_t)vg * HPG + h) * D + 2 * dt) = make_float2(o0[h], o1[h]);
    __syncthreads();
    const int stride = D + 2;
    float* mine = part + ((size_t)(b * n_heads + g * HPG) * MS + split) * stride;
    for (int i = tid; i < HPG * D; i += kBatThreads) {
        const int h = i / D, dd = i % D;
        float acc = 0.0f;
        for (int gg = 0; gg < VG; ++gg) acc += red[((size_t)gg * HPG + h) * D + dd];
        mine[(size_t)h * MS * stride + dd] = acc;
    }
    if (tid < HPG) {
        float* st = mine + (size_t)tid * MS * stride + D;
        st[0] = stat[tid][0];
        st[1] = stat[tid][1];
    }
    // The last CTA of (b, g) merges the splits (threadfence reduction).
    __threadfence();
    __syncthreads();
    unsigned int* cnt = counters + (size_t)b * kvh + g;
    if (tid == 0) last = atomicAdd(cnt, 1u) == (unsigned)(active - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    float* ls = reinterpret_cast<float*>(smem);  // [HPG][MS]
    for (int i = tid; i < HPG * active; i += kBatThreads) {
        const int h = i / active, s = i % active;
        const float* st = part + ((size_t)(b * n_heads + g * HPG + h) * MS + s) * stride + D;
        wsm[h][s] = st[0];
        ls[h * MS + s] = st[1];
    }
    __syncthreads();
    if (tid < HPG) {
        float M = -INFINITY;
        for (int s = 0; s < active; ++s) M = fmaxf(M, wsm[tid][s]);
        float L = 0.0f;
        for (int s = 0; s < active; ++s) {
            const float e = expf(wsm[tid][s] - M);
            wsm[tid][s] = e;
            L += ls[tid * MS + s] * e;
        }
        const float inv = 1.0f / fmaxf(L, 1e-20f);
        for (int s = 0; s < active; ++s) wsm[tid][s] *= inv;
    }
    __syncthreads();
    for (int i = tid; i < HPG * D; i += kBatThreads) {
        const int h = i / D, dd = i % D;
        const float* src = part + (size_t)(b * n_heads + g * HPG + h) * MS * stride + dd;
        float acc = 0.0f;
#pragma unroll 8
        for (int s = 0; s < active; ++s) acc = fmaf(wsm[h][s], src[(size_t)s * stride], acc);
        out[((long long)b * n_heads + g * HPG + h) * D + dd] = acc;
    }
    if (tid == 0) *cnt = 0u;
}

// The attention instantiation for a GQA group size (1, 2, 4 or 8) and a
// chunk of 32 or 128 context positions per CTA.
const void* attn_kernel_for(int hpg, int chunk) {
    if (chunk == 32) {
        switch (hpg) {
            case 1: return (const void*)bat_attn_kernel<1, 32>;
            case 2: return (const void*)bat_attn_kernel<2, 32>;
            case 4: return (const void*)bat_attn_kernel<4, 32>;
            case 8: return (const void*)bat_attn_kernel<8, 32>;
            default: return nullptr;
        }
    }
    switch (hpg) {
        case 1: return (const void*)bat_attn_kernel<1, 128>;
        case 2: return (const void*)bat_attn_kernel<2, 128>;
        case 4: return (const void*)bat_attn_kernel<4, 128>;
        case 8: return (const void*)bat_attn_kernel<8, 128>;
        default: return nullptr;
    }
}

// Dynamic shared memory of an attention CTA: the K and V chunks, reused for
// the value partials [VG][HPG][D] and the merge's sums [HPG][splits].
size_t attn_smem_for(int hpg, int D, int chunk) {
    size_t b = (size_t)2 * chunk * D * sizeof(__half);
    const size_t red = (size_t)(kBatThreads / (D / 2)) * hpg * D * sizeof(float);
    const size_t ls = (size_t)hpg * (kBatMaxCap / chunk) * sizeof(float);
    b = b > red ? b : red;
    return b > ls ? b : ls;
}

// token[b] = argmax key's index; out[step][b] = token; pos[b] += 1.
__global__ void bat_finish_kernel(const unsigned long long* keys, int B, int* token, int* pos, int* out,
                                  int* step, int max_steps) {
    griddep_wait();
    griddep_launch();
    const int s = *step;
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
        const int t = aexis_argmax_index(keys[b]);
        token[b] = t;
        if (s >= 0 && s < max_steps) out[(size_t)s * B + b] = t;
        pos[b] += 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) *step = s + 1;
}

}  // namespace

// ------------------------------------------------------- shared attention
bool split_attention_supported(int n_heads, int kvh, int D) {
    if (kvh <= 0 || n_heads % kvh) return false;
    const int hpg = n_heads / kvh;
    if (!attn_kernel_for(hpg, 128)) return false;
    const int dpt = 64 / hpg, tpp = D / dpt;
    return D >= 64 && D <= kBatMaxHeadDim && D % dpt == 0 && tpp >= 1 && tpp <= 32 && (tpp & (tpp - 1)) == 0;
}

int split_attention_max_cap() { return kBatMaxCap; }

size_t split_attention_part_floats(int B, int n_heads, int D, int chunk) {
    return (size_t)B * n_heads * (kBatMaxCap / chunk) * (D + 2);
}

cudaError_t split_attention_configure(int n_heads, int kvh, int D, int chunk) {
    const int hpg = n_heads / kvh;
    static size_t configured[64][2][4] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    const int ci = chunk == 32 ? 0 : 1, hi = hpg == 1 ? 0 : hpg == 2 ? 1 : hpg == 4 ? 2 : 3;
    const size_t smem = attn_smem_for(hpg, D, chunk);
    if (smem <= configured[dev][ci][hi]) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(attn_kernel_for(hpg, chunk), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e == cudaSuccess) configured[dev][ci][hi] = smem;
    return e;
}

cudaError_t launch_split_attention(const float* q, const __half* kc, const __half* vc, int cap, int D, int n_heads,
                                   int kvh, float scale, const int* pos, int B, float* part, unsigned int* counters,
                                   float* out, int* status, int chunk, cudaStream_t s) {
    const int hpg = n_heads / kvh;
    void* args[] = {(void*)&q, (void*)&kc, (void*)&vc, &cap, &D, &n_heads, &kvh, &scale, (void*)&pos, &part, &counters,
                    &out, &status};
    const int splits = (cap + chunk - 1) / chunk;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(splits, kvh, B);
    cfg.blockDim = dim3(kBatThreads);
    cfg.dynamicSmemBytes = attn_smem_for(hpg, D, chunk);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, attn_kernel_for(hpg, chunk), args);
}

// ------------------------------------------------------------------ host side
struct aexis_batch {
    aexis_decoder* d = nullptr;
    int max_batch = 0, cap = 0, max_steps = 0;
    int batch = 0;                       // sequences set by the last fill
    std::vector<int> host_pos;
    __half *kc = nullptr, *vc = nullptr; // [layers][max_batch][kvh][cap][D]
    float *cosv = nullptr, *sinv = nullptr;
    float *h = nullptr, *qkv = nullptr, *q = nullptr, *attn = nullptr, *gu = nullptr, *logits = nullptr;
    float* part = nullptr;
    void* xt = nullptr;
    unsigned int* counters = nullptr;    // [layers][max_batch][kvh]
    unsigned long long* keys = nullptr;  // [max_batch] argmax keys
    unsigned long long* seq_keys = nullptr;
    int* ctx = nullptr;                  // [max_batch] context lengths of the last fill
    int* ints = nullptr;                 // [0] step, [1..] tokens, then positions, then out [max_steps][batch]
    std::vector<void*> tiled;            // tensor-core copies: 4 per layer, then the lm_head
    cudaGraphExec_t exec = nullptr;
    int exec_batch = 0;
    // Tensor-core attention (k_batch_attn.cu, head_dim 128): caches stored
    // with swizzled rows, the split merge folded into the O projection's prep.
    bool tc_attn = false;
    int tc_attn_grid = 0;
};

namespace {

int bbind(aexis_batch* b) {
    return aexis_cuda_check(b->d->ctx, cudaSetDevice(b->d->ctx->device), "cudaSetDevice");
}

int balloc(aexis_batch* b, void** p, size_t bytes) {
    cudaError_t e = cudaMalloc(p, bytes);
    if (e == cudaSuccess) e = cudaMemset(*p, 0, bytes);
    return aexis_cuda_check(b->d->ctx, e, "batch alloc");
}

cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}


// Host copy of the per-sequence key: mix64(seed ^ mix64(sequence id)).
unsigned long long seq_key(unsigned long long seed, long long id) {
    return mix64(seed ^ mix64((unsigned long long)id));
}

cudaError_t gemm(aexis_batch* bt, const aexis_weights& w, const void* tiled, int B, float* y, int ldy, int accumulate,
                 cudaStream_t s) {
    TcLaunch a;
    a.w = &w;
    a.tiled = tiled;
    a.xt = bt->xt;
    a.m = B;
    a.split = 1;
    a.y = y;
    a.y_dtype = AEXIS_F32;
    a.ldy = ldy;
    a.accumulate = accumulate;
    a.sm_count = bt->d->ctx->sm_count;
    a.status = bt->d->ctx->status;
    a.pdl = true;
    return launch_gemm_tc_prepared(a, s);
}

cudaError_t enqueue_batch_step(aexis_batch* bt, cudaStream_t s, int B) {
    aexis_decoder* d = bt->d;
    const auto& c = d->cfg;
    const int D = c.head_dim, NH = c.n_heads, KVH = c.n_kv_heads, H = c.hidden, F = c.ffn;
    const int qd = NH * D, rows = qd + 2 * KVH * D;
    int* step = bt->ints;
    int* token = bt->ints + 1;
    int* pos = bt->ints + 1 + bt->max_batch;
    int* out = bt->ints + 1 + 2 * bt->max_batch;
    cudaError_t e;
    {
        const __half* tab = d->embed;
        int vocab = c.vocab, hidden = H;
        float* h = bt->h;
        void* args[] = {(void*)&tab, &vocab, &hidden, &token, &h};
        if ((e = launch_pdl((const void*)bat_embed_kernel, dim3((H + 255) / 256, B), dim3(256), 0, s, args)) !=
            cudaSuccess)
            return e;
    }
    const float scale = 1.0f / sqrtf((float)D);
    const size_t layer_kv = (size_t)bt->max_batch * KVH * bt->cap * D;
    for (int l = 0; l < c.n_layers; ++l) {
        auto& L = d->layers[l];
        __half* kc = bt->kc + (size_t)l * layer_kv;
        __half* vc = bt->vc + (size_t)l * layer_kv;
        if ((e = launch_tc_prep(1, bt->h, 0, H, B, H, L.norm[0], c.eps, 1, bt->xt, bt->qkv, rows, rows, true, s)) !=
            cudaSuccess)
            return e;
        if ((e = gemm(bt, L.qkv, bt->tiled[l * 4 + 0], B, bt->qkv, rows, 1, s)) != cudaSuccess) return e;
        if (bt->tc_attn) {
            // RoPE and the KV append happen inside the attention kernel.
            if ((e = launch_batch_tc_attention(bt->qkv, rows, bt->cosv, bt->sinv, c.rot_dim, kc, vc, bt->cap, NH, KVH,
                                               scale, pos, B, bt->part, bt->tc_attn_grid, d->ctx->status, s)) !=
                cudaSuccess)
                return e;
            if ((e = launch_batch_attn_merge_prep(bt->part, pos, B, NH, KVH, bt->tc_attn_grid, bt->xt, s)) !=
                cudaSuccess)
                return e;
        } else {
            const float* qkv = bt->qkv;
            int r = rows, hd = D, rot = c.rot_dim, nh = NH, nkv = KVH, cap = bt->cap, bb = B;
            const int* map = d->rope_map;
            const float* cs = bt->cosv;
            const float* sn = bt->sinv;
            const int* pp = pos;
            float* qo = bt->q;
            int swz = 0;
            void* args[] = {(void*)&qkv, &r, (void*)&map, (void*)&cs, (void*)&sn, (void*)&pp, &hd, &rot, &nh, &nkv,
                            &cap, &bb, &qo, &kc, &vc, &swz};
            if ((e = launch_pdl((const void*)bat_rope_kernel, dim3((rows + 255) / 256, B), dim3(256), 0, s, args)) !=
                cudaSuccess)
                return e;
            if ((e = launch_split_attention(bt->q, kc, vc, bt->cap, D, NH, KVH, scale, pos, B, bt->part,
                                            bt->counters + (size_t)l * bt->max_batch * KVH, bt->attn, d->ctx->status,
                                            kBatChunk, s)) != cudaSuccess)
                return e;
            if ((e = launch_tc_prep(0, bt->attn, 0, qd, B, qd, nullptr, 0.0f, 1, bt->xt, nullptr, 0, 0, true, s)) !=
                cudaSuccess)
                return e;
        }
        if ((e = gemm(bt, L.o, bt->tiled[l * 4 + 1], B, bt->h, H, 1, s)) != cudaSuccess) return e;
        if ((e = launch_tc_prep(1, bt->h, 0, H, B, H, L.norm[1], c.eps, 1, bt->xt, bt->gu, 2 * F, 2 * F, true, s)) !=
            cudaSuccess)
            return e;
        if ((e = gemm(bt, L.gateup, bt->tiled[l * 4 + 2], B, bt->gu, 2 * F, 1, s)) != cudaSuccess) return e;
        if ((e = launch_tc_prep(2, bt->gu, 0, 2 * F, B, F, nullptr, 0.0f, 1, bt->xt, nullptr, 0, 0, true, s)) !=
            cudaSuccess)
            return e;
        if ((e = gemm(bt, L.down, bt->tiled[l * 4 + 3], B, bt->h, H, 1, s)) != cudaSuccess) return e;
    }
    if ((e = launch_tc_prep(1, bt->h, 0, H, B, H, d->final_norm, c.eps, 1, bt->xt, nullptr, 0, 0, true, s)) !=
        cudaSuccess)
        return e;
    if ((e = gemm(bt, d->lm, bt->tiled[4 * c.n_layers], B, bt->logits, c.vocab, 0, s)) != cudaSuccess) return e;
    if ((e = launch_argmax_keys(bt->logits, B, c.vocab, c.vocab, 0, bt->keys, d->ctx->sm_count, s)) != cudaSuccess)
        return e;
    {
        const unsigned long long* keys = bt->keys;
        int bb = B, ms = bt->max_steps;
        void* args[] = {(void*)&keys, &bb, &token, &pos, &out, &step, &ms};
        e = launch_pdl((const void*)bat_finish_kernel, dim3(1), dim3(128), 0, s, args);
    }
    return e;
}

int capture_batch(aexis_batch* bt, int B) {
    aexis_ctx* ctx = bt->d->ctx;
    if (bt->exec && bt->exec_batch == B) return AEXIS_OK;
    if (bt->exec) {
        cudaGraphExecDestroy(bt->exec);
        bt->exec = nullptr;
    }
    cudaStream_t s = ctx->own_stream;
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return aexis_cuda_check(ctx, e, "begin capture");
    cudaError_t le = enqueue_batch_step(bt, s, B);
    e = cudaStreamEndCapture(s, &graph);
    if (le != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return aexis_cuda_check(ctx, le, "batch step launch (capture)");
    }
    if (e != cudaSuccess) return aexis_cuda_check(ctx, e, "end capture");
    e = cudaGraphInstantiateWithFlags(&bt->exec, graph, 0);
    cudaGraphDestroy(graph);
    if (e == cudaSuccess) bt->exec_batch = B;
    return aexis_cuda_check(ctx, e, "graph instantiate");
}

}  // namespace

AEXIS_API int aexis_cuda_batch_destroy(aexis_batch* bt) {
    if (!bt) return AEXIS_E_NULL;
    cudaSetDevice(bt->d->ctx->device);
    cudaStreamSynchronize(bt->d->ctx->stream);
    if (bt->exec) cudaGraphExecDestroy(bt->exec);
    for (void* p : bt->tiled)
        if (p) cudaFree(p);
    void* bufs[] = {bt->kc, bt->vc, bt->cosv, bt->sinv, bt->h, bt->qkv, bt->q, bt->attn, bt->gu, bt->logits,
                    bt->part, bt->xt, bt->counters, bt->keys, bt->seq_keys, bt->ctx, bt->ints};
    for (void* p : bufs)
        if (p) cudaFree(p);
    delete bt;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_batch_create(aexis_decoder* d, int max_batch, int kv_capacity, int max_steps,
                                      aexis_batch** out) {
    if (!d) return AEXIS_E_NULL;
    aexis_ctx* ctx = d->ctx;
    if (!out) return aexis_fail(ctx, AEXIS_E_NULL, "out is null");
    *out = nullptr;
    const auto& c = d->cfg;
    if (c.bits != 8 || c.lm_bits != 8)
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "batched decoding runs Q8 weights (bits=%d lm_bits=%d)", c.bits,
                          c.lm_bits);
    const int D = c.head_dim, qd = c.n_heads * D;
    if (d->hybrid)
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "batched decoding runs full-attention stacks only");
    if (c.hidden % 64 || qd % 64 || c.ffn % 64)
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "hidden, ffn and heads*head_dim must be multiples of 64");
    {
        // Attention layout: group 1, 2, 4 or 8; 64 / group query dims per
        // thread, head_dim / that a power of two <= 32; head_dim 64..256.
        if (!split_attention_supported(c.n_heads, c.n_kv_heads, D))
            return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "head_dim %d with %d query heads per KV head", D,
                              c.n_heads / c.n_kv_heads);
    }
    if (max_batch < 1 || max_batch > 128) return aexis_fail(ctx, AEXIS_E_RANGE, "max_batch %d (1..128)", max_batch);
    if (kv_capacity < 1 || kv_capacity > kBatMaxCap)
        return aexis_fail(ctx, AEXIS_E_RANGE, "kv_capacity %d (1..%d)", kv_capacity, kBatMaxCap);
    if (max_steps < 1) return aexis_fail(ctx, AEXIS_E_RANGE, "max_steps %d", max_steps);
    for (int l = 0; l < c.n_layers; ++l)
        if (d->layers[l].set_mask != 0x1FF)
            return aexis_fail(ctx, AEXIS_E_STATE, "layer %d weights incomplete (mask 0x%x)", l, d->layers[l].set_mask);
    if (!d->lm_set || !d->final_set || !d->embed_set)
        return aexis_fail(ctx, AEXIS_E_STATE, "lm_head/final norm/embedding not set");
    int rc = aexis_cuda_check(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    if (rc) return rc;
    aexis_batch* bt = new (std::nothrow) aexis_batch();
    if (!bt) return aexis_fail(ctx, AEXIS_E_STATE, "out of host memory");
    bt->d = d;
    bt->max_batch = max_batch;
    bt->cap = kv_capacity;
    bt->max_steps = max_steps;
    bt->host_pos.assign(max_batch, 0);
    const int KVH = c.n_kv_heads, H = c.hidden, F = c.ffn;
    const int rows = qd + 2 * KVH * D;
    const size_t kv = (size_t)c.n_layers * max_batch * KVH * kv_capacity * D;
    if (!rc) rc = balloc(bt, (void**)&bt->kc, kv * sizeof(__half));
    if (!rc) rc = balloc(bt, (void**)&bt->vc, kv * sizeof(__half));
    if (!rc) rc = balloc(bt, (void**)&bt->h, sizeof(float) * max_batch * H);
    if (!rc) rc = balloc(bt, (void**)&bt->qkv, sizeof(float) * max_batch * rows);
    if (!rc) rc = balloc(bt, (void**)&bt->q, sizeof(float) * max_batch * qd);
    if (!rc) rc = balloc(bt, (void**)&bt->attn, sizeof(float) * max_batch * qd);
    if (!rc) rc = balloc(bt, (void**)&bt->gu, sizeof(float) * max_batch * 2 * F);
    if (!rc) rc = balloc(bt, (void**)&bt->logits, sizeof(float) * max_batch * c.vocab);
    bt->tc_attn = batch_tc_attention_supported(c.n_heads, KVH, D, max_batch, kv_capacity);
    if (!rc) {
        size_t pf = split_attention_part_floats(max_batch, c.n_heads, D, kBatChunk);
        if (bt->tc_attn) pf = pf > batch_tc_attention_part_floats(max_batch, c.n_heads)
                                  ? pf : batch_tc_attention_part_floats(max_batch, c.n_heads);
        rc = balloc(bt, (void**)&bt->part, sizeof(float) * pf);
    }
    if (!rc) {
        const int kmax = H > qd ? (H > F ? H : F) : (qd > F ? qd : F);
        rc = balloc(bt, &bt->xt, gemm_tc_xt_bytes(max_batch, kmax, AEXIS_F32));
    }
    if (!rc) rc = balloc(bt, (void**)&bt->counters, sizeof(unsigned int) * c.n_layers * max_batch * KVH);
    if (!rc) rc = balloc(bt, (void**)&bt->keys, sizeof(unsigned long long) * max_batch);
    if (!rc) rc = balloc(bt, (void**)&bt->seq_keys, sizeof(unsigned long long) * max_batch);
    if (!rc) rc = balloc(bt, (void**)&bt->ctx, sizeof(int) * max_batch);
    if (!rc) rc = balloc(bt, (void**)&bt->ints, sizeof(int) * (1 + 2 * (size_t)max_batch + (size_t)max_steps * max_batch));
    if (!rc && c.rot_dim > 0) {
        std::vector<float> cs, sn;
        decoder_rope_tables(kv_capacity, c.rot_dim, c.rope_theta, cs, sn);
        rc = balloc(bt, (void**)&bt->cosv, sizeof(float) * cs.size());
        if (!rc) rc = balloc(bt, (void**)&bt->sinv, sizeof(float) * sn.size());
        if (!rc)
            rc = aexis_cuda_check(ctx, cudaMemcpy(bt->cosv, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice),
                                  "rope upload");
        if (!rc)
            rc = aexis_cuda_check(ctx, cudaMemcpy(bt->sinv, sn.data(), sizeof(float) * sn.size(), cudaMemcpyHostToDevice),
                                  "rope upload");
    }
    // Tensor-core copies of every linear (repacked once, read every step).
    if (!rc) {
        bt->tiled.assign(4 * (size_t)c.n_layers + 1, nullptr);
        for (int l = 0; l <= c.n_layers && !rc; ++l)
            for (int j = 0; j < (l < c.n_layers ? 4 : 1) && !rc; ++j) {
                const aexis_weights* w = l == c.n_layers ? &d->lm
                                         : j == 0       ? &d->layers[l].qkv
                                         : j == 1       ? &d->layers[l].o
                                         : j == 2       ? &d->layers[l].gateup
                                                        : &d->layers[l].down;
                void** dst = &bt->tiled[(size_t)l * 4 + j];
                rc = balloc(bt, dst, gemm_tc_tiled_bytes(w));
                if (!rc) rc = aexis_cuda_check(ctx, launch_repack_q8(w, *dst, ctx->stream), "weight repack");
            }
    }
    if (!rc) {
        rc = aexis_cuda_check(ctx, split_attention_configure(c.n_heads, c.n_kv_heads, D, kBatChunk),
                              "attention smem");
    }
    if (!rc && bt->tc_attn)
        rc = aexis_cuda_check(ctx, batch_tc_attention_configure(ctx->sm_count, &bt->tc_attn_grid), "attention smem");
    if (!rc) rc = aexis_cuda_check(ctx, cudaStreamSynchronize(ctx->stream), "batch setup");
    if (rc) {
        aexis_cuda_batch_destroy(bt);
        return rc;
    }
    *out = bt;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_batch_fill_context(aexis_batch* bt, int batch, const int32_t* ctx_lens, uint64_t seed,
                                            int64_t first_seq_id) {
    if (!bt) return AEXIS_E_NULL;
    aexis_ctx* ctx = bt->d->ctx;
    if (!ctx_lens) return aexis_fail(ctx, AEXIS_E_NULL, "ctx_lens is null");
    if (batch < 1 || batch > bt->max_batch)
        return aexis_fail(ctx, AEXIS_E_RANGE, "batch %d (1..%d)", batch, bt->max_batch);
    for (int i = 0; i < batch; ++i) {
        if (ctx_lens[i] < 0 || ctx_lens[i] >= bt->cap)
            return aexis_fail(ctx, AEXIS_E_RANGE, "context %d of sequence %d outside [0, %d)", ctx_lens[i], i, bt->cap);
    }
    int rc = bbind(bt);
    if (rc) return rc;
    std::vector<unsigned long long> keys(batch);
    for (int i = 0; i < batch; ++i) keys[i] = seq_key(seed, first_seq_id + i);
    cudaStream_t s = ctx->stream;
    cudaError_t e = cudaMemcpyAsync(bt->ctx, ctx_lens, sizeof(int) * batch, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess)
        e = cudaMemcpyAsync(bt->seq_keys, keys.data(), sizeof(unsigned long long) * batch, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) {
        const auto& c = bt->d->cfg;
        bat_fill_kernel<<<dim3(ctx->sm_count * 4, batch), 256, 0, s>>>(
            bt->kc, bt->vc, c.n_layers, bt->max_batch, c.n_kv_heads, bt->cap, c.head_dim, bt->ctx, bt->seq_keys,
            bt->ints + 1 + bt->max_batch, bt->tc_attn ? 1 : 0);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemsetAsync(bt->ints, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    rc = aexis_cuda_check(ctx, e, "context fill");
    if (rc) return rc;
    bt->batch = batch;
    for (int i = 0; i < batch; ++i) bt->host_pos[i] = ctx_lens[i];
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_batch_set_positions(aexis_batch* bt, int batch, const int32_t* positions) {
    if (!bt) return AEXIS_E_NULL;
    aexis_ctx* ctx = bt->d->ctx;
    if (!positions) return aexis_fail(ctx, AEXIS_E_NULL, "positions is null");
    if (batch < 1 || batch > bt->max_batch)
        return aexis_fail(ctx, AEXIS_E_RANGE, "batch %d (1..%d)", batch, bt->max_batch);
    for (int i = 0; i < batch; ++i)
        if (positions[i] < 0 || positions[i] >= bt->cap)
            return aexis_fail(ctx, AEXIS_E_RANGE, "position %d of sequence %d outside [0, %d)", positions[i], i,
                              bt->cap);
    int rc = bbind(bt);
    if (rc) return rc;
    cudaStream_t s = ctx->stream;
    cudaError_t e = cudaMemcpyAsync(bt->ints + 1 + bt->max_batch, positions, sizeof(int) * batch,
                                    cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(bt->ints, 0, sizeof(int), s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    rc = aexis_cuda_check(ctx, e, "position upload");
    if (rc) return rc;
    bt->batch = batch;
    for (int i = 0; i < batch; ++i) bt->host_pos[i] = positions[i];
    return AEXIS_OK;
}

static int batch_kv_args(aexis_batch* bt, int seq, int layer, int rows, const void* k, const void* v) {
    aexis_ctx* ctx = bt->d->ctx;
    if (!k || !v) return aexis_fail(ctx, AEXIS_E_NULL, "K/V buffer is null");
    if (seq < 0 || seq >= bt->max_batch)
        return aexis_fail(ctx, AEXIS_E_RANGE, "sequence %d outside [0, %d)", seq, bt->max_batch);
    if (layer < 0 || layer >= bt->d->cfg.n_layers)
        return aexis_fail(ctx, AEXIS_E_RANGE, "layer %d outside [0, %d)", layer, bt->d->cfg.n_layers);
    if (rows <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "rows=%d", rows);
    return bbind(bt);
}

static size_t batch_kv_offset(const aexis_batch* bt, int seq, int layer) {
    const auto& c = bt->d->cfg;
    return (((size_t)layer * bt->max_batch + seq) * c.n_kv_heads) * bt->cap * c.head_dim;
}

AEXIS_API int aexis_cuda_batch_kv_export(aexis_batch* bt, int seq, int layer, int rows, float* k_out, float* v_out) {
    if (!bt) return AEXIS_E_NULL;
    int rc = batch_kv_args(bt, seq, layer, rows, k_out, v_out);
    if (rc) return rc;
    aexis_ctx* ctx = bt->d->ctx;
    const int len = seq < bt->batch ? bt->host_pos[seq] : 0;
    if (rows < len) return aexis_fail(ctx, AEXIS_E_SHAPE, "rows %d < sequence length %d", rows, len);
    const auto& c = bt->d->cfg;
    const size_t off = batch_kv_offset(bt, seq, layer);
    return aexis_cuda_check(ctx, launch_kv_export(bt->kc + off, bt->vc + off, c.n_kv_heads, bt->cap, c.head_dim,
                                                  bt->tc_attn ? 1 : 0, len, rows, k_out, v_out, ctx->stream),
                            "kv export launch");
}

AEXIS_API int aexis_cuda_batch_kv_import(aexis_batch* bt, int seq, int layer, const float* k_in, const float* v_in,
                                         int rows, int length) {
    if (!bt) return AEXIS_E_NULL;
    int rc = batch_kv_args(bt, seq, layer, rows, k_in, v_in);
    if (rc) return rc;
    aexis_ctx* ctx = bt->d->ctx;
    if (length < 0 || length > rows || length >= bt->cap)
        return aexis_fail(ctx, AEXIS_E_RANGE, "length %d outside [0, min(rows %d, capacity %d - 1)]", length, rows,
                          bt->cap);
    const auto& c = bt->d->cfg;
    const size_t off = batch_kv_offset(bt, seq, layer);
    return aexis_cuda_check(ctx, launch_kv_import(k_in, v_in, c.n_kv_heads, bt->cap, c.head_dim, bt->tc_attn ? 1 : 0,
                                                  length, rows, bt->kc + off, bt->vc + off, ctx->stream),
                            "kv import launch");
}

AEXIS_API int aexis_cuda_batch_generate(aexis_batch* bt, const int32_t* first_tokens, int steps, int32_t* out_tokens) {
    if (!bt) return AEXIS_E_NULL;
    aexis_ctx* ctx = bt->d->ctx;
    if (!first_tokens) return aexis_fail(ctx, AEXIS_E_NULL, "first_tokens is null");
    if (bt->batch < 1) return aexis_fail(ctx, AEXIS_E_STATE, "no context: call aexis_cuda_batch_fill_context first");
    if (steps < 1 || steps > bt->max_steps)
        return aexis_fail(ctx, AEXIS_E_RANGE, "steps %d (1..%d)", steps, bt->max_steps);
    const int B = bt->batch;
    for (int i = 0; i < B; ++i)
        if (bt->host_pos[i] + steps > bt->cap)
            return aexis_fail(ctx, AEXIS_E_RANGE, "sequence %d: position %d + %d steps exceeds capacity %d", i,
                              bt->host_pos[i], steps, bt->cap);
    int rc = bbind(bt);
    if (rc) return rc;
    rc = capture_batch(bt, B);
    if (rc) return rc;
    cudaStream_t s = ctx->stream;
    cudaError_t e = cudaMemcpyAsync(bt->ints + 1, first_tokens, sizeof(int) * B, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(bt->ints, 0, sizeof(int), s);
    for (int i = 0; i < steps && e == cudaSuccess; ++i) e = cudaGraphLaunch(bt->exec, s);
    if (e == cudaSuccess && out_tokens)
        e = cudaMemcpyAsync(out_tokens, bt->ints + 1 + 2 * bt->max_batch, sizeof(int) * (size_t)steps * B,
                            cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    rc = aexis_cuda_check(ctx, e, "batch generate");
    if (rc) return rc;
    rc = aexis_check_status(ctx);
    if (rc) return rc;
    for (int i = 0; i < B; ++i) bt->host_pos[i] += steps;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_batch_positions(const aexis_batch* bt, int32_t* out) {
    if (!bt || !out) return AEXIS_E_NULL;
    for (int i = 0; i < bt->batch; ++i) out[i] = bt->host_pos[i];
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_batch_logits(aexis_batch* bt, float* out) {
    if (!bt) return AEXIS_E_NULL;
    if (!out) return aexis_fail(bt->d->ctx, AEXIS_E_NULL, "out is null");
    int rc = bbind(bt);
    if (rc) return rc;
    cudaError_t e = cudaMemcpy(out, bt->logits, sizeof(float) * (size_t)bt->batch * bt->d->cfg.vocab,
                               cudaMemcpyDeviceToHost);
    return aexis_cuda_check(bt->d->ctx, e, "logits read");
}
