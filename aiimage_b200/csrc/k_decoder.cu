// k_decoder.cu -- the fused batch-1 decode step of the synthetic decoder
// (Qwen35DecoderSession.DecodeCore + SelectNextToken, greedy), all layers
// full attention or Qwen3.5's hybrid stack of linear- and full-attention
// blocks.
//
// One step is a chain of kernels captured once into a CUDA graph, every edge a
// programmatic dependent launch (each kernel streams its weights while the
// previous one drains, then waits for its activation input):
//   embed      h = E[token] (fp16 table -> fp32), clear the argmax key
//   per full-attention layer
//              qkv   RMSNorm prologue + Q4/Q8 GEMV + RoPE + fp16 KV append
//              attn  split-K GQA decode attention, last CTA per KV head merges
//              o     GEMV, residual add into h
//   per linear-attention layer
//              in    RMSNorm prologue + GEMV to [q k v z b a] (fp32)
//              core  ShortConv + SiLU, Gated Delta Rule, gated per-head
//                    RMSNorm (lin_attn_decode_kernel, k_recurrent.cu)
//              out   GEMV, residual add into h
//   per layer  ffn1  RMSNorm prologue + fused gate|up GEMV + SiLU*up
//              ffn2  down GEMV, residual add into h
//   lm_head    RMSNorm prologue + GEMV, logits + fused greedy argmax key
//   finish     token = argmax, position += 1
// Position and token live in device memory, so the same graph replays for
// every step. Replaces ~869 Unity dispatches and 3 graph invocations per token
// (Qwen35DecoderSession.cs:463-585, 715-810).
#include <algorithm>
#include <cmath>
#include <cstring>
#include <new>

#include "decoder_internal.h"

#define AEXIS_API extern "C" __attribute__((visibility("default")))

namespace {

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

constexpr int kAttnSplits = 64;   // context splits per KV head (fixed at capture)
constexpr int kAttnThreads = 128;
constexpr int kMaxHeadDim = 256;
constexpr int kMaxGroup = 8;      // query heads per KV head
constexpr int kMinChunk = 32;     // fewest context positions per split
constexpr int kMaxChunk = 64;     // chunk bound at the largest supported capacity
// The Gated Delta Rule's norm eps (reference_ops.py gated_delta_rule default,
// the value the reference's GatedDeltaRule layer is exported with).
constexpr float kGdrEps = 1e-6f;

// h = E[token], key = 0. token_src[token_idx ? *token_idx : 0].
__global__ void dec_embed_kernel(const __half* table, int vocab, int hidden, const int* token,
                                 float* h, unsigned long long* key) {
    griddep_wait();
    griddep_launch();
    int t = *token;
    t = t < 0 ? 0 : (t >= vocab ? vocab - 1 : t);
    const __half* row = table + (long long)t * hidden;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
        h[i] = __half2float(row[i]);
    if (blockIdx.x == 0 && threadIdx.x == 0) *key = 0ull;
}

// Split-K decode attention for one KV head and one context split.
// q: fp32 [n_heads][D] (RoPE applied); caches: fp16 [kv_heads][cap][D].
// Context positions are cut into `active` splits of `chunk` positions
// (chunk = max(32, ceil(ctx / kAttnSplits))); CTAs past the active count exit.
// Scores s = (q . k) * scale; each split keeps (max m, sum l, o = sum e*v);
// the last CTA of a KV head merges the splits with weights
// w_s = e^(m_s - M) / sum_s l_s e^(m_s - M), computed once in shared memory,
// then out = sum_s w_s o_s with independent loads. Mathematically the
// reference's two-pass softmax (HLSL Pack4Matmul:485-547); no context cap
// beyond the cache capacity.
__global__ void __launch_bounds__(kAttnThreads) dec_attn_kernel(
    const float* q, const __half* kc, const __half* vc, int cap, int D, int n_heads, int n_kv,
    float scale, const int* pos_ptr, float* part, unsigned int* counters, float* out) {
    __shared__ float qs[kMaxGroup][kMaxHeadDim];
    __shared__ float sc[kMaxGroup][kMaxChunk];
    __shared__ float stat[kMaxGroup][2];
    __shared__ float wsm[kMaxGroup][kAttnSplits];
    __shared__ bool last;
    griddep_wait();
    griddep_launch();
    const int g = blockIdx.x, split = blockIdx.y;
    const int hpg = n_heads / n_kv;
    const int ctx = *pos_ptr + 1;
    int chunk = (ctx + kAttnSplits - 1) / kAttnSplits;
    chunk = chunk < kMinChunk ? kMinChunk : chunk;
    const int active = (ctx + chunk - 1) / chunk;
    if (split >= active) return;
    const int p0 = split * chunk, p1 = min(ctx, p0 + chunk);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int i = tid; i < hpg * D; i += kAttnThreads) qs[i / D][i % D] = q[(g * hpg + i / D) * D + i % D];
    __syncthreads();
    const __half* kb = kc + (long long)g * cap * D;
    const __half* vb = vc + (long long)g * cap * D;
    // Scores: one warp per position, each lane four consecutive dims.
    for (int p = p0 + warp; p < p1; p += kAttnThreads / 32) {
        float acc[kMaxGroup];
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) acc[h] = 0.0f;
        for (int d = lane * 4; d < D; d += 128) {
            const uint2 raw = *reinterpret_cast<const uint2*>(kb + (long long)p * D + d);
            const float2 k01 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
            const float2 k23 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h)
                if (h < hpg)
                    acc[h] = fmaf(qs[h][d + 3], k23.y, fmaf(qs[h][d + 2], k23.x,
                             fmaf(qs[h][d + 1], k01.y, fmaf(qs[h][d], k01.x, acc[h]))));
        }
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) {
            if (h >= hpg) break;
            float v = acc[h];
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            if (lane == 0) sc[h][p - p0] = v * scale;
        }
    }
    __syncthreads();
    // Per head: local max and exp-sum over this split (warp h handles head h).
    for (int h = warp; h < hpg; h += kAttnThreads / 32) {
        float m = -INFINITY;
        for (int i = lane; i < p1 - p0; i += 32) m = fmaxf(m, sc[h][i]);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float l = 0.0f;
        for (int i = lane; i < p1 - p0; i += 32) {
            const float e = expf(sc[h][i] - m);
            sc[h][i] = e;
            l += e;
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
        if (lane == 0) { stat[h][0] = m; stat[h][1] = l; }
    }
    __syncthreads();
    // o[h][d] = sum_p e[h][p] * v[p][d]; threads across d.
    const int stride = D + 2;
    for (int d = tid; d < D; d += kAttnThreads) {
        float o[kMaxGroup];
#pragma unroll
        for (int h = 0; h < kMaxGroup; ++h) o[h] = 0.0f;
        for (int p = p0; p < p1; ++p) {
            const float vv = __half2float(vb[(long long)p * D + d]);
#pragma unroll
            for (int h = 0; h < kMaxGroup; ++h)
                if (h < hpg) o[h] = fmaf(sc[h][p - p0], vv, o[h]);
        }
        for (int h = 0; h < hpg; ++h)
            part[((long long)(g * hpg + h) * kAttnSplits + split) * stride + d] = o[h];
    }
    if (tid < hpg) {
        float* st = part + ((long long)(g * hpg + tid) * kAttnSplits + split) * stride + D;
        st[0] = stat[tid][0];
        st[1] = stat[tid][1];
    }
    // Last CTA of this KV head merges the splits (threadfence reduction).
    __threadfence();
    __syncthreads();
    if (tid == 0) last = atomicAdd(counters + g, 1u) == (unsigned)(active - 1);
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = tid; i < hpg * active; i += kAttnThreads) {
        const int h = i / active, s = i % active;
        const float* st = part + ((long long)(g * hpg + h) * kAttnSplits + s) * stride + D;
        wsm[h][s] = st[0];
        sc[h][s] = st[1];
    }
    __syncthreads();
    if (tid < hpg) {
        float M = -INFINITY;
        for (int s = 0; s < active; ++s) M = fmaxf(M, wsm[tid][s]);
        float L = 0.0f;
        for (int s = 0; s < active; ++s) {
            const float e = expf(wsm[tid][s] - M);
            wsm[tid][s] = e;
            L += sc[tid][s] * e;
        }
        const float inv = 1.0f / fmaxf(L, 1e-20f);
        for (int s = 0; s < active; ++s) wsm[tid][s] *= inv;
    }
    __syncthreads();
    for (int i = tid; i < hpg * D; i += kAttnThreads) {
        const int h = i / D, d = i % D;
        const float* base = part + (long long)(g * hpg + h) * kAttnSplits * stride + d;
        float acc = 0.0f;
#pragma unroll 8
        for (int s = 0; s < active; ++s) acc = fmaf(wsm[h][s], base[(long long)s * stride], acc);
        out[(g * hpg + h) * D + d] = acc;
    }
    if (tid == 0) counters[g] = 0u;
}

// token = argmax(key); out_tokens[*step] = token while *step < max_out;
// position += 1.
__global__ void dec_finish_kernel(const unsigned long long* key, int* token, int* pos, int* out_tokens,
                                  int* step, int emit, int max_out) {
    griddep_wait();
    griddep_launch();
    if (threadIdx.x == 0 && blockIdx.x == 0) {
        if (emit) {
            const int t = aexis_argmax_index(*key);
            *token = t;
            const int s = *step;
            if (out_tokens && s >= 0 && s < max_out) out_tokens[s] = t;
            *step = s + 1;
        }
        *pos += 1;
    }
}

}  // namespace

// ------------------------------------------------------------------ host side


namespace {

int dbind(aexis_decoder* d) { return aexis_cuda_check(d->ctx, cudaSetDevice(d->ctx->device), "cudaSetDevice"); }

int alloc(aexis_decoder* d, void** p, size_t bytes, const char* what) {
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return aexis_cuda_check(d->ctx, e, what);
    e = cudaMemset(*p, 0, bytes);
    return aexis_cuda_check(d->ctx, e, what);
}

// Internal weight handle for a fused matrix of `n` rows x k.
int alloc_weights(aexis_decoder* d, aexis_weights& w, int bits, int group, int scale_dtype, int n, int k) {
    w.kind = bits == 4 ? WK_Q4 : WK_Q8;
    w.n = n;
    w.k = k;
    w.group = bits == 4 ? group : 0;
    w.scale_dtype = scale_dtype;
    w.data_bytes = (size_t)n * k / (bits == 4 ? 2 : 1);
    const size_t nscales = bits == 4 ? (size_t)n * (k / group) : (size_t)n;
    w.scale_bytes = nscales * (scale_dtype == AEXIS_F16 ? 2 : 4);
    int rc = alloc(d, &w.data, w.data_bytes + kWeightPad, "decoder weight alloc");
    if (rc == AEXIS_OK) rc = alloc(d, &w.scales, w.scale_bytes + kWeightPad, "decoder scale alloc");
    return rc;
}

void free_weights(aexis_weights& w) {
    if (w.data) cudaFree(w.data);
    if (w.scales) cudaFree(w.scales);
    if (w.frag) cudaFree(w.frag);
    if (w.frag_scales) cudaFree(w.frag_scales);
    w.data = w.scales = w.frag = w.frag_scales = nullptr;
}

// The tensor-core GEMV's fragment copy of a Q4 matrix (built once; rebuilt
// in place when the matrix is reloaded, so captured graphs stay valid).
int build_frag(aexis_decoder* d, aexis_weights& w) {
    if (!gemv_mma_eligible(&w)) return AEXIS_OK;
    cudaError_t e = cudaSuccess;
    if (!w.frag) {
        size_t sb = 0;
        const size_t wb = gemv_mma_frag_bytes(&w, &sb);
        e = cudaMalloc(&w.frag, wb);
        if (e == cudaSuccess) e = cudaMalloc(&w.frag_scales, sb);
    }
    if (e == cudaSuccess) e = launch_repack_frag(&w, d->ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(d->ctx->stream);
    return aexis_cuda_check(d->ctx, e, "decoder fragment repack");
}

// Copies logical rows [0, rows) of a packed matrix into internal rows
// dst_lo + dst_stride * perm[r] of `w` (perm empty = identity): the rows are
// permuted on the host, then one strided 2-D copy per array.
int scatter_rows(aexis_decoder* d, aexis_weights& w, const uint32_t* packed, const void* scales, int scale_dtype,
                 int rows, int dst_lo, int dst_stride, const std::vector<int>& perm) {
    const size_t row_bytes = w.data_bytes / w.n;
    const size_t srow = w.scale_bytes / w.n;
    if (scale_dtype != w.scale_dtype)
        return aexis_fail(d->ctx, AEXIS_E_SHAPE, "scale dtype %d differs from the decoder's (%d)", scale_dtype,
                          w.scale_dtype);
    const char* src = (const char*)packed;
    const char* ssrc = (const char*)scales;
    std::vector<char> tmp, stmp;
    if (!perm.empty()) {
        tmp.resize(row_bytes * rows);
        stmp.resize(srow * rows);
        for (int r = 0; r < rows; ++r) {
            std::memcpy(tmp.data() + (size_t)perm[r] * row_bytes, src + (size_t)r * row_bytes, row_bytes);
            std::memcpy(stmp.data() + (size_t)perm[r] * srow, ssrc + (size_t)r * srow, srow);
        }
        src = tmp.data();
        ssrc = stmp.data();
    }
    cudaError_t e = cudaMemcpy2D((char*)w.data + (size_t)dst_lo * row_bytes, row_bytes * dst_stride, src, row_bytes,
                                 row_bytes, rows, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = cudaMemcpy2D((char*)w.scales + (size_t)dst_lo * srow, srow * dst_stride, ssrc, srow, srow, rows,
                         cudaMemcpyHostToDevice);
    return aexis_cuda_check(d->ctx, e, "decoder weight upload");
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

// h += down(SiLU(gate(xn)) * up(xn)), xn = RMSNorm(h) * norm[1].
cudaError_t enqueue_ffn(aexis_decoder* d, aexis_decoder::Layer& L, cudaStream_t s) {
    cudaError_t e;
    GemvArgs f1;
    f1.status = d->ctx->status;
    f1.pdl = true;
    f1.x = d->h;
    f1.w = &L.gateup;
    f1.y = d->act;
    f1.epilogue = EPI_SWIGLU;
    f1.norm_gamma = L.norm[1];
    f1.norm_eps = d->cfg.eps;
    if ((e = launch_gemv(f1, d->ctx->sm_count, s)) != cudaSuccess) return e;
    GemvArgs f2;
    f2.status = d->ctx->status;
    f2.pdl = true;
    f2.x = d->act;
    f2.w = &L.down;
    f2.y = d->h;
    f2.epilogue = EPI_RESIDUAL;
    return launch_gemv(f2, d->ctx->sm_count, s);
}

// A linear-attention block's mixer: in_proj (RMSNorm prologue, fp32 [q k v
// z b a]), the fused conv + GDR + gated-norm kernel, out_proj added into h.
cudaError_t enqueue_linear_attention(aexis_decoder* d, aexis_decoder::Layer& L, cudaStream_t s) {
    const auto& c = d->cfg;
    cudaError_t e;
    GemvArgs in;
    in.status = d->ctx->status;
    in.pdl = true;
    in.x = d->h;
    in.w = &L.qkv;
    in.y = d->lin_proj;
    in.epilogue = EPI_STORE;
    in.norm_gamma = L.norm[0];
    in.norm_eps = c.eps;
    if ((e = launch_gemv(in, d->ctx->sm_count, s)) != cudaSuccess) return e;
    LinAttnDecode la;
    la.proj = d->lin_proj;
    la.conv_w = L.conv_w;
    la.conv_state = L.conv_state;
    la.a_log = L.lin_params;
    la.dt_bias = L.lin_params + c.lin_heads;
    la.gamma = L.lin_params + 2 * c.lin_heads;
    la.state = L.gdr_state;
    la.y = d->lin_y;
    la.heads = c.lin_heads;
    la.kdim = c.lin_kdim;
    la.vdim = c.lin_vdim;
    la.kernel = c.conv_kernel;
    la.gdr_eps = kGdrEps;
    la.norm_eps = c.eps;
    if ((e = launch_lin_attn_decode(la, s)) != cudaSuccess) return e;
    GemvArgs o;
    o.status = d->ctx->status;
    o.pdl = true;
    o.x = d->lin_y;
    o.w = &L.o;
    o.y = d->h;
    o.epilogue = EPI_RESIDUAL;
    return launch_gemv(o, d->ctx->sm_count, s);
}

// Enqueue one decode step (emit = 1: lm_head + greedy token; 0: prompt token).
cudaError_t enqueue_step(aexis_decoder* d, cudaStream_t s, int emit) {
    const auto& c = d->cfg;
    const int D = c.head_dim;
    int* token = d->ints;
    int* pos = d->ints + 1;
    int* step = d->ints + 2;
    cudaError_t e;
    {
        const __half* tab = d->embed;
        int vocab = c.vocab, hidden = c.hidden;
        float* h = d->h;
        unsigned long long* key = d->key;
        void* args[] = {(void*)&tab, &vocab, &hidden, &token, &h, &key};
        e = launch_pdl((const void*)dec_embed_kernel, dim3((hidden + 255) / 256), dim3(256), 0, s, args);
        if (e != cudaSuccess) return e;
    }
    const float scale = 1.0f / sqrtf((float)D);
    for (int l = 0; l < c.n_layers; ++l) {
        auto& L = d->layers[l];
        if (L.kind == AEXIS_LAYER_LINEAR_ATTENTION) {
            if ((e = enqueue_linear_attention(d, L, s)) != cudaSuccess) return e;
            if ((e = enqueue_ffn(d, L, s)) != cudaSuccess) return e;
            continue;
        }
        __half* kc = d->kcache + (size_t)L.attn_slot * c.n_kv_heads * c.kv_capacity * D;
        __half* vc = d->vcache + (size_t)L.attn_slot * c.n_kv_heads * c.kv_capacity * D;
        GemvArgs g;
        g.status = d->ctx->status;
        g.pdl = true;
        g.x = d->h;
        g.w = &L.qkv;
        g.y = d->q;
        g.epilogue = EPI_QKV_ROPE;
        g.norm_gamma = L.norm[0];
        g.norm_eps = c.eps;
        g.rope_cos = d->rope_cos;
        g.rope_sin = d->rope_sin;
        g.rope_map = d->rope_map;
        g.k_cache = kc;
        g.v_cache = vc;
        g.head_dim = D;
        g.kv_cap = c.kv_capacity;
        g.rot_dim = c.rot_dim;
        g.pos_ptr = pos;
        if ((e = launch_gemv(g, d->ctx->sm_count, s)) != cudaSuccess) return e;
        if (d->split_attn) {
            e = launch_split_attention(d->q, kc, vc, c.kv_capacity, D, c.n_heads, c.n_kv_heads, scale, pos, 1, d->part,
                                       d->counters + l * c.n_kv_heads, d->attn, d->ctx->status, 32, s);
            if (e != cudaSuccess) return e;
        } else {
            const float* qp = d->q;
            const __half* kcp = kc;
            const __half* vcp = vc;
            int cap = c.kv_capacity, hd = D, nh = c.n_heads, nkv = c.n_kv_heads;
            float sc = scale;
            const int* pp = pos;
            float* part = d->part;
            unsigned int* cnt = d->counters + l * c.n_kv_heads;
            float* out = d->attn;
            void* args[] = {(void*)&qp, (void*)&kcp, (void*)&vcp, &cap, &hd, &nh, &nkv, &sc, (void*)&pp, &part, &cnt, &out};
            e = launch_pdl((const void*)dec_attn_kernel, dim3(c.n_kv_heads, kAttnSplits), dim3(kAttnThreads), 0, s, args);
            if (e != cudaSuccess) return e;
        }
        GemvArgs o;
        o.status = d->ctx->status;
        o.pdl = true;
        o.x = d->attn;
        o.w = &L.o;
        o.y = d->h;
        o.epilogue = EPI_RESIDUAL;
        if ((e = launch_gemv(o, d->ctx->sm_count, s)) != cudaSuccess) return e;
        if ((e = enqueue_ffn(d, L, s)) != cudaSuccess) return e;
    }
    if (emit) {
        GemvArgs lm;
        lm.status = d->ctx->status;
        lm.pdl = true;
        lm.x = d->h;
        lm.w = &d->lm;
        lm.y = d->logits;
        lm.epilogue = EPI_LOGITS_ARGMAX;
        lm.norm_gamma = d->final_norm;
        lm.norm_eps = c.eps;
        lm.argmax_key = d->key;
        if ((e = launch_gemv(lm, d->ctx->sm_count, s)) != cudaSuccess) return e;
    }
    {
        const unsigned long long* key = d->key;
        int* outs = d->ints + 3;
        int em = emit;
        int mo = d->max_out;
        void* args[] = {(void*)&key, &token, &pos, &outs, &step, &em, &mo};
        e = launch_pdl((const void*)dec_finish_kernel, dim3(1), dim3(32), 0, s, args);
    }
    return e;
}

int capture(aexis_decoder* d, int emit, cudaGraphExec_t* exec) {
    aexis_ctx* ctx = d->ctx;
    cudaStream_t s = ctx->own_stream;
    cudaGraph_t graph = nullptr;
    cudaError_t e = cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal);
    if (e != cudaSuccess) return aexis_cuda_check(ctx, e, "begin capture");
    cudaError_t le = enqueue_step(d, s, emit);
    e = cudaStreamEndCapture(s, &graph);
    if (le != cudaSuccess) {
        if (graph) cudaGraphDestroy(graph);
        return aexis_cuda_check(ctx, le, "decode step launch (capture)");
    }
    if (e != cudaSuccess) return aexis_cuda_check(ctx, e, "end capture");
    e = cudaGraphInstantiateWithFlags(exec, graph, 0);
    cudaGraphDestroy(graph);
    return aexis_cuda_check(ctx, e, "graph instantiate");
}

int ready(aexis_decoder* d) {
    const auto& c = d->cfg;
    for (int l = 0; l < c.n_layers; ++l)
        if (d->layers[l].set_mask != 0x1FF)
            return aexis_fail(d->ctx, AEXIS_E_STATE, "layer %d weights incomplete (mask 0x%x)", l,
                              d->layers[l].set_mask);
    if (!d->lm_set || !d->final_set || !d->embed_set)
        return aexis_fail(d->ctx, AEXIS_E_STATE, "lm_head/final norm/embedding not set");
    if (!d->step_exec) {
        for (auto& L : d->layers) {
            aexis_weights* ws[4] = {&L.qkv, &L.o, &L.gateup, &L.down};
            for (aexis_weights* w : ws) {
                int rc = build_frag(d, *w);
                if (rc) return rc;
            }
        }
        int frc = build_frag(d, d->lm);
        if (frc) return frc;
        int rc = capture(d, 1, &d->step_exec);
        if (rc) return rc;
        rc = capture(d, 0, &d->prefill_exec);
        if (rc) return rc;
    }
    return AEXIS_OK;
}

// Host -> fp32 device vector from fp16 or fp32.
int upload_f32(aexis_decoder* d, float* dst, const void* src, int dtype, size_t count) {
    std::vector<float> tmp(count);
    if (dtype == AEXIS_F16) {
        const __half* hsrc = (const __half*)src;
        for (size_t i = 0; i < count; ++i) tmp[i] = __half2float(hsrc[i]);
    } else {
        std::memcpy(tmp.data(), src, count * sizeof(float));
    }
    return aexis_cuda_check(d->ctx, cudaMemcpy(dst, tmp.data(), count * sizeof(float), cudaMemcpyHostToDevice),
                            "norm upload");
}

// Whether generate runs the persistent greedy loop.
bool use_persist(aexis_decoder* d) {
    return d->persist_mode != 0 && decoder_persist_supported(d, d->ctx->sm_count);
}

// Replays `count` decode steps; emit = 1 uses the full step graph (lm_head,
// greedy token fed back on the device), emit = 0 the prompt-token graph.
int run_steps(aexis_decoder* d, int emit, int count) {
    cudaStream_t s = d->ctx->stream;
    for (int i = 0; i < count; ++i) {
        cudaError_t e = cudaGraphLaunch(emit ? d->step_exec : d->prefill_exec, s);
        if (e != cudaSuccess) return aexis_cuda_check(d->ctx, e, "graph launch");
    }
    return AEXIS_OK;
}

}  // namespace

void decoder_rope_tables(int cap, int rot_dim, float theta, std::vector<float>& cs, std::vector<float>& sn) {
    const int half = rot_dim / 2;
    cs.assign((size_t)cap * half, 0.0f);
    sn.assign((size_t)cap * half, 0.0f);
    for (int p = 0; p < cap; ++p)
        for (int j = 0; j < half; ++j) {
            const float inv = 1.0f / (float)std::pow((double)theta, (double)((float)j * (2.0f / (float)rot_dim)));
            const float ang = (float)p * inv;
            cs[(size_t)p * half + j] = (float)std::cos((double)ang);
            sn[(size_t)p * half + j] = (float)std::sin((double)ang);
        }
}

AEXIS_API int aexis_cuda_decoder_create(aexis_ctx* ctx, const aexis_decoder_config* cfg, aexis_decoder** out) {
    if (!ctx) return AEXIS_E_NULL;
    if (!cfg || !out) return aexis_fail(ctx, AEXIS_E_NULL, "cfg/out is null");
    *out = nullptr;
    const auto& c = *cfg;
    if (c.n_layers <= 0 || c.hidden <= 0 || c.n_heads <= 0 || c.n_kv_heads <= 0 || c.head_dim <= 0 || c.ffn <= 0 ||
        c.vocab <= 0 || c.kv_capacity <= 0)
        return aexis_fail(ctx, AEXIS_E_RANGE, "decoder dimensions must be positive");
    if ((c.bits != 4 && c.bits != 8) || (c.lm_bits != 4 && c.lm_bits != 8))
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "bits=%d lm_bits=%d (4 or 8)", c.bits, c.lm_bits);
    if (c.scale_dtype != AEXIS_F16 && c.scale_dtype != AEXIS_F32)
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "scale_dtype %d", c.scale_dtype);
    if (c.n_heads % c.n_kv_heads != 0 || c.n_heads / c.n_kv_heads > kMaxGroup)
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "n_heads/n_kv_heads must be an integer <= %d", kMaxGroup);
    if (c.head_dim % 2 != 0 || c.head_dim > kMaxHeadDim || c.rot_dim % 2 != 0 || c.rot_dim > c.head_dim ||
        c.rot_dim < 0)
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "head_dim=%d rot_dim=%d", c.head_dim, c.rot_dim);
    const int qd = c.n_heads * c.head_dim;
    if (c.hidden % 32 || c.ffn % 32 || qd % 32)
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "hidden, ffn and heads*head_dim must be multiples of 32");
    if (c.bits == 4 && (c.group <= 0 || c.hidden % c.group || c.ffn % c.group || qd % c.group))
        return aexis_fail(ctx, AEXIS_E_SHAPE, "group %d must divide hidden, ffn and heads*head_dim", c.group);
    if (c.lm_bits == 4 && (c.lm_group <= 0 || c.hidden % c.lm_group))
        return aexis_fail(ctx, AEXIS_E_SHAPE, "lm_group %d must divide hidden", c.lm_group);
    if ((long long)c.kv_capacity > (kAttnSplits * 64LL))
        return aexis_fail(ctx, AEXIS_E_RANGE, "kv_capacity %d > %d", c.kv_capacity, kAttnSplits * 64);
    bool hybrid = false;
    if (c.layer_types)
        for (int l = 0; l < c.n_layers; ++l) {
            if (c.layer_types[l] != AEXIS_LAYER_FULL_ATTENTION && c.layer_types[l] != AEXIS_LAYER_LINEAR_ATTENTION)
                return aexis_fail(ctx, AEXIS_E_RANGE, "layer_types[%d] = %d", l, c.layer_types[l]);
            hybrid |= c.layer_types[l] == AEXIS_LAYER_LINEAR_ATTENTION;
        }
    const long long lin_nv = (long long)c.lin_heads * c.lin_vdim;
    const long long lin_ch = 2LL * c.lin_heads * c.lin_kdim + lin_nv;  // conv channels
    const long long lin_rows = lin_ch + lin_nv + 2LL * c.lin_heads;    // in_proj rows
    if (hybrid) {
        if (!lin_attn_decode_supported(c.lin_heads, c.lin_kdim, c.lin_vdim, c.conv_kernel))
            return aexis_fail(ctx, AEXIS_E_UNSUPPORTED,
                              "linear attention heads=%d kdim=%d vdim=%d conv_kernel=%d (kdim a multiple of 4 up "
                              "to 256, vdim a multiple of 16 up to 128, kernel 1..8)",
                              c.lin_heads, c.lin_kdim, c.lin_vdim, c.conv_kernel);
        if (lin_rows > (1LL << 30) || lin_nv % 32 || (c.bits == 4 && lin_nv % c.group))
            return aexis_fail(ctx, AEXIS_E_SHAPE, "lin_heads*lin_vdim %lld must be a multiple of 32 and of the group",
                              lin_nv);
    }
    int rc = aexis_cuda_check(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
    if (rc) return rc;
    aexis_decoder* d = new (std::nothrow) aexis_decoder();
    if (!d) return aexis_fail(ctx, AEXIS_E_STATE, "out of host memory");
    d->ctx = ctx;
    d->cfg = c;
    d->cfg.layer_types = nullptr;  // the kinds live in layers[]
    d->hybrid = hybrid;
    d->layers.resize(c.n_layers);
    for (int l = 0; l < c.n_layers; ++l) {
        auto& L = d->layers[l];
        L.kind = c.layer_types ? c.layer_types[l] : AEXIS_LAYER_FULL_ATTENTION;
        if (L.kind == AEXIS_LAYER_FULL_ATTENTION) L.attn_slot = d->n_attn++;
    }
    const int kvd = c.n_kv_heads * c.head_dim;
    const int sdt = c.scale_dtype;
    for (auto& L : d->layers) {
        if (L.kind == AEXIS_LAYER_LINEAR_ATTENTION) {
            const size_t gdr = (size_t)c.lin_heads * c.lin_kdim * c.lin_vdim;
            if (!rc) rc = alloc_weights(d, L.qkv, c.bits, c.group, sdt, (int)lin_rows, c.hidden);
            if (!rc) rc = alloc_weights(d, L.o, c.bits, c.group, sdt, c.hidden, (int)lin_nv);
            if (!rc) rc = alloc(d, (void**)&L.conv_w, sizeof(float) * c.conv_kernel * lin_ch, "conv alloc");
            if (!rc) rc = alloc(d, (void**)&L.conv_state, sizeof(float) * c.conv_kernel * lin_ch, "conv alloc");
            if (!rc) rc = alloc(d, (void**)&L.gdr_state, sizeof(float) * gdr, "gdr alloc");
            if (!rc)
                rc = alloc(d, (void**)&L.lin_params, sizeof(float) * (2 * c.lin_heads + c.lin_vdim), "param alloc");
        } else {
            if (!rc) rc = alloc_weights(d, L.qkv, c.bits, c.group, sdt, qd + 2 * kvd, c.hidden);
            if (!rc) rc = alloc_weights(d, L.o, c.bits, c.group, sdt, c.hidden, qd);
        }
        if (!rc) rc = alloc_weights(d, L.gateup, c.bits, c.group, sdt, 2 * c.ffn, c.hidden);
        if (!rc) rc = alloc_weights(d, L.down, c.bits, c.group, sdt, c.hidden, c.ffn);
        if (!rc) rc = alloc(d, (void**)&L.norm[0], sizeof(float) * c.hidden, "norm alloc");
        if (!rc) rc = alloc(d, (void**)&L.norm[1], sizeof(float) * c.hidden, "norm alloc");
    }
    if (!rc) rc = alloc_weights(d, d->lm, c.lm_bits, c.lm_group, sdt, c.vocab, c.hidden);
    if (!rc) rc = alloc(d, (void**)&d->final_norm, sizeof(float) * c.hidden, "norm alloc");
    if (!rc) rc = alloc(d, (void**)&d->embed, sizeof(__half) * (size_t)c.vocab * c.hidden, "embedding alloc");
    const size_t kv = (size_t)(d->n_attn > 0 ? d->n_attn : 1) * c.n_kv_heads * c.kv_capacity * c.head_dim;
    if (!rc) rc = alloc(d, (void**)&d->kcache, sizeof(__half) * kv, "kv alloc");
    if (!rc) rc = alloc(d, (void**)&d->vcache, sizeof(__half) * kv, "kv alloc");
    if (!rc && hybrid) rc = alloc(d, (void**)&d->lin_proj, sizeof(float) * lin_rows, "alloc");
    if (!rc && hybrid) rc = alloc(d, (void**)&d->lin_y, sizeof(float) * lin_nv, "alloc");
    if (!rc) rc = alloc(d, (void**)&d->h, sizeof(float) * c.hidden, "alloc");
    if (!rc) rc = alloc(d, (void**)&d->q, sizeof(float) * qd, "alloc");
    if (!rc) rc = alloc(d, (void**)&d->attn, sizeof(float) * qd, "alloc");
    if (!rc) rc = alloc(d, (void**)&d->act, sizeof(float) * c.ffn, "alloc");
    if (!rc) rc = alloc(d, (void**)&d->logits, sizeof(float) * c.vocab, "alloc");
    // Decode attention: the bulk-copy split kernel (32-position chunks) where
    // the head shape allows it, else the direct-load kernel below.
    d->split_attn = split_attention_supported(c.n_heads, c.n_kv_heads, c.head_dim);
    {
        size_t pf = (size_t)c.n_heads * kAttnSplits * (c.head_dim + 2);
        if (d->split_attn) {
            const size_t sf = split_attention_part_floats(1, c.n_heads, c.head_dim, 32);
            pf = pf > sf ? pf : sf;
            if (!rc) rc = aexis_cuda_check(ctx, split_attention_configure(c.n_heads, c.n_kv_heads, c.head_dim, 32),
                                           "attention smem");
        }
        if (!rc) rc = alloc(d, (void**)&d->part, sizeof(float) * pf, "alloc");
    }
    if (!rc) rc = alloc(d, (void**)&d->counters, sizeof(unsigned int) * c.n_layers * c.n_kv_heads, "alloc");
    if (!rc) rc = alloc(d, (void**)&d->key, sizeof(unsigned long long), "alloc");
    d->max_out = 1 << 16;
    if (!rc) rc = alloc(d, (void**)&d->ints, sizeof(int) * (3 + d->max_out), "alloc");
    // QKV internal row order: per head, rotate-half pairs (j, j + rot/2)
    // adjacent, then the unrotated dims; V keeps its order.
    if (!rc) {
        std::vector<int> map;
        const int half = c.rot_dim / 2;
        auto emit_head = [&](int kind, int head, bool rotate) {
            if (rotate) {
                for (int j = 0; j < half; ++j) {
                    map.push_back((kind << 24) | (head << 12) | j);
                    map.push_back((kind << 24) | (head << 12) | (j + half));
                }
                for (int dd = c.rot_dim; dd < c.head_dim; ++dd) map.push_back((kind << 24) | (head << 12) | dd);
            } else {
                for (int dd = 0; dd < c.head_dim; ++dd) map.push_back((kind << 24) | (head << 12) | dd);
            }
        };
        for (int hh = 0; hh < c.n_heads; ++hh) emit_head(0, hh, true);
        for (int hh = 0; hh < c.n_kv_heads; ++hh) emit_head(1, hh, true);
        for (int hh = 0; hh < c.n_kv_heads; ++hh) emit_head(2, hh, false);
        d->qkv_perm = map;
        rc = alloc(d, (void**)&d->rope_map, sizeof(int) * map.size(), "alloc");
        if (!rc)
            rc = aexis_cuda_check(ctx, cudaMemcpy(d->rope_map, map.data(), sizeof(int) * map.size(), cudaMemcpyHostToDevice),
                                  "rope map upload");
    }
    // RoPE tables (Qwen35DecoderSession.CreateRopeTextures, :1660-1687).
    if (!rc && c.rot_dim > 0) {
        std::vector<float> cs, sn;
        decoder_rope_tables(c.kv_capacity, c.rot_dim, c.rope_theta, cs, sn);
        rc = alloc(d, (void**)&d->rope_cos, sizeof(float) * cs.size(), "alloc");
        if (!rc) rc = alloc(d, (void**)&d->rope_sin, sizeof(float) * sn.size(), "alloc");
        if (!rc) rc = aexis_cuda_check(ctx, cudaMemcpy(d->rope_cos, cs.data(), sizeof(float) * cs.size(), cudaMemcpyHostToDevice), "rope upload");
        if (!rc) rc = aexis_cuda_check(ctx, cudaMemcpy(d->rope_sin, sn.data(), sizeof(float) * sn.size(), cudaMemcpyHostToDevice), "rope upload");
    }
    if (rc) {
        aexis_cuda_decoder_destroy(d);
        return rc;
    }
    *out = d;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_decoder_destroy(aexis_decoder* d) {
    if (!d) return AEXIS_E_NULL;
    cudaSetDevice(d->ctx->device);
    cudaStreamSynchronize(d->ctx->stream);
    if (d->step_exec) cudaGraphExecDestroy(d->step_exec);
    if (d->prefill_exec) cudaGraphExecDestroy(d->prefill_exec);
    for (auto& L : d->layers) {
        free_weights(L.qkv);
        free_weights(L.o);
        free_weights(L.gateup);
        free_weights(L.down);
        float* lbufs[] = {L.norm[0], L.norm[1], L.conv_w, L.conv_state, L.gdr_state, L.lin_params};
        for (float* b : lbufs)
            if (b) cudaFree(b);
    }
    free_weights(d->lm);
    void* bufs[] = {d->final_norm, d->embed, d->rope_map, d->rope_cos, d->rope_sin, d->kcache, d->vcache, d->h, d->q,
                    d->attn, d->act, d->logits, d->part, d->counters, d->key, d->ints, d->persist_phases,
                    d->persist_sync, d->persist_stream, d->persist_off, d->lin_proj, d->lin_y};
    for (void* b : bufs)
        if (b) cudaFree(b);
    delete d;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_decoder_set_linear(aexis_decoder* d, int layer, int which, const uint32_t* packed,
                                            const void* scales, int scale_dtype) {
    if (!d) return AEXIS_E_NULL;
    if (!packed || !scales) return aexis_fail(d->ctx, AEXIS_E_NULL, "weights and scales must be configured together.");
    const auto& c = d->cfg;
    int rc = dbind(d);
    if (rc) return rc;
    const std::vector<int> none;
    if (layer == -1) {
        if (which != 7) return aexis_fail(d->ctx, AEXIS_E_RANGE, "layer -1 takes which=7 (lm_head)");
        rc = scatter_rows(d, d->lm, packed, scales, scale_dtype, c.vocab, 0, 1, none);
        if (!rc && d->lm.frag) rc = build_frag(d, d->lm);
        d->persist_packed = false;
        if (!rc) d->lm_set = 1;
        return rc;
    }
    if (layer < 0 || layer >= c.n_layers || which < 0 || which > 9 || which == 7)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "layer=%d which=%d", layer, which);
    auto& L = d->layers[layer];
    const bool lin = L.kind == AEXIS_LAYER_LINEAR_ATTENTION;
    if (lin ? (which <= 3) : (which >= 8))
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "which=%d does not exist in %s layer %d", which,
                          lin ? "linear-attention" : "full-attention", layer);
    const int D = c.head_dim, qd = c.n_heads * D, kvd = c.n_kv_heads * D;
    switch (which) {
        case 0:
        case 1:
        case 2: {
            // Each of Q, K, V fills its own contiguous internal range; inside it
            // rows follow the inverse of qkv_perm.
            const int kind = which;
            const int rows = kind == 0 ? qd : kvd;
            const int lo = kind == 0 ? 0 : (kind == 1 ? qd : qd + kvd);
            std::vector<int> dst(rows, -1);
            for (size_t i = 0; i < d->qkv_perm.size(); ++i) {
                const int m = d->qkv_perm[i];
                if ((m >> 24) == kind) dst[((m >> 12) & 0xFFF) * D + (m & 0xFFF)] = (int)i - lo;
            }
            rc = scatter_rows(d, L.qkv, packed, scales, scale_dtype, rows, lo, 1, dst);
        } break;
        case 3: rc = scatter_rows(d, L.o, packed, scales, scale_dtype, c.hidden, 0, 1, none); break;
        case 4: rc = scatter_rows(d, L.gateup, packed, scales, scale_dtype, c.ffn, 0, 2, none); break;
        case 5: rc = scatter_rows(d, L.gateup, packed, scales, scale_dtype, c.ffn, 1, 2, none); break;
        case 6: rc = scatter_rows(d, L.down, packed, scales, scale_dtype, c.hidden, 0, 1, none); break;
        case 8: rc = scatter_rows(d, L.qkv, packed, scales, scale_dtype, L.qkv.n, 0, 1, none); break;
        case 9: rc = scatter_rows(d, L.o, packed, scales, scale_dtype, c.hidden, 0, 1, none); break;
    }
    aexis_weights* w = which <= 2 || which == 8 ? &L.qkv : which == 3 || which == 9 ? &L.o
                     : which <= 5 ? &L.gateup : &L.down;
    if (!rc) {
        if (w->frag) rc = build_frag(d, *w);
        d->persist_packed = false;
    }
    if (!rc) L.set_mask |= 1 << (which == 8 ? 0 : which == 9 ? 3 : which);
    return rc;
}

AEXIS_API int aexis_cuda_layer_types_interval(int32_t n_layers, int32_t interval, int32_t* out) {
    if (!out) return AEXIS_E_NULL;
    if (n_layers < 0) return AEXIS_E_RANGE;
    for (int i = 0; i < n_layers; ++i)
        out[i] = interval <= 0 || (i + 1) % interval == 0 ? AEXIS_LAYER_FULL_ATTENTION : AEXIS_LAYER_LINEAR_ATTENTION;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_decoder_set_linear_attention(aexis_decoder* d, int layer, const void* conv, const void* a_log,
                                                      const void* dt_bias, const void* gamma, int dtype) {
    if (!d) return AEXIS_E_NULL;
    if (!conv || !a_log || !dt_bias || !gamma) return aexis_fail(d->ctx, AEXIS_E_NULL, "parameter array is null");
    if (dtype != AEXIS_F16 && dtype != AEXIS_F32) return aexis_fail(d->ctx, AEXIS_E_UNSUPPORTED, "dtype %d", dtype);
    const auto& c = d->cfg;
    if (layer < 0 || layer >= c.n_layers || d->layers[layer].kind != AEXIS_LAYER_LINEAR_ATTENTION)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "layer %d is not a linear-attention layer", layer);
    int rc = dbind(d);
    if (rc) return rc;
    auto& L = d->layers[layer];
    const size_t K = (size_t)c.conv_kernel;
    const size_t ch = 2 * (size_t)c.lin_heads * c.lin_kdim + (size_t)c.lin_heads * c.lin_vdim;
    auto at = [&](const void* p, size_t i) {
        return dtype == AEXIS_F16 ? __half2float(((const __half*)p)[i]) : ((const float*)p)[i];
    };
    // [channels][kernel] -> tap-major [kernel][channels]: a warp reads
    // consecutive channels of one tap.
    std::vector<float> w(K * ch);
    for (size_t g = 0; g < ch; ++g)
        for (size_t k = 0; k < K; ++k) w[k * ch + g] = at(conv, g * K + k);
    std::vector<float> prm(2 * (size_t)c.lin_heads + c.lin_vdim);
    for (int i = 0; i < c.lin_heads; ++i) {
        prm[i] = at(a_log, i);
        prm[c.lin_heads + i] = at(dt_bias, i);
    }
    for (int i = 0; i < c.lin_vdim; ++i) prm[2 * c.lin_heads + i] = at(gamma, i);
    rc = aexis_cuda_check(d->ctx, cudaMemcpy(L.conv_w, w.data(), sizeof(float) * w.size(), cudaMemcpyHostToDevice),
                          "conv upload");
    if (!rc)
        rc = aexis_cuda_check(d->ctx, cudaMemcpy(L.lin_params, prm.data(), sizeof(float) * prm.size(),
                                                 cudaMemcpyHostToDevice), "parameter upload");
    if (!rc) L.set_mask |= (1 << 1) | (1 << 2);
    return rc;
}

AEXIS_API int aexis_cuda_decoder_set_norm(aexis_decoder* d, int layer, int which, const void* gamma, int dtype) {
    if (!d) return AEXIS_E_NULL;
    if (!gamma) return aexis_fail(d->ctx, AEXIS_E_NULL, "gamma is null");
    if (dtype != AEXIS_F16 && dtype != AEXIS_F32) return aexis_fail(d->ctx, AEXIS_E_UNSUPPORTED, "dtype %d", dtype);
    int rc = dbind(d);
    if (rc) return rc;
    if (layer == -1) {
        rc = upload_f32(d, d->final_norm, gamma, dtype, d->cfg.hidden);
        if (!rc) d->final_set = 1;
        return rc;
    }
    if (layer < 0 || layer >= d->cfg.n_layers || which < 0 || which > 1)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "layer=%d which=%d", layer, which);
    rc = upload_f32(d, d->layers[layer].norm[which], gamma, dtype, d->cfg.hidden);
    if (!rc) d->layers[layer].set_mask |= 1 << (7 + which);
    return rc;
}

AEXIS_API int aexis_cuda_decoder_set_embedding(aexis_decoder* d, const void* table, int dtype) {
    if (!d) return AEXIS_E_NULL;
    if (!table) return aexis_fail(d->ctx, AEXIS_E_NULL, "table is null");
    int rc = dbind(d);
    if (rc) return rc;
    const size_t count = (size_t)d->cfg.vocab * d->cfg.hidden;
    if (dtype == AEXIS_F16) {
        rc = aexis_cuda_check(d->ctx, cudaMemcpy(d->embed, table, count * 2, cudaMemcpyHostToDevice), "embedding upload");
    } else if (dtype == AEXIS_F32) {
        std::vector<__half> tmp(count);
        const float* f = (const float*)table;
        for (size_t i = 0; i < count; ++i) tmp[i] = __float2half_rn(f[i]);
        rc = aexis_cuda_check(d->ctx, cudaMemcpy(d->embed, tmp.data(), count * 2, cudaMemcpyHostToDevice), "embedding upload");
    } else {
        return aexis_fail(d->ctx, AEXIS_E_UNSUPPORTED, "dtype %d", dtype);
    }
    if (!rc) d->embed_set = 1;
    return rc;
}

AEXIS_API int aexis_cuda_decoder_reset(aexis_decoder* d) {
    if (!d) return AEXIS_E_NULL;
    int rc = dbind(d);
    if (rc) return rc;
    d->host_pos = 0;
    const auto& c = d->cfg;
    cudaError_t e = cudaMemsetAsync(d->ints, 0, sizeof(int) * 3, d->ctx->stream);
    for (auto& L : d->layers) {
        if (L.kind != AEXIS_LAYER_LINEAR_ATTENTION || e != cudaSuccess) continue;
        const size_t ch = 2 * (size_t)c.lin_heads * c.lin_kdim + (size_t)c.lin_heads * c.lin_vdim;
        e = cudaMemsetAsync(L.conv_state, 0, sizeof(float) * c.conv_kernel * ch, d->ctx->stream);
        if (e == cudaSuccess)
            e = cudaMemsetAsync(L.gdr_state, 0, sizeof(float) * c.lin_heads * c.lin_kdim * c.lin_vdim, d->ctx->stream);
    }
    return aexis_cuda_check(d->ctx, e, "reset");
}

AEXIS_API int aexis_cuda_decoder_position(const aexis_decoder* d, int32_t* out) {
    if (!d || !out) return AEXIS_E_NULL;
    *out = d->host_pos;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_decoder_set_position(aexis_decoder* d, int32_t position) {
    if (!d) return AEXIS_E_NULL;
    if (position < 0 || position > d->cfg.kv_capacity)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "position %d outside [0, %d]", position, d->cfg.kv_capacity);
    int rc = dbind(d);
    if (rc) return rc;
    const int ints[3] = {0, position, 0};
    rc = aexis_cuda_check(d->ctx, cudaMemcpyAsync(d->ints, ints, sizeof(ints), cudaMemcpyHostToDevice, d->ctx->stream),
                          "position upload");
    if (!rc) rc = aexis_cuda_check(d->ctx, cudaStreamSynchronize(d->ctx->stream), "sync");
    if (!rc) d->host_pos = position;
    return rc;
}

static int kv_layer_args(aexis_decoder* d, int layer, int rows, const void* k, const void* v) {
    if (!k || !v) return aexis_fail(d->ctx, AEXIS_E_NULL, "K/V buffer is null");
    if (layer < 0 || layer >= d->cfg.n_layers)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "layer %d outside [0, %d)", layer, d->cfg.n_layers);
    if (d->layers[layer].kind != AEXIS_LAYER_FULL_ATTENTION)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "layer %d is linear attention: it has no KV cache", layer);
    if (rows <= 0) return aexis_fail(d->ctx, AEXIS_E_RANGE, "rows=%d", rows);
    return dbind(d);
}

static int recurrent_layer_args(aexis_decoder* d, int layer) {
    if (layer < 0 || layer >= d->cfg.n_layers || d->layers[layer].kind != AEXIS_LAYER_LINEAR_ATTENTION)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "layer %d is not a linear-attention layer", layer);
    return dbind(d);
}

// Both directions of the recurrent-cache copy (device to device, on the context stream).
static int recurrent_copy(aexis_decoder* d, int layer, float* conv_dst, const float* conv_src, float* gdr_dst,
                          const float* gdr_src) {
    const auto& c = d->cfg;
    const size_t ch = 2 * (size_t)c.lin_heads * c.lin_kdim + (size_t)c.lin_heads * c.lin_vdim;
    cudaError_t e = cudaSuccess;
    if (conv_dst && conv_src)
        e = cudaMemcpyAsync(conv_dst, conv_src, sizeof(float) * c.conv_kernel * ch, cudaMemcpyDeviceToDevice,
                            d->ctx->stream);
    if (e == cudaSuccess && gdr_dst && gdr_src)
        e = cudaMemcpyAsync(gdr_dst, gdr_src, sizeof(float) * c.lin_heads * c.lin_kdim * c.lin_vdim,
                            cudaMemcpyDeviceToDevice, d->ctx->stream);
    return aexis_cuda_check(d->ctx, e, "recurrent cache copy");
}

AEXIS_API int aexis_cuda_decoder_recurrent_export(aexis_decoder* d, int layer, float* conv_out, float* gdr_out) {
    if (!d) return AEXIS_E_NULL;
    int rc = recurrent_layer_args(d, layer);
    if (rc) return rc;
    const auto& L = d->layers[layer];
    return recurrent_copy(d, layer, conv_out, L.conv_state, gdr_out, L.gdr_state);
}

AEXIS_API int aexis_cuda_decoder_recurrent_import(aexis_decoder* d, int layer, const float* conv_in,
                                                  const float* gdr_in) {
    if (!d) return AEXIS_E_NULL;
    int rc = recurrent_layer_args(d, layer);
    if (rc) return rc;
    auto& L = d->layers[layer];
    return recurrent_copy(d, layer, L.conv_state, conv_in, L.gdr_state, gdr_in);
}

AEXIS_API int aexis_cuda_decoder_kv_export(aexis_decoder* d, int layer, int rows, float* k_out, float* v_out) {
    if (!d) return AEXIS_E_NULL;
    int rc = kv_layer_args(d, layer, rows, k_out, v_out);
    if (rc) return rc;
    if (rows < d->host_pos)
        return aexis_fail(d->ctx, AEXIS_E_SHAPE, "rows %d < sequence length %d", rows, d->host_pos);
    const auto& c = d->cfg;
    const size_t per = (size_t)c.n_kv_heads * c.kv_capacity * c.head_dim * d->layers[layer].attn_slot;
    return aexis_cuda_check(d->ctx, launch_kv_export(d->kcache + per, d->vcache + per, c.n_kv_heads,
                                                     c.kv_capacity, c.head_dim, 0, d->host_pos, rows, k_out, v_out,
                                                     d->ctx->stream), "kv export launch");
}

AEXIS_API int aexis_cuda_decoder_kv_import(aexis_decoder* d, int layer, const float* k_in, const float* v_in, int rows,
                                           int length) {
    if (!d) return AEXIS_E_NULL;
    int rc = kv_layer_args(d, layer, rows, k_in, v_in);
    if (rc) return rc;
    const auto& c = d->cfg;
    if (length < 0 || length > rows || length > c.kv_capacity)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "length %d outside [0, min(rows %d, capacity %d)]", length, rows,
                          c.kv_capacity);
    const size_t per = (size_t)c.n_kv_heads * c.kv_capacity * c.head_dim * d->layers[layer].attn_slot;
    return aexis_cuda_check(d->ctx, launch_kv_import(k_in, v_in, c.n_kv_heads, c.kv_capacity, c.head_dim, 0, length,
                                                     rows, d->kcache + per, d->vcache + per,
                                                     d->ctx->stream), "kv import launch");
}

AEXIS_API int aexis_cuda_decoder_prefill(aexis_decoder* d, const int32_t* tokens, int count, int32_t* next_token) {
    if (!d) return AEXIS_E_NULL;
    if (!tokens || !next_token) return aexis_fail(d->ctx, AEXIS_E_NULL, "tokens/next_token is null");
    if (count <= 0) return aexis_fail(d->ctx, AEXIS_E_RANGE, "count=%d", count);
    if (d->host_pos + count > d->cfg.kv_capacity)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "KV cache full: position %d + %d > capacity %d", d->host_pos, count,
                          d->cfg.kv_capacity);
    int rc = dbind(d);
    if (!rc) rc = ready(d);
    if (rc) return rc;
    cudaStream_t s = d->ctx->stream;
    for (int i = 0; i < count; ++i) {
        cudaError_t e = cudaMemcpyAsync(d->ints, tokens + i, sizeof(int), cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return aexis_cuda_check(d->ctx, e, "token upload");
        rc = run_steps(d, i == count - 1, 1);
        if (rc) return rc;
    }
    d->host_pos += count;
    rc = aexis_cuda_check(d->ctx, cudaMemcpyAsync(next_token, d->ints, sizeof(int), cudaMemcpyDeviceToHost, s), "readback");
    if (!rc) rc = aexis_cuda_check(d->ctx, cudaStreamSynchronize(s), "sync");
    if (!rc) rc = aexis_check_status(d->ctx);
    return rc;
}

AEXIS_API int aexis_cuda_decoder_step(aexis_decoder* d, int32_t token, int32_t* next_token) {
    return aexis_cuda_decoder_prefill(d, &token, 1, next_token);
}

AEXIS_API int aexis_cuda_decoder_generate(aexis_decoder* d, const int32_t* prompt, int n_prompt, int max_new,
                                          int32_t* out_tokens) {
    if (!d) return AEXIS_E_NULL;
    if (!prompt || !out_tokens) return aexis_fail(d->ctx, AEXIS_E_NULL, "prompt/out_tokens is null");
    if (n_prompt <= 0 || max_new <= 0 || max_new > d->max_out)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "n_prompt=%d max_new=%d", n_prompt, max_new);
    if (d->host_pos + n_prompt + max_new - 1 > d->cfg.kv_capacity)
        return aexis_fail(d->ctx, AEXIS_E_RANGE, "KV cache too small for %d + %d tokens", n_prompt, max_new);
    int rc = dbind(d);
    if (!rc) rc = ready(d);
    if (rc) return rc;
    cudaStream_t s = d->ctx->stream;
    if (use_persist(d)) {
        // Prompt tokens but the last: the prefill graph (no lm_head). Then
        // every emitting step in one persistent launch.
        for (int i = 0; i + 1 < n_prompt; ++i) {
            cudaError_t e = cudaMemcpyAsync(d->ints, prompt + i, sizeof(int), cudaMemcpyHostToDevice, s);
            if (e != cudaSuccess) return aexis_cuda_check(d->ctx, e, "token upload");
            rc = run_steps(d, 0, 1);
            if (rc) return rc;
        }
        cudaError_t e = cudaMemcpyAsync(d->ints, prompt + n_prompt - 1, sizeof(int), cudaMemcpyHostToDevice, s);
        if (e == cudaSuccess) e = cudaMemsetAsync(d->ints + 2, 0, sizeof(int), s);  // output cursor
        if (e != cudaSuccess) return aexis_cuda_check(d->ctx, e, "token upload");
        rc = aexis_cuda_check(d->ctx, decoder_persist_run(d, max_new, s), "persistent decode launch");
        if (rc) return rc;
        d->host_pos += n_prompt + max_new - 1;
        rc = aexis_cuda_check(d->ctx, cudaMemcpyAsync(out_tokens, d->ints + 3, sizeof(int) * max_new,
                                                      cudaMemcpyDeviceToHost, s), "readback");
        if (!rc) rc = aexis_cuda_check(d->ctx, cudaStreamSynchronize(s), "sync");
        if (!rc) rc = aexis_check_status(d->ctx);
        return rc;
    }
    // Prompt: one token upload + prefill graph per token, the last one emits.
    for (int i = 0; i < n_prompt; ++i) {
        cudaError_t e = cudaMemcpyAsync(d->ints, prompt + i, sizeof(int), cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return aexis_cuda_check(d->ctx, e, "token upload");
        if (i == 0) {
            e = cudaMemsetAsync(d->ints + 2, 0, sizeof(int), s);  // output cursor
            if (e != cudaSuccess) return aexis_cuda_check(d->ctx, e, "cursor reset");
        }
        rc = run_steps(d, i == n_prompt - 1, 1);
        if (rc) return rc;
    }
    // Greedy continuation: the finish kernel feeds each token to the next step
    // on the device; no host round trip until the end.
    rc = run_steps(d, 1, max_new - 1);
    if (rc) return rc;
    d->host_pos += n_prompt + max_new - 1;
    rc = aexis_cuda_check(d->ctx, cudaMemcpyAsync(out_tokens, d->ints + 3, sizeof(int) * max_new, cudaMemcpyDeviceToHost, s),
                          "readback");
    if (!rc) rc = aexis_cuda_check(d->ctx, cudaStreamSynchronize(s), "sync");
    if (!rc) rc = aexis_check_status(d->ctx);
    return rc;
}

AEXIS_API int aexis_cuda_decoder_set_schedule(aexis_decoder* d, int mode) {
    if (!d) return AEXIS_E_NULL;
    if (mode < -1 || mode > 1) return aexis_fail(d->ctx, AEXIS_E_RANGE, "mode=%d (-1, 0 or 1)", mode);
    int rc = dbind(d);
    if (rc) return rc;
    if (mode == 1 && !decoder_persist_supported(d, d->ctx->sm_count))
        return aexis_fail(d->ctx, AEXIS_E_UNSUPPORTED, "the persistent decode loop does not support this decoder");
    d->persist_mode = mode;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_decoder_schedule(aexis_decoder* d, int32_t* out) {
    if (!d || !out) return AEXIS_E_NULL;
    int rc = dbind(d);
    if (rc) return rc;
    *out = use_persist(d) ? 1 : 0;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_decoder_logits(aexis_decoder* d, float* out) {
    if (!d) return AEXIS_E_NULL;
    if (!out) return aexis_fail(d->ctx, AEXIS_E_NULL, "out is null");
    int rc = dbind(d);
    if (rc) return rc;
    rc = aexis_cuda_check(d->ctx, cudaMemcpyAsync(out, d->logits, sizeof(float) * d->cfg.vocab, cudaMemcpyDeviceToHost,
                                                  d->ctx->stream), "readback");
    if (!rc) rc = aexis_cuda_check(d->ctx, cudaStreamSynchronize(d->ctx->stream), "sync");
    return rc;
}
