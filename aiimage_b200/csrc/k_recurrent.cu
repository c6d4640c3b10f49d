// k_recurrent.cu -- decode kernels of the linear-attention blocks of Qwen3.5
// (18 of its 24 decoder blocks): the causal depthwise ShortConv with its
// streaming cache, and the recurrent Gated Delta Rule.
//
// Reference (paths relative to Packages/com.aexis/Runtime/):
//   AexisShortConvPack4       Resources/Aexis/AexisCommon.compute:623-678
//   AexisGatedDeltaRulePack4  Resources/Aexis/AexisCommon.compute:680-753
//   Ops.ShortConvPack4 / GatedDeltaRulePack4  Execution/Graph/AexisOps.cs:12593-12657
//   AexisGatedDeltaRuleLayer  Execution/Layers/AexisGatedDeltaRuleLayer.cs:32-98
//     (one dispatch per token, ping-pong state textures)
//
// The reference dispatches the Gated Delta Rule once per token, re-reading
// and re-writing the whole [heads, kdim, vdim] state each time. Here one
// launch runs any number of tokens: each CTA owns a 16-column slice of one
// head's state and keeps it in registers from the first token to the last,
// so the state crosses HBM once in and once out per call. For batch-1 decode
// (one token) the kernel is bound by that 2 x heads x kdim x vdim x 4 bytes
// and by launch latency.
#include <cooperative_groups.h>

#include "decoder_internal.h"

namespace {

constexpr int kConvMaxKernel = 16;

// AexisShortConvPack4 (COMMON:623-678). One thread per channel (group).
// Layouts: weight Pack4 CDHW [w=kernel, h=1, c=groups] (element (k, g) at
// ((g/4)*kernel + k)*4 + (g&3)); mixed/out [seq][ld], cache_in/cache_out
// [cache_len][ld], ld = ceil(groups/4)*4 (Pack4 linear rows).
//   out[t][g] = silu(sum_k hist(cache_len - kernel + t + 1 + k) * w[g][k])
//   hist(i)   = i < 0 ? 0 : i < cache_len ? cache_in[i] : mixed[i - cache_len]
//   cache_out[i] = hist(seq + i), the tail of [cache_in; mixed].
// All outputs are computed before the cache is rewritten, and cache_out[i]
// reads hist(seq + i) with seq + i > i, so cache_out may be cache_in itself.
__global__ void short_conv_kernel(const float* __restrict__ weight, const float* __restrict__ mixed,
                                  const float* cache_in, float* __restrict__ out, float* cache_out,
                                  int groups, int kernel, int seq, int cache_len) {
    const int g = blockIdx.x * blockDim.x + threadIdx.x;
    if (g >= groups) return;
    const long long ld = (long long)((groups + 3) / 4) * 4;
    float w[kConvMaxKernel];
#pragma unroll
    for (int k = 0; k < kConvMaxKernel; ++k)
        w[k] = k < kernel ? weight[((long long)(g >> 2) * kernel + k) * 4 + (g & 3)] : 0.0f;
    for (int t = 0; t < seq; ++t) {
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < kConvMaxKernel; ++k) {
            if (k < kernel) {
                const int hi = cache_len - kernel + t + 1 + k;
                const float x = hi < 0 ? 0.0f
                              : (hi < cache_len ? cache_in[hi * ld + g] : mixed[(hi - cache_len) * ld + g]);
                sum = fmaf(x, w[k], sum);
            }
        }
        out[t * ld + g] = sum / (1.0f + expf(-sum));
    }
    for (int i = 0; i < cache_len; ++i) {
        const int src = seq + i;
        cache_out[i * ld + g] = src < cache_len ? cache_in[src * ld + g] : mixed[(src - cache_len) * ld + g];
    }
}

struct GdrArgs {
    const float* a_log;     // [heads]
    const float* dt_bias;   // [heads]
    const float* b;         // [seq][heads]
    const float* a;         // [seq][heads]
    const float* q;         // Pack4 CDHW [w=kdim, h=heads, c=seq]
    const float* k;         // Pack4 CDHW [w=kdim, h=heads, c=seq]
    const float* v;         // Pack4 CDHW [w=vdim, h=heads, c=seq]
    const float* state_in;  // [heads][kdim][vdim4]
    float* out;             // Pack4 CDHW [w=vdim, h=heads, c=seq]
    float* state_out;       // [heads][kdim][vdim4]
    int heads, kdim, vdim, first, count;
    float eps;
};

constexpr int kGdrThreads = 128;   // 32 row groups x 4 column quads
constexpr int kGdrCols = 16;       // value columns per CTA

// AexisGatedDeltaRulePack4 (COMMON:680-753), for tokens first..first+count-1.
// Per token and head, with q, k the raw vectors:
//   decay = exp(-exp(a_log) * softplus(a + dt_bias)),  beta = sigmoid(b)
//   S    <- S * decay
//   mem   = (k / |k|) . S                  |x| = sqrt(sum x^2 + eps)
//   delta = (v - mem) * beta
//   S    <- S + (k / |k|) outer delta
//   out   = (q / |q|) . S / sqrt(kdim)
// Thread (r, qd) holds rows r, r+32, ... (RPT rows) of the CTA's columns
// 4qd..4qd+3: every dot product over rows is a partial sum per thread,
// three xor shuffles over the warp's 8 row groups and one pass over four
// warps' partials in shared memory. The two norms ride in the same reduction
// as `mem`. Columns past vdim (up to the Pack4 width vdim4) carry v = 0, as in
// the reference, which writes whole texels.
template <int RPT>
__global__ void __launch_bounds__(kGdrThreads) gdr_kernel(GdrArgs p) {
    const int tid = threadIdx.x;
    const int qd = tid & 3;
    const int r = tid >> 2;
    const int warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y;
    const int heads = p.heads, kdim = p.kdim, vdim = p.vdim;
    const int vdim4 = (vdim + 3) & ~3;
    const int c0 = blockIdx.x * kGdrCols + qd * 4;
    const bool col_ok = c0 < vdim4;

    __shared__ float red_a[4][4][6];
    __shared__ float red_b[4][4][4];

    float S[RPT][4];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        const int j = r + 32 * i;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < kdim && col_ok)
            s = *reinterpret_cast<const float4*>(p.state_in + ((long long)h * kdim + j) * vdim4 + c0);
        S[i][0] = s.x; S[i][1] = s.y; S[i][2] = s.z; S[i][3] = s.w;
    }
    const float ealog = expf(p.a_log[h]);
    const float dt = p.dt_bias[h];
    const float inv_sqrt_k = rsqrtf((float)kdim);

    // Per-token inputs, loaded one token ahead: the loads of token t+1 are in
    // flight while token t runs its two reductions (prefill is then bound by
    // the reductions, not by L2 latency).
    float qv[RPT], kv[RPT], vv[4], bb, xa;
    auto load_token = [&](int t, float (&qo)[RPT], float (&ko)[RPT], float (&vo)[4], float& bo, float& xo) {
        const int lane_t = t & 3;
        const long long qk_texel = ((long long)(t >> 2) * heads + h) * kdim;
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const int j = r + 32 * i;
            qo[i] = j < kdim ? p.q[(qk_texel + j) * 4 + lane_t] : 0.f;
            ko[i] = j < kdim ? p.k[(qk_texel + j) * 4 + lane_t] : 0.f;
        }
        const long long v_texel = ((long long)(t >> 2) * heads + h) * vdim;
#pragma unroll
        for (int c = 0; c < 4; ++c) vo[c] = c0 + c < vdim ? p.v[(v_texel + c0 + c) * 4 + lane_t] : 0.f;
        bo = p.b[(long long)t * heads + h];
        xo = p.a[(long long)t * heads + h] + dt;
    };
    const int t_end = p.first + p.count;
    load_token(p.first, qv, kv, vv, bb, xa);
    for (int t = p.first; t < t_end; ++t) {
        const int lane_t = t & 3;
        float qn[RPT], kn_[RPT], vn[4], bn = 0.f, xn = 0.f;
        if (t + 1 < t_end) load_token(t + 1, qn, kn_, vn, bn, xn);
        const float beta = 1.0f / (1.0f + expf(-bb));
        const float decay = expf(-ealog * (fmaxf(xa, 0.0f) + logf(1.0f + expf(-fabsf(xa)))));

        float part[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            part[0] = fmaf(qv[i], qv[i], part[0]);
            part[1] = fmaf(kv[i], kv[i], part[1]);
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                S[i][c] *= decay;
                part[2 + c] = fmaf(kv[i], S[i][c], part[2 + c]);
            }
        }
#pragma unroll
        for (int m = 4; m < 32; m <<= 1)
#pragma unroll
            for (int e = 0; e < 6; ++e) part[e] += __shfl_xor_sync(0xffffffffu, part[e], m);
        if (lane < 4) {
#pragma unroll
            for (int e = 0; e < 6; ++e) red_a[warp][qd][e] = part[e];
        }
        __syncthreads();
        float tot[6];
#pragma unroll
        for (int e = 0; e < 6; ++e) tot[e] = (red_a[0][qd][e] + red_a[1][qd][e]) + (red_a[2][qd][e] + red_a[3][qd][e]);
        const float qs = rsqrtf(tot[0] + p.eps);
        const float ks = rsqrtf(tot[1] + p.eps);

        const long long v_texel = ((long long)(t >> 2) * heads + h) * vdim;
        float delta[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) delta[c] = (vv[c] - tot[2 + c] * ks) * beta;
        float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const float kn = kv[i] * ks;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                S[i][c] = fmaf(kn, delta[c], S[i][c]);
                o[c] = fmaf(qv[i], S[i][c], o[c]);
            }
        }
#pragma unroll
        for (int m = 4; m < 32; m <<= 1)
#pragma unroll
            for (int c = 0; c < 4; ++c) o[c] += __shfl_xor_sync(0xffffffffu, o[c], m);
        if (lane < 4) {
#pragma unroll
            for (int c = 0; c < 4; ++c) red_b[warp][qd][c] = o[c];
        }
        __syncthreads();
        if (r == 0) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int col = c0 + c;
                if (col < vdim) {
                    const float sum = (red_b[0][qd][c] + red_b[1][qd][c]) + (red_b[2][qd][c] + red_b[3][qd][c]);
                    p.out[(v_texel + col) * 4 + lane_t] = sum * qs * inv_sqrt_k;
                }
            }
        }
        if (t + 1 < t_end) {
#pragma unroll
            for (int i = 0; i < RPT; ++i) { qv[i] = qn[i]; kv[i] = kn_[i]; }
#pragma unroll
            for (int c = 0; c < 4; ++c) vv[c] = vn[c];
            bb = bn;
            xa = xn;
        }
    }
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        const int j = r + 32 * i;
        if (j < kdim && col_ok)
            *reinterpret_cast<float4*>(p.state_out + ((long long)h * kdim + j) * vdim4 + c0) =
                make_float4(S[i][0], S[i][1], S[i][2], S[i][3]);
    }
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

// One decode step of a hybrid decoder's linear-attention block, after its
// in_proj GEMV: ShortConv + SiLU on the step's q/k/v channels, the Gated
// Delta Rule for one token, and the per-head gated RMSNorm, in one launch.
//   proj  = [q k v z b a] of this token (in_proj output, fp32)
//   q,k,v = silu(conv over [cache rows 1..K-1, proj]) (tap order as AexisShortConvPack4)
//   o     = GDR(q, k, v, b, a) as gdr_kernel, one token
//   y     = o * rsqrt(max(mean_head(o^2) + eps, 1e-20)) * gamma * silu(z)
// Grid (vdim/16, heads), one cluster of vdim/16 CTAs per head: CTA (x, h)
// owns columns 16x..16x+15 of head h's state (kept in registers as in
// gdr_kernel) and recomputes the conv of the head's q and k rows it needs
// (a few FMAs each) instead of reading them from another kernel. The
// per-head norm sums o^2 over the cluster's CTAs through distributed shared
// memory. The conv cache shifts in place after the first cluster barrier,
// when every CTA of the head has read it: q/k rows by the cluster's CTA 0,
// v columns by the CTA that owns them. The second barrier keeps every CTA's
// shared memory alive until the others have read it.
// Global memory is read in two batches, every load of a batch in flight at
// once: before griddepcontrol.wait the state, the conv cache rows and
// weights and the per-head parameters (none written by the previous kernel,
// the in_proj GEMV), after it the token's in_proj outputs. The cached conv
// rows stay in registers for the shift (KT - 1 predicated taps, KT >= K).
template <int RPT, int KT>
__global__ void __launch_bounds__(kGdrThreads) lin_attn_decode_kernel(LinAttnDecode p) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    const int tid = threadIdx.x;
    const int qd = tid & 3;
    const int r = tid >> 2;
    const int warp = tid >> 5, lane = tid & 31;
    const int h = blockIdx.y;
    const int heads = p.heads, kd = p.kdim, vd = p.vdim, K = p.kernel;
    const int nq = heads * kd;
    const int C = 2 * nq + heads * vd;                // conv channels
    const int c0 = blockIdx.x * kGdrCols + qd * 4;   // vd is a multiple of 16: always < vd
    constexpr int H = KT - 1;                         // cached taps held per channel

    __shared__ float red_a[4][4][6];
    __shared__ float red_b[4][4][4];
    __shared__ float ss_part;

    // Batch 1 (before the wait).
    float S[RPT][4];
    float hq[RPT][H], hk[RPT][H], hv[4][H];            // cache rows 1..K-1
    float wq[RPT][KT], wk[RPT][KT], wv[4][KT];          // conv taps 0..K-1
    auto load_channel = [&](int g, float (&hist)[H], float (&w)[KT]) {
#pragma unroll
        for (int k = 0; k < KT; ++k) {
            w[k] = k < K ? p.conv_w[k * C + g] : 0.0f;
            if (k < H) hist[k] = k + 1 < K ? p.conv_state[(k + 1) * C + g] : 0.0f;
        }
    };
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        const int j = r + 32 * i;
        float4 st = make_float4(0.f, 0.f, 0.f, 0.f);
        if (j < kd) {
            st = *reinterpret_cast<const float4*>(p.state + (h * kd + j) * vd + c0);
            load_channel(h * kd + j, hq[i], wq[i]);
            load_channel(nq + h * kd + j, hk[i], wk[i]);
        } else {
#pragma unroll
            for (int k = 0; k < KT; ++k) {
                wq[i][k] = wk[i][k] = 0.0f;
                if (k < H) hq[i][k] = hk[i][k] = 0.0f;
            }
        }
        S[i][0] = st.x; S[i][1] = st.y; S[i][2] = st.z; S[i][3] = st.w;
    }
    const int gv0 = 2 * nq + h * vd + c0;
    float gm[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        load_channel(gv0 + c, hv[c], wv[c]);
        gm[c] = p.gamma[c0 + c];
    }
    const float alog = p.a_log[h];
    const float dt = p.dt_bias[h];

    griddep_wait();
    griddep_launch();

    // Batch 2 (after the wait): this token's in_proj outputs.
    float xq[RPT], xk[RPT], xv[4], zv[4];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        const int j = r + 32 * i;
        xq[i] = j < kd ? p.proj[h * kd + j] : 0.0f;
        xk[i] = j < kd ? p.proj[nq + h * kd + j] : 0.0f;
    }
    const int zo = C + h * vd;        // z of this head
    const int bo = C + heads * vd;    // b, then a
#pragma unroll
    for (int c = 0; c < 4; ++c) {
        xv[c] = p.proj[gv0 + c];
        zv[c] = p.proj[zo + c0 + c];
    }
    const float bb = p.proj[bo + h];
    const float xa = p.proj[bo + heads + h] + dt;

    // conv: taps 0..K-2 over the cached rows, tap K-1 over this token, in order.
    auto conv = [&](const float (&hist)[H], const float (&w)[KT], float x) {
        float sum = 0.0f;
#pragma unroll
        for (int k = 0; k < H; ++k)
            if (k + 1 < K) sum = fmaf(hist[k], w[k], sum);
        float wl = w[0];
#pragma unroll
        for (int k = 1; k < KT; ++k)
            if (k == K - 1) wl = w[k];
        sum = fmaf(x, wl, sum);
        return sum / (1.0f + expf(-sum));
    };
    float qv[RPT], kv[RPT], vv[4];
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        const bool ok = r + 32 * i < kd;
        qv[i] = ok ? conv(hq[i], wq[i], xq[i]) : 0.0f;
        kv[i] = ok ? conv(hk[i], wk[i], xk[i]) : 0.0f;
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) vv[c] = conv(hv[c], wv[c], xv[c]);
    const float beta = 1.0f / (1.0f + expf(-bb));
    const float decay = expf(-expf(alog) * (fmaxf(xa, 0.0f) + logf(1.0f + expf(-fabsf(xa)))));
    const float inv_sqrt_k = rsqrtf((float)kd);

    float part[6] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        part[0] = fmaf(qv[i], qv[i], part[0]);
        part[1] = fmaf(kv[i], kv[i], part[1]);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            S[i][c] *= decay;
            part[2 + c] = fmaf(kv[i], S[i][c], part[2 + c]);
        }
    }
#pragma unroll
    for (int m = 4; m < 32; m <<= 1)
#pragma unroll
        for (int e = 0; e < 6; ++e) part[e] += __shfl_xor_sync(0xffffffffu, part[e], m);
    if (lane < 4) {
#pragma unroll
        for (int e = 0; e < 6; ++e) red_a[warp][qd][e] = part[e];
    }
    __syncthreads();
    float tot[6];
#pragma unroll
    for (int e = 0; e < 6; ++e) tot[e] = (red_a[0][qd][e] + red_a[1][qd][e]) + (red_a[2][qd][e] + red_a[3][qd][e]);
    const float qs = rsqrtf(tot[0] + p.gdr_eps);
    const float ks = rsqrtf(tot[1] + p.gdr_eps);
    float delta[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) delta[c] = (vv[c] - tot[2 + c] * ks) * beta;
    float o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        const float kn = kv[i] * ks;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            S[i][c] = fmaf(kn, delta[c], S[i][c]);
            o[c] = fmaf(qv[i], S[i][c], o[c]);
        }
    }
#pragma unroll
    for (int m = 4; m < 32; m <<= 1)
#pragma unroll
        for (int c = 0; c < 4; ++c) o[c] += __shfl_xor_sync(0xffffffffu, o[c], m);
    if (lane < 4) {
#pragma unroll
        for (int c = 0; c < 4; ++c) red_b[warp][qd][c] = o[c];
    }
    __syncthreads();
    // Threads 0..3 (r == 0) finish the CTA's 16 columns and their sum of squares.
    float ov[4] = {0.f, 0.f, 0.f, 0.f};
    if (warp == 0) {
        float ss = 0.0f;
        if (r == 0) {
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                ov[c] = ((red_b[0][qd][c] + red_b[1][qd][c]) + (red_b[2][qd][c] + red_b[3][qd][c])) * qs * inv_sqrt_k;
                ss = fmaf(ov[c], ov[c], ss);
            }
        }
        ss += __shfl_xor_sync(0xffffffffu, ss, 1);
        ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        if (lane == 0) ss_part = ss;
    }
    cluster.sync();  // partial sums visible; every CTA of the head has read the conv cache
    if (r == 0) {
        float total = 0.0f;
        const int nb = (int)cluster.num_blocks();
        for (int b = 0; b < nb; ++b) total += *cluster.map_shared_rank(&ss_part, b);
        const float inv = 1.0f / sqrtf(fmaxf(total / (float)vd + p.norm_eps, 1e-20f));
#pragma unroll
        for (int c = 0; c < 4; ++c)
            p.y[h * vd + c0 + c] = ov[c] * inv * gm[c] * (zv[c] / (1.0f + expf(-zv[c])));
    }
    cluster.barrier_arrive();
    // Conv cache: drop the oldest row, append this token (from registers).
    auto shift = [&](int g, const float (&hist)[H], float x) {
#pragma unroll
        for (int k = 0; k < H; ++k)
            if (k + 1 < K) p.conv_state[k * C + g] = hist[k];
        p.conv_state[(K - 1) * C + g] = x;
    };
    if (blockIdx.x == 0 && qd == 0) {
#pragma unroll
        for (int i = 0; i < RPT; ++i) {
            const int j = r + 32 * i;
            if (j < kd) {
                shift(h * kd + j, hq[i], xq[i]);
                shift(nq + h * kd + j, hk[i], xk[i]);
            }
        }
    }
    if (r == 0) {
#pragma unroll
        for (int c = 0; c < 4; ++c) shift(gv0 + c, hv[c], xv[c]);
    }
#pragma unroll
    for (int i = 0; i < RPT; ++i) {
        const int j = r + 32 * i;
        if (j < kd)
            *reinterpret_cast<float4*>(p.state + (h * kd + j) * vd + c0) =
                make_float4(S[i][0], S[i][1], S[i][2], S[i][3]);
    }
    cluster.barrier_wait();
}

}  // namespace

template <int KT>
static cudaError_t launch_lin_attn_rpt(const cudaLaunchConfig_t& cfg, const LinAttnDecode& a) {
    if (a.kdim <= 32) return cudaLaunchKernelEx(&cfg, lin_attn_decode_kernel<1, KT>, a);
    if (a.kdim <= 64) return cudaLaunchKernelEx(&cfg, lin_attn_decode_kernel<2, KT>, a);
    if (a.kdim <= 128) return cudaLaunchKernelEx(&cfg, lin_attn_decode_kernel<4, KT>, a);
    return cudaLaunchKernelEx(&cfg, lin_attn_decode_kernel<8, KT>, a);
}

bool lin_attn_decode_supported(int heads, int kdim, int vdim, int kernel) {
    // 32-bit indexing: the state and the in_proj rows stay below 2^30 elements.
    return heads > 0 && heads <= 65535 && kdim > 0 && kdim <= 256 && kdim % 4 == 0 && vdim % kGdrCols == 0 &&
           vdim > 0 && vdim / kGdrCols <= 8 && kernel >= 1 && kernel <= 8 &&
           (long long)heads * (2LL * kdim + 2LL * vdim + 2) < (1LL << 30) &&
           (long long)heads * kdim * vdim < (1LL << 30);
}

cudaError_t launch_lin_attn_decode(const LinAttnDecode& a, cudaStream_t s) {
    if (!lin_attn_decode_supported(a.heads, a.kdim, a.vdim, a.kernel)) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.vdim / kGdrCols, a.heads);
    cfg.blockDim = dim3(kGdrThreads);
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = a.vdim / kGdrCols;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    if (a.kernel <= 4) return launch_lin_attn_rpt<4>(cfg, a);
    return launch_lin_attn_rpt<8>(cfg, a);
}

cudaError_t launch_short_conv(const float* weight, const float* mixed, const float* cache_in, float* out,
                              float* cache_out, int groups, int kernel, int seq, int cache_len, cudaStream_t s) {
    if (kernel > kConvMaxKernel) return cudaErrorInvalidValue;
    const int threads = 128;
    short_conv_kernel<<<(groups + threads - 1) / threads, threads, 0, s>>>(weight, mixed, cache_in, out, cache_out,
                                                                          groups, kernel, seq, cache_len);
    return cudaGetLastError();
}

int gdr_max_kdim() { return 256; }

cudaError_t launch_gated_delta_rule(const float* a_log, const float* dt_bias, const float* b, const float* a,
                                    const float* q, const float* k, const float* v, const float* state_in,
                                    float* out, float* state_out, int heads, int kdim, int vdim, int first,
                                    int count, float eps, cudaStream_t s) {
    GdrArgs p{a_log, dt_bias, b, a, q, k, v, state_in, out, state_out, heads, kdim, vdim, first, count, eps};
    const int vdim4 = (vdim + 3) & ~3;
    dim3 grid((vdim4 + kGdrCols - 1) / kGdrCols, heads);
    if (kdim <= 32) gdr_kernel<1><<<grid, kGdrThreads, 0, s>>>(p);
    else if (kdim <= 64) gdr_kernel<2><<<grid, kGdrThreads, 0, s>>>(p);
    else if (kdim <= 128) gdr_kernel<4><<<grid, kGdrThreads, 0, s>>>(p);
    else if (kdim <= 256) gdr_kernel<8><<<grid, kGdrThreads, 0, s>>>(p);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}
