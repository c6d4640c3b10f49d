// k_gemv.cu -- batch-1 weight-only Q4 / Q8 dequant GEMV for sm_100a.
//
// Replaces the reference's AexisGemm2DPack4LinearTextureAFromLinear /
// ...TiledTextureAFromLinear kernels (HLSL Pack4Matmul:1038-1104, 2245-2300)
// and their weight read AexisGemm2DReadB (:707-734) for M = 1.
//
// Layout in HBM (kept as the reference packs it, so uploads are plain copies):
//   Q4: row n is k/2 contiguous bytes, element k at nibble (k & 1) of byte
//       k/2 (low nibble first); scales [n, k/group] (fp16 or fp32).
//   Q8: row n is k contiguous int8; one scale per row.
//
// Fast kernel ("activation-stationary streaming"): the activation vector is
// staged once per CTA in shared memory as fp32 (optionally RMS-normalised,
// which fuses the preceding RMSNorm layer), swizzled in 16-byte units so the
// per-lane chunk reads are bank-conflict free. Each warp owns R output rows at
// a time; lane l streams 16-byte chunks l, l+32, ... of those rows with
// non-allocating 128-bit loads, double-buffered one row block ahead. Int4 and
// int8 values become fp32 without conversion instructions: the packed bits are
// OR-ed under the exponent of 2^23 (LOP3 / PRMT), a packed fp32x2 add removes
// the bias, and packed fp32x2 FMAs accumulate. Int4 nibbles are decoded in
// place, shifted by 16^j inside the mantissa; the activation is pre-scaled by
// 16^-j in shared memory so the product is exact. Per-chunk (group) scales are
// applied once per 32 products. Rows are reduced with a reduce-scatter over the
// warp (R rows in 9 shuffles for R = 8).
//
// The generic kernel covers every other layout (odd k, groups that are not
// multiples of 16, ...) with the reference's exact flat indexing.
#include "gemv_dev.cuh"

namespace {

using namespace aexis_dev;

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

struct FastParams {
    const uint4* W;        // [n][row_u4] 16-byte chunks
    const void* S;         // scales
    int n, k;
    int nchunks;           // 16-byte chunks per row (= row_u4)
    int s_row;             // scales per row (group modes)
    int gshift;            // SMODE 1: scale index = chunk >> gshift
    const void* x;
    int a_dtype;
    const float* norm_gamma;
    float norm_eps;
    const float* bias;
    float alpha, beta;
    void* y;
    int y_dtype;
    int epi;
    // EPI_QKV_ROPE
    const float* rope_cos;
    const float* rope_sin;
    const int* rope_map;
    __half* k_cache;
    __half* v_cache;
    int head_dim, kv_cap, rot_dim;
    const int* pos_ptr;
    unsigned long long* argmax_key;
};

// Scale modes: 0 = one scale per row (Q8, Q4 with group == k), 1 = one scale
// per 16-byte chunk (Q4, group = 32 << gshift), 2 = two per chunk (Q4 group 16).
template <int BITS, typename ST, int SMODE, int R>
__global__ void __launch_bounds__(kThreads) gemv_fast_kernel(FastParams p);

}  // namespace

namespace {

template <int BITS, typename ST, int SMODE, int R>
__global__ void __launch_bounds__(kThreads) gemv_fast_kernel(FastParams p) {
    extern __shared__ float4 smem_act[];  // swizzled fp32 activations, k/4 units
    __shared__ float red[kWarps];
    constexpr int CPT = BITS == 4 ? 1 : 2;    // chunks per lane per tile
    constexpr int UPC = BITS == 4 ? 8 : 4;    // float4 activation units per chunk
    constexpr int TILE = 32 * CPT;            // chunks per tile
    constexpr int NS = SMODE == 2 ? 2 : 1;    // scales per chunk
    constexpr int LR = R == 8 ? 3 : R == 4 ? 2 : R == 2 ? 1 : 0;

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nt = (p.nchunks + TILE - 1) / TILE;
    const int nrb = (p.n + R - 1) / R;
    const int gw = blockIdx.x * kWarps + warp;
    const int tw = gridDim.x * kWarps;
    const long long items = (long long)(gw < nrb ? (nrb - 1 - gw) / tw + 1 : 0) * nt;
    const ST* S = reinterpret_cast<const ST*>(p.S);

    uint4 wb0[R][CPT], wb1[R][CPT];
    float sb0[R][CPT][NS], sb1[R][CPT][NS];

    auto load_item = [&](long long it, uint4 (&wb)[R][CPT], float (&sb)[R][CPT][NS]) {
        const int rb = gw + (int)(it / nt) * tw;
        const int t = (int)(it % nt);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int row = rb * R + r;
#pragma unroll
            for (int i = 0; i < CPT; ++i) {
                const int c = t * TILE + i * 32 + lane;
                const bool ok = row < p.n && c < p.nchunks;
                wb[r][i] = ok ? ldg_stream(p.W + (long long)row * p.nchunks + c) : make_uint4(0u, 0u, 0u, 0u);
                if constexpr (SMODE == 1) {
                    sb[r][i][0] = ok ? load_scale<ST>(S, (long long)row * p.s_row + (c >> p.gshift)) : 0.0f;
                } else if constexpr (SMODE == 2) {
                    sb[r][i][0] = ok ? load_scale<ST>(S, (long long)row * p.s_row + 2 * c) : 0.0f;
                    sb[r][i][1] = ok ? load_scale<ST>(S, (long long)row * p.s_row + 2 * c + 1) : 0.0f;
                }
            }
        }
    };

    // Weights do not depend on the producer of x: start streaming them before
    // waiting on the previous grid (programmatic dependent launch).
    if (items > 0) load_item(0, wb0, sb0);
    griddep_wait();

    // Stage x (optionally RMS-normalised) into shared memory, swizzled.
    {
        float* sa = reinterpret_cast<float*>(smem_act);
        const bool norm = p.norm_gamma != nullptr;
        float ss = 0.0f;
        for (int i = threadIdx.x; i < p.k; i += kThreads) {
            const float xv = aexis_load_act(p.x, p.a_dtype, i);
            const int u = i >> 2;
            float sv = xv;
            if (norm) ss = fmaf(xv, xv, ss);
            else if (BITS == 4) {
                const int j = i & 7;
                sv = xv * __uint_as_float((uint32_t)(127 - 4 * (j < 5 ? j : j - 3)) << 23);
            }
            sa[swz(u) * 4 + (i & 3)] = sv;
        }
        if (norm) {
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kWarps; ++w) tot += red[w];
            const float inv = 1.0f / sqrtf(fmaxf(tot / (float)p.k + p.norm_eps, 1e-20f));
            for (int i = threadIdx.x; i < p.k; i += kThreads) {
                const int idx = swz(i >> 2) * 4 + (i & 3);
                float sv = sa[idx] * inv * p.norm_gamma[i];
                if (BITS == 4) {
                    const int j = i & 7;
                    sv = sv * __uint_as_float((uint32_t)(127 - 4 * (j < 5 ? j : j - 3)) << 23);
                }
                sa[idx] = sv;
            }
        }
        __syncthreads();
    }
    griddep_launch();

    unsigned long long best_key = 0ull;  // EPI_LOGITS_ARGMAX running maximum
    float tot[R];
    unsigned long long racc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) { tot[r] = 0.0f; racc[r] = 0ull; }

    auto process = [&](long long it, const uint4 (&wb)[R][CPT], const float (&sb)[R][CPT][NS]) {
        const int rb = gw + (int)(it / nt) * tw;
        const int t = (int)(it % nt);
#pragma unroll
        for (int i = 0; i < CPT; ++i) {
            const int c = t * TILE + i * 32 + lane;
            if (c < p.nchunks) {
                float4 a[UPC];
#pragma unroll
                for (int q = 0; q < UPC; ++q) a[q] = smem_act[swz(c * UPC + q)];
#pragma unroll
                for (int r = 0; r < R; ++r) {
                    if constexpr (BITS == 4) {
                        if constexpr (SMODE == 0) {
                            tot[r] += sum2(dot_q4_chunk(wb[r][i], a));
                        } else if constexpr (SMODE == 1) {
                            tot[r] = fmaf(sum2(dot_q4_chunk(wb[r][i], a)), sb[r][i][0], tot[r]);
                        } else {
                            const uint4 w = wb[r][i];
                            const uint4 lo = make_uint4(w.x, w.y, 0u, 0u), hi = make_uint4(0u, 0u, w.z, w.w);
                            tot[r] = fmaf(sum2(dot_q4_chunk(lo, a)), sb[r][i][0], tot[r]);
                            tot[r] = fmaf(sum2(dot_q4_chunk(hi, a)), sb[r][i][1], tot[r]);
                        }
                    } else {
                        dot_q8_chunk(racc[r], wb[r][i], a);
                    }
                }
            }
        }
        if (t != nt - 1) return;
        // Row block complete: reduce-scatter the R row partials over the warp.
        float v[R];
#pragma unroll
        for (int r = 0; r < R; ++r) v[r] = (BITS == 8) ? sum2(racc[r]) : tot[r];
#pragma unroll
        for (int lvl = 0; lvl < LR; ++lvl) {
            const int s = 16 >> lvl;
            const int h = R >> (lvl + 1);
            const bool upper = (lane & s) != 0;
#pragma unroll
            for (int j = 0; j < h; ++j) {
                const float send = upper ? v[j] : v[j + h];
                const float keep = upper ? v[j + h] : v[j];
                v[j] = keep + __shfl_xor_sync(0xffffffffu, send, s);
            }
        }
#pragma unroll
        for (int s = 16 >> LR; s >= 1; s >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], s);
        const int rrow = LR == 0 ? 0 : (lane >> (5 - LR));
        const int row = rb * R + rrow;
        float val = v[0];
        if constexpr (SMODE == 0) {
            if (row < p.n) val *= load_scale<ST>(S, row);
        }
        const float partner = R >= 2 ? __shfl_xor_sync(0xffffffffu, val, 32 >> LR) : val;
        const bool leader = (lane & ((32 >> LR) - 1)) == 0;
        if (leader && row < p.n) {
            switch (p.epi) {
                case EPI_STORE: {
                    const float bb = p.bias ? p.beta * p.bias[row] : 0.0f;
                    aexis_store_out(p.y, p.y_dtype, row, p.alpha * (bb + val));
                } break;
                case EPI_STORE_TILED: {
                    const float bb = p.bias ? p.beta * p.bias[row] : 0.0f;
                    aexis_store_out(p.y, p.y_dtype, row, bb + p.alpha * val);
                } break;
                case EPI_RESIDUAL:
                    reinterpret_cast<float*>(p.y)[row] += p.alpha * val;
                    break;
                case EPI_SWIGLU:
                    if ((row & 1) == 0) {
                        const float g = val;
                        reinterpret_cast<float*>(p.y)[row >> 1] = g / (1.0f + expf(-g)) * partner;
                    }
                    break;
                case EPI_QKV_ROPE: {
                    const int desc = p.rope_map[row];
                    const int kind = desc >> 24, head = (desc >> 12) & 0xFFF, dim = desc & 0xFFF;
                    const int pos = *p.pos_ptr;
                    float out = val;
                    if (kind != 2 && dim < p.rot_dim) {
                        const int half = p.rot_dim >> 1;
                        const bool first = dim < half;
                        const int j = first ? dim : dim - half;
                        const float c = p.rope_cos[(long long)pos * half + j];
                        const float s = p.rope_sin[(long long)pos * half + j];
                        const float x0 = first ? val : partner, x1 = first ? partner : val;
                        out = first ? x0 * c - x1 * s : x0 * s + x1 * c;
                    }
                    if (kind == 0) {
                        reinterpret_cast<float*>(p.y)[head * p.head_dim + dim] = out;
                    } else {
                        __half* cache = kind == 1 ? p.k_cache : p.v_cache;
                        cache[((long long)head * p.kv_cap + pos) * p.head_dim + dim] = __float2half_rn(out);
                    }
                } break;
                case EPI_LOGITS_ARGMAX: {
                    reinterpret_cast<float*>(p.y)[row] = val;
                    const unsigned long long key = aexis_argmax_key(val, row);
                    best_key = key > best_key ? key : best_key;
                } break;
            }
        }
#pragma unroll
        for (int r = 0; r < R; ++r) { tot[r] = 0.0f; racc[r] = 0ull; }
    };

    for (long long it = 0; it < items; it += 2) {
        if (it + 1 < items) load_item(it + 1, wb1, sb1);
        process(it, wb0, sb0);
        if (it + 1 < items) {
            if (it + 2 < items) load_item(it + 2, wb0, sb0);
            process(it + 1, wb1, sb1);
        }
    }
    if (p.epi == EPI_LOGITS_ARGMAX) {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best_key, o);
            best_key = other > best_key ? other : best_key;
        }
        if (lane == 0 && best_key != 0ull) atomicMax(p.argmax_key, best_key);
    }
}

// Exact generic kernel: one warp per output row, the reference's flat index
// (row*k + kk) for any k, group and alignment.
template <typename ST>
__global__ void __launch_bounds__(kThreads) gemv_generic_kernel(
    const uint32_t* P, const ST* S, int bits, int group, int n, int k, const void* x, int a_dtype,
    const float* bias, float alpha, float beta, void* y, int y_dtype, int tiled, int residual) {
    griddep_wait();
    const int lane = threadIdx.x & 31;
    const long long row = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
    if (row >= n) return;
    float acc = 0.0f;
    for (int kk = lane; kk < k; kk += 32) {
        const long long index = row * k + kk;
        float w;
        if (bits == 4) {
            const uint32_t raw = (__ldg(P + (index >> 3)) >> ((index & 7) * 4)) & 0xFu;
            const int sv = raw >= 8u ? (int)raw - 16 : (int)raw;
            w = (float)sv * load_scale<ST>(S, group > 0 ? index / group : row);
        } else {
            const uint32_t raw = (__ldg(P + (index >> 2)) >> ((index & 3) * 8)) & 0xFFu;
            const int sv = raw >= 128u ? (int)raw - 256 : (int)raw;
            w = (float)sv * load_scale<ST>(S, row);
        }
        acc = fmaf(aexis_load_act(x, a_dtype, kk), w, acc);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
        const float bb = bias ? beta * bias[row] : 0.0f;
        if (residual) reinterpret_cast<float*>(y)[row] += alpha * acc;
        else aexis_store_out(y, y_dtype, row, tiled ? bb + alpha * acc : alpha * (bb + acc));
    }
}

template <int BITS, typename ST, int SMODE, int R>
cudaError_t launch_fast_t(const FastParams& fp, int sm_count, bool pdl, cudaStream_t stream) {
    auto kern = gemv_fast_kernel<BITS, ST, SMODE, R>;
    // The swizzle permutes 16-byte units inside groups of eight: pad the
    // buffer to whole groups so every swizzled unit is inside it.
    const size_t smem = (size_t)((fp.k + 31) / 32 * 32) * sizeof(float);
    static int occ = -1;  // resident CTAs per SM for this instantiation (queried once)
    static size_t occ_smem = 0;
    if (occ < 0 || occ_smem != smem) {
        if (smem > 48 * 1024) {
            cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess) return e;
        }
        int o = 0;
        cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, kThreads, smem);
        if (e != cudaSuccess) return e;
        occ = o > 0 ? o : 1;
        occ_smem = smem;
    }
    const int nrb = (fp.n + R - 1) / R;
    int blocks = (nrb + kWarps - 1) / kWarps;
    blocks = blocks < sm_count * occ ? blocks : sm_count * occ;
    if (blocks < 1) blocks = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, fp);
}

template <int BITS, typename ST, int SMODE>
cudaError_t launch_fast_r(const FastParams& fp, int R, int sm_count, bool pdl, cudaStream_t s) {
    switch (R) {
        case 8: return launch_fast_t<BITS, ST, SMODE, 8>(fp, sm_count, pdl, s);
        case 4: return launch_fast_t<BITS, ST, SMODE, 4>(fp, sm_count, pdl, s);
        case 2: return launch_fast_t<BITS, ST, SMODE, 2>(fp, sm_count, pdl, s);
        default: return launch_fast_t<BITS, ST, SMODE, 1>(fp, sm_count, pdl, s);
    }
}

template <typename ST>
cudaError_t launch_fast_s(const FastParams& fp, int bits, int smode, int R, int sm_count, bool pdl,
                          cudaStream_t s) {
    if (bits == 8) return launch_fast_r<8, ST, 0>(fp, R, sm_count, pdl, s);
    if (smode == 0) return launch_fast_r<4, ST, 0>(fp, R, sm_count, pdl, s);
    if (smode == 1) return launch_fast_r<4, ST, 1>(fp, R, sm_count, pdl, s);
    return launch_fast_r<4, ST, 2>(fp, R, sm_count, pdl, s);
}

// Scale mode of a Q4/Q8 weight for the fast kernel, or -1 when only the
// generic kernel can read it.
int fast_scale_mode(const aexis_weights* w, int* gshift) {
    *gshift = 0;
    if (w->kind == WK_Q8) return (w->k % 16 == 0 && w->k <= 49152) ? 0 : -1;
    if (w->kind != WK_Q4 || w->k % 32 != 0 || w->k > 49152) return -1;
    if (w->group == w->k) return 0;
    if (w->group == 16) return 2;
    if (w->group % 32 != 0) return -1;
    int g = w->group / 32, sh = 0;
    while ((1 << sh) < g) ++sh;
    if ((1 << sh) != g) return -1;
    *gshift = sh;
    return 1;
}

}  // namespace

const char* gemv_kernel_name(const aexis_weights* w) {
    if (gemv_mma_supported(w, AEXIS_F16)) return w->kind == WK_Q4 ? "q4_mma" : "q8_mma";
    if (gemv_stream_supported(w)) return w->kind == WK_Q4 ? "q4_stream" : "q8_stream";
    int gs;
    if (fast_scale_mode(w, &gs) < 0) return "generic";
    return w->kind == WK_Q4 ? "q4_fast" : "q8_fast";
}

cudaError_t launch_gemv(const GemvArgs& a, int sm_count, cudaStream_t stream) {
    const aexis_weights* w = a.w;
    if (gemv_mma_supported(w, a.a_dtype)) return launch_gemv_mma(a, sm_count, stream);
    if (gemv_stream_supported(w)) return launch_gemv_stream(a, sm_count, a.status, stream);
    int gshift = 0;
    const int smode = fast_scale_mode(w, &gshift);
    const bool pair_epi = a.epilogue == EPI_SWIGLU || a.epilogue == EPI_QKV_ROPE;
    if (a.epilogue == EPI_LOGITS_ARGMAX && smode < 0) return cudaErrorNotSupported;
    if (smode >= 0) {
        FastParams fp = {};
        fp.W = reinterpret_cast<const uint4*>(w->data);
        fp.S = w->scales;
        fp.n = w->n;
        fp.k = w->k;
        fp.nchunks = (int)((long long)w->k * (w->kind == WK_Q4 ? 4 : 8) / 128);
        fp.s_row = w->kind == WK_Q4 && w->group > 0 ? w->k / w->group : 1;
        fp.gshift = gshift;
        fp.x = a.x;
        fp.a_dtype = a.a_dtype;
        fp.norm_gamma = a.norm_gamma;
        fp.norm_eps = a.norm_eps;
        fp.bias = a.bias;
        fp.alpha = a.alpha;
        fp.beta = a.beta;
        fp.y = a.y;
        fp.y_dtype = a.y_dtype;
        fp.epi = a.epilogue;
        fp.rope_cos = a.rope_cos;
        fp.rope_sin = a.rope_sin;
        fp.rope_map = a.rope_map;
        fp.k_cache = a.k_cache;
        fp.v_cache = a.v_cache;
        fp.head_dim = a.head_dim;
        fp.kv_cap = a.kv_cap;
        fp.rot_dim = a.rot_dim;
        fp.pos_ptr = a.pos_ptr;
        fp.argmax_key = a.argmax_key;
        // Rows per warp: as many as keep every SM's warps supplied with rows.
        const int cpt = w->kind == WK_Q4 ? 1 : 2;
        const int target = sm_count * 16;
        int R = 8;
        while (R > 1 && (w->n + R - 1) / R < target) R >>= 1;
        (void)cpt;
        if (pair_epi && R < 2) R = 2;
        if (w->scale_dtype == AEXIS_F16)
            return launch_fast_s<__half>(fp, w->kind, smode, R, sm_count, a.pdl, stream);
        return launch_fast_s<float>(fp, w->kind, smode, R, sm_count, a.pdl, stream);
    }
    if (pair_epi) return cudaErrorNotSupported;
    const int tiled = a.epilogue == EPI_STORE_TILED, residual = a.epilogue == EPI_RESIDUAL;
    const int blocks = (w->n + kWarps - 1) / kWarps;
    const int bits = w->kind == WK_Q4 ? 4 : 8;
    if (w->scale_dtype == AEXIS_F16)
        gemv_generic_kernel<__half><<<blocks, kThreads, 0, stream>>>(
            reinterpret_cast<const uint32_t*>(w->data), reinterpret_cast<const __half*>(w->scales), bits,
            w->kind == WK_Q4 ? w->group : 0, w->n, w->k, a.x, a.a_dtype, a.bias, a.alpha, a.beta, a.y,
            a.y_dtype, tiled, residual);
    else
        gemv_generic_kernel<float><<<blocks, kThreads, 0, stream>>>(
            reinterpret_cast<const uint32_t*>(w->data), reinterpret_cast<const float*>(w->scales), bits,
            w->kind == WK_Q4 ? w->group : 0, w->n, w->k, a.x, a.a_dtype, a.bias, a.alpha, a.beta, a.y,
            a.y_dtype, tiled, residual);
    return cudaGetLastError();
}
