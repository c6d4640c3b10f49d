// k_gemv_stream.cu -- batch-1 Q4 / Q8 dequant GEMV, bulk-copy streaming version.
//
// Same contract as the register-streaming kernel in k_gemv.cu (AexisGemm2D-
// Pack4LinearTextureAFromLinear / ...Tiled..., HLSL Pack4Matmul:1038-1104,
// 2245-2300, with AexisGemm2DReadB :707-734 as the weight read), built for
// HBM streaming on B200:
//   * A persistent CTA per SM owns every gridDim.x-th tile of TR consecutive
//     output rows. Rows are contiguous in HBM, so a tile's weights are one
//     cp.async.bulk copy and its scales another. One producer thread keeps a
//     ring of S stages in shared memory full (mbarrier full/empty pairs,
//     evict-first L2 policy); eight consumer warps compute from it.
//   * The producer starts before griddepcontrol.wait: under programmatic
//     dependent launch the ring fills while the previous kernel is finishing,
//     and only the activation read waits for it.
//   * Consumers stage x once (with the optional fused RMSNorm) and keep their
//     lane's K-chunk of it in registers for every row. A row group of WPG
//     warps covers the K chunks of RPG rows; weights come from shared memory
//     with conflict-free 128-bit reads and are decoded with the fp32 magic-
//     number scheme of gemv_dev.cuh.
//   * Every barrier wait is bounded (about a second); a timeout is recorded
//     in the context status word and the kernel returns, after the producer
//     has waited (bounded) for its own copies in flight.
#include "gemv_stream.cuh"

namespace {

using namespace aexis_dev;

constexpr int kCW = 8;                       // consumer warps
constexpr int kStreamThreads = (kCW + 1) * 32;

// BITS 4/8; ST scale type; SMODE 0 per-row scale, 1 one scale per 16-byte
// chunk (group 32 << gshift), 2 two per chunk (group 16); A chunks per lane;
// WPG warps per row group; RPG rows per row group per tile.
template <int BITS, typename ST, int SMODE, int A, int WPG, int RPG>
__global__ void __launch_bounds__(kStreamThreads, A == 1 ? 2 : 1) gemv_stream_kernel(StreamParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int RG = kCW / WPG;
    constexpr int TR = RG * RPG;
    constexpr int EPC = BITS == 4 ? 32 : 16;  // elements per 16-byte chunk
    constexpr int NCT = 32 * WPG;
    constexpr int LR = RPG == 8 ? 3 : (RPG == 4 ? 2 : 1);

    const int S = p.stages;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + S;
    float* act_s = reinterpret_cast<float*>(smem + 128);
    float* red = act_s + p.act_floats;              // [2][RG][RPG][WPG]
    uint8_t* ring = reinterpret_cast<uint8_t*>(red + 2 * RG * RPG * WPG + 32);
    ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(ring) + 127) & ~uintptr_t(127));

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int my_tiles = (int)blockIdx.x < p.ntiles ? (p.ntiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, kCW);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kCW) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            int issued = 0;
            bool ok = true;
            for (int it = 0; it < my_tiles && ok; ++it) {
                const int s = it % S;
                if (it >= S && !mbar_wait(empty + s, ((it / S) & 1) ^ 1)) {
                    report_timeout(p.status);
                    ok = false;
                    break;
                }
                const int tile = (int)blockIdx.x + it * (int)gridDim.x;
                const int rows = min(TR, p.n - tile * TR);
                const uint32_t wb = (uint32_t)rows * p.row_bytes;
                const uint32_t sb = ((uint32_t)rows * p.srow_bytes + 15u) & ~15u;
                uint8_t* dst = ring + (size_t)s * p.stage_bytes;
                mbar_arrive_expect_tx(full + s, wb + sb);
                bulk_g2s(dst, p.W + (size_t)tile * TR * p.row_bytes, wb, full + s, pol);
                bulk_g2s(dst + p.w_tile_bytes, p.S + (size_t)tile * TR * p.srow_bytes, sb, full + s, pol);
                ++issued;
            }
            // No copy may still be landing when the CTA exits.
            for (int it = max(0, issued - S); it < issued; ++it)
                if (!mbar_wait(full + it % S, (it / S) & 1)) { report_timeout(p.status); break; }
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    griddep_wait();
    {
        // x -> shared memory in the pair-staged order of its chunk, pre-scaled
        // per field (optionally RMS-normalised first: the fused RMSNorm layer).
        constexpr int EPC_ = BITS == 4 ? 32 : 16;
        const bool norm = p.norm_gamma != nullptr;
        float ss = 0.0f;
        for (int i = threadIdx.x; i < p.k; i += kCW * 32) {
            const float xv = aexis_load_act(p.x, p.a_dtype, i);
            if (norm) ss = fmaf(xv, xv, ss);
            const int e = i % EPC_;
            act_s[i - e + act_pair_slot<BITS>(e)] = norm ? xv : xv * act_pair_prescale<BITS>(e);
        }
        if (norm) {
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) red[warp] = ss;
            named_sync(1, kCW * 32);
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kCW; ++w) tot += red[w];
            const float inv = 1.0f / sqrtf(fmaxf(tot / (float)p.k + p.norm_eps, 1e-20f));
            named_sync(1, kCW * 32);
            for (int i = threadIdx.x; i < p.k; i += kCW * 32) {
                const int e = i % EPC_;
                const int idx = i - e + act_pair_slot<BITS>(e);
                act_s[idx] = act_s[idx] * inv * p.norm_gamma[i] * act_pair_prescale<BITS>(e);
            }
        }
        named_sync(1, kCW * 32);
    }
    griddep_launch();

    const int rg = warp / WPG;
    const int tg = (warp % WPG) * 32 + lane;  // thread index within the row group
    constexpr int NP = EPC / 2;               // activation pairs per chunk
    unsigned long long a[A][NP];
#pragma unroll
    for (int ai = 0; ai < A; ++ai) {
        const int c = tg + ai * NCT;
#pragma unroll
        for (int q = 0; q < NP; ++q)
            a[ai][q] = c < p.nchunks ? reinterpret_cast<const unsigned long long*>(act_s)[c * NP + q] : 0ull;
    }
    const PairConsts kc = make_pair_consts<BITS>(p.zero);
    unsigned long long best_key = 0ull;
    // Set by any consumer warp whose bounded wait ran out; with WPG > 1 all
    // warps meet at the per-tile barrier and leave together.
    volatile int* abort_flag = reinterpret_cast<volatile int*>(red + 2 * RG * RPG * WPG);
    if (threadIdx.x == 0) *abort_flag = 0;
    named_sync(1, kCW * 32);

    for (int it = 0; it < my_tiles; ++it) {
        const int s = it % S;
        const bool ready = mbar_wait(full + s, (it / S) & 1);
        if (!ready) {
            report_timeout(p.status);
            *abort_flag = 1;
            if constexpr (WPG == 1) break;
        }
        const int tile = (int)blockIdx.x + it * (int)gridDim.x;
        const uint8_t* wt = ring + (size_t)s * p.stage_bytes;
        const uint8_t* st = wt + p.w_tile_bytes;
        float tot[RPG];
        unsigned long long r01[RPG], r23[RPG];  // per-row-scale accumulators (SMODE 0)
#pragma unroll
        for (int r = 0; r < RPG; ++r) { tot[r] = 0.0f; r01[r] = 0ull; r23[r] = 0ull; }
#pragma unroll
        for (int ai = 0; ai < A; ++ai) {
            const int c = tg + ai * NCT;
            if (ready && c < p.nchunks) {
#pragma unroll
                for (int r = 0; r < RPG; ++r) {
                    const int tr = rg * RPG + r;
                    const ulonglong2 w = *reinterpret_cast<const ulonglong2*>(wt + (size_t)tr * p.row_bytes + c * 16);
                    const ST* srow = reinterpret_cast<const ST*>(st + (size_t)tr * p.srow_bytes);
                    if constexpr (BITS == 4) {
                        if constexpr (SMODE == 0) {
                            dot_q4_pairs(w.x, w.y, a[ai], kc, r01[r], r23[r]);
                        } else {
                            unsigned long long c01 = 0ull, c23 = 0ull;
                            dot_q4_pairs(w.x, w.y, a[ai], kc, c01, c23);
                            if constexpr (SMODE == 1) {
                                tot[r] = fmaf(sum2u(c01) + sum2u(c23), to_float(srow[c >> p.gshift]), tot[r]);
                            } else {
                                tot[r] = fmaf(sum2u(c01), to_float(srow[2 * c]), tot[r]);
                                tot[r] = fmaf(sum2u(c23), to_float(srow[2 * c + 1]), tot[r]);
                            }
                        }
                    } else {
                        dot_q8_pairs(w.x, w.y, a[ai], kc, r01[r], r23[r]);
                    }
                }
            }
        }
        // Per-row scales (SMODE 0) are read before the stage is released.
        float rscale[RPG];
#pragma unroll
        for (int r = 0; r < RPG; ++r) {
            rscale[r] = 1.0f;
            if constexpr (SMODE == 0) {
                const int tr = rg * RPG + r;
                tot[r] = sum2u(r01[r]) + sum2u(r23[r]);
                if (ready && tile * TR + tr < p.n)
                    rscale[r] = to_float(*reinterpret_cast<const ST*>(st + (size_t)tr * p.srow_bytes));
            }
        }
        __syncwarp();
        if (ready && lane == 0) mbar_arrive(empty + s);

        // Reduce-scatter the RPG row partials over the warp; lane r then holds row r.
        float v[RPG];
#pragma unroll
        for (int r = 0; r < RPG; ++r) v[r] = tot[r];
#pragma unroll
        for (int lvl = 0; lvl < LR; ++lvl) {
            const int sh = 16 >> lvl;
            const int h = RPG >> (lvl + 1);
            const bool upper = (lane & sh) != 0;
#pragma unroll
            for (int j = 0; j < h; ++j) {
                const float send = upper ? v[j] : v[j + h];
                const float keep = upper ? v[j + h] : v[j];
                v[j] = keep + __shfl_xor_sync(0xffffffffu, send, sh);
            }
        }
#pragma unroll
        for (int sh = 16 >> LR; sh >= 1; sh >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], sh);
        float rv = __shfl_sync(0xffffffffu, v[0], (lane % RPG) << (5 - LR));
        if constexpr (WPG > 1) {
            float* rbuf = red + (it & 1) * RG * RPG * WPG;
            if (lane < RPG) rbuf[(rg * RPG + lane) * WPG + (warp % WPG)] = rv;
            named_sync(1, kCW * 32);
            if (*abort_flag) break;
            rv = 0.0f;
            if (lane < RPG) {
#pragma unroll
                for (int w = 0; w < WPG; ++w) rv += rbuf[(rg * RPG + lane) * WPG + w];
            }
        }
        const int row = tile * TR + rg * RPG + (lane % RPG);
        float sc = 1.0f;
#pragma unroll
        for (int r = 0; r < RPG; ++r)
            if ((lane % RPG) == r) sc = rscale[r];
        rv *= sc;
        const float partner = __shfl_xor_sync(0xffffffffu, rv, 1);
        if ((WPG == 1 || warp % WPG == 0) && lane < RPG && row < p.n) epilogue(p, row, rv, partner, best_key);
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

// Stage geometry chosen on the host for one weight.
struct StreamPlan {
    int wpg = 0, a = 0, rpg = 0, tr = 0, stages = 0, stage_bytes = 0, w_tile_bytes = 0, smem = 0, ntiles = 0;
};

template <int BITS, typename ST, int SMODE, int A, int WPG, int RPG>
cudaError_t launch_stream_t(const StreamParams& sp, int grid, int smem, bool pdl, cudaStream_t stream) {
    auto kern = gemv_stream_kernel<BITS, ST, SMODE, A, WPG, RPG>;
    static int configured_smem = 0;
    if (smem > configured_smem) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured_smem = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kStreamThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, sp);
}

template <int BITS, typename ST, int SMODE>
cudaError_t dispatch_geom(const StreamParams& sp, const StreamPlan& pl, int grid, bool pdl, cudaStream_t s) {
#define AEXIS_STREAM_CASE(A_, W_, R_)                                                   \
    if (pl.a == A_ && pl.wpg == W_ && pl.rpg == R_)                                     \
        return launch_stream_t<BITS, ST, SMODE, A_, W_, R_>(sp, grid, pl.smem, pdl, s);
    AEXIS_STREAM_CASE(1, 1, 8)
    AEXIS_STREAM_CASE(1, 1, 4)
    AEXIS_STREAM_CASE(1, 1, 2)
    AEXIS_STREAM_CASE(2, 1, 4)
    AEXIS_STREAM_CASE(2, 1, 2)
    AEXIS_STREAM_CASE(1, 2, 4)
    AEXIS_STREAM_CASE(2, 2, 4)
    AEXIS_STREAM_CASE(1, 4, 4)
    AEXIS_STREAM_CASE(2, 4, 4)
#undef AEXIS_STREAM_CASE
    return cudaErrorNotSupported;
}

}  // namespace

// Plans the tile geometry for `w` (0 when the streaming kernel cannot take it).
static int plan_stream(const aexis_weights* w, int sm_count, StreamPlan* pl, int* smode_out, int* gshift_out) {
    const int bits = w->kind == WK_Q4 ? 4 : (w->kind == WK_Q8 ? 8 : 0);
    if (!bits) return 0;
    if (bits == 4 && w->k % 32) return 0;
    if (bits == 8 && w->k % 16) return 0;
    int smode, gshift = 0;
    if (bits == 8) smode = 0;
    else if (w->group == w->k) smode = 0;
    else if (w->group == 16) smode = 2;
    else if (w->group % 32 == 0 && ((w->group / 32) & (w->group / 32 - 1)) == 0) {
        smode = 1;
        while ((32 << gshift) < w->group) ++gshift;
    } else return 0;
    const int nchunks = w->k * bits / 128;
    int wpg = 1;
    while (wpg < 4 && 64 * wpg < nchunks) wpg *= 2;
    if (64 * wpg < nchunks) return 0;                 // K beyond two chunks per lane of 4 warps
    const int a = nchunks > 32 * wpg ? 2 : 1;
    const int rg = 8 / wpg;
    const int row_bytes = w->k * bits / 8;
    const int sdt = w->scale_dtype == AEXIS_F16 ? 2 : 4;
    const int srow_bytes = smode == 0 ? sdt : (w->k / w->group) * sdt;
    // Rows per warp per tile: 8 when there are tiles for two CTAs per SM
    // (amortises the per-tile reduction), else 4, else 2 (small N: more tiles).
    int rpg = 4;
    if (wpg == 1 && a == 1 && (w->n + rg * 8 - 1) / (rg * 8) >= 2 * sm_count) rpg = 8;
    else if (wpg == 1 && (w->n + rg * 4 - 1) / (rg * 4) < sm_count) rpg = 2;
    const int tr = rg * rpg;
    const int w_tile = tr * row_bytes;
    const int s_tile = (tr * srow_bytes + 15) & ~15;
    const int stage = (w_tile + s_tile + 127) & ~127;
    int stages = (96 * 1024) / stage;
    stages = stages < 2 ? 2 : (stages > 8 ? 8 : stages);
    const int act_floats = (w->k + 31) / 32 * 32;
    const int smem = 128 + act_floats * 4 + (2 * rg * rpg * wpg + 32) * 4 + 128 + stages * stage;
    if (smem > 200 * 1024) return 0;
    pl->wpg = wpg;
    pl->a = a;
    pl->rpg = rpg;
    pl->tr = tr;
    pl->stages = stages;
    pl->stage_bytes = stage;
    pl->w_tile_bytes = w_tile;
    pl->smem = smem;
    pl->ntiles = (w->n + tr - 1) / tr;
    *smode_out = smode;
    *gshift_out = gshift;
    return 1;
}

bool gemv_stream_supported(const aexis_weights* w) {
    StreamPlan pl;
    int sm, gs;
    return plan_stream(w, 148, &pl, &sm, &gs) != 0;
}

cudaError_t launch_gemv_stream(const GemvArgs& a, int sm_count, int* status, cudaStream_t stream) {
    const aexis_weights* w = a.w;
    StreamPlan pl;
    int smode, gshift;
    if (!plan_stream(w, sm_count, &pl, &smode, &gshift)) return cudaErrorNotSupported;
    const int bits = w->kind == WK_Q4 ? 4 : 8;
    const int sdt = w->scale_dtype == AEXIS_F16 ? 2 : 4;
    StreamParams sp = {};
    sp.W = reinterpret_cast<const uint8_t*>(w->data);
    sp.S = reinterpret_cast<const uint8_t*>(w->scales);
    sp.n = w->n;
    sp.k = w->k;
    sp.nchunks = w->k * bits / 128;
    sp.row_bytes = w->k * bits / 8;
    sp.srow_bytes = smode == 0 ? sdt : (w->k / w->group) * sdt;
    sp.gshift = gshift;
    sp.ntiles = pl.ntiles;
    sp.stages = pl.stages;
    sp.stage_bytes = pl.stage_bytes;
    sp.w_tile_bytes = pl.w_tile_bytes;
    sp.act_floats = (w->k + 31) / 32 * 32;
    sp.x = a.x;
    sp.a_dtype = a.a_dtype;
    sp.norm_gamma = a.norm_gamma;
    sp.norm_eps = a.norm_eps;
    sp.bias = a.bias;
    sp.alpha = a.alpha;
    sp.beta = a.beta;
    sp.y = a.y;
    sp.y_dtype = a.y_dtype;
    sp.epi = a.epilogue;
    sp.rope_cos = a.rope_cos;
    sp.rope_sin = a.rope_sin;
    sp.rope_map = a.rope_map;
    sp.k_cache = a.k_cache;
    sp.v_cache = a.v_cache;
    sp.head_dim = a.head_dim;
    sp.kv_cap = a.kv_cap;
    sp.rot_dim = a.rot_dim;
    sp.pos_ptr = a.pos_ptr;
    sp.argmax_key = a.argmax_key;
    sp.status = status;
    sp.zero = 0;
    // Large matrices run two CTAs per SM; smaller ones one, which leaves room
    // for the next kernel's CTA to start streaming under programmatic launch.
    const int per_sm = (pl.rpg == 8 && 2 * pl.smem <= 220 * 1024) ? 2 : 1;
    const int grid = pl.ntiles < per_sm * sm_count ? pl.ntiles : per_sm * sm_count;
    if (bits == 8) {
        if (w->scale_dtype == AEXIS_F16) return dispatch_geom<8, __half, 0>(sp, pl, grid, a.pdl, stream);
        return dispatch_geom<8, float, 0>(sp, pl, grid, a.pdl, stream);
    }
    if (w->scale_dtype == AEXIS_F16) {
        if (smode == 0) return dispatch_geom<4, __half, 0>(sp, pl, grid, a.pdl, stream);
        if (smode == 1) return dispatch_geom<4, __half, 1>(sp, pl, grid, a.pdl, stream);
        return dispatch_geom<4, __half, 2>(sp, pl, grid, a.pdl, stream);
    }
    if (smode == 0) return dispatch_geom<4, float, 0>(sp, pl, grid, a.pdl, stream);
    if (smode == 1) return dispatch_geom<4, float, 1>(sp, pl, grid, a.pdl, stream);
    return dispatch_geom<4, float, 2>(sp, pl, grid, a.pdl, stream);
}
