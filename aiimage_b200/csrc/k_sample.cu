// k_sample.cu -- token sampling on the device: Qwen35Sampler.Select
// (Samples/AIImageApplicationExample/Runtime/Scripts/Qwen35DecoderSession.cs:
// 1823-1900) for `rows` logit rows at once.
//
// The reference copies the logits to the host, applies the repetition
// penalty over its history set, takes a temperature softmax over the whole
// vocabulary (float exp, double sum), sorts every probability, keeps the top
// k, then the top-p nucleus, and draws with System.Random.NextDouble. Here
// the probabilities never leave the GPU and nothing is fully sorted:
//   1. sample_prep_kernel: each CTA takes a segment of a row, applies the
//      penalty (history bitmap), writes the penalised scores when a penalty
//      applies, and leaves (max, sum exp((s - max)/T), greedy key) per
//      segment (an online softmax per thread, merged per CTA);
//   2. the top-k kernels (k_topk.cu) give the k largest penalised scores in
//      descending order, equal values by ascending index -- the first k of
//      the reference's descending probability order;
//   3. sample_finish_kernel: one warp per row merges the segments, turns the
//      k candidates into the reference's float probabilities
//      (float)(exp((s - max)/T) / sum), cuts the nucleus, scales the caller's
//      uniform draw by the kept mass and walks the cumulative sums.
// Greedy rows (temperature <= 0) and rows whose sum is not finite and
// positive take the first maximum of the penalised scores, as the reference's
// ArgMax does.
//
// top_k <= 0 (the whole vocabulary) and top_k > 64 take sample_full_kernel
// instead of steps 2-3: one CTA per row finds the nucleus cut and the drawn
// token without sorting, by a mass-weighted radix select over the
// probabilities' float bits (positive floats order like their bit patterns):
// a question "the first position in descending-probability order whose
// prefix mass reaches X" is answered with three histogram passes (12, 12 and
// 8 bits of the key, each bin holding the count and the exact fixed-point
// mass of its elements) and one pass over the elements equal to the found
// value, in index order. The prefix masses are exact sums of the
// probabilities in 2^-62 fixed point, where the reference sums them one by
// one in fp64: the two differ by about n * 2^-53 of the kept mass, so a draw
// closer than that to a cumulative boundary may pick the neighbouring token.
#include "aexis_internal.h"

#include <cfloat>

namespace {

constexpr int kSpThreads = 256;

struct SamplePartial {
    unsigned long long key;  // greedy key of the segment's first maximum
    double sum;              // sum of exp((s - m)/T) over the segment
    float m;                 // segment maximum (-inf when none)
    float pad;
};

__device__ __forceinline__ float penalise(float s, const uint32_t* hist_row, int i, float pen) {
    if (hist_row && ((hist_row[i >> 5] >> (i & 31)) & 1u)) s = s < 0.0f ? s * pen : s / pen;
    return s;
}

// Merge of two online-softmax states (m, s): the sum relative to the larger
// maximum. A NaN sum (a NaN score was seen) is sticky; otherwise a state with
// no finite maximum contributes nothing.
__device__ __forceinline__ void softmax_merge(float& m, double& s, float m2, double s2, float inv_t) {
    if (s != s) return;
    if (s2 != s2) { s = s2; return; }
    if (m2 == -INFINITY) return;
    if (m == -INFINITY) { m = m2; s = s2; return; }
    if (m2 > m) {
        s = s * (double)expf((m - m2) * inv_t) + s2;
        m = m2;
    } else {
        s = s + s2 * (double)expf((m2 - m) * inv_t);
    }
}

// Running state of the prep pass over a thread's scores, in index order:
// the first maximum (strict >, as the reference's ArgMax; NaN and -inf never
// become it) and the online softmax sum relative to that maximum. A quad of
// scores is summed in fp32 and folded into the fp64 sum once.
struct PrepState {
    float m = -INFINITY;  // running maximum
    int im = -1;          // its first index
    double s = 0.0;       // sum of exp((v - m)/T) over the scores seen (NaN once a NaN was seen)
    bool nan = false;
    template <int N>
    __device__ __forceinline__ void add(const float (&e)[N], int i, bool sample, float inv_t) {
        const float m_old = m;
#pragma unroll
        for (int c = 0; c < N; ++c) {
            nan |= e[c] != e[c];
            if (e[c] > m) { m = e[c]; im = i + c; }
        }
        if (!sample || m == -INFINITY) return;
        if (m > m_old) s = m_old == -INFINITY ? 0.0 : s * (double)expf((m_old - m) * inv_t);
        float q = 0.0f;
#pragma unroll
        for (int c = 0; c < N; ++c) q += expf((e[c] - m) * inv_t);
        s += (double)q;
    }
    __device__ __forceinline__ unsigned long long key() const {
        return im < 0 ? 0ull : aexis_argmax_key(m, im);
    }
};

// Segment [lo, hi) of one row. Rows whose base and stride allow it are read
// as float4 (`vec`), four loads in flight per thread before any arithmetic,
// so the pass runs at HBM rate rather than at one load latency per element.
__global__ void __launch_bounds__(kSpThreads) sample_prep_kernel(const float* __restrict__ logits, int width, int ld,
                                                                 const uint32_t* __restrict__ history, int hist_words,
                                                                 float pen, float temperature, int seg_len, bool vec,
                                                                 float* __restrict__ scores, int ld_scores,
                                                                 SamplePartial* __restrict__ parts) {
    const int row = blockIdx.y, seg = blockIdx.x;
    const int lo = seg * seg_len, hi = min(width, lo + seg_len);
    const float* x = logits + (long long)row * ld;
    const uint32_t* hrow = history ? history + (long long)row * hist_words : nullptr;
    float* srow = scores ? scores + (long long)row * ld_scores : nullptr;
    const bool sample = temperature > 0.0f;
    const float inv_t = sample ? 1.0f / temperature : 0.0f;
    PrepState st;
    int i0 = lo;
    if (vec) {
        // lo is a multiple of 4 (seg_len is); whole quads up to hi.
        const int q_lo = lo >> 2, q_hi = hi >> 2;
        const float4* x4 = reinterpret_cast<const float4*>(x);
        constexpr int U = 4;
        for (int q = q_lo + threadIdx.x; q < q_hi; q += U * kSpThreads) {
            float4 v[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int qq = q + u * kSpThreads;
                v[u] = qq < q_hi ? __ldcs(x4 + qq) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int qq = q + u * kSpThreads;
                if (qq >= q_hi) break;
                const int i = qq * 4;
                float e[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
                if (hrow) {
                    const uint32_t w = (hrow[i >> 5] >> (i & 31)) & 15u;
                    if (w) {  // rare: the history is sparse
#pragma unroll
                        for (int c = 0; c < 4; ++c)
                            if ((w >> c) & 1u) e[c] = e[c] < 0.0f ? e[c] * pen : e[c] / pen;
                    }
                }
                if (srow) *reinterpret_cast<float4*>(srow + i) = make_float4(e[0], e[1], e[2], e[3]);
                st.add(e, i, sample, inv_t);
            }
        }
        i0 = max(lo, q_hi * 4);   // a segment past the row's end (hi <= lo) reads nothing
    }
    for (int i = i0 + threadIdx.x; i < hi; i += kSpThreads) {
        const float v[1] = {penalise(x[i], hrow, i, pen)};
        if (srow) srow[i] = v[0];
        st.add(v, i, sample, inv_t);
    }
    unsigned long long key = st.key();
    // ArgMax keeps index 0 when nothing is greater than its score, a NaN or
    // -inf included: the key of element 0 itself covers that.
    if (lo == 0 && threadIdx.x == 0 && hi > 0) {
        const unsigned long long k0 = aexis_argmax_key(penalise(x[0], hrow, 0, pen), 0);
        key = k0 > key ? k0 : key;
    }
    float m = st.m;
    double s = st.s;
    if (st.nan) s = __longlong_as_double(0x7ff8000000000000ll);  // exp(NaN) poisons the reference's sum
    // Block merge: warps by shuffles, then warp 0 over the warps' states.
    __shared__ SamplePartial red[kSpThreads / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const double s2 = __shfl_xor_sync(0xffffffffu, s, o);
        key = k2 > key ? k2 : key;
        softmax_merge(m, s, m2, s2, inv_t);
    }
    if (lane == 0) red[warp] = SamplePartial{key, s, m, 0.0f};
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < kSpThreads / 32; ++w) {
            key = red[w].key > key ? red[w].key : key;
            softmax_merge(m, s, red[w].m, red[w].sum, inv_t);
        }
        parts[(long long)row * gridDim.x + seg] = SamplePartial{key, s, m, 0.0f};
    }
}

__global__ void sample_finish_kernel(const SamplePartial* __restrict__ parts, int segs, float temperature, int top_k,
                                     float top_p, int width, const float* __restrict__ cand_vals,
                                     const int32_t* __restrict__ cand_idx, int cand_ld,
                                     const double* __restrict__ uniforms, int32_t* __restrict__ out) {
    const int row = blockIdx.x, lane = threadIdx.x;
    const bool sample = temperature > 0.0f;
    const float inv_t = sample ? 1.0f / temperature : 0.0f;
    const int n_cand = sample ? (top_k < width ? top_k : width) : 0;
    // Candidates and the draw are loaded first, in parallel with the merge.
    const float* cv = cand_vals + (long long)row * cand_ld;
    const int32_t* ci = cand_idx + (long long)row * cand_ld;
    const float c_v0 = lane < n_cand ? cv[lane] : 0.0f, c_v1 = lane + 32 < n_cand ? cv[lane + 32] : 0.0f;
    const int c_i0 = lane < n_cand ? ci[lane] : 0, c_i1 = lane + 32 < n_cand ? ci[lane + 32] : 0;
    const double u = sample && lane == 0 ? uniforms[row] : 0.0;
    unsigned long long key = 0ull;
    float m = -INFINITY;
    double s = 0.0;
    for (int i = lane; i < segs; i += 32) {
        const SamplePartial p = parts[(long long)row * segs + i];
        key = p.key > key ? p.key : key;
        softmax_merge(m, s, p.m, p.sum, inv_t);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) {
        const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
        const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
        const double s2 = __shfl_xor_sync(0xffffffffu, s, o);
        key = k2 > key ? k2 : key;
        softmax_merge(m, s, m2, s2, inv_t);
    }
    // s is a NaN when any penalised score is a NaN (exp(NaN) poisons the sum
    // as in the reference); no finite maximum leaves s = 0.
    if (!sample || !(s > 0.0 && s <= DBL_MAX)) {
        if (lane == 0) out[row] = aexis_argmax_index(key);
        return;
    }
    int keep = n_cand;
    // The candidates' probabilities in parallel (one double division each);
    // the cumulative sums below stay sequential, in the reference's order.
    __shared__ float prob[64];
    __shared__ int32_t ix[64];
    if (lane < keep) {
        prob[lane] = (float)((double)expf((c_v0 - m) / temperature) / s);
        ix[lane] = c_i0;
    }
    if (lane + 32 < keep) {
        prob[lane + 32] = (float)((double)expf((c_v1 - m) / temperature) / s);
        ix[lane + 32] = c_i1;
    }
    __syncwarp();
    if (lane != 0) return;
    if (top_p < 1.0f) {
        double cumulative = 0.0;
        int nucleus = 0;
        while (nucleus < keep) {
            cumulative += prob[nucleus++];
            if (cumulative >= top_p) break;
        }
        keep = nucleus > 1 ? nucleus : 1;
    }
    double kept = 0.0;
    for (int j = 0; j < keep; ++j) kept += prob[j];
    if (!(kept > 0.0 && kept <= DBL_MAX)) {
        out[row] = aexis_argmax_index(key);
        return;
    }
    const double draw = u * kept;
    double cursor = 0.0;
    for (int j = 0; j < keep; ++j) {
        cursor += prob[j];
        if (draw <= cursor) {
            out[row] = ix[j];
            return;
        }
    }
    out[row] = ix[keep - 1];
}

// ---------------------------------------------------------------------------
// Whole-vocabulary selection (top_k <= 0 or > 64).
constexpr int kFullThreads = 1024;
constexpr int kFullBins = 4096;

struct FullShared {
    unsigned long long l1_mass[kFullBins];  // level 1 (key bits 31..20) of the whole row, kept for every query
    unsigned int l1_cnt[kFullBins];
    unsigned long long mass[kFullBins];     // levels 2 and 3 of the current query
    unsigned int cnt[kFullBins];
    unsigned long long wm[32];              // per-warp scan partials
    unsigned int wc[32];
    int bin;                                // bin found by the current level (-1: none)
    unsigned long long above_m;             // mass and count of the keys above the found ones
    unsigned int above_c;
    int idx;                                // index found by the tie pass
    unsigned long long total;               // mass of the whole row
    float m;
    double sum;
    unsigned long long key;
};

// 2^62: probabilities in [0, 1] as fixed point (a float's 24-bit mantissa
// times 2^62 is exact in double; the conversion truncates below 2^-62).
__device__ __forceinline__ unsigned long long prob_fx(float p) {
    return (unsigned long long)((double)p * 4611686018427387904.0);
}

// The reference's probability of one score: (float)(exp((s - max)/T) / sum).
__device__ __forceinline__ float full_prob(float sc, float m, float temperature, double sum) {
    return (float)((double)expf((sc - m) / temperature) / sum);
}

// Adds (fx, 1) to bin `bin` (>= 0; -1 adds nothing). When the whole warp
// shares one bin (a flat distribution) it adds once, reduced by shuffles;
// otherwise lane by lane.
__device__ __forceinline__ void full_hist_add(unsigned long long* mass, unsigned int* cnt, int bin,
                                              unsigned long long fx) {
    const int b0 = __shfl_sync(0xffffffffu, bin, 0);
    if (__all_sync(0xffffffffu, bin == b0)) {
        if (b0 < 0) return;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) fx += __shfl_xor_sync(0xffffffffu, fx, o);
        if ((threadIdx.x & 31) == 0) {
            atomicAdd(&mass[b0], fx);
            atomicAdd(&cnt[b0], 32u);
        }
    } else if (bin >= 0) {
        atomicAdd(&mass[bin], fx);
        atomicAdd(&cnt[bin], 1u);
    }
}

struct Found {
    int ok;                    // 0: the target exceeds the row's mass (by_mass) or count
    int pos;                   // 1-based position in descending-probability order
    int idx;                   // token at that position
    unsigned long long mass;   // prefix mass up to and including it
};

// Scans the histogram `nb` bins (mass/cnt) from the top for the bin where the
// prefix (starting at above_m / above_c) reaches `target`; sets sh.bin (-1
// when none), sh.above_m, sh.above_c. Every thread calls it.
__device__ void full_scan(const unsigned long long* mass, const unsigned int* cnt, int nb, unsigned long long above_m,
                          unsigned int above_c, unsigned long long target, bool by_mass, FullShared& sh) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int per = nb / kFullThreads > 0 ? nb / kFullThreads : 1;
    unsigned long long tm = 0;
    unsigned int tc = 0;
    const int b0 = tid * per;
    if (b0 < nb)
        for (int b = b0; b < b0 + per; ++b) {
            tm += mass[b];
            tc += cnt[b];
        }
    unsigned long long sm = tm;  // inclusive suffix over the lanes >= this one
    unsigned int sc = tc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const unsigned long long vm = __shfl_down_sync(0xffffffffu, sm, o);
        const unsigned int vc = __shfl_down_sync(0xffffffffu, sc, o);
        if (lane + o < 32) {
            sm += vm;
            sc += vc;
        }
    }
    __syncthreads();  // the previous user of sh.wm / sh.bin is done
    if (lane == 0) {
        sh.wm[warp] = sm;
        sh.wc[warp] = sc;
    }
    if (tid == 0) sh.bin = -1;
    __syncthreads();
    unsigned long long later_m = 0;  // the bins of later warps lie above this thread's
    unsigned int later_c = 0;
    for (int w = warp + 1; w < 32; ++w) {
        later_m += sh.wm[w];
        later_c += sh.wc[w];
    }
    unsigned long long run_m = above_m + later_m + (sm - tm);
    unsigned int run_c = above_c + later_c + (sc - tc);
    if (b0 < nb)
        for (int b = b0 + per - 1; b >= b0; --b) {
            const unsigned long long bm = mass[b];
            const unsigned int bc = cnt[b];
            const bool hit = by_mass ? (run_m < target && target <= run_m + bm)
                                     : (run_c < target && target <= run_c + bc);
            if (hit) {
                sh.bin = b;
                sh.above_m = run_m;
                sh.above_c = run_c;
            }
            run_m += bm;
            run_c += bc;
        }
    __syncthreads();
}

// The first position whose prefix mass (by_mass) or count (otherwise)
// reaches `target` (>= 1), over the row's probabilities in descending order,
// equal probabilities by ascending index. probs: the row's probabilities
// (written by the first pass); level 1 comes from sh.l1_*. Every thread calls it.
__device__ Found full_find(const float* __restrict__ probs, int width, unsigned long long target, bool by_mass,
                           FullShared& sh) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    full_scan(sh.l1_mass, sh.l1_cnt, kFullBins, 0, 0, target, by_mass, sh);
    if (sh.bin < 0) return Found{0, 0, 0, 0};
    unsigned int prefix = (unsigned)sh.bin << 20, pmask = 0xFFFu << 20;
    unsigned long long above_m = sh.above_m;
    unsigned int above_c = sh.above_c;
    const unsigned int* pbits = reinterpret_cast<const unsigned int*>(probs);
    for (int lv = 1; lv < 3; ++lv) {
        const int nb = lv == 1 ? 4096 : 256, sft = lv == 1 ? 8 : 0;
        for (int b = tid; b < nb; b += kFullThreads) {
            sh.mass[b] = 0;
            sh.cnt[b] = 0;
        }
        __syncthreads();
        for (int base = 0; base < width; base += kFullThreads) {
            const int i = base + tid;
            int bin = -1;
            unsigned long long fx = 0;
            if (i < width) {
                const unsigned int key = pbits[i];
                if ((key & pmask) == prefix) {
                    bin = (int)((key >> sft) & (unsigned)(nb - 1));
                    fx = prob_fx(__uint_as_float(key));
                }
            }
            full_hist_add(sh.mass, sh.cnt, bin, fx);
        }
        __syncthreads();
        full_scan(sh.mass, sh.cnt, nb, above_m, above_c, target, by_mass, sh);
        if (sh.bin < 0) return Found{0, 0, 0, 0};  // not reached: level 1 found the target's bin
        prefix |= (unsigned)sh.bin << sft;
        pmask |= (unsigned)(nb - 1) << sft;
        above_m = sh.above_m;
        above_c = sh.above_c;
    }
    // Every element left has the key `prefix`; the c-th of them by index is the answer.
    const unsigned long long tau_fx = prob_fx(__uint_as_float(prefix));
    unsigned int c;
    if (by_mass) {
        const unsigned long long need = target - above_m;  // > 0
        c = (unsigned int)((need + tau_fx - 1) / tau_fx);
    } else {
        c = (unsigned int)(target - above_c);
    }
    unsigned int run = 0;
    for (int base = 0; base < width; base += kFullThreads) {
        const int i = base + tid;
        const bool match = i < width && pbits[i] == prefix;
        const int tile = __syncthreads_count(match);
        if (run + (unsigned)tile >= c) {
            const unsigned bal = __ballot_sync(0xffffffffu, match);
            if (lane == 0) sh.wc[warp] = (unsigned)__popc(bal);
            __syncthreads();
            unsigned int before = run;
            for (int w = 0; w < warp; ++w) before += sh.wc[w];
            const unsigned int mine = before + (unsigned)__popc(bal & ((1u << lane) - 1u)) + 1u;
            if (match && mine == c) sh.idx = i;
            __syncthreads();
            return Found{1, (int)(above_c + c), sh.idx, above_m + (unsigned long long)c * tau_fx};
        }
        run += (unsigned)tile;
    }
    return Found{0, 0, 0, 0};  // not reached: the bin held at least c elements
}

__global__ void __launch_bounds__(kFullThreads, 1)
sample_full_kernel(const SamplePartial* __restrict__ parts, int segs, const float* __restrict__ scores, int ld,
                   float temperature, int top_k, float top_p, int width, const double* __restrict__ uniforms,
                   float* __restrict__ probs_all, int ld_p, int32_t* __restrict__ out) {
    extern __shared__ __align__(16) unsigned char full_smem[];
    FullShared& sh = *reinterpret_cast<FullShared*>(full_smem);
    const int row = blockIdx.x, tid = threadIdx.x;
    const bool sample = temperature > 0.0f;
    const float inv_t = sample ? 1.0f / temperature : 0.0f;
    if (tid < 32) {
        unsigned long long key = 0ull;
        float m = -INFINITY;
        double s = 0.0;
        for (int i = tid; i < segs; i += 32) {
            const SamplePartial p = parts[(long long)row * segs + i];
            key = p.key > key ? p.key : key;
            softmax_merge(m, s, p.m, p.sum, inv_t);
        }
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const unsigned long long k2 = __shfl_xor_sync(0xffffffffu, key, o);
            const float m2 = __shfl_xor_sync(0xffffffffu, m, o);
            const double s2 = __shfl_xor_sync(0xffffffffu, s, o);
            key = k2 > key ? k2 : key;
            softmax_merge(m, s, m2, s2, inv_t);
        }
        if (tid == 0) {
            sh.m = m;
            sh.sum = s;
            sh.key = key;
        }
    }
    for (int b = tid; b < kFullBins; b += kFullThreads) {
        sh.l1_mass[b] = 0;
        sh.l1_cnt[b] = 0;
    }
    __syncthreads();
    const float m = sh.m;
    const double sum = sh.sum;
    if (!sample || !(sum > 0.0 && sum <= DBL_MAX)) {
        if (tid == 0) out[row] = aexis_argmax_index(sh.key);
        return;
    }
    // One pass over the scores: the probabilities (kept for the later
    // passes) and the level-1 histogram every query starts from.
    const float* srow = scores + (long long)row * ld;
    float* probs = probs_all + (long long)row * ld_p;
    for (int base = 0; base < width; base += kFullThreads) {
        const int i = base + tid;
        int bin = -1;
        unsigned long long fx = 0;
        if (i < width) {
            const float pr = full_prob(srow[i], m, temperature, sum);
            probs[i] = pr;
            bin = (int)(__float_as_uint(pr) >> 20);
            fx = prob_fx(pr);
        }
        full_hist_add(sh.l1_mass, sh.l1_cnt, bin, fx);
    }
    __syncthreads();
    if (tid == 0) {
        unsigned long long t = 0;
        for (int b = 0; b < kFullBins; ++b) t += sh.l1_mass[b];
        sh.total = t;
    }
    __syncthreads();
    // keep = min(top_k, V) (all when top_k <= 0); kept = its prefix mass.
    int keep = width, keep_idx = -1;
    unsigned long long kept = sh.total;
    if (top_k > 0 && top_k < width) {
        const Found f = full_find(probs, width, (unsigned long long)top_k, false, sh);
        keep = f.pos;
        keep_idx = f.idx;
        kept = f.mass;
    }
    if (top_p < 1.0f) {
        // The nucleus: the first position whose cumulative reaches top_p, if within keep.
        const double tp = top_p > 0.0f ? (double)top_p : 0.0;
        unsigned long long target = (unsigned long long)ceil(tp * 4611686018427387904.0);
        if (target < 1) target = 1;
        const Found f = full_find(probs, width, target, true, sh);
        if (f.ok && f.pos <= keep) {
            keep = f.pos;
            keep_idx = f.idx;
            kept = f.mass;
        }
    }
    // The draw: the first position whose cumulative reaches u * kept.
    unsigned long long x = (unsigned long long)(uniforms[row] * (double)kept);
    if (x < 1) x = 1;
    if (x > kept) x = kept;
    const Found f = full_find(probs, width, x, true, sh);
    if (tid == 0) {
        int pick = f.ok ? f.idx : -1;
        if (!f.ok || f.pos > keep) pick = keep_idx >= 0 ? keep_idx : f.idx;
        out[row] = pick >= 0 ? pick : aexis_argmax_index(sh.key);
    }
}

__global__ void history_add_kernel(uint32_t* history, int rows, int hist_words, int width, const int32_t* tokens) {
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const int t = tokens[r];
    if (t >= 0 && t < width) atomicOr(history + (long long)r * hist_words + (t >> 5), 1u << (t & 31));
}

}  // namespace

// Segments per row: at least 1024 scores each, and about as many CTAs in
// total as fit on the GPU at once (8 of 256 threads per SM), so that enough
// loads are in flight to keep HBM busy.
int sample_segments(int rows, int width, int sm_count) {
    const int by_width = (width + 1023) / 1024;
    const int by_sms = (8 * sm_count) / rows;
    int segs = by_width < by_sms ? by_width : by_sms;
    return segs < 1 ? 1 : segs;
}

size_t sample_scratch_bytes(int rows, int width, int sm_count, bool scores, bool full) {
    const size_t ld_s = (size_t)((width + 3) & ~3);
    size_t b = (size_t)rows * sample_segments(rows, width, sm_count) * sizeof(SamplePartial);
    b = (b + 255) & ~(size_t)255;
    b += (size_t)rows * 64 * (sizeof(float) + sizeof(int32_t));
    b = (b + 255) & ~(size_t)255;
    if (scores) b += (size_t)rows * ld_s * sizeof(float);
    b = (b + 255) & ~(size_t)255;
    if (full) b += (size_t)rows * ld_s * sizeof(float);
    return b;
}

cudaError_t launch_sample(const float* logits, int rows, int width, int ld, const uint32_t* history, float pen,
                          float temperature, int top_k, float top_p, const double* uniforms, int32_t* out,
                          void* scratch, void* topk_scratch, int sm_count, cudaStream_t s) {
    const bool sample = temperature > 0.0f;
    const bool penalised = history != nullptr && pen != 1.0f;
    const int segs = sample_segments(rows, width, sm_count);
    const int seg_len = ((width + segs - 1) / segs + 3) & ~3;
    const bool vec = (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && (ld & 3) == 0;
    char* p = reinterpret_cast<char*>(scratch);
    SamplePartial* parts = reinterpret_cast<SamplePartial*>(p);
    size_t off = ((size_t)rows * segs * sizeof(SamplePartial) + 255) & ~(size_t)255;
    float* cand_vals = reinterpret_cast<float*>(p + off);
    int32_t* cand_idx = reinterpret_cast<int32_t*>(cand_vals + (size_t)rows * 64);
    off = (off + (size_t)rows * 64 * 8 + 255) & ~(size_t)255;
    const int ld_s = (width + 3) & ~3;
    float* scores = penalised ? reinterpret_cast<float*>(p + off) : nullptr;
    const int hist_words = (width + 31) / 32;
    sample_prep_kernel<<<dim3(segs, rows), kSpThreads, 0, s>>>(logits, width, ld, penalised ? history : nullptr,
                                                               hist_words, pen, temperature, seg_len, vec, scores,
                                                               ld_s, parts);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    if (sample && (top_k <= 0 || top_k > 64)) {
        // The whole vocabulary (or more candidates than the top-k kernels keep).
        const size_t smem = sizeof(FullShared);
        e = cudaFuncSetAttribute(sample_full_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
        size_t poff = ((size_t)rows * segs * sizeof(SamplePartial) + 255) & ~(size_t)255;
        poff = (poff + (size_t)rows * 64 * 8 + 255) & ~(size_t)255;
        if (penalised) poff += (size_t)rows * ld_s * sizeof(float);
        poff = (poff + 255) & ~(size_t)255;
        float* probs = reinterpret_cast<float*>(p + poff);
        sample_full_kernel<<<rows, kFullThreads, smem, s>>>(parts, segs, penalised ? scores : logits,
                                                            penalised ? ld_s : ld, temperature, top_k, top_p, width,
                                                            uniforms, probs, ld_s, out);
        return cudaGetLastError();
    }
    const int k = sample ? (top_k < width ? top_k : width) : 1;
    if (sample) {
        e = launch_topk(penalised ? scores : logits, rows, width, penalised ? ld_s : ld, k, cand_vals, cand_idx,
                        topk_scratch, sm_count, s);
        if (e != cudaSuccess) return e;
    }
    sample_finish_kernel<<<rows, 32, 0, s>>>(parts, segs, temperature, top_k, top_p, width, cand_vals, cand_idx, k,
                                              uniforms, out);
    return cudaGetLastError();
}

cudaError_t launch_history_add(uint32_t* history, int rows, int width, const int32_t* tokens, cudaStream_t s) {
    history_add_kernel<<<(rows + 127) / 128, 128, 0, s>>>(history, rows, (width + 31) / 32, width, tokens);
    return cudaGetLastError();
}
