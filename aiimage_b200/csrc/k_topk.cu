// k_topk.cu -- per-row top-k of a logit matrix by radix selection.
//
// Order: larger value first; equal values by ascending index (the argmax tie
// rule of AexisArgMaxPack4LinearMat, HLSL Pack4Matmul:645-686, extended to k
// entries); NaN never selected; -0 counts as +0. Every element has a unique
// 64-bit key (orderable value << 32 | ~index), so "the k largest keys" is the
// exact answer.
//
// One CTA per row. Histograms of the 32-bit order-preserving value (11, 11,
// then 10 bits) find the bin that holds the k-th largest value, refining only
// while that bin is too large for the candidate buffer. One more pass collects
// every element at or above the bin into shared memory, where a bitonic sort
// on the keys yields the answer. When a plateau of equal values is larger
// than the buffer, the values strictly above it are collected and the rest is
// filled with the plateau's lowest indices by an index-ordered scan.
#include "aexis_internal.h"

namespace {

constexpr int kThreads = 512;
constexpr int kBins = 2048;
constexpr int kCap = 2048;  // candidate buffer (keys)

__device__ __forceinline__ bool ord_of(float v, unsigned int& o) {
    if (v != v) return false;
    o = aexis_orderable(v == 0.0f ? 0.0f : v);
    return true;
}

__device__ __forceinline__ unsigned long long make_key(unsigned int o, int i) {
    return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned int)i);
}

__global__ void __launch_bounds__(kThreads) topk_radix_kernel(const float* logits, int width, int ld, int k,
                                                              float* vals, int32_t* idx) {
    __shared__ unsigned int hist[kBins];
    __shared__ unsigned long long cand[kCap];
    __shared__ unsigned int s_sel[4];   // bin, count above, bin count, flag
    __shared__ unsigned int s_ncand;
    __shared__ unsigned int warp_sum[kThreads / 32];
    const int row = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const float* x = logits + (long long)row * ld;

    unsigned int prefix = 0, pmask = 0;
    unsigned int need = (unsigned int)k;   // still to select below the fixed prefix
    unsigned int above = 0;                // selected so far strictly above the prefix
    unsigned int threshold = 0;            // collect o >= threshold
    bool plateau = false;
    const int shifts[3] = {21, 10, 0};
    const unsigned int dmask[3] = {0x7FFu, 0x7FFu, 0x3FFu};
    for (int lvl = 0; lvl < 3; ++lvl) {
        const int sh = shifts[lvl];
        for (int b = t; b < kBins; b += kThreads) hist[b] = 0u;
        __syncthreads();
        // Warp-uniform trip count; lanes that fall in the same bin add once.
        for (int start = 0; start < width; start += kThreads) {
            const int i = start + t;
            unsigned int o = 0;
            const bool in = i < width && ord_of(x[i], o) && (o & pmask) == prefix;
            const unsigned int bin = in ? (o >> sh) & dmask[lvl] : 0xFFFFFFFFu;
            const unsigned int peers = __match_any_sync(0xffffffffu, bin);
            if (in && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], (unsigned int)__popc(peers));
        }
        __syncthreads();
        // Suffix scan from the top bin: warp 0 finds the bin b with
        // count_above(b) < need <= count_above(b) + hist[b].
        if (warp == 0) {
            const int per = kBins / 32;
            unsigned int part = 0;
            for (int j = 0; j < per; ++j) part += hist[lane * per + j];
            // inclusive suffix sum over lanes (higher lanes = higher bins)
            unsigned int suf = part;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const unsigned int v = __shfl_down_sync(0xffffffffu, suf, o);
                if (lane + o < 32) suf += v;
            }
            const unsigned int above_lane = suf - part;  // bins of higher lanes
            const bool mine = above_lane < need && need <= suf;
            const unsigned int who = __ballot_sync(0xffffffffu, mine);
            if (who) {
                const int src = __ffs(who) - 1;
                if (lane == src) {
                    unsigned int c = above_lane;
                    for (int j = per - 1; j >= 0; --j) {
                        const unsigned int h = hist[lane * per + j];
                        if (c + h >= need) {
                            s_sel[0] = (unsigned int)(lane * per + j);
                            s_sel[1] = c;
                            s_sel[2] = h;
                            break;
                        }
                        c += h;
                    }
                    s_sel[3] = 1u;
                }
            } else if (lane == 0) {
                s_sel[3] = 0u;  // fewer than k valid values in this prefix
                s_sel[1] = suf;
            }
        }
        __syncthreads();
        if (s_sel[3] == 0u) {
            // Fewer than k selectable values: take all of them.
            threshold = prefix;
            above += s_sel[1];
            break;
        }
        const unsigned int b = s_sel[0], c_above = s_sel[1], h = s_sel[2];
        const unsigned int cut = prefix | (b << sh);
        if (above + c_above + h <= (unsigned int)kCap) {
            threshold = cut;
            break;
        }
        if (lvl == 2) {  // a plateau of equal values larger than the buffer
            threshold = cut;
            plateau = true;
            above += c_above;
            need -= c_above;
            break;
        }
        above += c_above;
        need -= c_above;
        prefix = cut;
        pmask |= dmask[lvl] << sh;
        __syncthreads();
    }
    __syncthreads();

    // Collect: every value at or above the threshold (strictly above for a plateau).
    if (t == 0) s_ncand = 0u;
    __syncthreads();
    for (int i = t; i < width; i += kThreads) {
        unsigned int o;
        if (ord_of(x[i], o) && (plateau ? o > threshold : o >= threshold)) {
            const unsigned int slot = atomicAdd(&s_ncand, 1u);
            if (slot < (unsigned int)kCap) cand[slot] = make_key(o, i);
        }
    }
    __syncthreads();
    if (plateau) {
        // Fill with the lowest indices equal to the threshold, in index order.
        unsigned int base_n = s_ncand < (unsigned int)kCap ? s_ncand : (unsigned int)kCap;
        unsigned int remaining = need;
        for (int start = 0; start < width && remaining > 0; start += kThreads) {
            const int i = start + t;
            unsigned int o = 0;
            const bool eq = i < width && ord_of(x[i], o) && o == threshold;
            const unsigned int bal = __ballot_sync(0xffffffffu, eq);
            if (lane == 0) warp_sum[warp] = __popc(bal);
            __syncthreads();
            unsigned int before = 0, total = 0;
            for (int w = 0; w < kThreads / 32; ++w) {
                if (w < warp) before += warp_sum[w];
                total += warp_sum[w];
            }
            const unsigned int rank = before + __popc(bal & ((1u << lane) - 1u));
            if (eq && rank < remaining && base_n + rank < (unsigned int)kCap) cand[base_n + rank] = make_key(o, i);
            const unsigned int took = total < remaining ? total : remaining;
            base_n += took;
            remaining -= took;
            __syncthreads();
        }
        if (t == 0) s_ncand = base_n;
        __syncthreads();
    }
    unsigned int n = s_ncand < (unsigned int)kCap ? s_ncand : (unsigned int)kCap;
    // Bitonic sort, descending, over the next power of two (padding keys 0).
    unsigned int np = 1;
    while (np < n) np <<= 1;
    for (unsigned int i = n + t; i < np; i += kThreads) cand[i] = 0ull;
    __syncthreads();
    for (unsigned int size = 2; size <= np; size <<= 1) {
        for (unsigned int stride = size >> 1; stride > 0; stride >>= 1) {
            for (unsigned int i = t; i < np; i += kThreads) {
                const unsigned int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long a = cand[i], b2 = cand[j];
                    if (desc ? (a < b2) : (a > b2)) {
                        cand[i] = b2;
                        cand[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }
    for (int j = t; j < k; j += kThreads) {
        float* vo = vals + (long long)row * k + j;
        int32_t* io = idx + (long long)row * k + j;
        if ((unsigned int)j < n && cand[j] != 0ull) {
            const unsigned long long key = cand[j];
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
    topk_radix_kernel<<<rows, kThreads, 0, s>>>(logits, width, ld, k, vals, idx);
    return cudaGetLastError();
}
