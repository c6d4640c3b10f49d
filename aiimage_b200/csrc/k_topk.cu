// k_topk.cu -- per-row top-k of a logit matrix.
//
// Order: larger value first; equal values by ascending index (the argmax tie
// rule of AexisArgMaxPack4LinearMat, HLSL Pack4Matmul:645-686, extended to k
// entries); NaN never selected; -0 counts as +0. Every element has a unique
// 64-bit key (orderable value << 32 | ~index), so "the k largest keys" is the
// exact answer; rows with fewer than k selectable values are padded with
// (-inf, -1).
//
// Wide rows (width >= kTkMinSampledWidth, 16-byte aligned rows) take two
// kernels that read the matrix once between them:
//   topk_sample_kernel  one CTA per row: the row's threshold t from 8192
//                       samples (32 chunks of 256 contiguous elements spread
//                       evenly over the row), the value of rank r among the
//                       256 threads' sample maxima, r chosen so that about
//                       4.5k elements of the row are >= t.
//   topk_filter_kernel  every CTA streams an equal contiguous share of the
//                       rows x width matrix with 128-bit loads, four values
//                       compared per warp vote (about two instructions per
//                       element); elements >= t are appended to the row's
//                       candidate list through per-warp shared buffers, one
//                       atomicAdd per flush. The CTA that finishes a row's
//                       last segment selects the row. With k <= n <= kTkCap
//                       candidates, the k largest candidate keys are the
//                       answer: at least k elements are >= t, so every
//                       element left out (< t) ranks below k of them.
//                       Otherwise the sample misjudged the row (plateaus,
//                       NaNs, values placed between the samples) and the CTA
//                       computes the row exactly.
// Selection: each warp sorts 64-key chunks in registers (bitonic network
// over shuffles) into a running top 64; three pairwise merges across warps.
// Narrow or unaligned rows take topk_exact_kernel: one CTA per row, per-warp
// candidate buffers whose thresholds rise as they fill.
#include "aexis_internal.h"

namespace {

constexpr int kTkWarps = 8;
constexpr int kTkThreads = kTkWarps * 32;
constexpr int kTkBuf = 256;             // candidate keys per warp
constexpr int kTkMaxK = 64;
constexpr int kTkChunks = 32;           // sample chunks per row
constexpr int kTkSamples = kTkChunks * kTkThreads;  // 8192 threshold samples per row
constexpr int kTkMaxRank = 64;          // largest rank used as threshold
constexpr int kTkCap = kTkWarps * kTkBuf;  // candidate keys kept per row (2048)
constexpr int kTkMinSampledWidth = 32768;

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

// Bounded waits (the peer exchange's flags): about a second of SM clock,
// then AEXIS_E_TIMEOUT in the context status word.
constexpr long long kTkWaitLimitCycles = 2000000000LL;
__device__ __forceinline__ void tk_report_timeout(int* status) {
    if (status) atomicCAS(status, 0, (int)AEXIS_E_TIMEOUT);
}

__device__ __forceinline__ unsigned int tk_key32(float v) {
    return v != v ? 0u : aexis_orderable(v == 0.0f ? 0.0f : v);  // NaN below everything
}

__device__ __forceinline__ float tk_value32(unsigned int hi) {
    return __uint_as_float((hi & 0x80000000u) ? (hi & 0x7FFFFFFFu) : ~hi);
}

__device__ __forceinline__ unsigned long long tk_key(float v, int i) {
    return ((unsigned long long)tk_key32(v) << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned int)i);
}

// 64 keys held two per lane (element h * 32 + lane in a[h]) sorted
// descending in registers (bitonic network; partners by shuffle).
__device__ __forceinline__ void warp_sort64_desc(unsigned long long (&a)[2], int lane) {
#pragma unroll
    for (int size = 2; size <= 64; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride == 32) {  // size 64: the lane's own pair, larger first
                const unsigned long long x = a[0], y = a[1];
                a[0] = x > y ? x : y;
                a[1] = x > y ? y : x;
            } else {
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const int i = h * 32 + lane;
                    const unsigned long long p = __shfl_xor_sync(0xffffffffu, a[h], stride);
                    const bool keep_max = ((i & stride) == 0) == ((i & size) == 0);
                    a[h] = keep_max ? (a[h] > p ? a[h] : p) : (a[h] < p ? a[h] : p);
                }
            }
        }
    }
}

// r <- the 64 largest of r and c (both sorted descending, two per lane),
// sorted descending: max(r[i], c[63 - i]) is bitonic and holds them, and six
// half-cleaner stages sort it.
__device__ __forceinline__ void warp_merge64_desc(unsigned long long (&r)[2], const unsigned long long (&c)[2],
                                                  int lane) {
    const unsigned long long c0 = __shfl_sync(0xffffffffu, c[1], 31 - lane);  // c[63 - lane]
    const unsigned long long c1 = __shfl_sync(0xffffffffu, c[0], 31 - lane);  // c[31 - lane]
    r[0] = r[0] > c0 ? r[0] : c0;
    r[1] = r[1] > c1 ? r[1] : c1;
    {
        const unsigned long long x = r[0], y = r[1];
        r[0] = x > y ? x : y;
        r[1] = x > y ? y : x;
    }
#pragma unroll
    for (int stride = 16; stride > 0; stride >>= 1) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const unsigned long long p = __shfl_xor_sync(0xffffffffu, r[h], stride);
            r[h] = (lane & stride) == 0 ? (r[h] > p ? r[h] : p) : (r[h] < p ? r[h] : p);
        }
    }
}

// The 64 largest of src[0, n) (n may be 0), sorted descending, two per lane;
// zero keys pad. Chunks c0, c0 + step, ... of 64 entries. GLOBAL: src is in
// global memory and is read through L2 (other CTAs of the running grid may
// have written it); else src is in shared memory.
template <bool GLOBAL>
__device__ __forceinline__ void warp_top64(const unsigned long long* src, int n, int c0, int step, int lane,
                                           unsigned long long (&r)[2]) {
    r[0] = r[1] = 0ull;
    for (int c = c0; c < n; c += step) {
        unsigned long long t[2];
        if (GLOBAL) {
            t[0] = c + lane < n ? __ldcg(src + c + lane) : 0ull;
            t[1] = c + 32 + lane < n ? __ldcg(src + c + 32 + lane) : 0ull;
        } else {
            t[0] = c + lane < n ? src[c + lane] : 0ull;
            t[1] = c + 32 + lane < n ? src[c + 32 + lane] : 0ull;
        }
        warp_sort64_desc(t, lane);
        warp_merge64_desc(r, t, lane);
    }
}

// Number of entries of L[0, len) (sorted descending) above key: a fixed
// sequence of probes, so that searches of several lists overlap.
template <int LMAX>
__device__ __forceinline__ int count_above(const unsigned long long* L, int len, unsigned long long key) {
    int pos = 0;
#pragma unroll
    for (int step = LMAX; step > 0; step >>= 1)
        if (pos + step <= len && L[pos + step - 1] > key) pos += step;
    return pos;
}

// Every warp holds a descending list of 64 keys in registers (two per lane);
// afterwards warp 0 holds the 64 largest of all of them, descending. Three
// levels of pairwise merges through xch (256 keys of shared memory).
// Block-wide; ends with the block synchronised.
__device__ void block_tree_merge(unsigned long long (&t)[2], int lane, int warp, unsigned long long* xch) {
#pragma unroll
    for (int d = 1; d < kTkWarps; d <<= 1) {
        if ((warp & (2 * d - 1)) == d) {
            xch[(warp >> 1) * 64 + lane] = t[0];
            xch[(warp >> 1) * 64 + 32 + lane] = t[1];
        }
        __syncthreads();
        if ((warp & (2 * d - 1)) == 0) {
            const int src = (warp + d) >> 1;
            const unsigned long long c[2] = {xch[src * 64 + lane], xch[src * 64 + 32 + lane]};
            warp_merge64_desc(t, c, lane);
        }
        __syncthreads();
    }
}

// The row threshold t: the value of rank r among the 256 threads' sample
// maxima (-inf when that maximum is NaN). Thread i's 32 samples are element
// i of each of 32 chunks of 256 contiguous elements spread evenly over the
// row (32 KB read). At least r samples are >= t, so the row holds at least as
// many elements >= t as above its r-th largest sample. Deterministic: every
// CTA that computes it for a row gets the same t. Block-wide (L: 256 keys of
// shared memory); ends with the block synchronised.
__device__ float row_threshold(const float* x, int width, int r, unsigned long long* L, float* thr_s) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int step = (width - kTkThreads) / (kTkChunks - 1);
    float f[kTkChunks];
#pragma unroll
    for (int c = 0; c < kTkChunks; ++c) f[c] = __ldg(x + c * step + tid);
    unsigned int m = 0u;
#pragma unroll
    for (int c = 0; c < kTkChunks; ++c) m = max(m, tk_key32(f[c]));
    // (maximum, thread) pairs are unique: sort each warp's 32 descending,
    // then rank every pair against the other warps' lists.
    unsigned long long v = ((unsigned long long)m << 32) | (unsigned int)tid;
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            const unsigned long long p = __shfl_xor_sync(0xffffffffu, v, stride);
            const bool keep_max = ((lane & stride) == 0) == ((lane & size) == 0);
            v = keep_max ? (v > p ? v : p) : (v < p ? v : p);
        }
    }
    L[tid] = v;
    __syncthreads();
    int rank = lane;
#pragma unroll
    for (int w = 0; w < kTkWarps; ++w)
        if (w != warp) rank += count_above<32>(L + 32 * w, 32, v);
    if (rank == r - 1) {
        const unsigned int kr = (unsigned int)(v >> 32);
        *thr_s = kr == 0u ? -INFINITY : tk_value32(kr);
    }
    __syncthreads();
    return *thr_s;
}

// Exact path: each warp's k largest keys of x[0, width) (the warps share
// the row by 32-quad blocks), left in t as a descending list of 64 (entries
// past the warp's k-th are real keys or zero). buf: kTkWarps * kTkBuf keys.
// Each warp streams its share in ascending index order into its buffer; a
// full buffer is cut to its k largest and its k-th key becomes the warp's
// threshold. Later elements have larger indices, so one equal to the
// threshold's value ranks below it: past a threshold only strictly larger
// values are candidates.
__device__ void warp_exact_list(const float* x, int width, int k, unsigned long long* buf, int lane, int warp,
                                unsigned long long (&t)[2]) {
    unsigned long long* wb = buf + warp * kTkBuf;
    const unsigned int lt = (1u << lane) - 1u;
    bool open = true;         // no threshold yet: every non-NaN value
    float thr_v = -INFINITY;  // else: values > thr_v
    int cnt = 0;              // warp-uniform
    // wb[0, cnt) -> its 64 largest, descending, in t and wb[0, 64).
    auto shrink = [&]() {
        __syncwarp();
        warp_top64<false>(wb, cnt, 0, 64, lane, t);
        __syncwarp();
        wb[lane] = t[0];
        wb[32 + lane] = t[1];
        __syncwarp();
        if (cnt >= k) {
            cnt = k;
            open = false;
            thr_v = tk_value32((unsigned int)(wb[k - 1] >> 32));
        }
    };
    auto pass = [&](float v) { return open ? v == v : v > thr_v; };

    int done = 0;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const float4* x4 = reinterpret_cast<const float4*>(x);
        const int quads = width >> 2;
        const float nan = __int_as_float(0x7fc00000);
        constexpr int kUnroll = 4;
        for (int base = warp * 32; base < quads; base += kUnroll * kTkThreads) {
            float4 v[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int q = base + u * kTkThreads + lane;
                v[u] = q < quads ? __ldg(x4 + q) : make_float4(nan, nan, nan, nan);
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const float m4 = fmaxf(fmaxf(v[u].x, v[u].y), fmaxf(v[u].z, v[u].w));
                if (!__any_sync(0xffffffffu, pass(m4))) continue;
                const int e = 4 * (base + u * kTkThreads + lane);
                const bool c0 = pass(v[u].x), c1 = pass(v[u].y), c2 = pass(v[u].z), c3 = pass(v[u].w);
                const int nc = (int)c0 + (int)c1 + (int)c2 + (int)c3;
                int incl = nc;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int tt = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += tt;
                }
                const int added = __shfl_sync(0xffffffffu, incl, 31);
                int pos = cnt + incl - nc;
                if (c0) wb[pos++] = tk_key(v[u].x, e);
                if (c1) wb[pos++] = tk_key(v[u].y, e + 1);
                if (c2) wb[pos++] = tk_key(v[u].z, e + 2);
                if (c3) wb[pos++] = tk_key(v[u].w, e + 3);
                cnt += added;
                if (cnt > kTkBuf - 128) shrink();  // room for the next 128
            }
        }
        done = 4 * quads;
    }
    for (int base = done + warp * 32; base < width; base += kTkThreads) {
        const int i = base + lane;
        const float v = i < width ? x[i] : __int_as_float(0x7fc00000);
        const bool c = pass(v);
        const unsigned int m = __ballot_sync(0xffffffffu, c);
        if (c) wb[cnt + __popc(m & lt)] = tk_key(v, i);
        cnt += __popc(m);
        if (cnt > kTkBuf - 32) shrink();
    }
    shrink();
}

// The k largest keys of a row, written as (value, index) pairs to
// vals/idx[0, k): from its candidate list cand_row[0, n) when
// k <= n <= kTkCap, else by the exact path over x_row. Block-wide, with the
// same n in every thread; no shared memory is read after its last barrier.
__device__ void select_row(const unsigned long long* cand_row, int n, const float* x_row, int width, int k,
                           unsigned long long* buf, unsigned long long* xch, float* vals, int32_t* idx) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    unsigned long long t[2];
    if (n >= k && n <= kTkCap)
        warp_top64<true>(cand_row, n, 64 * warp, 64 * kTkWarps, lane, t);  // chunks w, w + 8, ...
    else
        warp_exact_list(x_row, width, k, buf, lane, warp, t);
    block_tree_merge(t, lane, warp, xch);
    if (warp == 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = h * 32 + lane;
            if (j < k) {
                const unsigned long long key = t[h];
                vals[j] = key != 0ull ? tk_value32((unsigned int)(key >> 32)) : -INFINITY;
                idx[j] = key != 0ull ? (int32_t)(0xFFFFFFFFu - (unsigned int)(key & 0xFFFFFFFFull)) : -1;
            }
        }
    }
}

// Row `blockIdx.x`: thr[row] = row_threshold, cnt[row] = done[row] = 0.
__global__ void __launch_bounds__(kTkThreads) topk_sample_kernel(const float* logits, int width, int ld, int r,
                                                                  float* thr, int* cnt, int* done) {
    __shared__ unsigned long long L[kTkThreads];
    __shared__ float thr_s;
    const int row = blockIdx.x;
    griddep_wait();
    const float t = row_threshold(logits + (long long)row * ld, width, r, L, &thr_s);
    if (threadIdx.x == 0) {
        thr[row] = t;
        cnt[row] = 0;
        done[row] = 0;
    }
    griddep_launch();
}

// CTA b streams quads [total*b/G, total*(b+1)/G) of the rows x (width/4)
// quad matrix (plus the width % 4 tail of a row whose last quad it owns),
// one row segment at a time: the key of every element >= thr[row] is
// appended to cand[row][...] and counted in cnt[row]. Once a row's list
// passed kTkCap the warp stops appending to it (the count already says
// "overflow"). The CTA whose segment completes the row's quads (done[row]
// reaches width / 4) selects the row.
__global__ void __launch_bounds__(kTkThreads, 4) topk_filter_kernel(const float* logits, int rows, int width, int ld,
                                                                     int k, const float* thr, int* cnt, int* done,
                                                                     unsigned long long* cand, float* vals,
                                                                     int32_t* idx) {
    __shared__ unsigned long long buf[kTkWarps * kTkBuf];
    __shared__ unsigned long long xch[kTkThreads];
    __shared__ int last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    unsigned long long* wb = buf + warp * kTkBuf;
    const unsigned int lt = (1u << lane) - 1u;
    const int quads = width >> 2, rem = width & 3;
    const long long total = (long long)rows * quads;
    const long long g0 = total * blockIdx.x / gridDim.x, g1 = total * (blockIdx.x + 1) / gridDim.x;
    const float nan = __int_as_float(0x7fc00000);
    griddep_wait();
    for (long long g = g0; g < g1;) {
        const int row = (int)(g / quads);
        const int q0 = (int)(g - (long long)row * quads);
        const int q1 = (int)((long long)quads < q0 + (g1 - g) ? (long long)quads : q0 + (g1 - g));
        g += q1 - q0;
        const float* xr = logits + (long long)row * ld;
        const float tv = thr[row];
        const float4* x4 = reinterpret_cast<const float4*>(xr);
        int* row_cnt = cnt + row;
        unsigned long long* dst = cand + (long long)row * kTkCap;
        int wcnt = 0;       // keys in wb (warp-uniform)
        bool full = false;  // the row's list overflowed (warp-uniform)
        auto flush = [&]() {
            int base = 0;
            if (lane == 0) base = atomicAdd(row_cnt, wcnt);
            base = __shfl_sync(0xffffffffu, base, 0);
            for (int i = lane; i < wcnt; i += 32)
                if (base + i < kTkCap) dst[base + i] = wb[i];
            full = base + wcnt > kTkCap;
            wcnt = 0;
            __syncwarp();
        };
        constexpr int kUnroll = 4;
        for (int base = q0 + warp * 32; base < q1; base += kUnroll * kTkThreads) {
            float4 v[kUnroll];
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                const int q = base + u * kTkThreads + lane;
                v[u] = q < q1 ? __ldg(x4 + q) : make_float4(nan, nan, nan, nan);
            }
#pragma unroll
            for (int u = 0; u < kUnroll; ++u) {
                // fmaxf drops NaN, and NaN fails >=: NaN is never a candidate.
                const float m4 = fmaxf(fmaxf(v[u].x, v[u].y), fmaxf(v[u].z, v[u].w));
                if (!__any_sync(0xffffffffu, m4 >= tv) || full) continue;
                const int e = 4 * (base + u * kTkThreads + lane);
                const bool c0 = v[u].x >= tv, c1 = v[u].y >= tv, c2 = v[u].z >= tv, c3 = v[u].w >= tv;
                const int nc = (int)c0 + (int)c1 + (int)c2 + (int)c3;
                int incl = nc;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int t = __shfl_up_sync(0xffffffffu, incl, o);
                    if (lane >= o) incl += t;
                }
                const int added = __shfl_sync(0xffffffffu, incl, 31);
                int pos = wcnt + incl - nc;
                if (c0) wb[pos++] = tk_key(v[u].x, e);
                if (c1) wb[pos++] = tk_key(v[u].y, e + 1);
                if (c2) wb[pos++] = tk_key(v[u].z, e + 2);
                if (c3) wb[pos++] = tk_key(v[u].w, e + 3);
                wcnt += added;
                __syncwarp();
                if (wcnt > kTkBuf - 128) flush();  // room for the next 128
            }
        }
        if (rem != 0 && q1 == quads && warp == 0 && !full) {
            const int e = 4 * quads + lane;
            const float vv = lane < rem ? xr[e] : nan;
            const bool c = vv >= tv;
            const unsigned int m = __ballot_sync(0xffffffffu, c);
            if (c) wb[wcnt + __popc(m & lt)] = tk_key(vv, e);
            wcnt += __popc(m);
            __syncwarp();
        }
        if (wcnt > 0) flush();
        // Publish this segment's candidates, then count its quads.
        __threadfence();
        __syncthreads();
        if (tid == 0) last = atomicAdd(done + row, q1 - q0) + (q1 - q0) == quads;
        __syncthreads();
        if (last) {
            __threadfence();
            select_row(dst, __ldcg(row_cnt), xr, width, k, buf, xch, vals + (long long)row * k,
                       idx + (long long)row * k);
        }
    }
    griddep_launch();
}

// Row `blockIdx.x` by the exact path (narrow or unaligned rows).
__global__ void __launch_bounds__(kTkThreads) topk_exact_kernel(const float* logits, int width, int ld, int k,
                                                                 float* vals, int32_t* idx) {
    __shared__ unsigned long long buf[kTkWarps * kTkBuf];
    __shared__ unsigned long long xch[kTkThreads];
    const int row = blockIdx.x;
    griddep_wait();
    select_row(nullptr, -1, logits + (long long)row * ld, width, k, buf, xch, vals + (long long)row * k,
               idx + (long long)row * k);
    griddep_launch();
}

// Merge of per-shard results (vocab-sharded lm_head): `gathered` holds, for
// each of `lists` shards, rows x 8-byte greedy keys (global indices), then
// rows x k fp32 values and rows x k int32 LOCAL indices of the shard's top-k
// (launch_topk's output, descending, (-inf, -1) padded). Shard r's local
// index i is global r * shard_rows + i. Per row: the largest key (the
// greedy id, the scan's tie rule) and the k largest (value, global index)
// keys of the shards' lists (warp r loads list r, then the tree merge).
// With `flags` (the peer exchange: the receive buffer's header), the lists
// arrive from the other ranks' push kernels: thread 0 first waits, bounded,
// until every shard's flag of the call's parity holds the call's epoch (an
// acquire at system scope: the pushes released it after their data); a wait
// that runs out records AEXIS_E_TIMEOUT and the CTA writes nothing.
__global__ void __launch_bounds__(kTkThreads) topk_shard_merge_kernel(const int32_t* gathered, int lists, int rows,
                                                                       int k, int shard_rows, long long* ids,
                                                                       float* vals, int32_t* idx,
                                                                       int slot_words, const unsigned int* flags,
                                                                       int* status) {
    __shared__ unsigned long long xch[kTkThreads];
    __shared__ unsigned long long best[kTkWarps];
    __shared__ int arrived;
    const int row = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    griddep_wait();
    if (flags) {
        // The call's epoch (this rank's push stored it) picks the slot parity.
        const unsigned int e = *reinterpret_cast<const volatile unsigned int*>(flags + kPeerEpochWord);
        flags += (e & 1u) * kPeerMaxRanks;
        gathered += (size_t)(e & 1u) * lists * slot_words;
        if (threadIdx.x == 0) {
            int ok = 1;
            const long long t0 = clock64();
            for (int sh = 0; sh < lists && ok; ++sh) {
                for (;;) {
                    unsigned int f;
                    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(flags + sh) : "memory");
                    if (f == e) break;
                    if (clock64() - t0 > kTkWaitLimitCycles) {
                        tk_report_timeout(status);
                        ok = 0;
                        break;
                    }
                }
            }
            arrived = ok;
        }
        __syncthreads();
        if (!arrived) {
            griddep_launch();
            return;
        }
    }
    const size_t per = (size_t)slot_words;  // 32-bit words per shard
    unsigned long long t[2] = {0ull, 0ull};
    unsigned long long kmax = 0ull;
    if (warp < lists) {
        const int32_t* base = gathered + per * warp;
        const unsigned long long* keys = reinterpret_cast<const unsigned long long*>(base);
        const float* sv = reinterpret_cast<const float*>(base + (size_t)rows * 2) + (size_t)row * k;
        const int32_t* si = base + (size_t)rows * 2 + (size_t)rows * k + (size_t)row * k;
        kmax = __ldcg(keys + row);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = h * 32 + lane;
            if (j < k) {
                const int li = __ldcg(si + j);
                t[h] = li < 0 ? 0ull : tk_key(__ldcg(sv + j), warp * shard_rows + li);
            }
        }
    }
    if (lane == 0) best[warp] = kmax;
    block_tree_merge(t, lane, warp, xch);
    if (warp == 0) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const int j = h * 32 + lane;
            if (j < k) {
                const unsigned long long key = t[h];
                vals[(size_t)row * k + j] = key != 0ull ? tk_value32((unsigned int)(key >> 32)) : -INFINITY;
                idx[(size_t)row * k + j] = key != 0ull ? (int32_t)(0xFFFFFFFFu - (unsigned int)(key & 0xFFFFFFFFull)) : -1;
            }
        }
        if (lane == 0) {
            unsigned long long m = 0ull;
            for (int w = 0; w < kTkWarps; ++w) m = best[w] > m ? best[w] : m;
            ids[row] = (long long)aexis_argmax_index(m);
        }
    }
    griddep_launch();
}

bool topk_sampled(int width) { return width >= kTkMinSampledWidth; }

// Rank r whose sample value leaves about 4.5k of the row's elements above it
// (r / kTkSamples of the row). When the order of the values carries no
// pattern, the count above the r-th largest sample is about Gamma(r) x
// width / kTkSamples: at width 151936 and k = 50 (r = 13) a row holds fewer
// than k candidates with probability near 5e-6 and more than kTkCap
// practically never.
int topk_rank(int width, int k) {
    long long r = (9LL * k * kTkSamples + 2LL * width - 1) / (2LL * width);
    r = r < 1 ? 1 : r;
    return (int)(r > kTkMaxRank ? kTkMaxRank : r);
}

template <typename K, typename... Args>
cudaError_t launch_pdl(K kern, dim3 grid, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kTkThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

}  // namespace

// Scratch: cand[rows][kTkCap] keys, then thr[rows], cnt[rows], done[rows].
size_t topk_scratch_bytes(int rows, int width, int k, int sm_count) {
    (void)k;
    (void)sm_count;
    if (!topk_sampled(width)) return 16;
    return (size_t)rows * (kTkCap * sizeof(unsigned long long) + sizeof(float) + 2 * sizeof(int));
}

cudaError_t launch_topk(const float* logits, int rows, int width, int ld, int k, float* vals, int32_t* idx,
                        void* scratch, int sm_count, cudaStream_t s) {
    if (k < 1 || k > kTkMaxK) return cudaErrorInvalidValue;
    const bool aligned = (reinterpret_cast<uintptr_t>(logits) & 15) == 0 && (ld & 3) == 0;
    if (!topk_sampled(width) || !aligned)
        return launch_pdl(topk_exact_kernel, dim3(rows), s, logits, width, ld, k, vals, idx);
    unsigned long long* cand = reinterpret_cast<unsigned long long*>(scratch);
    float* thr = reinterpret_cast<float*>(cand + (size_t)rows * kTkCap);
    int* cnt = reinterpret_cast<int*>(thr + rows);
    int* done = cnt + rows;
    cudaError_t e =
        launch_pdl(topk_sample_kernel, dim3(rows), s, logits, width, ld, topk_rank(width, k), thr, cnt, done);
    if (e != cudaSuccess) return e;
    static int occ = 0;
    if (occ == 0) {
        int o = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, topk_filter_kernel, kTkThreads, 0) != cudaSuccess ||
            o < 1)
            o = 1;
        occ = o;
    }
    const long long total = (long long)rows * (width >> 2);
    long long blocks = (long long)sm_count * occ;
    const long long by_work = (total + 1023) / 1024;  // at least four quads per thread
    blocks = blocks < by_work ? blocks : by_work;
    return launch_pdl(topk_filter_kernel, dim3((unsigned int)(blocks < 1 ? 1 : blocks)), s, logits, rows, width, ld,
                      k, (const float*)thr, cnt, done, cand, vals, idx);
}

cudaError_t launch_topk_shard_merge(const int32_t* gathered, int lists, int rows, int k, int shard_rows, long long* ids,
                                    float* vals, int32_t* idx, cudaStream_t s) {
    if (lists < 1 || lists > kTkWarps || k < 1 || k > kTkMaxK) return cudaErrorInvalidValue;
    const unsigned int* no_flags = nullptr;
    int* no_status = nullptr;
    return launch_pdl(topk_shard_merge_kernel, dim3(rows), s, gathered, lists, rows, k, shard_rows, ids, vals, idx,
                      2 * rows + 2 * rows * k, no_flags, no_status);
}

namespace {

// The peer exchange: each rank pushes its packed result (keys + top-k lists)
// into slot `rank` of every rank's receive buffer (PeerRecv layout) with
// plain stores over NVLink, then, once every CTA's stores are fenced at
// system scope (the last CTA to arrive on the block counter knows), releases
// the epoch into flag[parity][rank] of every receive buffer.
struct PeerPtrs {
    char* p[kPeerMaxRanks];
};

__global__ void __launch_bounds__(kTkThreads) topk_peer_push_kernel(const int32_t* __restrict__ src, int words,
                                                                    PeerPtrs peers, int world, int rank,
                                                                    int slot_words) {
    griddep_wait();
    // This call's epoch: one past the last call's, which this rank's
    // previous push stored (every earlier kernel of the stream has finished).
    unsigned int* own = reinterpret_cast<unsigned int*>(peers.p[rank]);
    unsigned int* counter = own + kPeerCounterWord;
    const unsigned int epoch = *reinterpret_cast<volatile unsigned int*>(own + kPeerEpochWord) + 1u;
    const int parity = (int)(epoch & 1u);
    const size_t slot = (size_t)(parity * world + rank) * (size_t)slot_words;  // in 32-bit words
    const int n16 = words >> 2;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n16; i += gridDim.x * blockDim.x) {
        const int4 v = __ldcg(reinterpret_cast<const int4*>(src) + i);
        for (int p = 0; p < world; ++p)
            reinterpret_cast<int4*>(reinterpret_cast<int32_t*>(peers.p[p] + kPeerHeaderBytes) + slot)[i] = v;
    }
    if (blockIdx.x == 0 && threadIdx.x < (words & 3)) {
        const int i = (n16 << 2) + threadIdx.x;
        const int32_t v = __ldcg(src + i);
        for (int p = 0; p < world; ++p) (reinterpret_cast<int32_t*>(peers.p[p] + kPeerHeaderBytes) + slot)[i] = v;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0 && atomicAdd(counter, 1u) == gridDim.x - 1) {
        *counter = 0u;  // the next call's count
        __threadfence_system();
        for (int p = 0; p < world; ++p) {
            unsigned int* flag = reinterpret_cast<unsigned int*>(peers.p[p]) + parity * kPeerMaxRanks + rank;
            asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(epoch) : "memory");
        }
        own[kPeerEpochWord] = epoch;  // read by this call's merge and the next push
    }
    griddep_launch();
}

}  // namespace

int peer_slot_words(int rows, int k) { return ((2 * rows + 2 * rows * k) + 3) & ~3; }

size_t peer_recv_bytes(int world, int rows, int k) {
    return kPeerHeaderBytes + 2 * (size_t)world * (size_t)peer_slot_words(rows, k) * sizeof(int32_t);
}

cudaError_t launch_topk_peer_push(const int32_t* packed, int rows, int k, void* const* peers, int world, int rank,
                                  cudaStream_t s) {
    if (world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world) return cudaErrorInvalidValue;
    PeerPtrs pp = {};
    for (int p = 0; p < world; ++p) pp.p[p] = reinterpret_cast<char*>(peers[p]);
    const int words = 2 * rows + 2 * rows * k;
    const int blocks = ((words >> 2) + kTkThreads - 1) / kTkThreads;
    return launch_pdl(topk_peer_push_kernel, dim3(blocks < 1 ? 1 : (blocks > 64 ? 64 : blocks)), s, packed, words, pp,
                      world, rank, peer_slot_words(rows, k));
}

cudaError_t launch_topk_peer_merge(const void* recv, int world, int rows, int k, int shard_rows, long long* ids,
                                   float* vals, int32_t* idx, int* status, cudaStream_t s) {
    if (world < 1 || world > kPeerMaxRanks || k < 1 || k > kTkMaxK) return cudaErrorInvalidValue;
    const char* base = reinterpret_cast<const char*>(recv);
    const unsigned int* flags = reinterpret_cast<const unsigned int*>(base);
    const int32_t* gathered = reinterpret_cast<const int32_t*>(base + kPeerHeaderBytes);
    return launch_pdl(topk_shard_merge_kernel, dim3(rows), s, gathered, world, rows, k, shard_rows, ids, vals, idx,
                      peer_slot_words(rows, k), flags, status);
}

namespace {

// Greedy key of each row from its top-k list (the list's first entry is the
// row's largest value at its lowest index, -0 counted as +0, NaN never
// listed), so no second pass over the logits is needed. The one case the
// list cannot show is the ArgMax rule that a NaN at global index 0 wins
// (AexisArgMaxPack4LinearMat, HLSL Pack4Matmul:645-686): the shard holding
// index 0 reads that one element. An empty list (a row of NaN) gives key 0.
__global__ void topk_greedy_keys_kernel(const float* __restrict__ logits, int rows, int ld,
                                        const float* __restrict__ vals, const int32_t* __restrict__ idx, int k,
                                        long long offset, unsigned long long* __restrict__ keys) {
    griddep_wait();
    griddep_launch();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rows) return;
    const int i0 = idx[(long long)r * k];
    unsigned long long key = i0 >= 0 ? aexis_argmax_key(vals[(long long)r * k], (int)(offset + i0)) : 0ull;
    if (offset == 0) {
        const float x0 = logits[(long long)r * ld];
        if (x0 != x0) key = aexis_argmax_key(x0, 0);
    }
    keys[r] = key;
}

}  // namespace

cudaError_t launch_topk_greedy_keys(const float* logits, int rows, int ld, const float* vals, const int32_t* idx, int k,
                                    long long offset, unsigned long long* keys, cudaStream_t s) {
    return launch_pdl(topk_greedy_keys_kernel, dim3((rows + kTkThreads - 1) / kTkThreads), s, logits, rows, ld, vals,
                      idx, k, offset, keys);
}
