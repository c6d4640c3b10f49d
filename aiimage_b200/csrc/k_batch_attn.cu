// k_batch_attn.cu -- batched decode attention on the tensor cores (head_dim
// 128, up to 4 query heads per KV head).
//
// Same computation as the split attention of k_batch.cu (the reference's
// two-pass softmax, HLSL Pack4Matmul:485-547, with GQA kv = h / (H / Hkv)),
// laid out for mma.m16n8k16 (fp16 x fp16 -> fp32):
//   scores  S[p][col] = sum_d K[p][d] * B[d][col]: positions are the MMA rows
//           (A from the K chunk by ldmatrix), the query heads' fp16 hi parts
//           are B columns 0-3 and their lo parts columns 4-7, so one MMA per
//           16 dims gives both halves of an fp32-accurate dot product (K is
//           fp16 in the cache, the products are exact, the sums fp32);
//   values  O[d][col] = sum_p V[p][d] * P[p][col]: dims are the MMA rows (A =
//           V^T by ldmatrix.trans), the probabilities' hi / lo parts are B
//           columns 0-3 / 4-7.
// The work items are (sequence, KV head, 64-position chunk), in that order;
// CTA i of a fixed grid takes the equal contiguous share [T i / G, T (i+1) /
// G) of the T items of the step and streams its chunks through two
// shared-memory buffers (bulk copies, the next chunk in flight while one is
// computed). Consecutive chunks of one (sequence, KV head) in a CTA form a
// segment with an online softmax (running max m, sum l, rescaled O), and a
// segment leaves one partial (m, l, O) in the slot of its first chunk. The
// merge of a head's segments happens in launch_batch_attn_merge_prep, which
// also writes the O projection's fp16 hi / lo input tiles.
//
// The batch's KV caches are stored with the 16-byte chunks of every 128-byte
// half row XOR-swizzled by position & 7 (cache_dim in k_batch.cu), so a bulk
// copy of consecutive rows lands conflict-free for ldmatrix.
#include "decoder_internal.h"
#include "gemv_dev.cuh"
#include "mma_frag.cuh"

namespace {

using namespace aexis_dev;

constexpr int kTaD = 128;                  // head dim
constexpr int kTaC = 64;                   // positions per chunk
constexpr int kTaWarps = 4;
constexpr int kTaThreads = kTaWarps * 32;
constexpr int kTaMaxHpg = 4;
constexpr int kTaMaxB = 256;
constexpr int kTaSlots = 8192 / kTaC;      // partial slots per (sequence, query head)
constexpr int kTaRow = kTaD * 2;           // bytes per cache row
constexpr int kTaBuf = kTaC * kTaRow;      // one K or V chunk (16 KB)
constexpr int kTaPtStride = kTaC + 8;      // P^T row (halves), padded against bank conflicts
constexpr int kTaStride = kTaD + 2;        // partial: D values, then m and l

struct TaShared {
    __align__(128) uint8_t k[2][kTaBuf];
    __align__(128) uint8_t v[2][kTaBuf];
    float sc[kTaC][kTaMaxHpg];
    __align__(16) __half pt[8][kTaPtStride];  // rows 0-3: hi of head h, 4-7: lo
    float alpha[kTaMaxHpg], mrun[kTaMaxHpg], lrun[kTaMaxHpg];
    float qs[kTaMaxHpg][kTaD];                  // a segment's query heads after RoPE
    long long start[kTaMaxB + 1];               // item prefix over sequences
    int pos[kTaMaxB];                           // the step's positions
    uint64_t full[2];
};

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

// Generic-proxy writes to shared memory ordered before later bulk copies into it.
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Byte offset of (row p, 16-byte dim chunk ch) in a swizzled chunk buffer.
__device__ __forceinline__ int swz_off(int p, int ch) {
    return p * kTaRow + (((ch & 8) | ((ch & 7) ^ (p & 7))) << 4);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
}

// Chunks of a sequence at position p (ctx = p + 1 positions); 0 for p = -1.
__device__ __forceinline__ int seq_chunks(int p) { return (p + kTaC) / kTaC; }

// First item of CTA i of G over T items.
__device__ __forceinline__ long long cta_first(long long T, int i, int G) { return T * i / G; }

// Whether item `it` starts a CTA's share (T items over G CTAs).
__device__ __forceinline__ bool starts_share(long long T, int G, long long it) {
    const long long i = (it * G + T - 1) / T;  // the smallest i with T i / G >= it
    return i < G && cta_first(T, (int)i, G) == it;
}

// s[b] = items before sequence b (kvh chunk lists each), s[B] = T, and
// ps[b] = pos[b]. One warp (lane = its lane): the B <= kTaMaxB position loads
// are issued together, then a shuffle scan per 32 sequences.
__device__ void item_prefix(const int* pos, int B, int kvh, long long* s, int* ps, int lane) {
    constexpr int J = kTaMaxB / 32;
    int p[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int b = j * 32 + lane;
        p[j] = b < B ? pos[b] : -1;
    }
    long long carry = 0;
#pragma unroll
    for (int j = 0; j < J; ++j) {
        if (j * 32 < B) {  // uniform over the warp
            const int b = j * 32 + lane;
            const int n = kvh * seq_chunks(p[j]);
            int x = n;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, x, o);
                if (lane >= o) x += y;
            }
            if (b < B) {
                s[b] = carry + x - n;
                ps[b] = p[j];
            }
            carry += __shfl_sync(0xffffffffu, x, 31);
        }
    }
    if (lane == 0) s[B] = carry;
}

// Dim d (original order) of one head after RoPE (rotate-half over the first
// rot dims, HLSL Pack4PointwiseNorm:414-473) at the position whose cos / sin
// rows are cs / sn, from the head's rows in the decoder's internal order:
// pair (j, j + rot / 2) at rows 2 j, 2 j + 1, then dims rot.. in order.
__device__ __forceinline__ float rope_dim(const float* hr, int d, int rot, const float* cs, const float* sn) {
    // Branch-free, so that the loads of several calls issue together.
    const int half = rot >> 1;
    const bool rd = d < rot;
    const int j = rd ? (d < half ? d : d - half) : 0;
    const float x0 = __ldcg(hr + (rd ? 2 * j : d));
    const float x1 = __ldcg(hr + (rd ? 2 * j + 1 : d));
    const float c = rd ? __ldg(cs + j) : 1.0f;
    const float s = rd ? __ldg(sn + j) : 0.0f;
    return rd ? (d < half ? x0 * c - x1 * s : x0 * s + x1 * c) : x0;
}

// Position of dim d in a swizzled cache row at position p (16-byte chunks
// XOR p & 7 within each 128-byte half row).
__device__ __forceinline__ int swz_dim(int p, int d) {
    const int ch = d >> 3;
    return (((ch & 8) | ((ch & 7) ^ (p & 7))) << 3) | (d & 7);
}

// qkv: [B][rows] fp32, the QKV projection in the decoder's internal row
// order, before RoPE; cos / sin tables [position][rot / 2]; caches
// [B][kvh][cap][D] fp16, swizzled rows; part: [B][n_heads][kTaSlots][kTaStride].
// RoPE and the KV append are fused in: a segment's first chunk rotates its
// query heads while loading them, and the CTA whose item is the last chunk
// of (b, g) rotates the step's new K row (position pos[b]), writes it and the
// V row to the caches and patches both into its copy of the chunk.
__global__ void __launch_bounds__(kTaThreads, 3) bat_attn_tc_kernel(const float* qkv, int rows, const float* cosv,
                                                                   const float* sinv, int rot, __half* kc, __half* vc,
                                                                   int cap, int n_heads, int kvh, float scale,
                                                                   const int* pos, int B, float* part, int* status) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    TaShared& sh = *reinterpret_cast<TaShared*>(smem_raw);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int g8 = lane >> 2, tig = lane & 3;
    const int hpg = n_heads / kvh;
    const int G = gridDim.x, blk = blockIdx.x;
    // Before the wait on the previous kernel (programmatic dependent launch):
    // the positions (written by the previous step) and the cache rows below
    // them are final, so the item prefix and the first chunk's copies start
    // here; the QKV projection (the previous kernel's output) is read after.
    if (warp == 0) item_prefix(pos, B, kvh, sh.start, sh.pos, lane);
    // Zero both chunk buffers (rows past a chunk's end are read by the MMAs,
    // weighted 0) and P^T (columns of unused heads stay 0).
    for (int i = tid; i < 4 * kTaBuf / 16; i += kTaThreads) reinterpret_cast<uint4*>(&sh.k[0][0])[i] = make_uint4(0, 0, 0, 0);
    for (int i = tid; i < 8 * kTaPtStride / 2; i += kTaThreads) reinterpret_cast<uint32_t*>(&sh.pt[0][0])[i] = 0u;
    if (tid < kTaMaxHpg) sh.alpha[tid] = 0.0f;
    if (tid == 0) {
        mbar_init(&sh.full[0], 1);
        mbar_init(&sh.full[1], 1);
        fence_barrier_init();
    }
    fence_proxy_async_smem();
    __syncthreads();
    const long long T = sh.start[B];
    const long long i0 = cta_first(T, blk, G), i1 = cta_first(T, blk + 1, G);
    if (i0 >= i1) {
        griddep_wait();
        griddep_launch();
        return;
    }
    // (sequence, KV head, chunk) of an item; the cursor (a sequence index)
    // only moves forward.
    auto locate = [&](int& cur, long long it, int& b, int& g, int& c) {
        while (sh.start[cur + 1] <= it) ++cur;
        b = cur;
        const long long r = it - sh.start[cur];
        const int n = seq_chunks(sh.pos[cur]);
        g = (int)(r / n);
        c = (int)(r - (long long)g * n);
    };
    int cur_issue = 0, cur = 0;
    auto issue = [&](long long it, int buf) {  // thread 0
        int b, g, c;
        locate(cur_issue, it, b, g, c);
        const int ctx = sh.pos[b] + 1;
        const int np = min(kTaC, ctx - c * kTaC);
        const size_t row0 = ((size_t)b * kvh + g) * cap + (size_t)c * kTaC;
        const uint32_t bytes = (uint32_t)np * kTaRow;
        mbar_arrive_expect_tx(&sh.full[buf], 2 * bytes);
        bulk_g2s_plain(&sh.k[buf][0], kc + row0 * kTaD, bytes, &sh.full[buf]);
        bulk_g2s_plain(&sh.v[buf][0], vc + row0 * kTaD, bytes, &sh.full[buf]);
    };
    if (tid == 0) issue(i0, 0);
    griddep_wait();
    griddep_launch();

    uint32_t qf[8][2];     // B fragments of q (hi / lo columns), per 16-dim block
    float acc[2][4];       // O partials: rows d (2 m-tiles), columns 2 tig, 2 tig + 1
    int seg_c = 0;
    bool ok = true;
    long long fail_it = -1;
    for (long long it = i0; it < i1; ++it) {
        const int k = (int)(it - i0), buf = k & 1;
        int b, g, c;
        locate(cur, it, b, g, c);
        const int ctx = sh.pos[b] + 1;
        const int np = min(kTaC, ctx - c * kTaC);
        const int nch = seq_chunks(ctx - 1);
        const bool seg_start = it == i0 || c == 0;
        const bool seg_end = it + 1 == i1 || c + 1 == nch;
        const bool appends = c + 1 == nch;  // the chunk holds the step's new row, position ctx - 1
        const float* cs = cosv + (size_t)(ctx - 1) * (rot >> 1);
        const float* sn = sinv + (size_t)(ctx - 1) * (rot >> 1);
        if (tid == 0 && it + 1 < i1) issue(it + 1, buf ^ 1);  // that buffer was freed by the last barrier
        __half k_new = __float2half_rn(0.0f), v_new = k_new;
        int new_off = 0;
        if (appends) {  // thread tid = dim tid of the new K and V rows
            const int p = ctx - 1;
            const float* row = qkv + (size_t)b * rows;
            k_new = __float2half_rn(rope_dim(row + (size_t)(n_heads + g) * kTaD, tid, rot, cs, sn));
            v_new = __float2half_rn(__ldcg(row + (size_t)(n_heads + kvh + g) * kTaD + tid));
            const int sd = swz_dim(p, tid);
            const size_t at = (((size_t)b * kvh + g) * cap + p) * kTaD + sd;
            kc[at] = k_new;
            vc[at] = v_new;
            new_off = (p - c * kTaC) * kTaRow + sd * 2;
        }
        if (seg_start) {
            seg_c = c;
            {  // dim tid of the segment's query heads, after RoPE
                const float* qb = qkv + (size_t)b * rows + (size_t)g * hpg * kTaD;
                float qv[kTaMaxHpg];
#pragma unroll
                for (int h = 0; h < kTaMaxHpg; ++h) qv[h] = h < hpg ? rope_dim(qb + h * kTaD, tid, rot, cs, sn) : 0.0f;
#pragma unroll
                for (int h = 0; h < kTaMaxHpg; ++h) sh.qs[h][tid] = qv[h];
            }
            __syncthreads();
            // q columns: lane group g8 < 4 -> hi of head g8, 4..7 -> lo of head g8 - 4.
            const int hh = g8 & 3;
            const bool use = hh < hpg;
#pragma unroll
            for (int kb = 0; kb < 8; ++kb) {
#pragma unroll
                for (int r = 0; r < 2; ++r) {
                    const int d = kb * 16 + r * 8 + 2 * tig;
                    float x0 = use ? sh.qs[hh][d] : 0.0f;
                    float x1 = use ? sh.qs[hh][d + 1] : 0.0f;
                    if (g8 >= 4) {
                        x0 -= __half2float(__float2half_rn(x0));
                        x1 -= __half2float(__float2half_rn(x1));
                    }
                    qf[kb][r] = pack_half2(x0, x1);
                }
            }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[mt][e] = 0.0f;
            if (tid < kTaMaxHpg) {
                sh.mrun[tid] = -INFINITY;
                sh.lrun[tid] = 0.0f;
            }
        }
        if (!mbar_wait(&sh.full[buf], (uint32_t)((k >> 1) & 1))) {
            if (tid == 0) report_timeout(status);
            ok = false;
        }
        if (!__syncthreads_and(ok)) {
            fail_it = it;
            break;
        }
        if (appends) {
            // The copy read the row before this step's value; replace it. The
            // fence orders these writes before the buffer's next bulk copy.
            *reinterpret_cast<__half*>(&sh.k[buf][0] + new_off) = k_new;
            *reinterpret_cast<__half*>(&sh.v[buf][0] + new_off) = v_new;
            fence_proxy_async_smem();
            __syncthreads();
        }
        const uint8_t* kbuf = &sh.k[buf][0];
        const uint8_t* vbuf = &sh.v[buf][0];
        // Scores: warp w takes positions [16 w, 16 w + 16) of the chunk.
        {
            float s4[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            const int mi = lane >> 3, r8 = lane & 7;
            const int prow = 16 * warp + (mi & 1) * 8 + r8;
#pragma unroll
            for (int kb = 0; kb < 8; ++kb) {
                uint32_t a[4];
                ldsm_x4(a, kbuf + swz_off(prow, kb * 2 + (mi >> 1)));
                mma16816(s4, a, make_uint2(qf[kb][0], qf[kb][1]));
            }
            // Columns 2 tig, 2 tig + 1: hi of heads (2 tig, 2 tig + 1) for tig < 2,
            // lo of the same heads in the lanes with tig + 2.
#pragma unroll
            for (int e = 0; e < 4; ++e) s4[e] += __shfl_xor_sync(0xffffffffu, s4[e], 2);
            if (tig < 2) {
                const int p0 = 16 * warp + g8, p1 = p0 + 8;
                const int h0 = 2 * tig, h1 = h0 + 1;
                sh.sc[p0][h0] = p0 < np ? s4[0] * scale : -INFINITY;
                sh.sc[p0][h1] = p0 < np ? s4[1] * scale : -INFINITY;
                sh.sc[p1][h0] = p1 < np ? s4[2] * scale : -INFINITY;
                sh.sc[p1][h1] = p1 < np ? s4[3] * scale : -INFINITY;
            }
        }
        __syncthreads();
        // Online softmax, warp h for head h: the chunk's maximum, the rescale
        // of everything before it, the probabilities as fp16 hi / lo.
        if (warp < hpg) {
            const int h = warp;
            const float sa = sh.sc[lane][h], sb = sh.sc[lane + 32][h];
            float cm = fmaxf(sa, sb);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
            const float mold = sh.mrun[h];
            const float mnew = fmaxf(mold, cm);
            const float pa = expf(sa - mnew), pb = expf(sb - mnew);
            float ps = pa + pb;
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            const __half ha = __float2half_rn(pa), hb = __float2half_rn(pb);
            sh.pt[h][lane] = ha;
            sh.pt[h][lane + 32] = hb;
            sh.pt[4 + h][lane] = __float2half_rn(pa - __half2float(ha));
            sh.pt[4 + h][lane + 32] = __float2half_rn(pb - __half2float(hb));
            __syncwarp();
            if (lane == 0) {
                const float al = expf(mold - mnew);  // 0 before the first chunk (mold = -inf)
                sh.alpha[h] = al;
                sh.lrun[h] = sh.lrun[h] * al + ps;
                sh.mrun[h] = mnew;
            }
        }
        __syncthreads();
        // Values: warp w takes dims [32 w, 32 w + 32) (two 16-dim m-tiles).
        {
            const float a0 = sh.alpha[(2 * tig) & 3], a1 = sh.alpha[(2 * tig + 1) & 3];
            const int mi = lane >> 3, r8 = lane & 7;
#pragma unroll
            for (int mt = 0; mt < 2; ++mt) {
                acc[mt][0] *= a0;
                acc[mt][1] *= a1;
                acc[mt][2] *= a0;
                acc[mt][3] *= a1;
                const int dch = (32 * warp + 16 * mt) / 8 + (mi & 1);  // 16-byte dim chunk
#pragma unroll
                for (int pb = 0; pb < kTaC / 16; ++pb) {
                    uint32_t a[4];
                    ldsm_x4_t(a, vbuf + swz_off(pb * 16 + (mi >> 1) * 8 + r8, dch));
                    const __half* pr = &sh.pt[g8][pb * 16 + 2 * tig];
                    const uint2 bf = make_uint2(*reinterpret_cast<const uint32_t*>(pr),
                                                *reinterpret_cast<const uint32_t*>(pr + 8));
                    mma16816(acc[mt], a, bf);
                }
            }
        }
        if (seg_end) {
            // O[d][h] = hi column + lo column; lanes with tig < 2 hold heads 2 tig, 2 tig + 1.
            float o[2][4];
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int e = 0; e < 4; ++e) o[mt][e] = acc[mt][e] + __shfl_xor_sync(0xffffffffu, acc[mt][e], 2);
            if (tig < 2) {
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int h = 2 * tig + (e & 1);
                        const int d = 32 * warp + 16 * mt + g8 + (e >> 1) * 8;
                        if (h < hpg)
                            part[(((size_t)b * n_heads + (size_t)g * hpg + h) * kTaSlots + seg_c) * kTaStride + d] =
                                o[mt][e];
                    }
            }
            if (tid < hpg) {
                float* st = part + (((size_t)b * n_heads + (size_t)g * hpg + tid) * kTaSlots + seg_c) * kTaStride + kTaD;
                st[0] = sh.mrun[tid];
                st[1] = sh.lrun[tid];
            }
        }
        __syncthreads();  // both buffers and the softmax state are free for the next item
    }
    if (fail_it >= 0 && tid == 0) {
        // Copies still in flight (this item's, and the next one's) land before
        // the CTA exits (bounded waits).
        const int k = (int)(fail_it - i0);
        mbar_wait(&sh.full[k & 1], (uint32_t)((k >> 1) & 1));
        if (fail_it + 1 < i1) mbar_wait(&sh.full[(k + 1) & 1], (uint32_t)(((k + 1) >> 1) & 1));
    }
}

// Row b, query head h of the O projection's input: the merge of the head's
// segment partials (the slots of chunks that start a CTA share, and chunk
// 0), weights e^(m_s - M) / sum_s l_s e^(m_s - M), written as fp16 hi / lo
// into the tensor-core GEMM's prepared tiles (the layout of tc_prep: per
// 64-column block kb and row r, 128 bytes with 16-byte chunks XOR r & 7; lo
// rows at nb / 2 + b). Rows b >= B are zero. One thread per dim.
__global__ void __launch_bounds__(kTaD) bat_attn_merge_prep_kernel(const float* part, const int* pos, int B,
                                                                   int n_heads, int kvh, int G, int nb, uint8_t* xt) {
    __shared__ long long start[kTaMaxB + 1];
    __shared__ int ps[kTaMaxB];
    __shared__ float wsm[kTaSlots];
    __shared__ float red[kTaD / 32];
    __shared__ int vlist[kTaSlots];       // the valid slots, in increasing order
    __shared__ int wcount[kTaD / 32];
    griddep_wait();
    griddep_launch();
    const int b = blockIdx.x, h = blockIdx.y, d = threadIdx.x, lane = d & 31, warp = d >> 5;
    float v = 0.0f;
    if (b < B) {
        if (warp == 0) item_prefix(pos, B, kvh, start, ps, lane);
        __syncthreads();
        const long long T = start[B];
        const int n = seq_chunks(ps[b]), hpg = n_heads / kvh, g = h / hpg;
        const long long F = start[b] + (long long)g * n;
        const float* ph = part + ((size_t)b * n_heads + h) * kTaSlots * kTaStride;
        const bool valid = d < n && (d == 0 || starts_share(T, G, F + d));
        float mc = -INFINITY, lc = 0.0f;
        if (valid) {
            mc = __ldcg(ph + (size_t)d * kTaStride + kTaD);
            lc = __ldcg(ph + (size_t)d * kTaStride + kTaD + 1);
        }
        // The valid slots, compacted in increasing order, so that their
        // partial rows can be loaded together (they need no weights yet).
        const unsigned int bal = __ballot_sync(0xffffffffu, valid);
        if (lane == 0) wcount[warp] = __popc(bal);
        float M = mc;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
        if (lane == 0) red[warp] = M;
        __syncthreads();
        int off = 0, nval = 0;
#pragma unroll
        for (int w = 0; w < kTaD / 32; ++w) {
            off += w < warp ? wcount[w] : 0;
            nval += wcount[w];
        }
        if (valid) vlist[off + __popc(bal & ((1u << lane) - 1u))] = d;
        M = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
        __syncthreads();
        constexpr int kBatch = 8;
        float ov[kBatch];
#pragma unroll
        for (int j = 0; j < kBatch; ++j) ov[j] = j < nval ? __ldcg(ph + (size_t)vlist[j] * kTaStride + d) : 0.0f;
        const float e = valid ? expf(mc - M) : 0.0f;
        float L = lc * e;
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
        if (lane == 0) red[warp] = L;
        wsm[d] = e;
        __syncthreads();
        L = red[0] + red[1] + red[2] + red[3];
        // Same terms in the same order as a walk over every slot: the valid
        // slots by increasing index, skipping weights that underflow to 0.
        float acc = 0.0f;
        for (int i0 = 0; i0 < nval; i0 += kBatch) {
            if (i0 > 0)
#pragma unroll
                for (int j = 0; j < kBatch; ++j)
                    ov[j] = i0 + j < nval ? __ldcg(ph + (size_t)vlist[i0 + j] * kTaStride + d) : 0.0f;
#pragma unroll
            for (int j = 0; j < kBatch; ++j) {
                if (i0 + j < nval) {
                    const float w = wsm[vlist[i0 + j]];
                    if (w != 0.0f) acc = fmaf(w, ov[j], acc);
                }
            }
        }
        v = acc / fmaxf(L, 1e-20f);
    }
    const int col = h * kTaD + d, kb = col >> 6, cc = col & 63;
    const __half hi = __float2half_rn(v), lo = __float2half_rn(v - __half2float(hi));
    const int rlo = nb / 2 + b;
    *reinterpret_cast<__half*>(xt + ((size_t)kb * nb + b) * 128 + ((((cc >> 3) ^ (b & 7)) << 4)) + (cc & 7) * 2) = hi;
    *reinterpret_cast<__half*>(xt + ((size_t)kb * nb + rlo) * 128 + ((((cc >> 3) ^ (rlo & 7)) << 4)) + (cc & 7) * 2) = lo;
}

cudaError_t launch_pdl_ex(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args) {
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

}  // namespace

bool batch_tc_attention_supported(int n_heads, int kvh, int D, int max_batch, int cap) {
    return D == kTaD && kvh > 0 && n_heads % kvh == 0 && n_heads / kvh <= kTaMaxHpg && max_batch <= kTaMaxB &&
           cap <= kTaSlots * kTaC;
}

size_t batch_tc_attention_part_floats(int B, int n_heads) {
    return (size_t)B * n_heads * kTaSlots * kTaStride;
}

cudaError_t batch_tc_attention_configure(int sm_count, int* grid) {
    cudaError_t e = cudaFuncSetAttribute(bat_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sizeof(TaShared));
    if (e != cudaSuccess) return e;
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, bat_attn_tc_kernel, kTaThreads, sizeof(TaShared));
    if (e != cudaSuccess) return e;
    *grid = sm_count * (occ < 1 ? 1 : occ);
    return cudaSuccess;
}

cudaError_t launch_batch_tc_attention(const float* qkv, int rows, const float* cosv, const float* sinv, int rot,
                                      __half* kc, __half* vc, int cap, int n_heads, int kvh, float scale,
                                      const int* pos, int B, float* part, int grid, int* status, cudaStream_t s) {
    if (rot < 0 || rot > kTaD || (rot & 1)) return cudaErrorInvalidValue;
    void* args[] = {(void*)&qkv, &rows, (void*)&cosv, (void*)&sinv, &rot, (void*)&kc, (void*)&vc, &cap, &n_heads,
                    &kvh, &scale, (void*)&pos, &B, &part, &status};
    return launch_pdl_ex((const void*)bat_attn_tc_kernel, dim3(grid), dim3(kTaThreads), sizeof(TaShared), s, args);
}

cudaError_t launch_batch_attn_merge_prep(const float* part, const int* pos, int B, int n_heads, int kvh, int grid,
                                         void* xt, cudaStream_t s) {
    int nb = tc_width(B, AEXIS_F32);
    uint8_t* xtp = reinterpret_cast<uint8_t*>(xt);
    void* args[] = {(void*)&part, (void*)&pos, &B, &n_heads, &kvh, &grid, &nb, &xtp};
    return launch_pdl_ex((const void*)bat_attn_merge_prep_kernel, dim3(nb / 2, n_heads), dim3(kTaD), 0, s, args);
}
