// k_decoder_persist.cu -- the batch-1 greedy decode loop as one persistent
// kernel: every decode step of a generate call, every layer, in one
// cooperative launch with one CTA per SM.
//
// Same computation as the per-step graph of k_decoder.cu (Qwen35DecoderSession
// DecodeCore + SelectNextToken, greedy; Qwen35DecoderSession.cs:463-585,
// 715-810), the same fragment-layout weights and the same numerics (fp32
// activations as fp16 hi + lo MMA operands, fp32 sums). What changes is the
// schedule. In the graph, each of the ~120 kernels of a step waits for its
// predecessor to finish and drain before it reads its input. Here a step is
// a sequence of phases separated by a grid barrier:
//   per layer  QKV   RMSNorm + GEMV + RoPE + fp16 KV append (layer 0 reads
//                    the token's embedding row and seeds the residual h)
//              ATT   split attention over 32-position chunks; the last CTA
//                    of a KV head merges the splits
//              O     GEMV, residual add into h
//              GU    RMSNorm + gate|up GEMV + SiLU * up
//              DOWN  GEMV, residual add into h
//   lm_head    RMSNorm + GEMV, logits + greedy key (atomicMax)
// and the weights never wait for a barrier: warp 0 of every CTA streams the
// CTA's share of every GEMV phase, in phase order and across steps, through
// a ring of bulk copies (units of 16 rows x 512 K: 4 KB of fragment words and
// 512 B of scales), as far ahead as the ring allows. The 16 consumer warps
// run the phases: after a barrier they stage the input vector as MMA
// fragments, take their units from the ring (unit j of a phase by warp
// j % 16), leave per-unit row partials in shared memory, then sum the K
// chunks of each row and apply the epilogue.
//
// The grid barrier is a monotonically increasing arrival counter; every
// spin (barrier, ring) is bounded and a CTA that gives up records
// AEXIS_E_TIMEOUT and raises an abort flag that ends every other CTA's waits.
// Values produced by other CTAs are read through L2 (ld.global.cg): L1 is not
// coherent between SMs.
#include <cmath>
#include <vector>

#include "decoder_internal.h"
#include "gemv_dev.cuh"
#include "mma_frag.cuh"

namespace {

using namespace aexis_dev;

constexpr int kPW = 16;                     // consumer warps
constexpr int kPConsumers = kPW * 32;       // 512
constexpr int kPThreads = kPConsumers + 32; // + the producer warp
constexpr int kPChunkK = 512;               // K per unit
constexpr int kPUnitW = kPChunkK / 16 * 128;  // 4096 B of Q4 fragment words (32 k16 blocks)
constexpr int kPUnitS = kPChunkK / 32 * 16 * 2;  // 512 B of fp16 scales (16 groups x 16 rows)
constexpr int kPStage = kPUnitW + kPUnitS;  // 4608 B
constexpr int kPStages = 32;                // a multiple of kPW
constexpr int kPGroup = 4;                  // stages filled by one bulk copy (a super-stage)
constexpr int kPSupers = kPStages / kPGroup;
constexpr int kPChunk = 32;                 // attention positions per split
constexpr int kPHeadDim = 128;
constexpr int kPMaxHpg = 4;
constexpr int kPMaxSplits = 64;             // 2048 positions
constexpr int kPMaxK = 4096;                // largest GEMV K (x fragments in shared memory)
constexpr int kPMaxRed = 68 * 2 * 16;       // row partials: tiles x chunks x 16 (lm_head at 148 SMs)

enum { PH_GEMV = 0, PH_ATTN = 1 };

struct PPhase {
    int kind;
    int n, k, ntiles, nchunks;
    const uint8_t* W;      // fragment words
    const uint8_t* S;      // fragment scales (fp16)
    const float* x;        // input vector; nullptr: the token's embedding row
    const float* gamma;    // RMSNorm weight (nullable)
    int epi;               // EPI_QKV_ROPE, EPI_RESIDUAL, EPI_SWIGLU, EPI_LOGITS_ARGMAX
    float* y;
    __half* kc;            // this layer's caches [kvh][cap][D]
    __half* vc;
    int merge;             // x = the attention output, merged here from the split partials
};

struct PArgs {
    const PPhase* phases;
    int nphases;           // phases of one step
    int nsteps;
    const __half* embed;
    int vocab, hidden;
    float* h;
    const int* rope_map;
    const float* rope_cos;
    const float* rope_sin;
    int rot_dim, kv_cap, n_heads, kvh;
    float eps, attn_scale;
    float* q;
    float* attn;
    float* part;           // [n_heads][kPMaxSplits][D + 2]
    unsigned long long* keys;  // [2], zero at launch
    const uint8_t* stream;     // every CTA's units of one step, CTA-major (persist_pack_kernel)
    const long long* stream_off;  // [G + 1]: CTA b's units start at unit stream_off[b]
    int* ints;             // [0] token, [1] position, [2] output cursor, [3..] output tokens
    int max_out;
    unsigned int* bar;     // arrival counter, zero at launch
    int* abort_flag;       // zero at launch
    int* status;
};

constexpr int kPMaxHeads = kPMaxK / kPHeadDim;

struct PShared {
    __half xs[2 * kPMaxK + 64];      // x fragments: hi, lo (+ a zero block)
    float red[kPMaxRed];             // row partials [tile][chunk][16]
    float redn[kPW];
    float mw[kPMaxHeads][kPMaxSplits];  // attention split weights (O phase)
    float ml[kPMaxHeads][kPMaxSplits];
};

struct AShared {
    __align__(16) __half k[kPChunk * kPHeadDim];
    __align__(16) __half v[kPChunk * kPHeadDim];
    float qv[kPMaxHpg][kPHeadDim];
    float sc[kPChunk][kPMaxHpg];
    float stat[kPMaxHpg][2];
    float ored[8][kPMaxHpg][kPHeadDim];
};

__device__ __forceinline__ unsigned int ld_acquire(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void csync() { named_sync(1, kPConsumers); }

__device__ __forceinline__ void red_release_add(unsigned int* p, unsigned int v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Grid barrier over the consumer warps of every CTA: arrival `index`
// (0-based) completes when the arrival counter reaches (index + 1) *
// gridDim.x. The arrival is a release (it publishes every write the CTA's
// consumer warps made before the CTA barrier), the polls are acquires. False
// when this CTA gave up (timeout, or another CTA's abort).
__device__ bool grid_sync(const PArgs& a, unsigned int index, int* s_flag) {
    csync();
    if (threadIdx.x == 32) {
        red_release_add(a.bar, 1u);
        const unsigned int target = (index + 1u) * gridDim.x;
        int ok = 1;
        if (ld_acquire(a.bar) < target) {
            const long long t0 = clock64();
            for (unsigned int n = 1; ld_acquire(a.bar) < target; ++n) {
                if ((n & 31u) == 0u) {
                    if (*(volatile int*)a.abort_flag) {
                        ok = 0;
                        break;
                    }
                    if (clock64() - t0 > kWaitLimitCycles) {
                        report_timeout(a.status);
                        atomicExch(a.abort_flag, 1);
                        ok = 0;
                        break;
                    }
                }
            }
        }
        *s_flag = ok;
    }
    csync();
    return *s_flag != 0;
}

// Units of CTA b in a GEMV phase: its tiles b, b + G, ... times the K chunks.
__device__ __forceinline__ int phase_units(const PPhase& p, int b, int G) {
    const int tiles = p.ntiles > b ? (p.ntiles - b + G - 1) / G : 0;
    return tiles * p.nchunks;
}

// Warps per unit (K split inside a unit) so that a phase with few units per
// CTA still keeps the 16 consumer warps busy: 1, 2, 4 or 8.
__device__ __forceinline__ int warps_per_unit(int U) {
    int nw = 1;
    while (nw < 8 && U * nw * 2 <= kPW) nw <<= 1;
    return nw;
}

// x (or the token's embedding row) -> fp16 hi/lo B fragments in sh.xs,
// RMS-normalised first when the phase has a gamma (the fused RMSNorm layer).
// Fragment order as in the tensor-core GEMV: for every four k16 blocks, lane
// t (0..3) owns 32 contiguous bytes (blocks kb..kb+3, registers b0 b1 each);
// the lo plane follows the hi plane in the same order. One L2 round trip:
// every thread loads its (at most kPMaxK / 512) values once.
__device__ void stage_x(const PArgs& a, const PPhase& p, int token, int pos, PShared& sh) {
    constexpr int kPer = kPMaxK / kPConsumers;
    const int t = threadIdx.x - 32, lane = t & 31, warp = t >> 5;
    const int k = p.k, nkb = k >> 4;
    float v[kPer];
    if (p.merge) {
        // The attention output, head h = e / D: the splits' partial sums o_s
        // with weights e^(m_s - M) / sum_s l_s e^(m_s - M) (the reference's
        // two-pass softmax, HLSL Pack4Matmul:485-547, merged over splits).
        constexpr int D = kPHeadDim, stride = D + 2;
        constexpr int kBatch = 16;  // splits whose partials are in flight at once
        const int nh = k / D, nsplit = (pos + kPChunk) / kPChunk;
        // The first kBatch splits of this thread's two elements: loads issued
        // now, before (and independent of) the split weights.
        float o[2][kBatch];
#pragma unroll
        for (int j = 0; j < 2; ++j) {
            const int e = t + j * kPConsumers;
            const int h = e / D, dd = e - h * D;
            const float* src = a.part + (size_t)h * kPMaxSplits * stride + dd;
#pragma unroll
            for (int sp = 0; sp < kBatch; ++sp)
                o[j][sp] = e < k && sp < nsplit ? __ldcg(src + (size_t)sp * stride) : 0.0f;
        }
        for (int i = t; i < nh * nsplit; i += kPConsumers) {
            const int h = i / nsplit, sp = i - h * nsplit;
            const float* st = a.part + ((size_t)h * kPMaxSplits + sp) * stride + D;
            sh.mw[h][sp] = __ldcg(st);
            sh.ml[h][sp] = __ldcg(st + 1);
        }
        csync();
        for (int h = warp; h < nh; h += kPW) {
            float M = -INFINITY;
            for (int sp = lane; sp < nsplit; sp += 32) M = fmaxf(M, sh.mw[h][sp]);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, o));
            float L = 0.0f;
            for (int sp = lane; sp < nsplit; sp += 32) {
                const float e = expf(sh.mw[h][sp] - M);
                sh.mw[h][sp] = e;
                L += sh.ml[h][sp] * e;
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) L += __shfl_xor_sync(0xffffffffu, L, o);
            const float inv = 1.0f / fmaxf(L, 1e-20f);
            __syncwarp();
            for (int sp = lane; sp < nsplit; sp += 32) sh.mw[h][sp] *= inv;
        }
        csync();
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int e = t + j * kPConsumers;
            float acc = 0.0f;
            if (e < k) {
                const int h = e / D, dd = e - h * D;
                const float* src = a.part + (size_t)h * kPMaxSplits * stride + dd;
                if (j < 2) {
#pragma unroll
                    for (int sp = 0; sp < kBatch; ++sp)
                        if (sp < nsplit) acc = fmaf(sh.mw[h][sp], o[j][sp], acc);
                } else {
                    for (int sp = 0; sp < kBatch && sp < nsplit; ++sp)
                        acc = fmaf(sh.mw[h][sp], __ldcg(src + (size_t)sp * stride), acc);
                }
                for (int sp = kBatch; sp < nsplit; ++sp) acc = fmaf(sh.mw[h][sp], __ldcg(src + (size_t)sp * stride), acc);
            }
            v[j] = acc;
        }
    } else {
        const __half* erow = a.embed + (long long)token * a.hidden;
        const bool emb = p.x == nullptr;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int e = t + j * kPConsumers;
            v[j] = e < k ? (emb ? __half2float(erow[e]) : __ldcg(p.x + e)) : 0.0f;
        }
    }
    float gm[kPer];  // the norm weights, read together with x
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int e = t + j * kPConsumers;
        gm[j] = p.gamma != nullptr && e < k ? __ldg(p.gamma + e) : 1.0f;
    }
    if (p.gamma != nullptr) {
        float ss = 0.0f;
#pragma unroll
        for (int j = 0; j < kPer; ++j) ss = fmaf(v[j], v[j], ss);
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) sh.redn[warp] = ss;
        csync();
        float tot = 0.0f;
#pragma unroll
        for (int w = 0; w < kPW; ++w) tot += sh.redn[w];
        const float inv = 1.0f / sqrtf(fmaxf(tot / (float)k + a.eps, 1e-20f));
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
            const int e = t + j * kPConsumers;
            if (e < k) v[j] = v[j] * inv * gm[j];
        }
    }
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
        const int e = t + j * kPConsumers;
        if (e < k) {
            const int slot = q4_x_slot(e);
            const __half hi = __float2half_rn(v[j]);
            sh.xs[slot] = hi;
            sh.xs[nkb * 16 + slot] = __float2half_rn(v[j] - __half2float(hi));
        }
    }
    if (t < 8) reinterpret_cast<uint32_t*>(sh.xs + 2 * nkb * 16)[t] = 0u;  // the zero block
    csync();
}

// One warp's share of a unit (16 rows x 512 K, K chunk c): IT four-block
// steps from step q0, copied out of the ring stage into registers so the
// stage can be released before the MMAs run: a 16-byte word per step (the
// lane's A fragments of four k16 blocks) and the lane's row-pair scales of
// the step's two groups.
template <int IT>
struct UnitRegs {
    uint4 w[IT];
    uint32_t sc[2 * IT];
};

template <int IT>
__device__ __forceinline__ void unit_load(const uint8_t* st, int q0, int lane, UnitRegs<IT>& r) {
    const uint32_t* sc = reinterpret_cast<const uint32_t*>(st + kPUnitW) + (lane >> 2);  // (row g, row g + 8)
#pragma unroll
    for (int i = 0; i < IT; ++i) {
        r.w[i] = *reinterpret_cast<const uint4*>(st + ((size_t)(q0 + i) * 32 + lane) * 16);
        r.sc[2 * i] = sc[(2 * (q0 + i)) * 8];
        r.sc[2 * i + 1] = sc[(2 * (q0 + i) + 1) * 8];
    }
}

// Rows g and g + 8 (g = lane / 4; valid in lanes with lane % 4 == 0) of the
// warp's share. B column 0 carries x hi (lanes 0-3), column 1 x lo (lanes
// 4-7), the other columns zero, so one MMA per k16 block gives both partial
// sums. Groups of 32 K: a fresh accumulator every two blocks, its column sum
// added to the row sum with the group's scale.
template <int IT>
__device__ __forceinline__ void unit_mma(const UnitRegs<IT>& r, const __half* xs, int nkb, int c, int q0, int lane,
                                         float& y0, float& y1) {
    const uint4* xz = reinterpret_cast<const uint4*>(xs + 2 * nkb * 16);
    const uint4* xb_ptr = lane < 4 ? reinterpret_cast<const uint4*>(xs) + lane * 2
                                   : (lane < 8 ? reinterpret_cast<const uint4*>(xs + nkb * 16) + (lane - 4) * 2 : xz);
    const int xstep = lane < 8 ? 8 : 0;  // uint4 per four blocks
    y0 = 0.0f;
    y1 = 0.0f;
#pragma unroll
    for (int i = 0; i < IT; ++i) {
        const uint32_t words[4] = {r.w[i].x, r.w[i].y, r.w[i].z, r.w[i].w};
        const int xb = (c * (kPChunkK / 64) + q0 + i) * xstep;
        const uint4 b01 = xb_ptr[xb], b23 = xb_ptr[xb + 1];
        const uint2 bf[4] = {make_uint2(b01.x, b01.y), make_uint2(b01.z, b01.w), make_uint2(b23.x, b23.y),
                             make_uint2(b23.z, b23.w)};
        float acc[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t af[4];
            decode_frag(words[j], af);
            if ((j & 1) == 0) mma16816_zc(acc, af, bf[j]);
            else mma16816(acc, af, bf[j]);
            if (j & 1) {
                const __half2 s2 = *reinterpret_cast<const __half2*>(&r.sc[2 * i + (j >> 1)]);
                y0 = fmaf(acc[0] + acc[1], __low2float(s2), y0);
                y1 = fmaf(acc[2] + acc[3], __high2float(s2), y1);
            }
        }
    }
}

// The units of warp group gi (units gi, gi + NG, ...), NW = 8 / IT warps per
// unit, this warp's share starting at step sub * IT. Each unit's stage is
// released as soon as its share is in registers.
template <int IT>
__device__ __forceinline__ bool run_units(const PArgs& a, const PPhase& p, const uint8_t* ring, uint64_t* full,
                                          uint64_t* empty, unsigned long long seq, int U, PShared& sh, int lane,
                                          int warp) {
    constexpr int NW = 8 / IT, NG = kPW / NW;
    const int gi = warp / NW, sub = warp % NW, q0 = sub * IT;
    const int nkb = p.k >> 4;
    for (int j = gi; j < U; j += NG) {
        const unsigned long long i = seq + (unsigned long long)j;
        const int s = (int)(i % kPStages);
        if (!mbar_wait(full + s / kPGroup, (uint32_t)((i / kPStages) & 1))) {
            if (lane == 0) {
                report_timeout(a.status);
                atomicExch(a.abort_flag, 1);
            }
            return false;
        }
        UnitRegs<IT> r;
        unit_load<IT>(ring + (size_t)s * kPStage, q0, lane, r);
        __syncwarp();
        if (lane == 0) mbar_arrive_cnt(empty + s / kPGroup, IT);
        float y0, y1;
        unit_mma<IT>(r, sh.xs, nkb, j % p.nchunks, q0, lane, y0, y1);
        if ((lane & 3) == 0) {
            sh.red[(j * NW + sub) * 16 + (lane >> 2)] = y0;
            sh.red[(j * NW + sub) * 16 + (lane >> 2) + 8] = y1;
        }
    }
    return true;
}

// Per-row operands of an epilogue that do not depend on the MMA: the
// residual input (EPI_RESIDUAL, final since the last barrier) or the RoPE
// destination and angle (EPI_QKV_ROPE). Read at the start of a phase so the
// loads overlap the staging and the MMAs.
struct RowPre {
    float resid, c, s;
    int desc;
};

__device__ __forceinline__ RowPre row_pre(const PArgs& a, const PPhase& p, int row, int pos) {
    RowPre r = {0.0f, 1.0f, 0.0f, 0};
    if (p.epi == EPI_RESIDUAL) {
        r.resid = __ldcg(p.y + row);
    } else if (p.epi == EPI_QKV_ROPE) {
        r.desc = __ldg(a.rope_map + row);
        const int kind = r.desc >> 24, dim = r.desc & 0xFFF;
        if (kind != 2 && dim < a.rot_dim) {
            const int half = a.rot_dim >> 1;
            const int j = dim < half ? dim : dim - half;
            r.c = __ldg(a.rope_cos + (long long)pos * half + j);
            r.s = __ldg(a.rope_sin + (long long)pos * half + j);
        }
    }
    return r;
}

// One row's output (the graph's GEMV epilogues, with cross-CTA values read
// through L2). partner: the value of row ^ 1; pre: row_pre of the row.
__device__ __forceinline__ void persist_epilogue(const PArgs& a, const PPhase& p, int row, float val, float partner,
                                                 const RowPre& pre, int pos, unsigned long long& best) {
    switch (p.epi) {
        case EPI_RESIDUAL:
            p.y[row] = pre.resid + val;
            break;
        case EPI_SWIGLU:
            if ((row & 1) == 0) p.y[row >> 1] = val / (1.0f + expf(-val)) * partner;
            break;
        case EPI_QKV_ROPE: {
            const int desc = pre.desc;
            const int kind = desc >> 24, head = (desc >> 12) & 0xFFF, dim = desc & 0xFFF;
            float out = val;
            if (kind != 2 && dim < a.rot_dim) {
                const bool first = dim < (a.rot_dim >> 1);
                const float x0 = first ? val : partner, x1 = first ? partner : val;
                out = first ? x0 * pre.c - x1 * pre.s : x0 * pre.s + x1 * pre.c;
            }
            if (kind == 0) {
                a.q[head * kPHeadDim + dim] = out;
            } else {
                __half* cache = kind == 1 ? p.kc : p.vc;
                cache[((long long)head * a.kv_cap + pos) * kPHeadDim + dim] = __float2half_rn(out);
            }
        } break;
        case EPI_LOGITS_ARGMAX: {
            p.y[row] = val;
            const unsigned long long key = aexis_argmax_key(val, row);
            best = key > best ? key : best;
        } break;
    }
}

// A GEMV phase on the consumer warps. seq: this CTA's unit counter (the same
// sequence the producer fills the ring in). NW warps share a unit (K split);
// the NG = 16 / NW warp groups take units g, g + NG, ... Consecutive fills of
// a stage are units kPStages apart, so the same group takes them, in order
// (NG divides the ring depth). False when a ring wait gave up.
__device__ bool gemv_phase(const PArgs& a, const PPhase& p, const uint8_t* ring, uint64_t* full, uint64_t* empty,
                           unsigned long long& seq, int token, int pos, unsigned long long* key, PShared& sh) {
    const int t = threadIdx.x - 32, lane = t & 31, warp = t >> 5;
    const int b = blockIdx.x, G = gridDim.x;
    const int U = phase_units(p, b, G);
    const int tl_count = U / p.nchunks;
    // The epilogue operands of the row this thread finishes first.
    RowPre pre0 = {0.0f, 1.0f, 0.0f, 0};
    if (t < tl_count * 16) {
        const int row = (b + (t >> 4) * G) * 16 + (t & 15);
        if (row < p.n) pre0 = row_pre(a, p, row, pos);
    }
    if (U == 0) return true;  // nothing to multiply: no input to stage
    stage_x(a, p, token, pos, sh);
    const int NW = warps_per_unit(U);
    bool ok;
    switch (NW) {
        case 8: ok = run_units<1>(a, p, ring, full, empty, seq, U, sh, lane, warp); break;
        case 4: ok = run_units<2>(a, p, ring, full, empty, seq, U, sh, lane, warp); break;
        case 2: ok = run_units<4>(a, p, ring, full, empty, seq, U, sh, lane, warp); break;
        default: ok = run_units<8>(a, p, ring, full, empty, seq, U, sh, lane, warp); break;
    }
    seq += (unsigned long long)U;
    csync();
    unsigned long long best = 0ull;
    const int parts = p.nchunks * NW;
    for (int e = t; e < tl_count * 16; e += kPConsumers) {
        const int tl = e >> 4, r = e & 15;
        const float* rp = sh.red + tl * parts * 16;
        float v = 0.0f, pv = 0.0f;
        for (int c = 0; c < parts; ++c) {
            v += rp[c * 16 + r];
            pv += rp[c * 16 + (r ^ 1)];
        }
        const int row = (b + tl * G) * 16 + r;
        if (row < p.n) persist_epilogue(a, p, row, v, pv, e == t ? pre0 : row_pre(a, p, row, pos), pos, best);
    }
    if (p.epi == EPI_LOGITS_ARGMAX) {
#pragma unroll
        for (int o = 16; o >= 1; o >>= 1) {
            const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
            best = other > best ? other : best;
        }
        if (lane == 0 && best != 0ull) atomicMax(key, best);
    }
    return ok;
}

// An attention phase: items (KV head g, 32-position split) of ctx = pos + 1
// positions, item i on CTA i % G. Per item: K and V of the split into shared
// memory, scores (q . k) * scale for the hpg query heads of g (GQA kv = h /
// (H / Hkv)), split max m, sum l and o = sum e * v into the partials; the O
// phase that follows merges the splits while staging its input.
// This thread's K and V row slice of the CTA's first attention item, for
// every position but the newest (the QKV phase writes that one): read before
// the barrier that precedes the attention phase.
__device__ __forceinline__ void attn_prefetch(const PArgs& a, const PPhase& att, int pos, uint4& kpre, uint4& vpre) {
    const int t = threadIdx.x - 32;
    const int ctx = pos + 1;
    const int nsplit = (ctx + kPChunk - 1) / kPChunk;
    const int item = blockIdx.x;
    if (item >= a.kvh * nsplit) return;
    const int g = item / nsplit, split = item - g * nsplit;
    const int p0 = split * kPChunk, np = min(kPChunk, ctx - p0);
    const int pp = t >> 4, d8 = (t & 15) * 8;
    if (pp < np && p0 + pp != pos) {
        const size_t off = ((size_t)g * a.kv_cap + p0 + pp) * kPHeadDim + d8;
        kpre = __ldcg(reinterpret_cast<const uint4*>(att.kc + off));
        vpre = __ldcg(reinterpret_cast<const uint4*>(att.vc + off));
    }
}

__device__ void attn_phase(const PArgs& a, const PPhase& p, int pos, AShared& as, uint4 kpre, uint4 vpre) {
    const int t = threadIdx.x - 32, lane = t & 31, warp = t >> 5;
    const int hpg = a.n_heads / a.kvh;
    const int ctx = pos + 1;
    const int nsplit = (ctx + kPChunk - 1) / kPChunk;
    const int items = a.kvh * nsplit;
    constexpr int D = kPHeadDim, stride = D + 2;
    for (int item = blockIdx.x; item < items; item += gridDim.x) {
        const int g = item / nsplit, split = item - g * nsplit;
        const int p0 = split * kPChunk, np = min(kPChunk, ctx - p0);
        {
            const int pp = t >> 4, d8 = (t & 15) * 8;
            if (pp < np) {
                uint4 kr = kpre, vr = vpre;
                if (item != (int)blockIdx.x || p0 + pp == pos) {
                    const size_t off = ((size_t)g * a.kv_cap + p0 + pp) * D + d8;
                    kr = __ldcg(reinterpret_cast<const uint4*>(p.kc + off));
                    vr = __ldcg(reinterpret_cast<const uint4*>(p.vc + off));
                }
                *reinterpret_cast<uint4*>(as.k + pp * D + d8) = kr;
                *reinterpret_cast<uint4*>(as.v + pp * D + d8) = vr;
            }
            for (int i = t; i < hpg * D; i += kPConsumers) as.qv[i / D][i % D] = __ldcg(a.q + g * hpg * D + i);
        }
        csync();
        // Scores: 16 threads per position, 8 dims each.
        {
            const int pp = t >> 4, d8 = (t & 15) * 8;
            float acc[kPMaxHpg] = {0.0f, 0.0f, 0.0f, 0.0f};
            if (pp < np) {
                const uint4 raw = *reinterpret_cast<const uint4*>(as.k + pp * D + d8);
                const __half2* k2 = reinterpret_cast<const __half2*>(&raw);
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 kf = __half22float2(k2[e]);
#pragma unroll
                    for (int h = 0; h < kPMaxHpg; ++h)
                        if (h < hpg) acc[h] = fmaf(as.qv[h][d8 + 2 * e + 1], kf.y, fmaf(as.qv[h][d8 + 2 * e], kf.x, acc[h]));
                }
            }
#pragma unroll
            for (int h = 0; h < kPMaxHpg; ++h)
#pragma unroll
                for (int o = 8; o >= 1; o >>= 1) acc[h] += __shfl_xor_sync(0xffffffffu, acc[h], o);
            if ((t & 15) == 0 && pp < np)
#pragma unroll
                for (int h = 0; h < kPMaxHpg; ++h)
                    if (h < hpg) as.sc[pp][h] = acc[h] * a.attn_scale;
        }
        csync();
        if (warp < hpg) {
            const int h = warp;
            float m = -INFINITY;
            for (int i = lane; i < np; i += 32) m = fmaxf(m, as.sc[i][h]);
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
            float l = 0.0f;
            for (int i = lane; i < np; i += 32) {
                const float e = expf(as.sc[i][h] - m);
                as.sc[i][h] = e;
                l += e;
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
            if (lane == 0) {
                as.stat[h][0] = m;
                as.stat[h][1] = l;
            }
        }
        csync();
        // Values: dims (2 dp, 2 dp + 1), positions pg, pg + 8, ...
        {
            const int dp = t & 63, pg = t >> 6;
            float o0[kPMaxHpg] = {0.0f, 0.0f, 0.0f, 0.0f}, o1[kPMaxHpg] = {0.0f, 0.0f, 0.0f, 0.0f};
            for (int pp = pg; pp < np; pp += 8) {
                const float2 v = __half22float2(*reinterpret_cast<const __half2*>(as.v + pp * D + 2 * dp));
#pragma unroll
                for (int h = 0; h < kPMaxHpg; ++h)
                    if (h < hpg) {
                        const float e = as.sc[pp][h];
                        o0[h] = fmaf(e, v.x, o0[h]);
                        o1[h] = fmaf(e, v.y, o1[h]);
                    }
            }
#pragma unroll
            for (int h = 0; h < kPMaxHpg; ++h)
                if (h < hpg) *reinterpret_cast<float2*>(&as.ored[pg][h][2 * dp]) = make_float2(o0[h], o1[h]);
        }
        csync();
        for (int i = t; i < hpg * D; i += kPConsumers) {
            const int h = i / D, dd = i - h * D;
            float acc = 0.0f;
#pragma unroll
            for (int pg = 0; pg < 8; ++pg) acc += as.ored[pg][h][dd];
            a.part[((size_t)(g * hpg + h) * kPMaxSplits + split) * stride + dd] = acc;
        }
        if (t < hpg) {
            float* st = a.part + ((size_t)(g * hpg + t) * kPMaxSplits + split) * stride + D;
            st[0] = as.stat[t][0];
            st[1] = as.stat[t][1];
        }
        csync();
    }
}

// The persistent loop's weight stream: CTA b's units of one step (its tiles
// b, b + G, ... of every GEMV phase in phase order, K chunks in order), each
// unit 4 KB of fragment words then 512 B of scales, contiguous from unit
// stream_off[b]. One CTA per destination CTA, 16-byte copies.
__global__ void persist_pack_kernel(const PPhase* phases, int nphases, uint8_t* stream, const long long* stream_off) {
    const int b = blockIdx.x, G = gridDim.x;
    uint8_t* dst = stream + (size_t)stream_off[b] * kPStage;
    for (int ph = 0; ph < nphases; ++ph) {
        const PPhase& p = phases[ph];
        if (p.kind != PH_GEMV) continue;
        const int U = phase_units(p, b, G);
        for (int j = 0; j < U; ++j, dst += kPStage) {
            const size_t unit = (size_t)(b + (j / p.nchunks) * G) * p.nchunks + (j % p.nchunks);
            const uint4* w = reinterpret_cast<const uint4*>(p.W + unit * kPUnitW);
            const uint4* sc = reinterpret_cast<const uint4*>(p.S + unit * kPUnitS);
            for (int i = threadIdx.x; i < kPStage / 16; i += blockDim.x)
                reinterpret_cast<uint4*>(dst)[i] = i < kPUnitW / 16 ? w[i] : sc[i - kPUnitW / 16];
        }
    }
}

__global__ void __launch_bounds__(kPThreads, 1) decoder_persist_kernel(PArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)kPStages * kPStage);  // per super-stage
    uint64_t* empty = full + kPSupers;
    uint8_t* scratch = reinterpret_cast<uint8_t*>(full + 2 * kPStages);
    PShared& sh = *reinterpret_cast<PShared*>(scratch);
    AShared& as = *reinterpret_cast<AShared*>(scratch);  // the attention phases reuse the same bytes
    __shared__ int s_flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int b = blockIdx.x;
    if (threadIdx.x == 0) {
        for (int m = 0; m < kPSupers; ++m) {
            mbar_init(full + m, 1);
            mbar_init(empty + m, 8 * kPGroup);  // per unit, its warps arrive with their four-block steps (8 in all)
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        // This CTA's units of one step are contiguous in a.stream (units
        // [stream_off[b], stream_off[b + 1])); every step reads them again.
        // One bulk copy fills kPGroup consecutive stages (a super-stage).
        if (lane != 0) return;
        const uint64_t pol = policy_evict_first();
        const long long u0 = a.stream_off[b], ustep = a.stream_off[b + 1] - u0;
        const uint8_t* base = a.stream + (size_t)u0 * kPStage;
        const long long total = ustep * a.nsteps;
        long long fills = 0;
        for (long long i = 0; i < total; i += kPGroup, ++fills) {
            const int m = (int)(fills % kPSupers);
            if (fills >= kPSupers && !mbar_wait(empty + m, (uint32_t)(((fills / kPSupers) - 1) & 1))) break;
            if ((fills & 63) == 0 && *(volatile int*)a.abort_flag) break;
            const int n = (int)(total - i < kPGroup ? total - i : kPGroup);
            uint8_t* dst = ring + (size_t)m * kPGroup * kPStage;
            mbar_arrive_expect_tx(full + m, (uint32_t)n * kPStage);
            long long src = i % ustep;  // the step stream wraps around
            for (int done = 0; done < n;) {
                const int take = (int)(ustep - src < n - done ? ustep - src : n - done);
                bulk_g2s(dst + (size_t)done * kPStage, base + (size_t)src * kPStage, (uint32_t)take * kPStage, full + m,
                         pol);
                done += take;
                src = 0;
            }
        }
        // Copies still in flight land before the CTA may exit: the last
        // kPSupers fills are the latest fill of distinct super-stages.
        for (long long f = fills > kPSupers ? fills - kPSupers : 0; f < fills; ++f)
            if (!mbar_wait(full + (int)(f % kPSupers), (uint32_t)((f / kPSupers) & 1))) break;
        return;
    }

    // -------------------------------------------------------------- consumers
    const int t = threadIdx.x - 32;
    int token = __ldcg(a.ints);
    token = token < 0 ? 0 : (token >= a.vocab ? a.vocab - 1 : token);  // the embedding clamp of the graph path
    int pos = __ldcg(a.ints + 1);
    const int cursor = __ldcg(a.ints + 2);
    unsigned long long seq = 0ull;
    unsigned int nb = 0u;
    uint4 kpre = make_uint4(0u, 0u, 0u, 0u), vpre = kpre;
    for (int step = 0; step < a.nsteps; ++step) {
        unsigned long long* key = a.keys + (step & 1);
        for (int ph = 0; ph < a.nphases; ++ph) {
            const PPhase& p = a.phases[ph];
            if (p.kind == PH_GEMV) {
                if (ph == 0 && b == 0)  // the residual stream starts at the embedding row
                    for (int i = t; i < a.hidden; i += kPConsumers)
                        a.h[i] = __half2float(a.embed[(long long)token * a.hidden + i]);
                gemv_phase(a, p, ring, full, empty, seq, token, pos, key, sh);
                if (ph + 1 < a.nphases && a.phases[ph + 1].kind == PH_ATTN)
                    attn_prefetch(a, a.phases[ph + 1], pos, kpre, vpre);
            } else {
                // The other key buffer was last read before the previous barrier.
                if (ph == 1 && b == 0 && t == 0) a.keys[(step + 1) & 1] = 0ull;
                attn_phase(a, p, pos, as, kpre, vpre);
            }
            if (!grid_sync(a, nb++, &s_flag)) return;
        }
        token = aexis_argmax_index(__ldcg(key));
        if (b == 0 && t == 0 && cursor + step >= 0 && cursor + step < a.max_out) a.ints[3 + cursor + step] = token;
        ++pos;
    }
    if (b == 0 && t == 0) {
        a.ints[0] = token;
        a.ints[1] = pos;
        a.ints[2] = cursor + a.nsteps;
    }
}

constexpr size_t kPSyncBytes = 2048;

size_t persist_smem_bytes() {
    size_t u = sizeof(PShared) > sizeof(AShared) ? sizeof(PShared) : sizeof(AShared);
    return (size_t)kPStages * kPStage + 2 * kPStages * sizeof(uint64_t) + u;
}

}  // namespace

// Whether the persistent kernel runs this decoder: Q4 group-32 weights and
// lm_head with fp16 scales, every K a multiple of 512, head_dim 128, at most
// 4 query heads per KV head, contexts up to 2048, the row partials of every
// GEMV phase within the shared-memory budget, and a device that can hold
// one CTA per SM resident (cooperative launch).
bool decoder_persist_supported(const aexis_decoder* d, int sm_count) {
    const auto& c = d->cfg;
    if (d->hybrid) return false;  // the phase table covers full-attention layers only
    if (c.bits != 4 || c.lm_bits != 4 || c.group != 32 || c.lm_group != 32 || c.scale_dtype != AEXIS_F16) return false;
    if (c.head_dim != kPHeadDim || c.n_heads % c.n_kv_heads || c.n_heads / c.n_kv_heads > kPMaxHpg) return false;
    if (c.kv_capacity > kPChunk * kPMaxSplits) return false;
    const int qd = c.n_heads * c.head_dim;
    const int ks[3] = {c.hidden, qd, c.ffn};
    for (int k : ks)
        if (k % kPChunkK || k > kPMaxK) return false;
    auto red_ok = [&](int n, int k) {
        const int tiles = (n + 15) / 16;
        return (long long)((tiles + sm_count - 1) / sm_count) * (k / kPChunkK) * 16 <= kPMaxRed;
    };
    const int kvd = c.n_kv_heads * c.head_dim;
    if (!red_ok(qd + 2 * kvd, c.hidden) || !red_ok(c.hidden, qd) || !red_ok(2 * c.ffn, c.hidden) ||
        !red_ok(c.hidden, c.ffn) || !red_ok(c.vocab, c.hidden))
        return false;
    int dev = 0, coop = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess || !coop) return false;
    int maxsm = 0;
    if (cudaDeviceGetAttribute(&maxsm, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return false;
    return persist_smem_bytes() <= (size_t)maxsm;
}

// Runs `nsteps` greedy steps from the device state (ints[0] token, [1]
// position, [2] output cursor), one cooperative launch. The phase table is
// built on first use (pointers only; weights reloaded in place keep it valid).
cudaError_t decoder_persist_run(aexis_decoder* d, int nsteps, cudaStream_t s) {
    const auto& c = d->cfg;
    const int G = d->ctx->sm_count;
    cudaError_t e = cudaSuccess;
    if (!d->persist_phases) {
        std::vector<PPhase> ph;
        auto gemv = [&](const aexis_weights& w, const float* x, const float* gamma, int epi, float* y, __half* kc,
                        __half* vc) {
            PPhase p = {};
            p.kind = PH_GEMV;
            p.n = w.n;
            p.k = w.k;
            p.ntiles = (w.n + 15) / 16;
            p.nchunks = w.k / kPChunkK;
            p.W = reinterpret_cast<const uint8_t*>(w.frag);
            p.S = reinterpret_cast<const uint8_t*>(w.frag_scales);
            p.x = x;
            p.gamma = gamma;
            p.epi = epi;
            p.y = y;
            p.kc = kc;
            p.vc = vc;
            ph.push_back(p);
        };
        for (int l = 0; l < c.n_layers; ++l) {
            const auto& L = d->layers[l];
            __half* kc = d->kcache + (size_t)l * c.n_kv_heads * c.kv_capacity * c.head_dim;
            __half* vc = d->vcache + (size_t)l * c.n_kv_heads * c.kv_capacity * c.head_dim;
            gemv(L.qkv, l == 0 ? nullptr : d->h, L.norm[0], EPI_QKV_ROPE, d->q, kc, vc);
            PPhase at = {};
            at.kind = PH_ATTN;
            at.kc = kc;
            at.vc = vc;
            ph.push_back(at);
            gemv(L.o, d->attn, nullptr, EPI_RESIDUAL, d->h, nullptr, nullptr);
            ph.back().merge = 1;
            gemv(L.gateup, d->h, L.norm[1], EPI_SWIGLU, d->act, nullptr, nullptr);
            gemv(L.down, d->act, nullptr, EPI_RESIDUAL, d->h, nullptr, nullptr);
        }
        gemv(d->lm, d->h, d->final_norm, EPI_LOGITS_ARGMAX, d->logits, nullptr, nullptr);
        for (const PPhase& p : ph)
            if (p.kind == PH_GEMV && (!p.W || !p.S)) return cudaErrorNotSupported;
        // The weight stream: CTA b's units of one step from unit off[b].
        std::vector<long long> off(G + 1, 0);
        for (int b = 0; b < G; ++b) {
            long long u = 0;
            for (const PPhase& p : ph)
                if (p.kind == PH_GEMV) u += (long long)(p.ntiles > b ? (p.ntiles - b + G - 1) / G : 0) * p.nchunks;
            off[b + 1] = off[b] + u;
        }
        if (!d->persist_off) e = cudaMalloc(&d->persist_off, sizeof(long long) * (G + 1));
        if (e != cudaSuccess) return e;
        e = cudaMemcpy(d->persist_off, off.data(), sizeof(long long) * (G + 1), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return e;
        if (!d->persist_stream) e = cudaMalloc(&d->persist_stream, (size_t)off[G] * kPStage + 16);
        if (e != cudaSuccess) return e;
        d->persist_packed = false;
        if (!d->persist_sync) e = cudaMalloc(&d->persist_sync, kPSyncBytes);
        if (e != cudaSuccess) return e;
        e = cudaFuncSetAttribute(decoder_persist_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)persist_smem_bytes());
        if (e != cudaSuccess) return e;
        // The phase table last: its presence marks the state as built.
        void* buf = nullptr;
        e = cudaMalloc(&buf, sizeof(PPhase) * ph.size());
        if (e != cudaSuccess) return e;
        e = cudaMemcpy(buf, ph.data(), sizeof(PPhase) * ph.size(), cudaMemcpyHostToDevice);
        if (e != cudaSuccess) {
            cudaFree(buf);
            return e;
        }
        d->persist_phases = buf;
        d->persist_nphases = (int)ph.size();
    }
    if (!d->persist_packed) {  // first use, or weights reloaded since
        persist_pack_kernel<<<G, 256, 0, s>>>(reinterpret_cast<const PPhase*>(d->persist_phases), d->persist_nphases,
                                              reinterpret_cast<uint8_t*>(d->persist_stream),
                                              reinterpret_cast<const long long*>(d->persist_off));
        e = cudaGetLastError();
        if (e != cudaSuccess) return e;
        d->persist_packed = true;
    }
    // u32 [0]: the barrier's arrival counter; [32] the abort flag; bytes
    // [256, 272): the two greedy keys.
    e = cudaMemsetAsync(d->persist_sync, 0, kPSyncBytes, s);
    if (e != cudaSuccess) return e;
    PArgs a = {};
    a.phases = reinterpret_cast<const PPhase*>(d->persist_phases);
    a.stream = reinterpret_cast<const uint8_t*>(d->persist_stream);
    a.stream_off = reinterpret_cast<const long long*>(d->persist_off);
    a.nphases = d->persist_nphases;
    a.nsteps = nsteps;
    a.embed = d->embed;
    a.vocab = c.vocab;
    a.hidden = c.hidden;
    a.h = d->h;
    a.rope_map = d->rope_map;
    a.rope_cos = d->rope_cos;
    a.rope_sin = d->rope_sin;
    a.rot_dim = c.rot_dim;
    a.kv_cap = c.kv_capacity;
    a.n_heads = c.n_heads;
    a.kvh = c.n_kv_heads;
    a.eps = c.eps;
    a.attn_scale = 1.0f / sqrtf((float)c.head_dim);
    a.q = d->q;
    a.attn = d->attn;
    a.part = d->part;
    unsigned int* sync = reinterpret_cast<unsigned int*>(d->persist_sync);
    a.bar = sync;
    a.abort_flag = reinterpret_cast<int*>(sync + 32);
    a.keys = reinterpret_cast<unsigned long long*>(sync + 64);
    a.ints = d->ints;
    a.max_out = d->max_out;
    a.status = d->ctx->status;
    void* args[] = {&a};
    return cudaLaunchCooperativeKernel((const void*)decoder_persist_kernel, dim3(G), dim3(kPThreads), args,
                                       persist_smem_bytes(), s);
}
