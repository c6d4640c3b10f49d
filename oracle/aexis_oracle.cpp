// aexis_oracle.cpp -- CPU restatement of the Aexis quantized-decoder hot path.
//
// TEST INFRASTRUCTURE ONLY. This file is the parity checker for libaexis_cuda.
// Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg (and
// `bench.py --impl reference`) load it. The product never links or calls it.
//
// Every function restates one piece of the reference's arithmetic, in fp32,
// in the reference's own summation order, and cites the file:line it follows.
// Paths are relative to the reference checkout (newzjh/AIImage); the short
// forms are
//   HLSL_MM  = Packages/com.aexis/Runtime/Resources/Aexis/Includes/KernelGroups/AexisKernels.Pack4Matmul.hlsl
//   HLSL_PN  = .../KernelGroups/AexisKernels.Pack4PointwiseNorm.hlsl
//   HLSL_EW  = .../KernelGroups/AexisKernels.Pack4Elementwise.hlsl
//   HLSL_BT  = .../KernelGroups/AexisKernels.BufferTensor.hlsl
//   COMMON   = Packages/com.aexis/Runtime/Resources/Aexis/AexisCommon.compute
//   SESSION  = Packages/com.aexis/Runtime/Execution/Graph/AexisGraphSession.cs
//   DECODER  = Packages/com.aexis/Samples/AIImageApplicationExample/Runtime/Scripts/Qwen35DecoderSession.cs
//   GOLDEN   = Packages/com.aexis/Samples/AIImageApplicationExample/Editor/NcnnLinearCmdPack4GoldenTests.cs
//
// Pinning: the reference's known-answer tests (int8 packing, Q8 Gemm + bias,
// argmax 13/17 and tiled 34/37, SDPA mask/causal and KV-cache concat with the
// CreateValues inputs) are restated in tests/test_oracle_pins.py and must pass
// against this file before any GPU comparison is trusted.
//
// Build: oracle/Makefile (g++ -O3 -fopenmp -ffp-contract=off). No fast-math:
// fp32 rounding follows IEEE single precision, one rounding per operation, as
// the HLSL source states it (no contraction into fused multiply-adds).

#include <cstdint>
#include <cstring>
#include <cmath>
#include <cfloat>
#include <vector>
#include <algorithm>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_API extern "C" __attribute__((visibility("default")))

namespace {

// C# Mathf.RoundToInt is Math.Round (midpoint to even). nearbyintf under the
// default FE_TONEAREST rounding mode is the same function.
inline int round_to_int_even(float v) { return (int)std::nearbyintf(v); }

inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

// AexisGemm2DReadB (HLSL_MM:707-734) with _MatTransB != 0: element (col, kk)
// of a [N, K] weight lives at flat index col*K + kk.
//   Q4: nibble (index & 7) of word index >> 3, two's complement, times
//       S[index / blk] (blk > 0) or S[col] (blk == 0).
//   Q8: byte (index & 3) of word index >> 2, two's complement, times S[col].
inline float read_b(int bits, const uint32_t* P, const float* S, int blk,
                    int64_t col, int64_t K, int64_t kk) {
    int64_t index = col * K + kk;
    if (bits == 4) {
        uint32_t packed = P[index >> 3];
        uint32_t raw = (packed >> ((index & 7) * 4)) & 0xFu;
        int sv = raw >= 8u ? (int)raw - 16 : (int)raw;
        int64_t si = blk > 0 ? index / blk : col;
        return (float)sv * S[si];
    }
    uint32_t packed = P[index >> 2];
    uint32_t raw = (packed >> ((index & 3) * 8)) & 0xFFu;
    int sv = raw >= 128u ? (int)raw - 256 : (int)raw;
    return (float)sv * S[col];
}

}  // namespace

// ---------------------------------------------------------------------------
// Weight quantizers: AexisGraphSession.NewInt8WeightOnlyUpload(float[], ...)
// (SESSION:12834-12885) and NewInt4WeightOnlyUpload(float[], ...)
// (SESSION:12912-12964). Per output channel: scale = maxAbs/127 (or /7),
// 1 when the channel is all zero; q = clamp(RoundToInt(v / scale)); packed
// by the flat source index (4 bytes or 8 nibbles per uint32, low first).
// `packed` must be zeroed by the caller and hold ceil(n*k/4) (or /8) words.
// ---------------------------------------------------------------------------
ORACLE_API void oracle_quantize_rows(int bits, const float* data, int out_ch, int per_ch,
                                     int contiguous, uint32_t* packed, float* scales) {
    const float qmax = bits == 4 ? 7.0f : 127.0f;
    const int lim = bits == 4 ? 7 : 127;
    for (int oc = 0; oc < out_ch; ++oc) {
        float max_abs = 0.0f;
        for (int vi = 0; vi < per_ch; ++vi) {
            int64_t si = contiguous ? (int64_t)oc * per_ch + vi : (int64_t)vi * out_ch + oc;
            max_abs = std::max(max_abs, std::fabs(data[si]));
        }
        float scale = max_abs > 0.0f ? max_abs / qmax : 1.0f;
        scales[oc] = scale;
        for (int vi = 0; vi < per_ch; ++vi) {
            int64_t si = contiguous ? (int64_t)oc * per_ch + vi : (int64_t)vi * out_ch + oc;
            int q = clampi(round_to_int_even(data[si] / scale), -lim, lim);
            if (bits == 4) {
                packed[si >> 3] |= ((uint32_t)q & 0xFu) << ((si & 7) * 4);
            } else {
                packed[si >> 2] |= (uint32_t)(uint8_t)(int8_t)q << ((si & 3) * 8);
            }
        }
    }
}

// Dequantize a whole [N, K] weight with AexisGemm2DReadB (HLSL_MM:707-734).
ORACLE_API void oracle_dequant(int bits, const uint32_t* P, const float* S, int blk,
                               int n, int k, float* out) {
#pragma omp parallel for schedule(static)
    for (int col = 0; col < n; ++col)
        for (int kk = 0; kk < k; ++kk)
            out[(int64_t)col * k + kk] = read_b(bits, P, S, blk, col, k, kk);
}

// ---------------------------------------------------------------------------
// AexisGemm2DPack4LinearTextureAFromLinear_Impl (HLSL_MM:1038-1104), transB,
// bias broadcast per column (broadcastTypeC = 4, AexisResolveGemm2DBias
// HLSL_MM:688-705):
//   acc = useC ? beta * C[col] : 0
//   for kk in 0..K-1: acc += a[row, kk] * ReadB(col, kk)      (fp32, in order)
//   y[row, col] = acc * alpha
// The packed-int8 fast path (HLSL_MM:1059-1088) sums the same terms in the
// same order, so one loop covers both. Rows are independent; a block of rows
// is walked together so each row keeps its own sequential k order.
// ---------------------------------------------------------------------------
namespace {
template <bool kTiled>
void gemm_impl(const float* a, int lda, int m, int k, int bits, const uint32_t* P,
               const float* S, int blk, int n, const float* bias, float alpha, float beta,
               float* y, int ldy) {
    constexpr int RB = 8;
    const int nblocks = (n + RB - 1) / RB;
#pragma omp parallel for schedule(static)
    for (int b = 0; b < nblocks * m; ++b) {
        const int row = b / nblocks;
        const int c0 = (b % nblocks) * RB;
        const int cn = std::min(RB, n - c0);
        float acc[RB];
        for (int j = 0; j < cn; ++j)
            acc[j] = (!kTiled && bias) ? beta * bias[c0 + j] : 0.0f;
        const float* arow = a + (int64_t)row * lda;
        for (int kk = 0; kk < k; ++kk) {
            const float av = arow[kk];
            for (int j = 0; j < cn; ++j) {
                float prod = av * read_b(bits, P, S, blk, c0 + j, k, kk);
                acc[j] = acc[j] + prod;
            }
        }
        for (int j = 0; j < cn; ++j) {
            float out;
            if (kTiled) {
                // AexisGemm2DPack4TiledTextureAFrom*_Impl (HLSL_MM:2245-2300):
                // bias resolved after the loop: beta*C + acc*alpha.
                float bterm = bias ? beta * bias[c0 + j] : 0.0f;
                out = bterm + acc[j] * alpha;
            } else {
                out = acc[j] * alpha;
            }
            y[(int64_t)row * ldy + c0 + j] = out;
        }
    }
}
}  // namespace

ORACLE_API void oracle_gemm(const float* a, int lda, int m, int k, int bits, const uint32_t* P,
                            const float* S, int blk, int n, const float* bias, float alpha,
                            float beta, float* y, int ldy) {
    gemm_impl<false>(a, lda, m, k, bits, P, S, blk, n, bias, alpha, beta, y, ldy);
}

ORACLE_API void oracle_gemm_tiled(const float* a, int lda, int m, int k, int bits,
                                  const uint32_t* P, const float* S, int blk, int n,
                                  const float* bias, float alpha, float beta, float* y, int ldy) {
    gemm_impl<true>(a, lda, m, k, bits, P, S, blk, n, bias, alpha, beta, y, ldy);
}

// The A operand of AexisGemm2DPack4LinearTextureAFromPack4_Impl
// (HLSL_MM:1106-1190, inputPacked = true in Ops.Gemm2DPack4LinearTextureA,
// AexisOps.cs:3649-3683) as a row-major [m][k] matrix: the kernel walks
// logicalPack = 0, 1, ... with packX = logicalPack % width, packSlice =
// logicalPack / width, stops at the first packSlice >= slices, and uses lane
// kk & 3 of texel (packX, row, packSlice) for kk = 4*logicalPack + lane < K
// (AexisGemm2DPack4LinearTextureAReadPack4, HLSL_MM:880-891). A texture array
// [slices][height][width] of float4 is stored flat as
// ((slice*height + row)*width + x)*4 + lane. Values past the last slice are
// never added; 0 stands in for them (acc + 0 = acc).
ORACLE_API void oracle_read_pack4a(const float* a, int width, int height, int slices, int m, int k, float* out) {
    for (int row = 0; row < m; ++row)
        for (int kk = 0; kk < k; ++kk) {
            const int pack = kk >> 2, x = pack % std::max(1, width), sl = pack / std::max(1, width);
            out[(int64_t)row * k + kk] =
                sl < slices ? a[(((int64_t)sl * height + row) * width + x) * 4 + (kk & 3)] : 0.0f;
        }
}

// W8A8 activation fake-quantisation, AexisQuantizeGemmActivationForInt8
// (HLSL_MM:792-800): q = clamp(round(v / scale) + zp), back to (q - zp)*scale.
ORACLE_API void oracle_quantize_activation_int8(const float* x, int count, float scale, int zp,
                                                int is_unsigned, float* out) {
    for (int i = 0; i < count; ++i) {
        int q = (int)std::nearbyintf(x[i] / scale) + zp;
        q = is_unsigned ? clampi(q, 0, 255) : clampi(q, -128, 127);
        out[i] = (float)(q - zp) * scale;
    }
}

// ---------------------------------------------------------------------------
// AexisRmsNormPack4LinearMat (COMMON:4531-4563), one logical row of width W:
//   sumSquare = sum_i x_i^2                         (sequential, fp32)
//   invRms    = rsqrt(max(sumSquare / W + eps, 1e-20))
//   y_i       = x_i * invRms * gamma[clamp(i, 0, affineSize - 1)]   (if affine)
// rsqrt is written as 1/sqrtf; the HLSL intrinsic is not correctly rounded
// either, so parity with it is by tolerance.
// ---------------------------------------------------------------------------
ORACLE_API void oracle_rmsnorm(const float* x, int rows, int width, int ld, const float* gamma,
                               int affine_size, float eps, float* y, int ldy) {
    for (int r = 0; r < rows; ++r) {
        const float* xr = x + (int64_t)r * ld;
        float ss = 0.0f;
        for (int i = 0; i < width; ++i) ss = ss + xr[i] * xr[i];
        float inv = 1.0f / std::sqrt(std::max(ss / (float)width + eps, 1e-20f));
        for (int i = 0; i < width; ++i) {
            float v = xr[i] * inv;
            if (gamma && affine_size > 0) v = v * gamma[clampi(i, 0, affine_size - 1)];
            y[(int64_t)r * ldy + i] = v;
        }
    }
}

// Pack4 CDHW element (x, y, z=0, channel c) of a [W, H, 1, C] tensor:
// slice c/4, texel ((slice*H + y)*W + x), lane c&3.
static inline int64_t pack4_cdhw(int W, int H, int x, int y, int c) {
    return (((int64_t)(c >> 2) * H + y) * W + x) * 4 + (c & 3);
}

// AexisRotaryEmbedPack4_Impl (HLSL_PN:414-473). src/out are Pack4 CDHW
// [embedDim, seqLen, 1, numHeads]; cos/sin are linear [seqLen, embedDim/2].
// Rotate-half: j < half -> x_j*c - x_{j+half}*s, else x_j'*s + x_{j'+half}*c.
// Interleaved: pairs (2j, 2j+1). An element whose partner is out of range is
// copied through (HLSL_PN:452-456).
ORACLE_API void oracle_rope(const float* src, int embed_dim, int seq_len, int num_heads,
                            const float* cosv, const float* sinv, int interleaved, float* out) {
    const int half = std::max(1, embed_dim / 2);
    for (int head = 0; head < num_heads; ++head)
        for (int seq = 0; seq < seq_len; ++seq)
            for (int e = 0; e < embed_dim; ++e) {
                int pair0, pair1, ci;
                bool first;
                if (interleaved) {
                    int j = e / 2;
                    pair0 = j * 2; pair1 = pair0 + 1; ci = seq * half + j; first = (e & 1) == 0;
                } else {
                    int j2 = e < half ? e : e - half;
                    pair0 = j2; pair1 = half + j2; ci = seq * half + j2; first = e < half;
                }
                int64_t o = pack4_cdhw(embed_dim, seq_len, e, seq, head);
                if (pair1 >= embed_dim) { out[o] = src[o]; continue; }
                float c = cosv[ci], s = sinv[ci];
                float x0 = src[pack4_cdhw(embed_dim, seq_len, pair0, seq, head)];
                float x1 = src[pack4_cdhw(embed_dim, seq_len, pair1, seq, head)];
                out[o] = first ? x0 * c - x1 * s : x0 * s + x1 * c;
            }
}

// AexisAppendSequencePack4CDHW_Impl (HLSL_EW:84-98): copy `rows` texel rows
// of `current` to rows offset.. of `cache` ([width, cache_rows, slices] float4
// texels); rows that fall outside the cache are dropped.
ORACLE_API void oracle_append_sequence(const float* current, int width, int rows, int slices,
                                       int offset, float* cache, int cache_rows) {
    for (int z = 0; z < slices; ++z)
        for (int y = 0; y < rows; ++y) {
            int dy = offset + y;
            if (dy < 0 || dy >= cache_rows) continue;
            for (int x = 0; x < width; ++x)
                for (int l = 0; l < 4; ++l)
                    cache[(((int64_t)z * cache_rows + dy) * width + x) * 4 + l] =
                        current[(((int64_t)z * rows + y) * width + x) * 4 + l];
        }
}

// AexisConcatSequencePack4CDHW_Impl (HLSL_EW:64-81): out rows [0, aH) from a,
// [aH, aH+bH) from b, the rest zero.
ORACLE_API void oracle_concat_sequence(const float* a, int a_rows, const float* b, int b_rows,
                                       int width, int slices, float* out, int out_rows) {
    for (int z = 0; z < slices; ++z)
        for (int y = 0; y < out_rows; ++y)
            for (int x = 0; x < width; ++x)
                for (int l = 0; l < 4; ++l) {
                    float v = 0.0f;
                    if (y < a_rows) v = a[(((int64_t)z * a_rows + y) * width + x) * 4 + l];
                    else if (y < a_rows + b_rows)
                        v = b[(((int64_t)z * b_rows + (y - a_rows)) * width + x) * 4 + l];
                    out[(((int64_t)z * out_rows + y) * width + x) * 4 + l] = v;
                }
}

// AexisSdpaAttentionPack4CDHW_Impl (HLSL_MM:420-557). q/out: Pack4 CDHW
// [embed, srcLen, 1, heads]; k/v: [embed (outEmbed for v), dstLen, 1, groups];
// mask: single-channel Pack4 [maskW, maskH] (value at lane 0 of each texel).
//   s = scale * sum_i q_i k_i; causal col > row + offset -> -1e20, else
//   s += mask[row, col] when inside the mask; p = exp(s - max) / max(sum, 1e-20);
//   out = sum_col p_col * v_col.                      GQA: kv = head / (H/G).
// The HLSL kernel returns without writing when dstLen > 4096 (a groupshared
// capacity limit, HLSL_MM:432); the restatement has no such cap.
ORACLE_API void oracle_sdpa(const float* q, const float* k, const float* v, int src_len,
                            int dst_len, int embed_dim, int out_embed_dim, int num_heads,
                            int num_groups, float scale, const float* mask, int mask_w,
                            int mask_h, int causal, int causal_offset, float* out) {
    const int hpg = std::max(1, num_heads / num_groups);
    const int off = std::max(0, causal_offset);
#pragma omp parallel for collapse(2) schedule(static)
    for (int row = 0; row < src_len; ++row)
        for (int head = 0; head < num_heads; ++head) {
            const int kh = std::min(std::max(0, num_groups - 1), head / hpg);
            std::vector<float> sc(dst_len);
            for (int col = 0; col < dst_len; ++col) {
                float s = 0.0f;
                for (int i = 0; i < embed_dim; ++i)
                    s = s + q[pack4_cdhw(embed_dim, src_len, i, row, head)] *
                            k[pack4_cdhw(embed_dim, dst_len, i, col, kh)];
                s = s * scale;
                if (causal && col > row + off) s = -1.0e20f;
                else if (mask && col < mask_w && row < mask_h)
                    s = s + mask[((int64_t)row * mask_w + col) * 4];
                sc[col] = s;
            }
            float mx = -FLT_MAX;
            for (int col = 0; col < dst_len; ++col) mx = std::max(mx, sc[col]);
            float sum = 0.0f;
            for (int col = 0; col < dst_len; ++col) { sc[col] = std::exp(sc[col] - mx); sum = sum + sc[col]; }
            float inv = 1.0f / std::max(sum, 1e-20f);
            for (int col = 0; col < dst_len; ++col) sc[col] = sc[col] * inv;
            for (int ox = 0; ox < out_embed_dim; ++ox) {
                float acc = 0.0f;
                for (int col = 0; col < dst_len; ++col)
                    acc = acc + sc[col] * v[pack4_cdhw(out_embed_dim, dst_len, ox, col, kh)];
                out[pack4_cdhw(out_embed_dim, src_len, ox, row, head)] = acc;
            }
        }
}

// AexisArgMaxPack4LinearMat_Impl (HLSL_MM:645-686) and Qwen35Sampler.ArgMax
// (DECODER:1902-1908): the first index holding the maximum wins (strict >),
// starting from index 0. Logits are row-major with row stride ld.
ORACLE_API void oracle_argmax(const float* logits, int rows, int width, int ld, int32_t* out) {
    for (int r = 0; r < rows; ++r) {
        const float* x = logits + (int64_t)r * ld;
        int best = 0;
        float bv = 0.0f;
        for (int i = 0; i < width; ++i)
            if (i == 0 || x[i] > bv) { bv = x[i]; best = i; }
        out[r] = best;
    }
}

// Top-k per row: the k largest logits in descending order; equal values are
// ordered by ascending index (the argmax tie rule extended to k entries). NaN
// is never selected; a row with fewer than k other values is padded with
// (-inf, -1).
ORACLE_API void oracle_topk(const float* logits, int rows, int width, int ld, int k,
                            float* out_vals, int32_t* out_idx) {
    for (int r = 0; r < rows; ++r) {
        const float* x = logits + (int64_t)r * ld;
        std::vector<int> ord;
        ord.reserve(width);
        for (int i = 0; i < width; ++i)
            if (x[i] == x[i]) ord.push_back(i);
        const int kk = std::min<int>(k, (int)ord.size());
        std::partial_sort(ord.begin(), ord.begin() + kk, ord.end(), [&](int a, int b) {
            if (x[a] != x[b]) return x[a] > x[b];
            return a < b;
        });
        for (int j = 0; j < k; ++j) {
            out_vals[(int64_t)r * k + j] = j < kk ? x[ord[j]] : -INFINITY;
            out_idx[(int64_t)r * k + j] = j < kk ? ord[j] : -1;
        }
    }
}

// AexisEmbedValue (HLSL_BT:37-62): word = clamp(word, 0, inputDim-1);
// index = word*numOutput + p; Q4 scale S[index/blk]; Q8 scale S[word];
// bits == 32 reads a plain fp32 table. Bias is added per output p.
ORACLE_API void oracle_embed(const int32_t* words, int count, int bits, const uint32_t* P,
                             const float* S, int blk, const float* table_f32, int input_dim,
                             int num_output, const float* bias, float* out) {
    for (int q = 0; q < count; ++q) {
        int w = clampi(words[q], 0, input_dim - 1);
        for (int p = 0; p < num_output; ++p) {
            int64_t wi = (int64_t)w * num_output + p;
            float v;
            if (bits == 4) {
                uint32_t raw = (P[wi >> 3] >> ((wi & 7) * 4)) & 0xFu;
                int sv = raw >= 8u ? (int)raw - 16 : (int)raw;
                v = (float)sv * S[wi / blk];
            } else if (bits == 8) {
                uint32_t raw = (P[wi >> 2] >> ((wi & 3) * 8)) & 0xFFu;
                int sv = raw >= 128u ? (int)raw - 256 : (int)raw;
                v = (float)sv * S[w];
            } else {
                v = table_f32[wi];
            }
            if (bias) v = v + bias[p];
            out[(int64_t)q * num_output + p] = v;
        }
    }
}

// AexisApplySwishLinearScalar (HLSL_MM:91-94): x / (1 + exp(-x)).
ORACLE_API void oracle_swish(const float* x, int count, float* y) {
    for (int i = 0; i < count; ++i) y[i] = x[i] / (1.0f + std::exp(-x[i]));
}

// SwiGLU as the reference composes it: Swish layer on the gate, BinaryOp
// multiply with the up projection (HLSL_MM:118-128,205-218).
ORACLE_API void oracle_swiglu(const float* gate, const float* up, int count, float* y) {
    for (int i = 0; i < count; ++i) {
        float g = gate[i] / (1.0f + std::exp(-gate[i]));
        y[i] = g * up[i];
    }
}

// ---------------------------------------------------------------------------
// fp32 -> fp16 (IEEE binary16, round to nearest even, with subnormals, inf and
// NaN), then back to fp32. The fp16 KV cache stores values through this.
// ---------------------------------------------------------------------------
static inline uint16_t f32_to_f16_bits(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t absx = x & 0x7FFFFFFFu;
    if (absx >= 0x7F800000u) return (uint16_t)(sign | 0x7C00u | (absx > 0x7F800000u ? 0x200u : 0u));
    if (absx >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u);  // rounds to >= 65520 -> inf
    int e = (int)(absx >> 23) - 127;
    uint32_t mant = absx & 0x7FFFFFu;
    if (e >= -14) {  // normal half
        uint32_t h = ((uint32_t)(e + 15) << 10) | (mant >> 13);
        uint32_t rem = mant & 0x1FFFu;
        if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1;
        return (uint16_t)(sign | h);
    }
    if (e < -25) return (uint16_t)sign;  // below half the smallest subnormal
    mant |= 0x800000u;                   // subnormal half: value = mant * 2^(e-23)
    int shift = -e - 1;                  // so that result unit is 2^-24
    uint32_t h = mant >> shift;
    uint32_t rem = mant & ((1u << shift) - 1u);
    uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (h & 1u))) h += 1;
    return (uint16_t)(sign | h);
}

static inline float f16_bits_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) x = sign;
        else {  // subnormal: m * 2^-24
            float v = (float)m * 5.9604644775390625e-8f;
            std::memcpy(&x, &v, 4);
            x |= sign;
        }
    } else if (e == 31) x = sign | 0x7F800000u | (m << 13);
    else x = sign | ((e + 112) << 23) | (m << 13);
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

ORACLE_API float oracle_round_f16(float v) { return f16_bits_to_f32(f32_to_f16_bits(v)); }

ORACLE_API void oracle_f32_to_f16(const float* x, int64_t count, uint16_t* out) {
    for (int64_t i = 0; i < count; ++i) out[i] = f32_to_f16_bits(x[i]);
}

// RoPE tables as Qwen35DecoderSession.CreateRopeTextures builds them
// (DECODER:1660-1687), generalised from RopeHalfDimension=32 to rot_dim/2:
//   invFreq_j = 1 / pow(theta, j * (2 / rot_dim)),  angle = pos * invFreq_j,
//   cos/sin evaluated in double and rounded to fp32 (Mathf.Cos/Sin).
ORACLE_API void oracle_rope_tables(int positions, int rot_dim, float theta, float* cosv,
                                   float* sinv) {
    const int half = rot_dim / 2;
    for (int p = 0; p < positions; ++p)
        for (int j = 0; j < half; ++j) {
            float inv = 1.0f / (float)std::pow((double)theta, (double)((float)j * (2.0f / (float)rot_dim)));
            float angle = (float)p * inv;
            cosv[(int64_t)p * half + j] = (float)std::cos((double)angle);
            sinv[(int64_t)p * half + j] = (float)std::sin((double)angle);
        }
}

// ---------------------------------------------------------------------------
// Synthetic decoder (the Qwen3.5-0.8B-shaped full-attention stack used for
// measurement, or with layer_types the hybrid stack whose linear-attention
// blocks are linear_attention_block below), composed from the restated
// layers the way the reference's
// decode loop drives them (DecodeCore DECODER:469-585, layer plugins
// AexisRMSNormLayer / AexisGemmLayer / AexisRotaryEmbedLayer / AexisSdpaLayer):
//   h = Embed(token)
//   per layer: xn = RMSNorm(h); q,k,v = Gemm(xn); RoPE(q), RoPE(k) (rotate
//     half over the first rot_dim dims); KV append at `pos` (fp16 cache);
//     a = SDPA(q, K[0..pos], V[0..pos]) with GQA; h += Gemm_o(a);
//     xn = RMSNorm(h); h += Gemm_down(Swish(Gemm_gate(xn)) * Gemm_up(xn))
//   logits = Gemm_lm(RMSNorm_final(h)); next = ArgMax(logits)
// Activations are fp32 (as the reference's Qwen session runs them,
// DECODER:1748-1766); the KV cache holds fp16.
// ---------------------------------------------------------------------------
struct OracleDecoderCfg {
    int32_t n_layers, hidden, n_heads, n_kv_heads, head_dim, ffn, vocab, kv_capacity;
    int32_t rot_dim, bits, group, lm_bits, lm_group;
    float theta, eps;
    // Hybrid stacks (Qwen3.5: DECODER:167-172, 6 attention caches and 18
    // conv/GDR caches). layer_types[l] = 1 makes layer l a linear-attention
    // block; null or 0 everywhere is the all-full-attention stack.
    int32_t lin_heads, lin_kdim, lin_vdim, conv_kernel;
    const int32_t* layer_types;
};

// The linear-attention restatements further down (one token of each per
// decode step here).
ORACLE_API void oracle_short_conv(const float* weight, const float* mixed, const float* cache_in, float* out,
                                  float* cache_out, int groups, int kernel, int seq, int cache_len);
ORACLE_API void oracle_gated_delta_rule(const float* a_log, const float* dt_bias, const float* b, const float* a,
                                        const float* q, const float* k, const float* v, const float* state_in,
                                        float* out, float* state_out, int heads, int kdim, int vdim, int first,
                                        int count, float eps);

namespace {
struct OLinear { const uint32_t* P = nullptr; const float* S = nullptr; int n = 0, k = 0, bits = 4, blk = 0; };
struct OLayer {
    OLinear lin[7];  // a linear-attention layer uses lin[0] as in_proj, lin[3] as out_proj
    const float* norm[2] = {nullptr, nullptr};
    int kind = 0;    // 0 full attention, 1 linear attention
    // Linear attention: ShortConv weight in its Pack4 layout, per-head a_log
    // and dt_bias, the gated norm's gain, and the two recurrent caches.
    std::vector<float> conv_w, a_log, dt_bias, gamma;
    std::vector<float> conv_state;  // [conv_kernel][channels]
    std::vector<float> gdr_state;   // [lin_heads][lin_kdim][lin_vdim]
};
struct ODecoder {
    OracleDecoderCfg c;
    std::vector<OLayer> layers;
    OLinear lm;
    const float* final_norm = nullptr;
    const float* embed = nullptr;
    std::vector<float> kcache, vcache;  // [layer][kvh][cap][D], fp16-rounded values
    std::vector<float> cosv, sinv;
    int pos = 0;
};

void run_linear(const OLinear& L, const float* x, float* y) {
    oracle_gemm(x, L.k, 1, L.k, L.bits, L.P, L.S, L.blk, L.n, nullptr, 1.0f, 1.0f, y, L.n);
}

// Rotate-half RoPE for one head vector (HLSL_PN:414-473 with seq=1).
void rope_head(float* x, int D, int rot, const float* c, const float* s) {
    const int half = rot / 2;
    std::vector<float> t(x, x + D);
    for (int e = 0; e < rot; ++e) {
        int j = e < half ? e : e - half;
        float x0 = t[j], x1 = t[j + half];
        x[e] = e < half ? x0 * c[j] - x1 * s[j] : x0 * s[j] + x1 * c[j];
    }
}
}  // namespace

ORACLE_API void* oracle_decoder_create(const OracleDecoderCfg* cfg) {
    ODecoder* d = new ODecoder();
    d->c = *cfg;
    const auto& c = d->c;
    d->layers.resize(c.n_layers);
    const int q_n = c.n_heads * c.head_dim, kv_n = c.n_kv_heads * c.head_dim;
    const int shapes[7][2] = {{q_n, c.hidden}, {kv_n, c.hidden}, {kv_n, c.hidden}, {c.hidden, q_n},
                              {c.ffn, c.hidden}, {c.ffn, c.hidden}, {c.hidden, c.ffn}};
    const int l_nq = c.lin_heads * c.lin_kdim, l_nv = c.lin_heads * c.lin_vdim;
    const int l_ch = 2 * l_nq + l_nv;
    for (int l = 0; l < c.n_layers; ++l) {
        OLayer& L = d->layers[l];
        L.kind = c.layer_types ? c.layer_types[l] : 0;
        for (int w = 0; w < 7; ++w) {
            int n = shapes[w][0], k = shapes[w][1];
            if (L.kind == 1 && w == 0) n = l_ch + l_nv + 2 * c.lin_heads;  // [q k v z b a]
            if (L.kind == 1 && w == 3) k = l_nv;
            L.lin[w].n = n;
            L.lin[w].k = k;
            L.lin[w].bits = c.bits;
            L.lin[w].blk = c.bits == 4 ? (c.group > 0 ? c.group : k) : 0;
        }
        if (L.kind == 1) {
            L.conv_state.assign((size_t)c.conv_kernel * l_ch, 0.0f);
            L.gdr_state.assign((size_t)c.lin_heads * c.lin_kdim * c.lin_vdim, 0.0f);
        }
    }
    d->lm.n = c.vocab;
    d->lm.k = c.hidden;
    d->lm.bits = c.lm_bits;
    d->lm.blk = c.lm_bits == 4 ? (c.lm_group > 0 ? c.lm_group : c.hidden) : 0;
    size_t kvsz = (size_t)c.n_layers * c.n_kv_heads * c.kv_capacity * c.head_dim;
    d->kcache.assign(kvsz, 0.0f);
    d->vcache.assign(kvsz, 0.0f);
    d->cosv.resize((size_t)c.kv_capacity * (c.rot_dim / 2));
    d->sinv.resize((size_t)c.kv_capacity * (c.rot_dim / 2));
    oracle_rope_tables(c.kv_capacity, c.rot_dim, c.theta, d->cosv.data(), d->sinv.data());
    return d;
}

ORACLE_API void oracle_decoder_destroy(void* h) { delete (ODecoder*)h; }

namespace {
// splitmix64 finaliser (Steele, Lea and Flood, OOPSLA 2014).
uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
}  // namespace

// Synthetic context of a batched-decoding benchmark sequence (no reference
// counterpart: the reference fills its cache by running a prompt). Positions
// [0, ctx) of every layer's K (kind 0) and V (kind 1) cache hold the fp16
// rounding of u = (mix64(key ^ idx) >> 40) * 2^-24 - 0.5 with
// key = mix64(seed ^ mix64(seq_id)), idx = ((((l*2 + kind)*256 + h)*65536 + p)*256 + d);
// the next position becomes ctx. Returns -2 when ctx >= capacity.
ORACLE_API int oracle_decoder_fill_context(void* h, int ctx, uint64_t seed, int64_t seq_id) {
    ODecoder* d = (ODecoder*)h;
    const auto& c = d->c;
    if (ctx < 0 || ctx >= c.kv_capacity) return -2;
    const uint64_t key = mix64(seed ^ mix64((uint64_t)seq_id));
    const int D = c.head_dim, KVH = c.n_kv_heads;
    for (int l = 0; l < c.n_layers; ++l)
        for (int kind = 0; kind < 2; ++kind) {
            float* cache = (kind == 0 ? d->kcache : d->vcache).data() + (size_t)l * KVH * c.kv_capacity * D;
            for (int hh = 0; hh < KVH; ++hh)
                for (int p = 0; p < ctx; ++p)
                    for (int i = 0; i < D; ++i) {
                        const uint64_t idx =
                            ((((uint64_t)l * 2 + kind) * 256 + hh) * 65536 + (uint64_t)p) * 256 + (uint64_t)i;
                        const uint64_t r = mix64(key ^ idx);
                        const float u = (float)(r >> 40) * (1.0f / 16777216.0f) - 0.5f;
                        cache[((size_t)hh * c.kv_capacity + p) * D + i] = oracle_round_f16(u);
                    }
        }
    d->pos = ctx;
    return 0;
}
// CreateInitialState (DECODER:376-400): position 0, conv and GDR caches zero.
ORACLE_API void oracle_decoder_reset(void* h) {
    ODecoder* d = (ODecoder*)h;
    d->pos = 0;
    for (auto& L : d->layers) {
        std::fill(L.conv_state.begin(), L.conv_state.end(), 0.0f);
        std::fill(L.gdr_state.begin(), L.gdr_state.end(), 0.0f);
    }
}
// Layer `layer`'s cache (kind 0 = K, 1 = V) as [kv_heads][capacity][head_dim]
// fp32 (the fp16-rounded values the decoder attends over).
ORACLE_API void oracle_decoder_kv(void* h, int layer, int kind, float* out) {
    ODecoder* d = (ODecoder*)h;
    const auto& c = d->c;
    const size_t per = (size_t)c.n_kv_heads * c.kv_capacity * c.head_dim;
    const float* src = (kind == 0 ? d->kcache : d->vcache).data() + per * layer;
    std::memcpy(out, src, per * sizeof(float));
}
ORACLE_API int oracle_decoder_position(void* h) { return ((ODecoder*)h)->pos; }

// which: 0 q, 1 k, 2 v, 3 o, 4 gate, 5 up, 6 down; 8 in_proj and 9 out_proj
// of a linear-attention layer; layer -1 = lm_head. The arrays are borrowed,
// not copied: the caller keeps them alive.
ORACLE_API void oracle_decoder_set_linear(void* h, int layer, int which, const uint32_t* P,
                                          const float* S) {
    ODecoder* d = (ODecoder*)h;
    const int slot = which == 8 ? 0 : which == 9 ? 3 : which;
    OLinear& L = layer < 0 ? d->lm : d->layers[layer].lin[slot];
    L.P = P;
    L.S = S;
}

// A linear-attention layer's small parameters (copied): conv [channels][kernel]
// (the reference operator's weight=[groups, kernel], reference_ops.py:36-60),
// a_log and dt_bias [lin_heads], gamma [lin_vdim] (the gated RMSNorm's gain,
// shared by every head).
ORACLE_API void oracle_decoder_set_linear_attention(void* h, int layer, const float* conv, const float* a_log,
                                                    const float* dt_bias, const float* gamma) {
    ODecoder* d = (ODecoder*)h;
    const auto& c = d->c;
    OLayer& L = d->layers[layer];
    const int K = c.conv_kernel, ch = 2 * c.lin_heads * c.lin_kdim + c.lin_heads * c.lin_vdim;
    // Pack4 CDHW [w = kernel, h = 1, c = channels] (RecurrentLoadShortConvWeight, COMMON:586-592).
    L.conv_w.assign((size_t)((ch + 3) / 4) * 4 * K, 0.0f);
    for (int g = 0; g < ch; ++g)
        for (int k = 0; k < K; ++k) L.conv_w[((size_t)(g / 4) * K + k) * 4 + (g & 3)] = conv[(size_t)g * K + k];
    L.a_log.assign(a_log, a_log + c.lin_heads);
    L.dt_bias.assign(dt_bias, dt_bias + c.lin_heads);
    L.gamma.assign(gamma, gamma + c.lin_vdim);
}

// A linear-attention layer's caches: conv [conv_kernel][channels] (the
// reference's cache_conv texture, rows = taps) and GDR [heads][kdim][vdim]
// (cache_gdr, texel x = column / 4, y = key row, slice = head).
ORACLE_API void oracle_decoder_recurrent(void* h, int layer, float* conv_out, float* gdr_out) {
    const OLayer& L = ((ODecoder*)h)->layers[layer];
    if (conv_out) std::memcpy(conv_out, L.conv_state.data(), L.conv_state.size() * sizeof(float));
    if (gdr_out) std::memcpy(gdr_out, L.gdr_state.data(), L.gdr_state.size() * sizeof(float));
}

// which: 0 attention norm, 1 ffn norm; layer -1 = final norm.
ORACLE_API void oracle_decoder_set_norm(void* h, int layer, int which, const float* gamma) {
    ODecoder* d = (ODecoder*)h;
    if (layer < 0) d->final_norm = gamma;
    else d->layers[layer].norm[which] = gamma;
}

ORACLE_API void oracle_decoder_set_embedding(void* h, const float* table) {
    ((ODecoder*)h)->embed = table;
}

namespace {
// Qwen3.5's linear-attention decoder block for one token (the 18 blocks
// `ShortConv + GatedDeltaRule` of the hybrid stack, UNITY_IMPLEMENTATION_PLAN
// "topology": three of them before each cache-SDPA block), with the Qwen3-Next
// GatedDeltaNet composition around the two custom operators:
//   xn = RMSNorm(h); [q k v z b a] = Gemm_in(xn)
//   [q k v] = ShortConv+SiLU([q k v]) (streaming cache of conv_kernel rows)
//   o = GatedDeltaRule(q, k, v, b, a) per head (state [heads][kdim][vdim])
//   y = RMSNorm_head(o) * gamma * SiLU(z); h += Gemm_out(y)
//   xn = RMSNorm(h); h += Gemm_down(Swish(Gemm_gate(xn)) * Gemm_up(xn))
// The operators are the restatements above (ShortConv COMMON:623-678, GDR
// COMMON:680-753, eps 1e-6 as reference_ops.py:88); the norms are
// oracle_rmsnorm with the model's eps.
void linear_attention_block(ODecoder* d, OLayer& L, float* hs) {
    const auto& c = d->c;
    const int H = c.hidden, Hl = c.lin_heads, kd = c.lin_kdim, vd = c.lin_vdim, K = c.conv_kernel;
    const int nq = Hl * kd, nv = Hl * vd, ch = 2 * nq + nv;
    std::vector<float> xn(H), proj(L.lin[0].n), conv(ch), o(nv), y(nv), out(H);
    oracle_rmsnorm(hs, 1, H, H, L.norm[0], H, c.eps, xn.data(), H);
    run_linear(L.lin[0], xn.data(), proj.data());
    oracle_short_conv(L.conv_w.data(), proj.data(), L.conv_state.data(), conv.data(), L.conv_state.data(), ch, K, 1,
                      K);
    // One token in the GDR's Pack4 CDHW layout (sequence packed by 4: lane 0).
    std::vector<float> qp((size_t)nq * 4, 0.0f), kp((size_t)nq * 4, 0.0f), vp((size_t)nv * 4, 0.0f);
    std::vector<float> op((size_t)nv * 4, 0.0f), st(L.gdr_state.size());
    for (int i = 0; i < nq; ++i) {
        qp[(size_t)i * 4] = conv[i];
        kp[(size_t)i * 4] = conv[nq + i];
    }
    for (int i = 0; i < nv; ++i) vp[(size_t)i * 4] = conv[2 * nq + i];
    const float* z = proj.data() + ch;
    const float* b = z + nv;
    const float* a = b + Hl;
    oracle_gated_delta_rule(L.a_log.data(), L.dt_bias.data(), b, a, qp.data(), kp.data(), vp.data(),
                            L.gdr_state.data(), op.data(), st.data(), Hl, kd, vd, 0, 1, 1e-6f);
    L.gdr_state.swap(st);
    for (int i = 0; i < nv; ++i) o[i] = op[(size_t)i * 4];
    oracle_rmsnorm(o.data(), Hl, vd, vd, L.gamma.data(), vd, c.eps, y.data(), vd);
    for (int i = 0; i < nv; ++i) y[i] = y[i] * (z[i] / (1.0f + std::exp(-z[i])));
    run_linear(L.lin[3], y.data(), out.data());
    for (int i = 0; i < H; ++i) hs[i] = hs[i] + out[i];
    std::vector<float> g(c.ffn), u(c.ffn), act(c.ffn), dn(H);
    oracle_rmsnorm(hs, 1, H, H, L.norm[1], H, c.eps, xn.data(), H);
    run_linear(L.lin[4], xn.data(), g.data());
    run_linear(L.lin[5], xn.data(), u.data());
    oracle_swiglu(g.data(), u.data(), c.ffn, act.data());
    run_linear(L.lin[6], act.data(), dn.data());
    for (int i = 0; i < H; ++i) hs[i] = hs[i] + dn[i];
}
}  // namespace

// One token at the current position. When want_logits is 0 the lm_head is
// skipped (prompt tokens before the last) and -1 is returned; otherwise the
// greedy token is returned, logits (if non-null) receive the fp32 logits and
// margin (if non-null) the gap between the best and second-best logit.
ORACLE_API int oracle_decoder_step(void* h, int token, int want_logits, float* logits,
                                   float* margin) {
    ODecoder* d = (ODecoder*)h;
    const auto& c = d->c;
    if (d->pos >= c.kv_capacity) return -2;
    const int H = c.hidden, D = c.head_dim, NH = c.n_heads, KVH = c.n_kv_heads;
    const int half = c.rot_dim / 2;
    const int pos = d->pos;
    std::vector<float> hs(H), xn(H), q(NH * D), k(KVH * D), v(KVH * D), att(NH * D), o(H);
    std::vector<float> g(c.ffn), u(c.ffn), act(c.ffn), dn(H);
    int tok = clampi(token, 0, c.vocab - 1);
    for (int i = 0; i < H; ++i) hs[i] = d->embed[(int64_t)tok * H + i];
    const float* cs = d->cosv.data() + (size_t)pos * half;
    const float* sn = d->sinv.data() + (size_t)pos * half;
    const float scale = 1.0f / std::sqrt((float)D);
    const int hpg = std::max(1, NH / KVH);
    for (int l = 0; l < c.n_layers; ++l) {
        OLayer& L = d->layers[l];
        if (L.kind == 1) {
            linear_attention_block(d, L, hs.data());
            continue;
        }
        oracle_rmsnorm(hs.data(), 1, H, H, L.norm[0], H, c.eps, xn.data(), H);
        run_linear(L.lin[0], xn.data(), q.data());
        run_linear(L.lin[1], xn.data(), k.data());
        run_linear(L.lin[2], xn.data(), v.data());
        for (int hh = 0; hh < NH; ++hh) rope_head(q.data() + hh * D, D, c.rot_dim, cs, sn);
        for (int hh = 0; hh < KVH; ++hh) rope_head(k.data() + hh * D, D, c.rot_dim, cs, sn);
        float* kc = d->kcache.data() + (size_t)l * KVH * c.kv_capacity * D;
        float* vc = d->vcache.data() + (size_t)l * KVH * c.kv_capacity * D;
        for (int hh = 0; hh < KVH; ++hh)
            for (int i = 0; i < D; ++i) {
                kc[((size_t)hh * c.kv_capacity + pos) * D + i] = oracle_round_f16(k[hh * D + i]);
                vc[((size_t)hh * c.kv_capacity + pos) * D + i] = oracle_round_f16(v[hh * D + i]);
            }
        const int L_ctx = pos + 1;
#pragma omp parallel for schedule(static)
        for (int hh = 0; hh < NH; ++hh) {
            const int kh = std::min(KVH - 1, hh / hpg);
            std::vector<float> sc(L_ctx);
            const float* qh = q.data() + hh * D;
            for (int col = 0; col < L_ctx; ++col) {
                const float* kr = kc + ((size_t)kh * c.kv_capacity + col) * D;
                float s = 0.0f;
                for (int i = 0; i < D; ++i) s = s + qh[i] * kr[i];
                sc[col] = s * scale;
            }
            float mx = -FLT_MAX;
            for (int col = 0; col < L_ctx; ++col) mx = std::max(mx, sc[col]);
            float sum = 0.0f;
            for (int col = 0; col < L_ctx; ++col) { sc[col] = std::exp(sc[col] - mx); sum = sum + sc[col]; }
            float inv = 1.0f / std::max(sum, 1e-20f);
            for (int col = 0; col < L_ctx; ++col) sc[col] = sc[col] * inv;
            for (int i = 0; i < D; ++i) {
                float acc = 0.0f;
                for (int col = 0; col < L_ctx; ++col)
                    acc = acc + sc[col] * vc[((size_t)kh * c.kv_capacity + col) * D + i];
                att[hh * D + i] = acc;
            }
        }
        run_linear(L.lin[3], att.data(), o.data());
        for (int i = 0; i < H; ++i) hs[i] = hs[i] + o[i];
        oracle_rmsnorm(hs.data(), 1, H, H, L.norm[1], H, c.eps, xn.data(), H);
        run_linear(L.lin[4], xn.data(), g.data());
        run_linear(L.lin[5], xn.data(), u.data());
        oracle_swiglu(g.data(), u.data(), c.ffn, act.data());
        run_linear(L.lin[6], act.data(), dn.data());
        for (int i = 0; i < H; ++i) hs[i] = hs[i] + dn[i];
    }
    d->pos += 1;
    if (!want_logits) return -1;
    oracle_rmsnorm(hs.data(), 1, H, H, d->final_norm, H, c.eps, xn.data(), H);
    std::vector<float> lg(c.vocab);
    run_linear(d->lm, xn.data(), lg.data());
    int32_t best = 0;
    oracle_argmax(lg.data(), 1, c.vocab, c.vocab, &best);
    if (margin) {
        float second = -FLT_MAX;
        for (int i = 0; i < c.vocab; ++i)
            if (i != best) second = std::max(second, lg[i]);
        *margin = lg[best] - second;
    }
    if (logits) std::memcpy(logits, lg.data(), sizeof(float) * c.vocab);
    return best;
}

ORACLE_API int oracle_num_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// ---------------------------------------------------------------------------
// Linear-attention decode layers of Qwen3.5 (COMMON = Packages/com.aexis/
// Runtime/Resources/Aexis/AexisCommon.compute). Pinned against the
// reference's own fp32 NumPy gold operators (Tools/Qwen35NcnnBaseline/
// reference_ops.py:36-152) through tests/golden/recurrent_ops.npz.
// ---------------------------------------------------------------------------

// AexisShortConvPack4 (COMMON:623-678). weight: Pack4 CDHW [w=kernel, h=1,
// c=groups] (RecurrentLoadShortConvWeight, COMMON:586-592); mixed/out
// [seq][ld], cache_in/cache_out [cache_len][ld], ld = ceil(groups/4)*4
// (RecurrentLoad2, COMMON:574-578). The cache rows are the tail of
// [cache_in; mixed] (COMMON:630-648); each output sums the kernel window in
// order, then SiLU = sum / (1 + exp(-sum)) (COMMON:657-674).
ORACLE_API void oracle_short_conv(const float* weight, const float* mixed, const float* cache_in, float* out,
                                  float* cache_out, int groups, int kernel, int seq, int cache_len) {
    const int64_t ld = (int64_t)((groups + 3) / 4) * 4;
    auto hist = [&](int i, int g) -> float {
        if (i < 0) return 0.0f;
        return i < cache_len ? cache_in[i * ld + g] : mixed[(i - cache_len) * ld + g];
    };
    for (int t = 0; t < seq; ++t)
        for (int g = 0; g < groups; ++g) {
            float sum = 0.0f;
            for (int k = 0; k < kernel; ++k) {
                float w = weight[((int64_t)(g / 4) * kernel + k) * 4 + (g & 3)];
                sum = sum + hist(cache_len - kernel + t + 1 + k, g) * w;
            }
            out[t * ld + g] = sum / (1.0f + std::exp(-sum));
        }
    std::vector<float> tail((size_t)std::max(cache_len, 0) * groups);
    for (int i = 0; i < cache_len; ++i)
        for (int g = 0; g < groups; ++g) tail[(size_t)i * groups + g] = hist(seq + i, g);
    for (int i = 0; i < cache_len; ++i)
        for (int g = 0; g < groups; ++g) cache_out[i * ld + g] = tail[(size_t)i * groups + g];
}

// AexisGatedDeltaRulePack4 (COMMON:680-753), one dispatch per token as
// AexisGatedDeltaRuleLayer issues them (AexisGatedDeltaRuleLayer.cs:71-78),
// for tokens first..first+count-1. q/k/v/out are Pack4 CDHW with the sequence
// packed by 4 (RecurrentLoadGdrTensor, COMMON:600-604); a/b are [seq][heads]
// and a_log/dt_bias [heads] (RecurrentLoadLinearScalar, COMMON:594-598); the
// state is [heads][kdim][vdim4] (texel x = column / 4, y = key row, slice =
// head). Per token: norms by rsqrt(sum + eps) (COMMON:689-700), beta and
// decay (:701-706), memory over the decayed state (:708-714), delta (:716-
// 722), state update and projection (:723-731), scaled by rsqrt(kdim)
// (:732). Columns past vdim read v = 0 (the HLSL writes whole texels).
ORACLE_API void oracle_gated_delta_rule(const float* a_log, const float* dt_bias, const float* b, const float* a,
                                        const float* q, const float* k, const float* v, const float* state_in,
                                        float* out, float* state_out, int heads, int kdim, int vdim, int first,
                                        int count, float eps) {
    const int vdim4 = (vdim + 3) / 4 * 4;
    const size_t n_state = (size_t)heads * kdim * vdim4;
    std::vector<float> cur(state_in, state_in + n_state), next(n_state);
    auto gdr = [&](const float* t_, int64_t tok, int h, int j, int W) -> float {
        return t_[(((tok / 4) * heads + h) * (int64_t)W + j) * 4 + (tok & 3)];
    };
    for (int tok = first; tok < first + count; ++tok) {
        for (int h = 0; h < heads; ++h) {
            float qn2 = 0.0f, kn2 = 0.0f;
            for (int j = 0; j < kdim; ++j) {
                float qj = gdr(q, tok, h, j, kdim), kj = gdr(k, tok, h, j, kdim);
                qn2 = qn2 + qj * qj;
                kn2 = kn2 + kj * kj;
            }
            const float q_scale = 1.0f / std::sqrt(qn2 + eps);
            const float k_scale = 1.0f / std::sqrt(kn2 + eps);
            const float bb = b[(int64_t)tok * heads + h], aa = a[(int64_t)tok * heads + h];
            const float alog = a_log[h], dt = dt_bias[h];
            const float beta = 1.0f / (1.0f + std::exp(-bb));
            const float x = aa + dt;
            const float decay = std::exp(-std::exp(alog) * (std::max(x, 0.0f) + std::log(1.0f + std::exp(-std::fabs(x)))));
            for (int c = 0; c < vdim4; ++c) {
                float memory = 0.0f;
                for (int j = 0; j < kdim; ++j) {
                    float kj = gdr(k, tok, h, j, kdim) * k_scale;
                    memory = memory + kj * (cur[((size_t)h * kdim + j) * vdim4 + c] * decay);
                }
                const float val = c < vdim ? gdr(v, tok, h, c, vdim) : 0.0f;
                const float delta = (val - memory) * beta;
                float projected = 0.0f;
                for (int j = 0; j < kdim; ++j) {
                    float kj = gdr(k, tok, h, j, kdim) * k_scale;
                    float qj = gdr(q, tok, h, j, kdim) * q_scale;
                    size_t si = ((size_t)h * kdim + j) * vdim4 + c;
                    float updated = cur[si] * decay + kj * delta;
                    next[si] = updated;
                    projected = projected + qj * updated;
                }
                projected = projected * (1.0f / std::sqrt((float)kdim));
                if (c < vdim) out[(((int64_t)(tok / 4) * heads + h) * vdim + c) * 4 + (tok & 3)] = projected;
            }
        }
        cur.swap(next);
    }
    std::memcpy(state_out, cur.data(), sizeof(float) * n_state);
}

// ---------------------------------------------------------------------------
// Qwen35Sampler.Select (DECODER:1847-1892) for `rows` logit rows, with the
// NextDouble draw of each row given in `uniforms` (the System.Random stream
// is the caller's). history: NULL or a bitmap [rows][ceil(width/32)] (bit i
// of word i/32 = token i is in the history set, DECODER:1840-1844).
//   scores = logits with the repetition penalty on history tokens (:1852-1853)
//   greedy when temperature <= 0 (:1855-1856), ArgMax = first maximum (:1894-1900)
//   value_i = (float)exp((s_i - max)/T), sum in double (:1858-1866); fallback
//   to ArgMax when the sum is not finite and positive (:1867-1868)
//   p_i = (float)(value_i / sum); order by p descending (:1869-1872); equal
//   probabilities keep ascending index here (the reference's Array.Sort is
//   unstable, so its order among exact ties is unspecified)
//   keep = min(TopK, V) (TopK <= 0: V), nucleus while cumulative < TopP (:1873-1884)
//   draw = u * kept mass, first cumulative >= draw (:1886-1894)
// margin[r] (optional): distance of the draw, and of the nucleus cut, from
// the nearest cumulative boundary, relative to the kept mass (a GPU/CPU
// difference in the last bits can only change the token when it is tiny).
// ---------------------------------------------------------------------------
ORACLE_API void oracle_sample(const float* logits, int rows, int width, int ld, const uint32_t* history,
                              float pen, float temperature, int top_k, float top_p, const double* uniforms,
                              int32_t* out, double* margin) {
    const int words = (width + 31) / 32;
    for (int r = 0; r < rows; ++r) {
        std::vector<float> scores(logits + (int64_t)r * ld, logits + (int64_t)r * ld + width);
        if (history)
            for (int i = 0; i < width; ++i)
                if ((history[(int64_t)r * words + i / 32] >> (i % 32)) & 1u)
                    scores[i] = scores[i] < 0.0f ? scores[i] * pen : scores[i] / pen;
        auto argmax = [&]() {
            int best = 0;
            for (int i = 1; i < width; ++i)
                if (scores[i] > scores[best]) best = i;
            return best;
        };
        if (margin) margin[r] = 1.0;
        if (temperature <= 0.0f) { out[r] = argmax(); continue; }
        const float mx = scores[argmax()];
        std::vector<float> prob(width);
        double sum = 0.0;
        for (int i = 0; i < width; ++i) {
            float value = std::exp((scores[i] - mx) / temperature);
            prob[i] = value;
            sum += value;
        }
        if (!std::isfinite(sum) || sum <= 0.0) { out[r] = argmax(); continue; }
        for (int i = 0; i < width; ++i) prob[i] = (float)(prob[i] / sum);
        int keep = top_k > 0 ? std::min(top_k, width) : width;
        std::vector<int> order(width);
        for (int i = 0; i < width; ++i) order[i] = i;
        auto by_prob = [&](int a, int b) { return prob[a] > prob[b] || (prob[a] == prob[b] && a < b); };
        std::partial_sort(order.begin(), order.begin() + keep, order.end(), by_prob);
        double cut_margin = 1.0;
        if (top_p < 1.0f) {
            double cumulative = 0.0;
            int nucleus = 0;
            while (nucleus < keep) {
                cumulative += prob[order[nucleus++]];
                cut_margin = std::min(cut_margin, std::fabs(cumulative - (double)top_p));
                if (cumulative >= top_p) break;
            }
            keep = std::max(1, nucleus);
        }
        double kept = 0.0;
        for (int i = 0; i < keep; ++i) kept += prob[order[i]];
        if (!std::isfinite(kept) || kept <= 0.0) { out[r] = argmax(); continue; }
        const double sample = uniforms[r] * kept;
        double cursor = 0.0, prev = 0.0;
        int pick = order[keep - 1];
        double dm = 1.0;
        for (int i = 0; i < keep; ++i) {
            prev = cursor;
            cursor += prob[order[i]];
            if (sample <= cursor) {
                pick = order[i];
                dm = std::min(sample - prev, cursor - sample) / kept;
                break;
            }
        }
        out[r] = pick;
        if (margin) margin[r] = std::min(dm, cut_margin);
    }
}
