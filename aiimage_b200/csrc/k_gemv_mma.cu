// k_gemv_mma.cu -- batch-1 Q4 / Q8 dequant GEMV with the multiply-accumulate
// on the tensor cores (mma.m16n8k16, fp16 x fp16 -> fp32).
//
// Same contract as the CUDA-core kernels (AexisGemm2DPack4LinearTexture-
// AFromLinear / ...Tiled..., HLSL Pack4Matmul:1038-1104, 2245-2300, weight
// read AexisGemm2DReadB :707-734). The CUDA-core decode spends about four
// instructions per weight (isolate, exact magic-number subtract, FMA, plus
// overhead) and cannot keep up with HBM. Here the weights are the A operand of
// m16n8k16 MMAs: a 4-bit value and an fp16 activation are both exact in fp16,
// the products are exact and the sums are fp32, so the arithmetic keeps the
// reference's fp32 semantics up to summation order. Per 8 weights a thread
// spends one shift, four LOP3 (nibble pairs under the fp16 exponent of 1024)
// and four HADD2/HFMA2 (exact removal of the offset), plus one MMA.
//
// Q8 works the same way with two words per lane and block (bytes placed under
// the fp16 exponent by PRMT, one HSUB2 per pair) and one scale per row.
//
// Layout (built from the reference packing at upload, launch_repack_frag):
//   * Q4 weights: 16-row tiles; per tile and per four k16 blocks, 32 lanes x
//     16 bytes, the word of k16 block kb for lane L = (g, t) holding, in byte
//     i, the two's complement nibbles of rows g (low) and g + 8 (high) at
//     k = 16 kb + 4t + i: the int8 MMA's A fragment of a k32 chunk is two
//     such words masked, the fp16 decode (decode_frag) reads k in the order
//     (4t, 4t + 2), (4t + 1, 4t + 3) and the B fragments follow it;
//   * Q8 weights: per lane and k16 block two words of offset-binary bytes
//     (repack_q8_frag_kernel);
//   * scales: per tile [group][8][2], the scales of rows r and r + 8 adjacent.
// Both are padded to a multiple of 8 tiles (rows past n decode to zero).
//
// Kernel: a producer warp bulk-copies one 16-row tile (weights and scales)
// per ring stage; the 8 consumer warps form 8 / KW groups that take the
// stages in turn, the KW warps of a group splitting K (KW = 1 for large N:
// one warp per tile, no cross-warp reduction). Each
// scale group accumulates in a fresh fp32 fragment and is added to the row sum
// with its scale (fp32 FMA). fp32 activations ride as fp16 hi + lo (two MMAs).
// The activation vector is staged once in fragment order (optionally through
// the fused RMSNorm); only lanes 0-3 carry it (column 0 of B), the others
// multiply zeros. Every barrier wait is bounded.
#include "gemv_stream.cuh"
#include "mma_frag.cuh"

namespace {

using namespace aexis_dev;

constexpr int kMW = 8;                     // consumer warps
constexpr int kMmaThreads = (kMW + 1) * 32;

struct MmaParams {
    StreamParams sp;       // W / S: fragment-layout copies; n, k, x, epilogue fields as for the stream kernel
    int nkb;               // K / 16
    int gk;                // k16 blocks per scale group
    int tile_wbytes, tile_sbytes;
    int units;             // 16-row tiles (one per ring stage)
    int ring_stages, stage_bytes;
};

// Q4 repack: one thread per (tile, k16 block, lane) word (layout above).
template <typename ST>
__global__ void repack_q4_frag_kernel(const uint32_t* src, const ST* scales, int n, int k, int group, int ntiles_pad,
                                      uint32_t* dst, ST* dst_s) {
    const int nkb = k / 16;
    const int kw = k / 8;  // source words per row
    const long long total = (long long)ntiles_pad * nkb * 32;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const int kb = (int)((i >> 5) % nkb);
        const long long t = (i >> 5) / nkb;
        const int g = lane >> 2, tig = lane & 3;
        const long long r0 = t * 16 + g, r1 = r0 + 8;
        const int k0 = kb * 16 + 4 * tig;
        auto nib = [&](long long r, int kk) -> uint32_t {
            if (r >= n) return 0u;
            return (src[r * kw + (kk >> 3)] >> (4 * (kk & 7))) & 15u;
        };
        // Byte i: rows g (low nibble) and g + 8 (high nibble) at k0 + i.
        uint32_t word = 0u;
#pragma unroll
        for (int i = 0; i < 4; ++i) word |= (nib(r0, k0 + i) | (nib(r1, k0 + i) << 4)) << (8 * i);
        dst[(t * nkb + (kb >> 2) * 4) * 32 + (long long)lane * 4 + (kb & 3)] = word;
    }
    // Scales: [tile][group][8][2], rows g and g + 8 adjacent.
    const int ng = group > 0 ? k / group : 1;
    const long long stotal = (long long)ntiles_pad * ng * 16;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < stotal;
         i += (long long)gridDim.x * blockDim.x) {
        const int row16 = (int)((i >> 1) & 7) + 8 * (int)(i & 1);
        const int grp = (int)((i >> 4) % ng);
        const long long t = (i >> 4) / ng;
        const long long r = t * 16 + row16;
        dst_s[i] = r < n ? scales[r * ng + grp] : ST(0.0f);
    }
}

// Q8 repack: the two words of lane L for k16 block kb hold its A fragment as
// offset-binary bytes u = q + 128: word 0 = (row g: k0, k0+1), (row g+8: k0,
// k0+1); word 1 = the same at k0+8, k0+9. Per tile and four blocks a lane's 8
// words are contiguous. Scales: one per row, [tile][8][2].
template <typename ST>
__global__ void repack_q8_frag_kernel(const uint32_t* src, const ST* scales, int n, int k, int ntiles_pad,
                                      uint32_t* dst, ST* dst_s) {
    const int nkb = k / 16;
    const int kw = k / 4;  // source words per row
    const long long total = (long long)ntiles_pad * nkb * 32;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int lane = (int)(i & 31);
        const int kb = (int)((i >> 5) % nkb);
        const long long t = (i >> 5) / nkb;
        const int g = lane >> 2, tig = lane & 3;
        const long long r0 = t * 16 + g, r1 = r0 + 8;
        const int k0 = kb * 16 + 2 * tig;
        auto u = [&](long long r, int kk) -> uint32_t {
            if (r >= n) return 128u;
            return ((src[r * kw + (kk >> 2)] >> (8 * (kk & 3))) & 0xFFu) ^ 0x80u;
        };
        const uint32_t w0 = u(r0, k0) | (u(r0, k0 + 1) << 8) | (u(r1, k0) << 16) | (u(r1, k0 + 1) << 24);
        const uint32_t w1 = u(r0, k0 + 8) | (u(r0, k0 + 9) << 8) | (u(r1, k0 + 8) << 16) | (u(r1, k0 + 9) << 24);
        const long long o = (t * nkb + (kb >> 2) * 4) * 64 + (long long)lane * 8 + (kb & 3) * 2;
        dst[o] = w0;
        dst[o + 1] = w1;
    }
    const long long stotal = (long long)ntiles_pad * 16;
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < stotal;
         i += (long long)gridDim.x * blockDim.x) {
        const int row16 = (int)((i >> 1) & 7) + 8 * (int)(i & 1);
        const long long r = (i >> 4) * 16 + row16;
        dst_s[i] = r < n ? scales[r] : ST(0.0f);
    }
}

// Scales of rows g and g + 8 (adjacent in the fragment layout).
__device__ __forceinline__ void load_scale_pair(const __half* p, float& s0, float& s1) {
    const __half2 h = *reinterpret_cast<const __half2*>(p);
    s0 = __low2float(h);
    s1 = __high2float(h);
}
__device__ __forceinline__ void load_scale_pair(const float* p, float& s0, float& s1) {
    const float2 f = *reinterpret_cast<const float2*>(p);
    s0 = f.x;
    s1 = f.y;
}

// The int8 path: Q4 group-32 weights with fp16 activations. Each scale group
// (k32 chunk) of the activations becomes a 23-bit fixed-point vector
// x_int = x 2^-E, E from the group's largest magnitude: values within eleven
// octaves of it (every fp16 value, up to outliers 2048 times the rest) are
// exact, smaller ones round at 2^(E-1), i.e. 2^-23 of the group maximum,
// the size of an fp32 rounding of a sum that maximum dominates. x_int is
// split into balanced int8 digits x_int = 65536 d2 + 256 d1 + d0, and the
// m16n8k32 MMAs take the weights straight from their nibbles (s8_frag) and
// give exact int32 digit sums. Four groups share an accumulator: group j of
// a window puts d2 / d1 in B columns 2j / 2j + 1 of tile A and d0 in column
// 2j of tile B, so lane (g, t) ends the window holding group t's three
// digit sums for rows g and g + 8.
// It pays where a CTA streams many tiles (the activations are quantised once
// per CTA): plan_mma picks it for N >= 8 x 16 x SM-count rows.
template <int XF, int GK, int BITS>
constexpr bool kS8Able = XF == 1 && GK == 2 && BITS == 4;

// Bytes of the staged activations: fp16 B fragments [XF][nkb * 4] uint2 plus
// a 32-byte zero block, or for the int8 path the B tiles A and B (each per
// window of four groups, two halves x 32 lanes x 16 bytes) and per group
// {8 sum d2, 8 sum d1, 8 sum d0, 2^E}.
__host__ __device__ inline int mma_x_bytes(bool s8, int xf, int nkb) {
    return s8 ? nkb * 256 + nkb * 8 : xf * nkb * 32 + 32;
}

// ST scale type; XF 1: fp16 activations, 2: fp32 as fp16 hi + lo; KW warps
// per tile (K split); GK 2: scale groups of two k16 blocks (group 32) with
// static group ends, 0: any group length (tracked at run time).
template <typename ST, int XF, int KW, int GK, int BITS, bool S8P>
__global__ void __launch_bounds__(kMmaThreads, 2) gemv_mma_kernel(MmaParams mp) {
    constexpr int NG = kMW / KW;  // warp groups; group it % NG takes unit it
    const StreamParams& p = mp.sp;
    extern __shared__ __align__(128) uint8_t smem[];
    const int S = mp.ring_stages;  // a multiple of NG
    const int SPG = S / NG;        // stages per group
    constexpr bool S8 = S8P && kS8Able<XF, GK, BITS>;
    uint8_t* ring = smem;
    uint8_t* xreg = smem + (size_t)S * mp.stage_bytes;  // staged activations (mma_x_bytes)
    uint2* xs = reinterpret_cast<uint2*>(xreg);
    float* red = reinterpret_cast<float*>(xreg + mma_x_bytes(S8, XF, mp.nkb));  // [2][kMW][16]
    uint64_t* full = reinterpret_cast<uint64_t*>(red + 2 * kMW * 16);
    uint64_t* empty = full + S;
    volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);
    float* redn = reinterpret_cast<float*>(const_cast<int*>(abort_flag) + 4);  // [kMW] RMSNorm partials

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int my_units = (int)blockIdx.x < mp.units ? (mp.units - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, KW);
        }
        *abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kMW) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = policy_evict_first();
            const uint32_t wb = (uint32_t)mp.tile_wbytes, sb = (uint32_t)mp.tile_sbytes;
            int issued = 0;
            for (int it = 0; it < my_units; ++it) {
                // Unit it belongs to group it % NG (its j-th unit), which owns
                // the private sub-ring of stages g, g + NG, ...
                const int j = it / NG;
                const int s = it % NG + NG * (j % SPG);
                if (j >= SPG && !mbar_wait(empty + s, ((j / SPG) & 1) ^ 1)) {
                    report_timeout(p.status);
                    break;
                }
                if (*abort_flag) break;
                const size_t u = (size_t)blockIdx.x + (size_t)it * gridDim.x;
                uint8_t* dst = ring + (size_t)s * mp.stage_bytes;
                mbar_arrive_expect_tx(full + s, wb + sb);
                bulk_g2s(dst, p.W + u * wb, wb, full + s, pol);
                bulk_g2s(dst + wb, p.S + u * sb, sb, full + s, pol);
                ++issued;
            }
            // The last S units issued are the last fills of S distinct stages.
            for (int it = max(0, issued - S); it < issued; ++it) {
                const int j = it / NG;
                if (!mbar_wait(full + it % NG + NG * (j % SPG), (j / SPG) & 1)) {
                    report_timeout(p.status);
                    break;
                }
            }
        }
        return;
    }

    // -------------------------------------------------------------- consumers
    griddep_wait();
    {
        // x -> B fragments: element e of k16 block kb sits in lane t = (e % 8) / 2,
        // register e / 8, half e % 2 (fp16 hi, and lo for XF 2), optionally
        // RMS-normalised first (the fused RMSNorm layer).
        const int tid = threadIdx.x;
        const bool norm = p.norm_gamma != nullptr;
        float inv = 1.0f;
        if (norm) {
            float ss = 0.0f;
            for (int i = tid; i < p.k; i += kMW * 32) {
                const float v = aexis_load_act(p.x, p.a_dtype, i);
                ss = fmaf(v, v, ss);
            }
#pragma unroll
            for (int o = 16; o >= 1; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) redn[warp] = ss;
            named_sync(1, kMW * 32);
            float tot = 0.0f;
#pragma unroll
            for (int w = 0; w < kMW; ++w) tot += redn[w];
            inv = 1.0f / sqrtf(fmaxf(tot / (float)p.k + p.norm_eps, 1e-20f));
        }
        if constexpr (S8) {
            uint4* bt = reinterpret_cast<uint4*>(xreg);
            for (int i = tid; i < mp.nkb * 16; i += kMW * 32) bt[i] = make_uint4(0u, 0u, 0u, 0u);
            named_sync(1, kMW * 32);
            int4* gq = reinterpret_cast<int4*>(xreg + (size_t)mp.nkb * 256);
            for (int q = warp; q < (p.k >> 5); q += kMW) {  // one warp per group, lane = element
                const int e = q * 32 + lane;
                float v = aexis_load_act(p.x, p.a_dtype, e);
                if (norm) v = v * inv * p.norm_gamma[e];
                if (p.act_quant) v = aexis_act_code(v, p.act_scale, p.act_zero_point, p.act_unsigned);
                float amax = fabsf(v);
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                int xi = 0;
                float ge = 0.0f;
                if (!(amax <= 3.402823466e38f)) {
                    ge = __int_as_float(0x7fc00000);  // Inf or NaN in the group: the rows become NaN
                } else if (amax > 0.0f) {
                    int ex;
                    frexpf(amax, &ex);  // amax = m 2^ex, m in [0.5, 1)
                    xi = __float2int_rn(ldexpf(v, 22 - ex));  // |xi| <= 2^22
                    ge = ldexpf(1.0f, ex - 22);
                }
                const int d0 = ((xi + 128) & 255) - 128, x1 = (xi - d0) >> 8;
                const int d1 = ((x1 + 128) & 255) - 128, d2 = (x1 - d1) >> 8;  // |d2| <= 64
                int X0 = d0, X1 = d1, X2 = d2;
#pragma unroll
                for (int o = 16; o >= 1; o >>= 1) {
                    X0 += __shfl_xor_sync(0xffffffffu, X0, o);
                    X1 += __shfl_xor_sync(0xffffffffu, X1, o);
                    X2 += __shfl_xor_sync(0xffffffffu, X2, o);
                }
                // Element k = lane: window q / 4, MMA j = q % 4 (half j / 2, slot j % 2),
                // B row k -> lane t = (k % 16) / 4, byte k % 4 of register b0 (k < 16) or b1.
                const int j = q & 3, t = (lane & 15) >> 2;
                uint8_t* half = xreg + (size_t)((q >> 2) * 2 + (j >> 1)) * 32 * 16;
                uint8_t* half_b = half + (size_t)mp.nkb * 128;
                const int off = ((j & 1) * 2 + (lane >> 4)) * 4 + (lane & 3);
                half[(2 * j * 4 + t) * 16 + off] = (uint8_t)d2;
                half[((2 * j + 1) * 4 + t) * 16 + off] = (uint8_t)d1;
                half_b[(2 * j * 4 + t) * 16 + off] = (uint8_t)d0;
                if (lane == 0) gq[q] = make_int4(8 * X2, 8 * X1, 8 * X0, __float_as_int(ge));
            }
        } else {
            // Fragment order: for every four k16 blocks, lane t (0..3) owns 32
            // contiguous bytes (blocks kb..kb+3, registers b0 b1 each).
            __half* xh = reinterpret_cast<__half*>(xs);
            for (int e = tid; e < p.k; e += kMW * 32) {
                float v = aexis_load_act(p.x, p.a_dtype, e);
                if (norm) v = v * inv * p.norm_gamma[e];
                if (p.act_quant) v = aexis_act_code(v, p.act_scale, p.act_zero_point, p.act_unsigned);
                int slot;
                if constexpr (BITS == 4) {
                    slot = q4_x_slot(e);
                } else {
                    const int kb = e >> 4, w16 = e & 15;
                    slot = (((((kb >> 2) * 4 + ((w16 & 7) >> 1)) * 4 + (kb & 3)) * 2) + (w16 >> 3)) * 2 + (w16 & 1);
                }
                const __half hi = __float2half_rn(v);
                xh[slot] = hi;
                if constexpr (XF == 2) xh[(size_t)mp.nkb * 16 + slot] = __float2half_rn(v - __half2float(hi));
            }
            if (tid < 8) reinterpret_cast<uint32_t*>(xs + (size_t)XF * mp.nkb * 4)[tid] = 0u;  // zero block
        }
        named_sync(1, kMW * 32);
    }
    griddep_launch();

    const int grp = warp / KW, ks = warp % KW;
    const int kb_per = mp.nkb / KW;
    const int kb0 = ks * kb_per;
    const int g = lane >> 2, tig = lane & 3;
    // B fragment sources: lanes 0-3 read their column-0 slice, the others a
    // zero block (column 1..7 of B), so every lane loads unconditionally.
    const uint4* xzero = reinterpret_cast<const uint4*>(xs + (size_t)XF * mp.nkb * 4);
    const uint4* xhi = lane < 4 ? reinterpret_cast<const uint4*>(xs) + lane * 2 : xzero;
    const uint4* xlo = lane < 4 ? reinterpret_cast<const uint4*>(xs + (size_t)mp.nkb * 4) + lane * 2 : xzero;
    const int xstep = lane < 4 ? 8 : 0;  // uint4 per four blocks
    unsigned long long best_key = 0ull;

    // This group's local-th unit sits in its private stage grp + NG * (local % SPG),
    // fill local / SPG: the group waits for fill f of a stage only after it
    // consumed fill f - 1. Slot and fill parity advance by one per unit.
    int slot = 0, local = 0;
    uint32_t fill_par = 0;
    for (int it = grp; it < my_units; it += NG, ++local) {
        const int s = grp + NG * slot;
        // Warp-uniform, so that the MMAs and shuffles below see the whole warp.
        const bool ready = __all_sync(0xffffffffu, mbar_wait(full + s, fill_par));
        if (++slot == SPG) {
            slot = 0;
            fill_par ^= 1u;
        }
        if (!ready) {
            report_timeout(p.status);
            *abort_flag = 1;
        }
        const size_t u = (size_t)blockIdx.x + (size_t)it * gridDim.x;  // 16-row tile
        const uint8_t* wt = ring + (size_t)s * mp.stage_bytes;
        // Scales: [group][8][2], the pair (row g, row g + 8) adjacent.
        const ST* st = reinterpret_cast<const ST*>(wt + mp.tile_wbytes) + g * 2;
        float y0 = 0.0f, y1 = 0.0f;  // rows g and g + 8 (column 0: lanes with tig == 0)
        if constexpr (S8) {
            if (ready) {
                // Windows of four groups (k128): two 16-byte weight loads (words
                // W0 W1 of each group), two B loads, four MMAs into one
                // accumulator; lane (g, t) then scales group 4w + t.
                const int wpw = (mp.nkb >> 3) / KW, w0 = ks * wpw;
                const uint4* wv = reinterpret_cast<const uint4*>(wt) + lane;
                const uint4* bv = reinterpret_cast<const uint4*>(xreg) + lane;
                const uint4* bv0 = reinterpret_cast<const uint4*>(xreg + (size_t)mp.nkb * 128) + lane;
                const int4* gq = reinterpret_cast<const int4*>(xreg + (size_t)mp.nkb * 256);
#pragma unroll 2
                for (int w = w0; w < w0 + wpw; ++w) {
                    const uint4 wa = wv[(2 * w) * 32], wb = wv[(2 * w + 1) * 32];
                    const uint4 ba = bv[(2 * w) * 32], bb = bv[(2 * w + 1) * 32];
                    const uint4 ea = bv0[(2 * w) * 32], eb = bv0[(2 * w + 1) * 32];
                    int c[4], d[4];
                    uint32_t a[4];
                    s8_frag(wa.x, wa.y, a);
                    mma_s8_zc(c, a, make_uint2(ba.x, ba.y));
                    mma_s8_zc(d, a, make_uint2(ea.x, ea.y));
                    s8_frag(wa.z, wa.w, a);
                    mma_s8(c, a, make_uint2(ba.z, ba.w));
                    mma_s8(d, a, make_uint2(ea.z, ea.w));
                    s8_frag(wb.x, wb.y, a);
                    mma_s8(c, a, make_uint2(bb.x, bb.y));
                    mma_s8(d, a, make_uint2(eb.x, eb.y));
                    s8_frag(wb.z, wb.w, a);
                    mma_s8(c, a, make_uint2(bb.z, bb.w));
                    mma_s8(d, a, make_uint2(eb.z, eb.w));
                    const int q = 4 * w + tig;
                    const int4 gi = gq[q];
                    float s0, s1;
                    load_scale_pair(st + q * 16, s0, s1);
                    // Row g (weights u = q + 8): digit sums minus 8 sum(d); row
                    // g + 8 (weights 16 q): the digit sums, 1/16 in the factor.
                    const float f0 = fmaf((float)(c[0] - gi.x), 65536.0f,
                                          fmaf((float)(c[1] - gi.y), 256.0f, (float)(d[0] - gi.z)));
                    const float f1 = fmaf((float)c[2], 65536.0f, fmaf((float)c[3], 256.0f, (float)d[2]));
                    const float ge = __int_as_float(gi.w);
                    y0 = fmaf(f0, s0 * ge, y0);
                    y1 = fmaf(f1, s1 * (ge * 0.0625f), y1);
                }
                y0 += __shfl_xor_sync(0xffffffffu, y0, 1);
                y0 += __shfl_xor_sync(0xffffffffu, y0, 2);
                y1 += __shfl_xor_sync(0xffffffffu, y1, 1);
                y1 += __shfl_xor_sync(0xffffffffu, y1, 2);
            }
        } else if (ready) {
            float c[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            int gi = kb0 / mp.gk, gpos = kb0 - gi * mp.gk;  // runtime group tracking (GK == 0)
#pragma unroll 2
            for (int kb = kb0; kb < kb0 + kb_per; kb += 4) {
                // This lane's words of blocks kb..kb+3: one (Q4) or two (Q8) per block.
                uint32_t words[2 * 4];
                if constexpr (BITS == 4) {
                    const uint4 wq = *reinterpret_cast<const uint4*>(wt + ((size_t)(kb >> 2) * 32 + lane) * 16);
                    words[0] = wq.x; words[1] = wq.y; words[2] = wq.z; words[3] = wq.w;
                } else {
                    const uint4* wp = reinterpret_cast<const uint4*>(wt + ((size_t)(kb >> 2) * 32 + lane) * 32);
                    const uint4 w01 = wp[0], w23 = wp[1];
                    words[0] = w01.x; words[1] = w01.y; words[2] = w01.z; words[3] = w01.w;
                    words[4] = w23.x; words[5] = w23.y; words[6] = w23.z; words[7] = w23.w;
                }
                const uint4 bh01 = xhi[(kb >> 2) * xstep], bh23 = xhi[(kb >> 2) * xstep + 1];
                uint4 bl01 = make_uint4(0u, 0u, 0u, 0u), bl23 = bl01;
                if constexpr (XF == 2) {
                    bl01 = xlo[(kb >> 2) * xstep];
                    bl23 = xlo[(kb >> 2) * xstep + 1];
                }
                const uint2 bh[4] = {make_uint2(bh01.x, bh01.y), make_uint2(bh01.z, bh01.w),
                                     make_uint2(bh23.x, bh23.y), make_uint2(bh23.z, bh23.w)};
                const uint2 blo[4] = {make_uint2(bl01.x, bl01.y), make_uint2(bl01.z, bl01.w),
                                      make_uint2(bl23.x, bl23.y), make_uint2(bl23.z, bl23.w)};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t a[4];
                    if constexpr (BITS == 4) decode_frag(words[j], a);
                    else decode_frag8(words[2 * j], words[2 * j + 1], a);
                    if constexpr (GK == 2) {
                        // Static groups of two blocks: fresh accumulator on even j.
                        if ((j & 1) == 0) mma16816_zc(c, a, bh[j]);
                        else mma16816(c, a, bh[j]);
                        if constexpr (XF == 2) mma16816(c, a, blo[j]);
                        if (j & 1) {
                            float s0, s1;
                            load_scale_pair(st + ((kb + j) >> 1) * 16, s0, s1);
                            y0 = fmaf(c[0], s0, y0);
                            y1 = fmaf(c[2], s1, y1);
                        }
                    } else {
                        mma16816(c, a, bh[j]);
                        if constexpr (XF == 2) mma16816(c, a, blo[j]);
                        if (++gpos == mp.gk) {
                            float s0, s1;
                            load_scale_pair(st + gi * 16, s0, s1);
                            y0 = fmaf(c[0], s0, y0);
                            y1 = fmaf(c[2], s1, y1);
                            c[0] = c[1] = c[2] = c[3] = 0.0f;
                            gpos = 0;
                            ++gi;
                        }
                    }
                }
            }
            if (GK == 0 && gpos != 0) {  // one scale per row: this warp's share of the single group
                float s0, s1;
                load_scale_pair(st, s0, s1);
                y0 = fmaf(c[0], s0, y0);
                y1 = fmaf(c[2], s1, y1);
            }
        }
        __syncwarp();
        if (ready && lane == 0) mbar_arrive(empty + s);

        // Add the KW partials of each row (KW > 1), then the epilogue (lanes
        // 0-15 of the group's first warp; the pair partner of row r is r ^ 1).
        float* rb = red + ((local & 1) * NG + grp) * KW * 16;
        if (tig == 0) {
            rb[ks * 16 + g] = y0;
            rb[ks * 16 + g + 8] = y1;
        }
        if constexpr (KW > 1) named_sync(2 + grp, KW * 32);
        else __syncwarp();
        if (*abort_flag) break;
        if (ks == 0) {
            float v = 0.0f;
            if (lane < 16)
#pragma unroll
                for (int w = 0; w < KW; ++w) v += rb[w * 16 + lane];
            const float partner = __shfl_xor_sync(0xffffffffu, v, 1);
            const long long row = (long long)u * 16 + lane;
            if (lane < 16 && row < p.n) epilogue(p, (int)row, v, partner, best_key);
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

struct MmaPlan {
    int kw = 0, units = 0, stages = 0, stage_bytes = 0, smem = 0, per_sm = 1;
    bool s8 = false;  // the int8 path (kS8Able, many tiles per CTA)
};

int frag_tiles_padded(int n) { return ((n + 15) / 16 + 7) / 8 * 8; }

int scale_groups(const aexis_weights* w) { return w->kind == WK_Q4 && w->group > 0 ? w->k / w->group : 1; }

// Bytes of one 16-row tile of fragment words.
int tile_wbytes(const aexis_weights* w) { return (w->kind == WK_Q8 ? 16 : 8) * w->k; }

// K split: enough (tile, K-share) units for every consumer warp of two CTAs
// per SM (KW = 1 when the tiles alone suffice; up to 8 warps on one tile for
// small N), within the alignment the fragment layout and the scale groups
// allow. Ring: one tile per stage, as deep as the shared-memory budget of two
// CTAs per SM allows (at least 3), else one CTA per SM.
bool plan_mma(const aexis_weights* w, int xf, int sm_count, MmaPlan& pl) {
    const int nkb = w->k / 16;
    const int gk = w->kind == WK_Q4 && w->group > 0 ? w->group / 16 : nkb;
    const int ntiles = (w->n + 15) / 16;
    const int st = w->scale_dtype == AEXIS_F16 ? 2 : 4;
    const int stage = tile_wbytes(w) + scale_groups(w) * 16 * st;
    // The int8 path (fp16 activations, Q4 group 32, K a multiple of 128).
    const bool s8 = xf == 1 && w->kind == WK_Q4 && gk == 2 && nkb % 8 == 0 && ntiles >= 8 * sm_count;
    const int fixed = mma_x_bytes(s8, xf, nkb) + 2 * kMW * 16 * 4 + 16 * 16 + 64 + kMW * 4 + 128;
    const int want = 2 * sm_count * kMW;  // warp units that fill two CTAs per SM
    int kw0 = 1;
    while (kw0 < 8 && (long long)ntiles * kw0 < want) kw0 <<= 1;
    for (int per_sm = 2; per_sm >= 1; --per_sm) {
        const int budget = per_sm == 2 ? 113 * 1024 : 227 * 1024;
        int S = (budget - fixed) / stage;
        S = S > 16 ? 16 : S;
        if (S < (per_sm == 2 ? 3 : 2)) continue;
        // Every warp group owns S / NG stages: NG = 8 / kw must not exceed S.
        // Preferred split first, then larger, then smaller ones that still fit.
        int kw_min = 1;
        while (kw_min < 8 && kMW / kw_min > S) kw_min <<= 1;
        const int pref = kw0 > kw_min ? kw0 : kw_min;
        auto fits = [&](int kw) {
            return nkb % (kw * 4) == 0 && ((nkb / kw) % gk == 0 || gk == nkb) && (!s8 || (nkb / 8) % kw == 0);
        };
        int kw = 0;
        for (int c = pref; c <= 8 && !kw; c <<= 1)
            if (fits(c)) kw = c;
        for (int c = pref >> 1; c >= kw_min && !kw; c >>= 1)
            if (fits(c)) kw = c;
        if (!kw) continue;
        S -= S % (kMW / kw);
        pl.kw = kw;
        pl.units = ntiles;
        pl.stages = S;
        pl.stage_bytes = stage;
        pl.smem = S * stage + fixed;
        pl.per_sm = per_sm;
        pl.s8 = s8;
        return true;
    }
    return false;
}

template <typename ST, int XF, int KW, int GK, int BITS, bool S8P>
cudaError_t launch_mma_t(const MmaParams& mp, int grid, int smem, bool pdl, cudaStream_t stream) {
    static int configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (smem > configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(gemv_mma_kernel<ST, XF, KW, GK, BITS, S8P>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        configured[dev] = smem;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kMmaThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, gemv_mma_kernel<ST, XF, KW, GK, BITS, S8P>, mp);
}

template <typename ST, int XF, int GK, int BITS, bool S8P = false>
cudaError_t launch_mma_kw(const MmaParams& mp, int kw, int grid, int smem, bool pdl, cudaStream_t s) {
    switch (kw) {
        case 1: return launch_mma_t<ST, XF, 1, GK, BITS, S8P>(mp, grid, smem, pdl, s);
        case 2: return launch_mma_t<ST, XF, 2, GK, BITS, S8P>(mp, grid, smem, pdl, s);
        case 4: return launch_mma_t<ST, XF, 4, GK, BITS, S8P>(mp, grid, smem, pdl, s);
        default: return launch_mma_t<ST, XF, 8, GK, BITS, S8P>(mp, grid, smem, pdl, s);
    }
}

// Q4 with groups of 32 takes the static group path; Q8 (one scale per row)
// and other Q4 groups the run-time one.
template <typename ST, int XF>
cudaError_t launch_mma_gk(const MmaParams& mp, int bits, int kw, bool s8, int grid, int smem, bool pdl,
                          cudaStream_t s) {
    if (bits == 8) return launch_mma_kw<ST, XF, 0, 8>(mp, kw, grid, smem, pdl, s);
    if (mp.gk == 2) {
        if constexpr (XF == 1)
            if (s8) return launch_mma_kw<ST, XF, 2, 4, true>(mp, kw, grid, smem, pdl, s);
        return launch_mma_kw<ST, XF, 2, 4>(mp, kw, grid, smem, pdl, s);
    }
    return launch_mma_kw<ST, XF, 0, 4>(mp, kw, grid, smem, pdl, s);
}

}  // namespace

bool gemv_mma_eligible(const aexis_weights* w) {
    if ((w->kind != WK_Q4 && w->kind != WK_Q8) || w->k % 64 != 0 || w->n <= 0) return false;
    if (w->kind == WK_Q4 && w->group > 0 && (w->group % 16 != 0 || w->k % w->group != 0)) return false;
    MmaPlan pl;
    return plan_mma(w, 2, 148, pl);
}

size_t gemv_mma_frag_bytes(const aexis_weights* w, size_t* scale_bytes) {
    const size_t tiles = (size_t)frag_tiles_padded(w->n);
    if (scale_bytes)
        *scale_bytes = tiles * scale_groups(w) * 16 * (w->scale_dtype == AEXIS_F16 ? 2 : 4);
    return tiles * (size_t)tile_wbytes(w);
}

cudaError_t launch_repack_frag(const aexis_weights* w, cudaStream_t s) {
    const int tiles = frag_tiles_padded(w->n);
    if (w->kind == WK_Q8) {
        if (w->scale_dtype == AEXIS_F16)
            repack_q8_frag_kernel<__half><<<148 * 8, 256, 0, s>>>(
                reinterpret_cast<const uint32_t*>(w->data), reinterpret_cast<const __half*>(w->scales), w->n, w->k,
                tiles, reinterpret_cast<uint32_t*>(w->frag), reinterpret_cast<__half*>(w->frag_scales));
        else
            repack_q8_frag_kernel<float><<<148 * 8, 256, 0, s>>>(
                reinterpret_cast<const uint32_t*>(w->data), reinterpret_cast<const float*>(w->scales), w->n, w->k,
                tiles, reinterpret_cast<uint32_t*>(w->frag), reinterpret_cast<float*>(w->frag_scales));
        return cudaGetLastError();
    }
    if (w->scale_dtype == AEXIS_F16)
        repack_q4_frag_kernel<__half><<<148 * 8, 256, 0, s>>>(
            reinterpret_cast<const uint32_t*>(w->data), reinterpret_cast<const __half*>(w->scales), w->n, w->k,
            w->group, tiles, reinterpret_cast<uint32_t*>(w->frag), reinterpret_cast<__half*>(w->frag_scales));
    else
        repack_q4_frag_kernel<float><<<148 * 8, 256, 0, s>>>(
            reinterpret_cast<const uint32_t*>(w->data), reinterpret_cast<const float*>(w->scales), w->n, w->k,
            w->group, tiles, reinterpret_cast<uint32_t*>(w->frag), reinterpret_cast<float*>(w->frag_scales));
    return cudaGetLastError();
}

bool gemv_mma_supported(const aexis_weights* w, int a_dtype) {
    return w->frag && w->frag_scales && (a_dtype == AEXIS_F16 || a_dtype == AEXIS_F32);
}

cudaError_t launch_gemv_mma(const GemvArgs& a, int sm_count, cudaStream_t stream) {
    const aexis_weights* w = a.w;
    const int xf = a.a_dtype == AEXIS_F16 ? 1 : 2;
    MmaPlan pl;
    if (!plan_mma(w, xf, sm_count, pl)) return cudaErrorNotSupported;
    MmaParams mp = {};
    StreamParams& sp = mp.sp;
    sp.W = reinterpret_cast<const uint8_t*>(w->frag);
    sp.S = reinterpret_cast<const uint8_t*>(w->frag_scales);
    sp.n = w->n;
    sp.k = w->k;
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
    sp.status = a.status;
    sp.act_quant = a.act_quant;
    sp.act_scale = a.act_scale;
    sp.act_zero_point = a.act_zero_point;
    sp.act_unsigned = a.act_unsigned;
    mp.nkb = w->k / 16;
    mp.gk = w->kind == WK_Q4 && w->group > 0 ? w->group / 16 : mp.nkb;
    mp.tile_wbytes = tile_wbytes(w);
    mp.tile_sbytes = scale_groups(w) * 16 * (w->scale_dtype == AEXIS_F16 ? 2 : 4);
    mp.units = pl.units;
    mp.ring_stages = pl.stages;
    mp.stage_bytes = pl.stage_bytes;
    const int grid = pl.units < pl.per_sm * sm_count ? pl.units : pl.per_sm * sm_count;
    const int bits = w->kind == WK_Q8 ? 8 : 4;
    if (w->scale_dtype == AEXIS_F16) {
        if (xf == 1) return launch_mma_gk<__half, 1>(mp, bits, pl.kw, pl.s8, grid, pl.smem, a.pdl, stream);
        return launch_mma_gk<__half, 2>(mp, bits, pl.kw, pl.s8, grid, pl.smem, a.pdl, stream);
    }
    if (xf == 1) return launch_mma_gk<float, 1>(mp, bits, pl.kw, pl.s8, grid, pl.smem, a.pdl, stream);
    return launch_mma_gk<float, 2>(mp, bits, pl.kw, pl.s8, grid, pl.smem, a.pdl, stream);
}
