// gemv_dev.cuh -- device helpers shared by the GEMV kernels (k_gemv.cu,
// k_gemv_stream.cu): int4 / int8 unpacking into fp32 with packed fp32x2
// arithmetic, async-proxy barriers and bulk copies, bounded waits.
#pragma once

#include "aexis_internal.h"

namespace aexis_dev {

__device__ __forceinline__ uint4 ldg_stream(const uint4* p) {
    uint4 r;
    asm("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
        : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
        : "l"(p));
    return r;
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

// acc.{x,y} += (as_float(f0) + m0, as_float(f1) + m1) * (a0, a1), with packed
// fp32x2 add and FMA (each lane rounds exactly as the scalar op would).
__device__ __forceinline__ void mac2(unsigned long long& acc, uint32_t f0, uint32_t f1, float m0,
                                     float m1, float a0, float a1) {
    asm("{\n\t.reg .b64 f, m, a, d;\n\t"
        "mov.b64 f, {%1, %2};\n\t"
        "mov.b64 m, {%3, %4};\n\t"
        "mov.b64 a, {%5, %6};\n\t"
        "add.rn.f32x2 d, f, m;\n\t"
        "fma.rn.f32x2 %0, d, a, %0;\n\t}"
        : "+l"(acc)
        : "r"(f0), "r"(f1), "f"(m0), "f"(m1), "f"(a0), "f"(a1));
}

__device__ __forceinline__ float sum2(unsigned long long acc) {
    return __uint_as_float((uint32_t)acc) + __uint_as_float((uint32_t)(acc >> 32));
}

// Int4 magic constants: (nibble-field ^ 8<<4j') | 0x4B000000 read as fp32 is
// 2^23 + (u ^ 8) * 16^j'; subtracting 2^23 + 8 * 16^j' leaves q * 16^j'.
constexpr uint32_t kQ4X0 = 0x4B000008u, kQ4X1 = 0x4B000080u, kQ4X2 = 0x4B000800u,
                   kQ4X3 = 0x4B008000u, kQ4X4 = 0x4B080000u;
#define Q4M(x) (-__uint_as_float(x))

// 32 int4 products of one 16-byte chunk against 32 pre-scaled activations.
__device__ __forceinline__ unsigned long long dot_q4_chunk(const uint4 w, const float4* a) {
    unsigned long long acc = 0ull;
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t v = words[i];
        const uint32_t vh = v >> 12;
        const float4 a0 = a[2 * i], a1 = a[2 * i + 1];
        mac2(acc, (v & 0xFu) ^ kQ4X0, (v & 0xF0u) ^ kQ4X1, Q4M(kQ4X0), Q4M(kQ4X1), a0.x, a0.y);
        mac2(acc, (v & 0xF00u) ^ kQ4X2, (v & 0xF000u) ^ kQ4X3, Q4M(kQ4X2), Q4M(kQ4X3), a0.z, a0.w);
        mac2(acc, (v & 0xF0000u) ^ kQ4X4, (vh & 0xF00u) ^ kQ4X2, Q4M(kQ4X4), Q4M(kQ4X2), a1.x, a1.y);
        mac2(acc, (vh & 0xF000u) ^ kQ4X3, (vh & 0xF0000u) ^ kQ4X4, Q4M(kQ4X3), Q4M(kQ4X4), a1.z, a1.w);
    }
    return acc;
}

// 16 int8 products of one 16-byte chunk. Bytes are biased by 128 (XOR), moved
// under the 2^23 exponent with PRMT, and the 2^23 + 128 bias is subtracted.
__device__ __forceinline__ void dot_q8_chunk(unsigned long long& acc, const uint4 w, const float4* a) {
    const uint32_t words[4] = {w.x, w.y, w.z, w.w};
    const float m = -__uint_as_float(0x4B000080u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t v = words[i] ^ 0x80808080u;
        const float4 av = a[i];
        mac2(acc, __byte_perm(v, 0x4B000000u, 0x7650), __byte_perm(v, 0x4B000000u, 0x7651), m, m,
             av.x, av.y);
        mac2(acc, __byte_perm(v, 0x4B000000u, 0x7652), __byte_perm(v, 0x4B000000u, 0x7653), m, m,
             av.z, av.w);
    }
}

// Physical 16-byte unit of logical unit u in the swizzled activation buffer.
__device__ __forceinline__ int swz(int u) { return u ^ ((u >> 3) & 7); }

template <typename ST>
__device__ __forceinline__ float load_scale(const ST* s, long long i);
template <>
__device__ __forceinline__ float load_scale<float>(const float* s, long long i) { return __ldg(s + i); }
template <>
__device__ __forceinline__ float load_scale<__half>(const __half* s, long long i) {
    return __half2float(__ldg(s + i));
}


// --------------------------------------------------- pair-form int4 / int8 dot
// A 16-byte chunk is read as two 64-bit halves {w0, w1} and {w2, w3}. Field j
// of both words of a half is isolated by one 64-bit AND/XOR, so each decoded
// fp32 pair is born in an aligned register pair and feeds the packed fp32x2
// add/FMA directly. The activations are staged in the matching pair order
// (see act_pair_index) and pre-scaled by the field's 16^-j' (int4) or
// 256^-j' (int8) so every product is exact before its single rounding.
//
// acc += (((x & m) ^ c) as fp32x2 + b) * a, with one three-input LOP3
// (truth table 0x6A = (a & b) ^ c) per 32-bit half. m and c arrive in
// registers (PairConsts) so the assembler keeps each isolate as one LOP3.
__device__ __forceinline__ void mac_pair(unsigned long long& acc, unsigned long long x, uint32_t m, uint32_t c,
                                         unsigned long long b, unsigned long long a) {
    asm("{\n\t.reg .b32 xl, xh, tl, th;\n\t.reg .b64 t;\n\t"
        "mov.b64 {xl, xh}, %1;\n\t"
        "lop3.b32 tl, xl, %2, %3, 0x6A;\n\t"
        "lop3.b32 th, xh, %2, %3, 0x6A;\n\t"
        "mov.b64 t, {tl, th};\n\t"
        "add.rn.f32x2 t, t, %4;\n\t"
        "fma.rn.f32x2 %0, t, %5, %0;\n\t}"
        : "+l"(acc)
        : "l"(x), "r"(m), "r"(c), "l"(b), "l"(a));
}

__device__ __forceinline__ unsigned long long dup64(uint32_t v) {
    return ((unsigned long long)v << 32) | v;
}

// Field constants of the int4 / int8 decode: for field j' the mask, the XOR
// (sign flip + 2^23 exponent) and the negated magic (2^23 + bias * 2^(w*j'))
// as fp32x2 bits. Built from a runtime zero so they stay in registers.
struct PairConsts {
    uint32_t m[5], c[5];
    unsigned long long b[5];
};

template <int BITS>
__device__ __forceinline__ PairConsts make_pair_consts(uint32_t zero) {
    PairConsts k;
#pragma unroll
    for (int j = 0; j < 5; ++j) {
        const uint32_t mask = BITS == 4 ? (0xFu << (4 * j)) : (j < 2 ? 0xFFu << (8 * j) : 0u);
        const uint32_t x = BITS == 4 ? (0x4B000000u | (8u << (4 * j))) : (0x4B000000u | (j < 2 ? 0x80u << (8 * j) : 0u));
        k.m[j] = mask | zero;
        k.c[j] = x | zero;
        k.b[j] = dup64(__float_as_uint(-__uint_as_float(x))) | zero;
    }
    return k;
}

// One int4 chunk: x01 = {w0, w1}, x23 = {w2, w3}; a[0..7] pairs of words
// (0,1), a[8..15] of words (2,3), index j = nibble. Nibbles 5..7 are read
// from the halves shifted right by 12 (the 64-bit shift only pollutes bits
// 20..31 of the low word, which no mask selects).
__device__ __forceinline__ void dot_q4_pairs(unsigned long long x01, unsigned long long x23,
                                             const unsigned long long* a, const PairConsts& k,
                                             unsigned long long& acc01, unsigned long long& acc23) {
    const unsigned long long h01 = x01 >> 12, h23 = x23 >> 12;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int jp = j < 5 ? j : j - 3;
        mac_pair(acc01, j < 5 ? x01 : h01, k.m[jp], k.c[jp], k.b[jp], a[j]);
        mac_pair(acc23, j < 5 ? x23 : h23, k.m[jp], k.c[jp], k.b[jp], a[8 + j]);
    }
}

// One int8 chunk (16 values): a[0..3] pairs of words (0,1), a[4..7] of (2,3);
// bytes 2, 3 come from the halves shifted right by 16.
__device__ __forceinline__ void dot_q8_pairs(unsigned long long x01, unsigned long long x23,
                                             const unsigned long long* a, const PairConsts& k,
                                             unsigned long long& acc01, unsigned long long& acc23) {
    const unsigned long long h01 = x01 >> 16, h23 = x23 >> 16;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int jp = j & 1;
        mac_pair(acc01, j < 2 ? x01 : h01, k.m[jp], k.c[jp], k.b[jp], a[j]);
        mac_pair(acc23, j < 2 ? x23 : h23, k.m[jp], k.c[jp], k.b[jp], a[4 + j]);
    }
}

// Position of activation element e of a chunk in the pair-staged order
// (fp32 slot within the chunk) and its pre-scale.
template <int BITS>
__device__ __forceinline__ int act_pair_slot(int e) {
    constexpr int FPW = BITS == 4 ? 8 : 4;  // fields per 32-bit word
    const int w = e / FPW, j = e % FPW;
    return ((w >> 1) * FPW + j) * 2 + (w & 1);
}
template <int BITS>
__device__ __forceinline__ float act_pair_prescale(int e) {
    if (BITS == 4) {
        const int j = e & 7;
        return __uint_as_float((uint32_t)(127 - 4 * (j < 5 ? j : j - 3)) << 23);
    }
    return (e & 1) ? __uint_as_float((uint32_t)(127 - 8) << 23) : 1.0f;
}

__device__ __forceinline__ float sum2u(unsigned long long acc) {
    return __uint_as_float((uint32_t)acc) + __uint_as_float((uint32_t)(acc >> 32));
}

template <typename T>
__device__ __forceinline__ float to_float(T v);
template <>
__device__ __forceinline__ float to_float<float>(float v) { return v; }
template <>
__device__ __forceinline__ float to_float<__half>(__half v) { return __half2float(v); }

// ---------------------------------------------------------------- async copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

// Makes mbarrier initialisation visible to the async proxy (bulk copies).
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}

// Arrival counting `count` of the barrier's expected arrivals.
__device__ __forceinline__ void mbar_arrive_cnt(uint64_t* bar, uint32_t count) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
                 "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, p;\n\t}"
                 : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
    return ok != 0;
}

// Every wait on a barrier is bounded: about one second of SM clock, after
// which the caller records AEXIS_E_TIMEOUT in the context's status word and
// returns instead of spinning forever.
constexpr long long kWaitLimitCycles = 2000000000LL;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
        if (clock64() - t0 > kWaitLimitCycles) return false;
    return true;
}

__device__ __forceinline__ void report_timeout(int* status) {
    if (status) atomicCAS(status, 0, (int)AEXIS_E_TIMEOUT);
}

// Global -> shared bulk copy (no tensor map), completing on `bar` with
// `bytes` transaction bytes. dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
        : "memory");
}

// Same copy without an L2 policy hint.
__device__ __forceinline__ void bulk_g2s_plain(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// L2 policy for weights that are read once per call.
__device__ __forceinline__ uint64_t policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}

// Named barrier over the first `threads` threads of the CTA (id 1..15).
__device__ __forceinline__ void named_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

}  // namespace aexis_dev
