// mma_frag.cuh -- register-level pieces of the tensor-core GEMVs
// (k_gemv_mma.cu, k_decoder_persist.cu): exact fp16 decode of packed Q4 / Q8
// A fragments and the m16n8k16 MMA (fp16 x fp16 -> fp32).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace aexis_dev {

__device__ __forceinline__ uint32_t lop3_f16pair(uint32_t q, uint32_t mask) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(q), "r"(mask), "r"(0x64006400u));  // (q & mask) | c
    return r;
}

// The A fragment of one k16 block from its packed word: fp16 pairs of q.
__device__ __forceinline__ void decode_frag(uint32_t q, uint32_t (&a)[4]) {
    const __half2 off = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));     // 1032
    const __half2 inv16 = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));   // 1/16
    const __half2 off16 = __halves2half2(__ushort_as_half(0xD480), __ushort_as_half(0xD480));   // -72
    const uint32_t q8 = q >> 8;
    uint32_t t0 = lop3_f16pair(q, 0x000F000Fu), t1 = lop3_f16pair(q, 0x00F000F0u);
    uint32_t t2 = lop3_f16pair(q8, 0x000F000Fu), t3 = lop3_f16pair(q8, 0x00F000F0u);
    __half2 h0 = __hsub2(*reinterpret_cast<__half2*>(&t0), off);           // (1024 + u) - 1032 = q
    __half2 h1 = __hfma2(*reinterpret_cast<__half2*>(&t1), inv16, off16);  // (1024 + 16u) / 16 - 72 = q
    __half2 h2 = __hsub2(*reinterpret_cast<__half2*>(&t2), off);
    __half2 h3 = __hfma2(*reinterpret_cast<__half2*>(&t3), inv16, off16);
    a[0] = *reinterpret_cast<uint32_t*>(&h0);
    a[1] = *reinterpret_cast<uint32_t*>(&h1);
    a[2] = *reinterpret_cast<uint32_t*>(&h2);
    a[3] = *reinterpret_cast<uint32_t*>(&h3);
}

// The A fragment of one k16 block from its two Q8 words: PRMT puts each
// offset-binary byte under the fp16 exponent of 1024, HSUB2 removes 1152.
__device__ __forceinline__ void decode_frag8(uint32_t w0, uint32_t w1, uint32_t (&a)[4]) {
    const __half2 off = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
    const uint32_t t0 = __byte_perm(w0, 0x64646464u, 0x4140), t1 = __byte_perm(w0, 0x64646464u, 0x4342);
    const uint32_t t2 = __byte_perm(w1, 0x64646464u, 0x4140), t3 = __byte_perm(w1, 0x64646464u, 0x4342);
    __half2 h0 = __hsub2(*reinterpret_cast<const __half2*>(&t0), off);
    __half2 h1 = __hsub2(*reinterpret_cast<const __half2*>(&t1), off);
    __half2 h2 = __hsub2(*reinterpret_cast<const __half2*>(&t2), off);
    __half2 h3 = __hsub2(*reinterpret_cast<const __half2*>(&t3), off);
    a[0] = *reinterpret_cast<uint32_t*>(&h0);
    a[1] = *reinterpret_cast<uint32_t*>(&h1);
    a[2] = *reinterpret_cast<uint32_t*>(&h2);
    a[3] = *reinterpret_cast<uint32_t*>(&h3);
}

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint2 b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}

// d = a b (accumulator input zero).
__device__ __forceinline__ void mma16816_zc(float (&c)[4], const uint32_t (&a)[4], uint2 b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=f"(c[0]), "=f"(c[1]), "=f"(c[2]), "=f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "f"(0.0f));
}

}  // namespace aexis_dev
