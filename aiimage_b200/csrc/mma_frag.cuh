// mma_frag.cuh -- register-level pieces of the tensor-core GEMVs
// (k_gemv_mma.cu, k_decoder_persist.cu): exact fp16 decode of packed Q4 / Q8
// A fragments, the fp16 B-fragment order of Q4 tiles and the m16n8k16 MMA
// (fp16 x fp16 -> fp32).
#pragma once
#include <cstdint>
#include <cuda_fp16.h>

namespace aexis_dev {

// (q & mask) ^ c in one LOP3: c's bits inside the mask flip bits of q, those
// outside it are set.
__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t q, uint32_t mask, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(q), "r"(mask), "r"(c));
    return r;
}

// Q4 A fragments. A tile word of lane (g, t) holds, for one k16 half of a
// k32 chunk (k = 4 t + i, i = 0..3, within the half), byte i = the two's
// complement nibbles of rows g (low nibble) and g + 8 (high nibble). The
// same words feed the int8 MMA (m16n8k32) directly and the fp16 MMA
// (m16n8k16) through this decode, whose k order within the block is
// a0 / a1 = (4t, 4t + 2), a2 / a3 = (4t + 1, 4t + 3): the B fragments are
// staged in that order. Exact: the nibble, made offset-binary by the XOR,
// sits under the fp16 exponent of 1024 and the bias is removed by HSUB2 (or
// HFMA2 with 1/16 for the nibbles at bit 4).
__device__ __forceinline__ void decode_frag(uint32_t q, uint32_t (&a)[4]) {
    const __half2 off = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));     // 1032
    const __half2 inv16 = __halves2half2(__ushort_as_half(0x2C00), __ushort_as_half(0x2C00));   // 1/16
    const __half2 off16 = __halves2half2(__ushort_as_half(0xD480), __ushort_as_half(0xD480));   // -72
    const uint32_t q8 = q >> 8;
    uint32_t t0 = lop3_and_xor(q, 0x000F000Fu, 0x64086408u), t1 = lop3_and_xor(q, 0x00F000F0u, 0x64806480u);
    uint32_t t2 = lop3_and_xor(q8, 0x000F000Fu, 0x64086408u), t3 = lop3_and_xor(q8, 0x00F000F0u, 0x64806480u);
    __half2 h0 = __hsub2(*reinterpret_cast<__half2*>(&t0), off);           // (1024 + u) - 1032 = q
    __half2 h1 = __hfma2(*reinterpret_cast<__half2*>(&t1), inv16, off16);  // (1024 + 16u) / 16 - 72 = q
    __half2 h2 = __hsub2(*reinterpret_cast<__half2*>(&t2), off);
    __half2 h3 = __hfma2(*reinterpret_cast<__half2*>(&t3), inv16, off16);
    a[0] = *reinterpret_cast<uint32_t*>(&h0);
    a[1] = *reinterpret_cast<uint32_t*>(&h1);
    a[2] = *reinterpret_cast<uint32_t*>(&h2);
    a[3] = *reinterpret_cast<uint32_t*>(&h3);
}

// Half-slot of activation element e in the fp16 B fragments of Q4 tiles: per
// four k16 blocks, lane t owns 32 contiguous bytes (blocks vb..vb + 3,
// registers b0 b1, two halves each) holding k = 4t + {0, 2} (b0) and
// 4t + {1, 3} (b1) of each block, the order decode_frag gives the A side.
__device__ __forceinline__ int q4_x_slot(int e) {
    const int vb = e >> 4, j = e & 15, t = j >> 2, i = j & 3;
    return ((((vb >> 2) * 4 + t) * 4 + (vb & 3)) * 2 + (i & 1)) * 2 + (i >> 1);
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

// The int8 A fragment (m16n8k32) of one k32 chunk of a Q4 tile from its two
// words: row g as offset-binary bytes u = q + 8 (low nibbles, XOR 8), row
// g + 8 as 16 q (high nibbles in place, two's complement).
__device__ __forceinline__ void s8_frag(uint32_t w0, uint32_t w1, uint32_t (&a)[4]) {
    a[0] = lop3_and_xor(w0, 0x0F0F0F0Fu, 0x08080808u);
    a[1] = w0 & 0xF0F0F0F0u;
    a[2] = lop3_and_xor(w1, 0x0F0F0F0Fu, 0x08080808u);
    a[3] = w1 & 0xF0F0F0F0u;
}

__device__ __forceinline__ void mma_s8(int (&c)[4], const uint32_t (&a)[4], uint2 b) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y));
}

// d = a b (accumulator input zero).
__device__ __forceinline__ void mma_s8_zc(int (&c)[4], const uint32_t (&a)[4], uint2 b) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b.x), "r"(b.y), "r"(0));
}

}  // namespace aexis_dev
