// gemv_stream.cuh -- parameters and per-row epilogues shared by the batch-1
// GEMV kernels that stream row tiles through a bulk-copy ring
// (k_gemv_stream.cu: CUDA-core decode; k_gemv_mma.cu: tensor-core decode).
#pragma once
#include "gemv_dev.cuh"

namespace aexis_dev {

struct StreamParams {
    const uint8_t* W;   // [n][row_bytes]
    const uint8_t* S;   // [n][srow_bytes]
    int n, k, nchunks, row_bytes, srow_bytes, gshift;
    int ntiles, stages, stage_bytes, w_tile_bytes, act_floats;
    const void* x;
    int a_dtype;
    const float* norm_gamma;
    float norm_eps;
    const float* bias;
    float alpha, beta;
    void* y;
    int y_dtype;
    int epi;
    const float* rope_cos;
    const float* rope_sin;
    const int* rope_map;
    __half* k_cache;
    __half* v_cache;
    int head_dim, kv_cap, rot_dim;
    const int* pos_ptr;
    unsigned long long* argmax_key;
    int* status;
    uint32_t zero;   // 0, opaque to the compiler (keeps decode constants in registers)
    int act_quant;   // W8A8 codes instead of x (gemv_mma_kernel)
    float act_scale;
    int act_zero_point, act_unsigned;
};

// Output of one row (lane-local), shared with the register-streaming kernel's
// epilogue semantics. `partner` is the value of the paired row (row ^ 1).
__device__ __forceinline__ void epilogue(const StreamParams& p, int row, float val, float partner,
                                         unsigned long long& best_key) {
    switch (p.epi) {
        case EPI_STORE: {
            const float bb = p.bias ? p.beta * p.bias[row] : 0.0f;
            aexis_store_out(p.y, p.y_dtype, row, p.alpha * (bb + val));
        } break;
        case EPI_STORE_TILED: {
            const float bb = p.bias ? p.beta * p.bias[row] : 0.0f;
            aexis_store_out(p.y, p.y_dtype, row, bb + p.alpha * val);
        } break;
        case EPI_RESIDUAL:
            reinterpret_cast<float*>(p.y)[row] += p.alpha * val;
            break;
        case EPI_SWIGLU:
            if ((row & 1) == 0) reinterpret_cast<float*>(p.y)[row >> 1] = val / (1.0f + expf(-val)) * partner;
            break;
        case EPI_QKV_ROPE: {
            const int desc = p.rope_map[row];
            const int kind = desc >> 24, head = (desc >> 12) & 0xFFF, dim = desc & 0xFFF;
            const int pos = *p.pos_ptr;
            float out = val;
            if (kind != 2 && dim < p.rot_dim) {
                const int half = p.rot_dim >> 1;
                const bool first = dim < half;
                const int j = first ? dim : dim - half;
                const float c = p.rope_cos[(long long)pos * half + j];
                const float s = p.rope_sin[(long long)pos * half + j];
                const float x0 = first ? val : partner, x1 = first ? partner : val;
                out = first ? x0 * c - x1 * s : x0 * s + x1 * c;
            }
            if (kind == 0) {
                reinterpret_cast<float*>(p.y)[head * p.head_dim + dim] = out;
            } else {
                __half* cache = kind == 1 ? p.k_cache : p.v_cache;
                cache[((long long)head * p.kv_cap + pos) * p.head_dim + dim] = __float2half_rn(out);
            }
        } break;
        case EPI_LOGITS_ARGMAX: {
            reinterpret_cast<float*>(p.y)[row] = val;
            const unsigned long long key = aexis_argmax_key(val, row);
            best_key = key > best_key ? key : best_key;
        } break;
    }
}

}  // namespace aexis_dev
