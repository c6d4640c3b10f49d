// aexis_internal.h -- shared declarations of libaexis_cuda (not part of the ABI).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cstdint>
#include <cstdio>
#include <string>
#include <vector>

#include "../../include/aexis_cuda.h"

// Weight storage kinds held by an aexis_weights handle.
enum aexis_wkind { WK_Q4 = 4, WK_Q8 = 8, WK_F16 = 16, WK_F32 = 32 };

struct aexis_weights {
    int kind = 0;            // aexis_wkind
    int n = 0, k = 0;        // [n, k] logical shape
    int group = 0;           // Q4 scale block along the flat index (divides k)
    int scale_dtype = AEXIS_F32;
    void* data = nullptr;    // device: packed words (Q4/Q8) or dense values
    void* scales = nullptr;  // device: fp32 or fp16 scales (Q4/Q8)
    size_t data_bytes = 0, scale_bytes = 0;
    // Q8 weights repacked into 128-row x 64-k blocks for the tensor-core
    // batched GEMM, built on the first batched call.
    void* tc_tiled = nullptr;
    // Q4 weights and scales in the MMA-fragment layout of the tensor-core
    // GEMV (k_gemv_mma.cu), built at upload when the shape allows it.
    void* frag = nullptr;
    void* frag_scales = nullptr;
};

struct aexis_ctx {
    int device = 0;
    int sm_count = 0;
    cudaStream_t own_stream = nullptr;
    cudaStream_t stream = nullptr;
    std::string err;
    // Grow-only device scratch (split-K attention partials, argmax keys).
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    // Device status word: kernels whose bounded waits run out record
    // AEXIS_E_TIMEOUT here; aexis_cuda_sync reports and clears it.
    int* status = nullptr;
    // W8A8 activation fake-quantisation (Ops.SetInt8ActivationQuantization):
    // when enabled, aexis_cuda_gemm* first writes the activations' integer
    // codes (q - zero_point) as fp16 into act_q and multiplies by act_scale in
    // the epilogue.
    int act_quant = 0;
    float act_scale = 1.0f;
    int act_zero_point = 0;
    int act_unsigned = 0;
    void* act_q = nullptr;
    size_t act_q_bytes = 0;
    // Device sampler partials, candidates and penalised scores (grow-only).
    void* samp = nullptr;
    size_t samp_bytes = 0;
    // Row-major copy of a Pack4 texture-array activation (aexis_cuda_gemm_pack4a
    // with more than one slice; grow-only).
    void* pack_a = nullptr;
    size_t pack_a_bytes = 0;
    // aexis_cuda_gemm_topk: the logits between its GEMM and its top-k (grow-only).
    void* fused = nullptr;
    size_t fused_bytes = 0;
};

// Records `msg` on the context and returns `code`.
int aexis_fail(aexis_ctx* ctx, int code, const char* fmt, ...);
// Checks a CUDA call; on failure records "<what>: <cuda error>" and returns E_CUDA.
int aexis_cuda_check(aexis_ctx* ctx, cudaError_t e, const char* what);
// Returns a device buffer of at least `bytes` (grow-only, owned by ctx).
int aexis_scratch(aexis_ctx* ctx, size_t bytes, void** out);
// Reads (and clears) the context status word after a synchronize: returns
// the recorded error (AEXIS_E_TIMEOUT) or AEXIS_OK.
int aexis_check_status(aexis_ctx* ctx);

// ---------------------------------------------------------------- launchers
// Every launcher enqueues on `stream` and returns the launch's cudaError_t.

// Epilogue of the batch-1 GEMV kernels.
enum gemv_epilogue {
    EPI_STORE = 0,      // y[n] = alpha * (beta*bias[n] + acc)      (bias may be null)
    EPI_STORE_TILED,    // y[n] = beta*bias[n] + alpha * acc
    EPI_RESIDUAL,       // y[n] (fp32) += acc                        (decoder residual add)
    EPI_SWIGLU,         // rows (2i, 2i+1) = (gate_i, up_i): y[i] = silu(gate)*up
    EPI_QKV_ROPE,       // decoder QKV: RoPE on row pairs, q -> fp32, k/v -> fp16 cache
    EPI_LOGITS_ARGMAX,  // y[n] (fp32) = acc, and the greedy key max-reduced into *argmax_key
};

struct GemvArgs {
    const void* x = nullptr;      // activation [k] (a_dtype)
    int a_dtype = AEXIS_F32;
    const aexis_weights* w = nullptr;
    const float* bias = nullptr;
    float alpha = 1.0f, beta = 1.0f;
    void* y = nullptr;
    int y_dtype = AEXIS_F32;
    int epilogue = EPI_STORE;
    // Optional RMSNorm prologue on x (decoder): x <- x*rsqrt(max(mean(x^2)+eps,1e-20))*gamma.
    const float* norm_gamma = nullptr;
    float norm_eps = 0.0f;
    // EPI_QKV_ROPE extras.
    const float* rope_cos = nullptr;   // [rot_dim/2] row of this position
    const float* rope_sin = nullptr;
    const int* rope_map = nullptr;     // per internal row: packed destination descriptor
    __half* k_cache = nullptr;         // [kv_heads][cap][head_dim] of this layer
    __half* v_cache = nullptr;
    int head_dim = 0, kv_cap = 0, q_rows = 0, kv_rows = 0, rot_dim = 0;
    const int* pos_ptr = nullptr;      // device position (decoder graph)
    unsigned long long* argmax_key = nullptr;  // EPI_LOGITS_ARGMAX target
    int* status = nullptr;             // context status word (bounded-wait timeouts)
    bool pdl = false;                  // launch with programmatic dependent launch
    // W8A8: stage the activation codes (aexis_act_code) instead of x (gemv_mma only).
    int act_quant = 0;
    float act_scale = 1.0f;
    int act_zero_point = 0, act_unsigned = 0;
};

// y = W x for one activation row; picks the fast streaming kernel when the
// weight layout allows it, else the exact generic kernel.
cudaError_t launch_gemv(const GemvArgs& a, int sm_count, cudaStream_t stream);
// Reports which kernel launch_gemv would use.
const char* gemv_kernel_name(const aexis_weights* w);
// The bulk-copy streaming GEMV (k_gemv_stream.cu): whether it takes `w`, and
// its launch.
bool gemv_stream_supported(const aexis_weights* w);
// Tensor-core Q4/Q8 GEMV (k_gemv_mma.cu): shapes with a fragment copy (K a
// multiple of 64; Q4 groups a multiple of 16); the copy's sizes and builder.
bool gemv_mma_eligible(const aexis_weights* w);
size_t gemv_mma_frag_bytes(const aexis_weights* w, size_t* scale_bytes);
cudaError_t launch_repack_frag(const aexis_weights* w, cudaStream_t s);
bool gemv_mma_supported(const aexis_weights* w, int a_dtype);
cudaError_t launch_gemv_mma(const GemvArgs& a, int sm_count, cudaStream_t stream);
cudaError_t launch_gemv_stream(const GemvArgs& a, int sm_count, int* status, cudaStream_t stream);
// Bytes of padding after every weight and scale allocation: bulk copies of a
// partial last tile round their size up to 16 bytes.
constexpr size_t kWeightPad = 256;

// Batched Q8 GEMM on tcgen05 (k_gemm_tc.cu).
bool gemm_tc_supported(const aexis_weights* w, int m, int a_dtype);
size_t gemm_tc_tiled_bytes(const aexis_weights* w);
size_t gemm_tc_xt_bytes(int m, int k, int a_dtype);
cudaError_t launch_repack_q8(const aexis_weights* w, void* tiled, cudaStream_t s);
cudaError_t launch_gemm_tc(const aexis_weights* w, const void* tiled, const void* x, int a_dtype, int lda, int m,
                           void* xt, const float* bias, float alpha, float beta, void* y, int y_dtype, int ldy,
                           int tiled_epi, int sm_count, int* status, cudaStream_t s);
// MMA width (rows of the prepared activations) for m rows; fp32 (split) doubles it.
int tc_width(int m, int a_dtype);
// Prepare activations for the tensor-core GEMM: op 0 copy, 1 RMSNorm with
// gamma, 2 SwiGLU of interleaved gate/up pairs; split = fp16 hi + lo rows.
// Optionally zeroes zero[m][zero_n] (row stride zero_ld). pdl: launched as a
// programmatic dependent of the previous kernel on the stream.
cudaError_t launch_tc_prep(int op, const void* x, int x_f16, int lda, int m, int k, const float* gamma, float eps,
                           int split, void* xt, float* zero, int zero_ld, int zero_n, bool pdl, cudaStream_t s);
struct TcLaunch {
    const aexis_weights* w = nullptr;
    const void* tiled = nullptr;  // launch_repack_q8 layout of w
    const void* xt = nullptr;     // launch_tc_prep output
    int m = 0, split = 0;
    const float* bias = nullptr;
    float alpha = 1.0f, beta = 1.0f;
    void* y = nullptr;
    int y_dtype = AEXIS_F32, ldy = 0;
    int tiled_epi = 0;
    int accumulate = 0;  // y += result (fp32 atomics); allows splitting K over CTAs
    int k_splits = 0;    // 0: automatic
    int sm_count = 148;
    int* status = nullptr;
    bool pdl = false;
};
cudaError_t launch_gemm_tc_prepared(const TcLaunch& a, cudaStream_t s);

cudaError_t launch_dequant(const aexis_weights* w, float* out, cudaStream_t s);
// One bounded wait on a flag nothing sets (zeroed first): records
// AEXIS_E_TIMEOUT in `status` after limit_cycles of SM clock.
cudaError_t launch_selftest_wait(int* flag, long long limit_cycles, int* status, cudaStream_t s);
cudaError_t launch_rmsnorm(const void* x, int x_dtype, int rows, int width, int ld,
                           const float* gamma, int affine_size, float eps, void* y, int y_dtype,
                           cudaStream_t s);
cudaError_t launch_rope(const float* src, int embed_dim, int seq_len, int num_heads,
                        const float* cosv, const float* sinv, int interleaved, float* out,
                        cudaStream_t s);
cudaError_t launch_kv_append(const float* cur, int width, int rows, int slices, int offset,
                             float* cache, int cache_rows, cudaStream_t s);
cudaError_t launch_kv_concat(const float* a, int a_rows, const float* b, int b_rows, int width,
                             int slices, float* out, int out_rows, cudaStream_t s);
cudaError_t launch_sdpa(const float* q, const float* k, const float* v, int src_len, int dst_len,
                        int embed_dim, int out_embed_dim, int num_heads, int num_groups,
                        float scale, const float* mask, int mask_w, int mask_h, int causal,
                        int causal_offset, float* out, cudaStream_t s);
size_t sdpa_smem_bytes(int dst_len);
cudaError_t launch_argmax(const float* logits, int rows, int width, int ld, int32_t* out,
                          unsigned long long* keys, int sm_count, cudaStream_t s);
cudaError_t launch_argmax_keys(const float* logits, int rows, int width, int ld, long long offset,
                               unsigned long long* keys, int sm_count, cudaStream_t s);
// Per-row top-k (k <= 64): scratch of topk_scratch_bytes() device bytes.
size_t topk_scratch_bytes(int rows, int width, int k, int sm_count);
// Merge of the shards' packed argmax keys and top-k lists (k_topk.cu).
cudaError_t launch_topk_shard_merge(const int32_t* gathered, int lists, int rows, int k, int shard_rows, long long* ids,
                                    float* vals, int32_t* idx, cudaStream_t s);
// The peer exchange of the same packed results (k_topk.cu). Every rank owns a
// receive buffer, mapped into every other rank's process (CUDA IPC):
//   u32 words [0, 16): flags [2][kPeerMaxRanks], flag[parity][s] = the epoch
//                      of the last call whose result from shard s is in place;
//   u32 word 16: the push kernel's CTA counter, word 17: the epoch of this
//                rank's last push (both for its own buffer only);
//   from byte 256: slots int32 [2][world][peer_slot_words], parity = epoch & 1.
// The push takes the next epoch, writes rank's packed result into every
// buffer's slot and releases the flags; the merge waits for all flags of the
// epoch, then merges. Nothing of a call is on the host, so a call can be
// captured in a CUDA graph.
constexpr int kPeerMaxRanks = 8;
constexpr int kPeerCounterWord = 16;
constexpr int kPeerEpochWord = 17;
constexpr size_t kPeerHeaderBytes = 256;
int peer_slot_words(int rows, int k);
size_t peer_recv_bytes(int world, int rows, int k);
cudaError_t launch_topk_peer_push(const int32_t* packed, int rows, int k, void* const* peers, int world, int rank,
                                  cudaStream_t s);
cudaError_t launch_topk_peer_merge(const void* recv, int world, int rows, int k, int shard_rows, long long* ids,
                                   float* vals, int32_t* idx, int* status, cudaStream_t s);
// Greedy keys (aexis_argmax_key, global indices) from per-row top-k lists.
cudaError_t launch_topk_greedy_keys(const float* logits, int rows, int ld, const float* vals, const int32_t* idx, int k,
                                    long long offset, unsigned long long* keys, cudaStream_t s);
cudaError_t launch_topk(const float* logits, int rows, int width, int ld, int k, float* vals, int32_t* idx,
                        void* scratch, int sm_count, cudaStream_t s);
cudaError_t launch_embed(const int32_t* words, int count, const aexis_weights* table,
                         const float* bias, float* out, cudaStream_t s);
cudaError_t launch_swish(const float* x, int count, float* y, cudaStream_t s);
cudaError_t launch_swiglu(const float* g, const float* u, int count, float* y, cudaStream_t s);
// AexisQuantizeGemmActivationForInt8 codes: out[r*k + i] = (half)(clamp(rint(a/scale) + zp) - zp).
cudaError_t launch_act_quant_i8(const void* a, int a_dtype, int lda, int m, int k, float scale, int zero_point,
                                int is_unsigned, __half* out, cudaStream_t s);
// Pack4 texture-array activation [slices][height][width][4] -> row-major [m][k]
// (the inputPacked A of AexisGemm2DPack4LinearTextureAFromPack4).
cudaError_t launch_gather_pack4a(const void* a, int a_dtype, int width, int height, int slices, int m, int k,
                                 void* out, cudaStream_t s);
// Device sampler (k_sample.cu). `topk_scratch` holds topk_scratch_bytes(rows, width, min(top_k, width)).
// `full`: room for the whole-vocabulary path's probabilities (top_k <= 0 or > 64).
size_t sample_scratch_bytes(int rows, int width, int sm_count, bool scores, bool full);
cudaError_t launch_sample(const float* logits, int rows, int width, int ld, const uint32_t* history, float pen,
                          float temperature, int top_k, float top_p, const double* uniforms, int32_t* out,
                          void* scratch, void* topk_scratch, int sm_count, cudaStream_t s);
cudaError_t launch_history_add(uint32_t* history, int rows, int width, const int32_t* tokens, cudaStream_t s);
// Linear-attention decode kernels (k_recurrent.cu).
cudaError_t launch_short_conv(const float* weight, const float* mixed, const float* cache_in, float* out,
                              float* cache_out, int groups, int kernel, int seq, int cache_len, cudaStream_t s);
int gdr_max_kdim();
cudaError_t launch_gated_delta_rule(const float* a_log, const float* dt_bias, const float* b, const float* a,
                                    const float* q, const float* k, const float* v, const float* state_in,
                                    float* out, float* state_out, int heads, int kdim, int vdim, int first,
                                    int count, float eps, cudaStream_t s);

// Device helpers shared by kernels.
#ifdef __CUDACC__
__device__ __forceinline__ float aexis_load_act(const void* p, int dtype, long long i) {
    return dtype == AEXIS_F16 ? __half2float(reinterpret_cast<const __half*>(p)[i])
                              : reinterpret_cast<const float*>(p)[i];
}
// W8A8 activation code (AexisQuantizeGemmActivationForInt8, HLSL Pack4Matmul:
// 792-800): q = clamp(round(v / scale) + zp) over [-128, 127] or [0, 255]
// (unsigned), rounding half to even; returns the integer q - zp, which the
// GEMMs multiply exactly and scale by `scale` in their epilogue.
__device__ __forceinline__ float aexis_act_code(float v, float scale, int zp, int is_unsigned) {
    float qf = rintf(__fdiv_rn(v, scale));
    qf = fminf(fmaxf(qf, -1.0e6f), 1.0e6f);   // clamp before the integer conversion
    int q = (int)qf + zp;
    const int lo = is_unsigned ? 0 : -128, hi = is_unsigned ? 255 : 127;
    q = q < lo ? lo : (q > hi ? hi : q);
    return (float)(q - zp);
}
__device__ __forceinline__ void aexis_store_out(void* p, int dtype, long long i, float v) {
    if (dtype == AEXIS_F16) reinterpret_cast<__half*>(p)[i] = __float2half_rn(v);
    else reinterpret_cast<float*>(p)[i] = v;
}
// Order-preserving map of an fp32 value to uint32 (larger float -> larger key).
__device__ __forceinline__ unsigned int aexis_orderable(float v) {
    unsigned int b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
// Greedy-selection key: orderable value in the high word, (~index) in the low
// word, so the maximum key is the largest value at the lowest index -- the
// strict > scan of AexisArgMaxPack4LinearMat (HLSL Pack4Matmul:645-686). -0
// counts as +0; a NaN never wins unless it is at index 0 (where it wins, as in
// the scan).
__device__ __forceinline__ unsigned long long aexis_argmax_key(float v, int idx) {
    unsigned int hi;
    if (v != v) hi = idx == 0 ? 0xFFFFFFFFu : 0u;
    else hi = aexis_orderable(v == 0.0f ? 0.0f : v);
    return ((unsigned long long)hi << 32) | (unsigned long long)(0xFFFFFFFFu - (unsigned int)idx);
}
__device__ __forceinline__ int aexis_argmax_index(unsigned long long key) {
    return key == 0ull ? 0 : (int)(0xFFFFFFFFu - (unsigned int)(key & 0xFFFFFFFFull));
}
#endif
