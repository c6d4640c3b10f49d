// decoder_internal.h -- the decoder object shared by the batch-1 step graph
// (k_decoder.cu) and the batched decode path (k_batch.cu).
#pragma once
#include <vector>

#include "aexis_internal.h"

struct aexis_decoder {
    aexis_ctx* ctx = nullptr;
    aexis_decoder_config cfg = {};
    struct Layer {
        // A linear-attention layer keeps in_proj in qkv and out_proj in o.
        aexis_weights qkv, o, gateup, down;
        float* norm[2] = {nullptr, nullptr};
        // bit w set once linear w was loaded (in_proj bit 0, out_proj bit 3,
        // the linear-attention parameters bits 1 and 2); bits 7,8 the norms
        int set_mask = 0;
        int kind = AEXIS_LAYER_FULL_ATTENTION;
        int attn_slot = -1;             // full attention: index of its KV cache
        float* conv_w = nullptr;        // linear attention: [conv_kernel][channels]
        float* lin_params = nullptr;    // a_log [heads], dt_bias [heads], gamma [vdim]
        float* conv_state = nullptr;    // [conv_kernel][channels]
        float* gdr_state = nullptr;     // [heads][kdim][vdim]
    };
    std::vector<Layer> layers;
    int n_attn = 0;                 // full-attention layers (KV caches)
    bool hybrid = false;            // some layer is linear attention
    float* lin_proj = nullptr;      // in_proj output of the current linear-attention layer
    float* lin_y = nullptr;         // its gated-norm output (out_proj input)
    aexis_weights lm;
    int lm_set = 0;
    float* final_norm = nullptr;
    __half* embed = nullptr;
    int embed_set = 0, final_set = 0;
    int* rope_map = nullptr;        // [qkv rows]
    float* rope_cos = nullptr;      // [cap][rot/2]
    float* rope_sin = nullptr;
    __half* kcache = nullptr;       // [full-attention layers][kv][cap][D]
    __half* vcache = nullptr;
    float *h = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr, *part = nullptr;
    unsigned int* counters = nullptr;
    unsigned long long* key = nullptr;
    int* ints = nullptr;            // [0] token, [1] pos, [2] step, [3..] out tokens
    int max_out = 0;
    int host_pos = 0;
    cudaGraphExec_t step_exec = nullptr, prefill_exec = nullptr;
    std::vector<int> qkv_perm;      // internal row -> logical (kind, head, dim)
    bool split_attn = false;        // decode attention by launch_split_attention
    // Persistent greedy loop (k_decoder_persist.cu): 0 never (default), 1
    // always (generate fails where unsupported), -1 where supported.
    int persist_mode = 0;
    void* persist_phases = nullptr;  // device phase table of one step
    int persist_nphases = 0;
    void* persist_sync = nullptr;    // arrival counter, abort flag, greedy keys
    void* persist_stream = nullptr;  // every CTA's weight units of one step, CTA-major
    void* persist_off = nullptr;     // [sm_count + 1] unit offsets into persist_stream
    bool persist_packed = false;     // persist_stream matches the current weights
};

// One decode step of a linear-attention block after its in_proj GEMV
// (k_recurrent.cu): ShortConv + SiLU, the Gated Delta Rule and the gated
// per-head RMSNorm, one cluster of vdim/16 CTAs per head, launched as a
// programmatic dependent of the previous kernel.
struct LinAttnDecode {
    const float* proj = nullptr;     // in_proj output [q k v z b a]
    const float* conv_w = nullptr;   // [kernel][channels]
    float* conv_state = nullptr;     // [kernel][channels], shifted in place
    const float* a_log = nullptr;    // [heads]
    const float* dt_bias = nullptr;  // [heads]
    const float* gamma = nullptr;    // [vdim]
    float* state = nullptr;          // [heads][kdim][vdim], updated in place
    float* y = nullptr;              // [heads][vdim], the out_proj input
    int heads = 0, kdim = 0, vdim = 0, kernel = 0;
    float gdr_eps = 1e-6f, norm_eps = 1e-6f;
};
bool lin_attn_decode_supported(int heads, int kdim, int vdim, int kernel);
cudaError_t launch_lin_attn_decode(const LinAttnDecode& a, cudaStream_t s);

// One layer of one sequence's KV cache (fp16 [kvh][cap][D], rows swizzled
// when swz) to and from Pack4 CDHW fp32 [w = D, h = rows, c = kvh]
// (k_kvstate.cu). Export writes every texel, zero past len; import rounds
// positions [0, len) to fp16.
cudaError_t launch_kv_export(const __half* kc, const __half* vc, int kvh, int cap, int D, int swz, int len, int rows,
                             float* k_out, float* v_out, cudaStream_t s);
cudaError_t launch_kv_import(const float* k_in, const float* v_in, int kvh, int cap, int D, int swz, int len, int rows,
                             __half* kc, __half* vc, cudaStream_t s);

// The persistent greedy loop: whether it runs this decoder, and `nsteps`
// greedy steps from the device state (ints[0] token, [1] position, [2]
// output cursor) in one cooperative launch.
bool decoder_persist_supported(const aexis_decoder* d, int sm_count);
cudaError_t decoder_persist_run(aexis_decoder* d, int nsteps, cudaStream_t s);

// cos/sin tables [cap][rot/2] of Qwen35DecoderSession.CreateRopeTextures
// (Qwen35DecoderSession.cs:1660-1687): inv = 1 / theta^(j * 2/rot) in fp32,
// angle = pos * inv in fp32, cos/sin evaluated in double and rounded.
void decoder_rope_tables(int cap, int rot_dim, float theta, std::vector<float>& cs, std::vector<float>& sn);

// Split decode attention over fp16 KV caches [B][kv][cap][D] (k_batch.cu):
// sequence b's query heads q[b][n_heads][D] attend positions [0, pos[b]],
// chunk (32 or 128) positions per CTA, K and V of a chunk staged by bulk
// copies, the last CTA of (b, kv head) merging the splits into out[b][..][D].
// part: split_attention_part_floats() floats; counters: [B][kv], zero, left
// zero. Launched as a programmatic dependent of the previous kernel.
bool split_attention_supported(int n_heads, int kvh, int D);
int split_attention_max_cap();
size_t split_attention_part_floats(int B, int n_heads, int D, int chunk);
cudaError_t split_attention_configure(int n_heads, int kvh, int D, int chunk);
cudaError_t launch_split_attention(const float* q, const __half* kc, const __half* vc, int cap, int D, int n_heads,
                                   int kvh, float scale, const int* pos, int B, float* part, unsigned int* counters,
                                   float* out, int* status, int chunk, cudaStream_t s);

// Batched decode attention on the tensor cores (k_batch_attn.cu): head_dim
// 128, <= 4 query heads per KV head, caches [B][kvh][cap][D] stored with
// swizzled rows. The attention takes the QKV projection before RoPE (internal
// row order, rows per sequence) and does RoPE and the KV append itself. A
// fixed grid (from configure) streams the step's (sequence,
// KV head, 64-position chunk) items, one partial per CTA segment into `part`
// (batch_tc_attention_part_floats floats); the merge prep combines a head's
// partials into the O projection's prepared fp16 hi / lo input (the
// launch_tc_prep layout for B rows, fp32 split). Both are programmatic
// dependents of the previous kernel.
bool batch_tc_attention_supported(int n_heads, int kvh, int D, int max_batch, int cap);
size_t batch_tc_attention_part_floats(int B, int n_heads);
cudaError_t batch_tc_attention_configure(int sm_count, int* grid);
cudaError_t launch_batch_tc_attention(const float* qkv, int rows, const float* cosv, const float* sinv, int rot,
                                      __half* kc, __half* vc, int cap, int n_heads, int kvh, float scale,
                                      const int* pos, int B, float* part, int grid, int* status, cudaStream_t s);
cudaError_t launch_batch_attn_merge_prep(const float* part, const int* pos, int B, int n_heads, int kvh, int grid,
                                         void* xt, cudaStream_t s);
