/*
 * aexis_cuda.h -- C ABI of libaexis_cuda, the B200 (sm_100a) backend for the
 * Aexis quantized-decoder hot path.
 *
 * Each entry point replaces one AexisOps / AexisGraphSession method of the
 * reference (paths relative to Packages/com.aexis/Runtime/ in newzjh/AIImage;
 * "Ops" = Execution/Graph/AexisOps.cs, "Session" = Execution/Graph/
 * AexisGraphSession.cs). Argument meaning and validation follow the cited
 * method; where the reference throws, the call returns the matching status:
 *   ArgumentNullException        -> AEXIS_E_NULL
 *   ArgumentOutOfRangeException  -> AEXIS_E_RANGE
 *   ArgumentException            -> AEXIS_E_SHAPE
 *   NotSupportedException        -> AEXIS_E_UNSUPPORTED
 *   InvalidOperationException    -> AEXIS_E_STATE
 * and aexis_cuda_last_error(ctx) holds the message. No C++ exception crosses
 * this boundary.
 *
 * Memory: "device" pointers are CUDA device memory owned by the caller;
 * "host" pointers are host memory the call copies from or to before it
 * returns. Tensors keep the reference's logical Pack4 layouts:
 *   - a 2-D [rows, W] matrix is row-major with a caller-given row stride
 *     (Pack4 linear storage uses stride ceil(W/4)*4);
 *   - a CDHW tensor [W, H, 1, C] stores element (x, y, c) at
 *     ((c/4 * H + y) * W + x) * 4 + (c & 3).
 * All device work is enqueued on the context's stream and is asynchronous;
 * aexis_cuda_sync() waits for it. A context is not thread-safe; use one per
 * GPU (and per host thread).
 */
#ifndef AEXIS_CUDA_H_
#define AEXIS_CUDA_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AEXIS_CUDA_ABI_VERSION 1

typedef enum aexis_status {
    AEXIS_OK = 0,
    AEXIS_E_NULL = 1,
    AEXIS_E_RANGE = 2,
    AEXIS_E_SHAPE = 3,
    AEXIS_E_UNSUPPORTED = 4,
    AEXIS_E_STATE = 5,
    AEXIS_E_CUDA = 6,
    AEXIS_E_TIMEOUT = 7
} aexis_status;

typedef enum aexis_dtype {
    AEXIS_F32 = 0,
    AEXIS_F16 = 1
} aexis_dtype;

typedef struct aexis_ctx aexis_ctx;
typedef struct aexis_weights aexis_weights;
typedef struct aexis_decoder aexis_decoder;

/* ------------------------------------------------------------------ context */

/* ABI version of the loaded library (AEXIS_CUDA_ABI_VERSION). No reference
 * counterpart; lets a binding check it loaded a matching library. */
int aexis_cuda_abi_version(void);

/* new AexisOps() (Ops constructor): binds `device` and creates the context's
 * stream. Checks that the device is sm_100. */
int aexis_cuda_create(int device, aexis_ctx** out);

/* AexisOps.Dispose (Ops): frees the context's stream and scratch. */
int aexis_cuda_destroy(aexis_ctx* ctx);

/* Last error message of the context ("" when none). A NULL ctx returns the
 * message of the last failed aexis_cuda_create on this thread. */
const char* aexis_cuda_last_error(const aexis_ctx* ctx);

/* Enqueue subsequent work on a caller-owned cudaStream_t; NULL is the CUDA
 * legacy default stream. Until the first call the context uses a stream of
 * its own. The reference records into a CommandBuffer
 * (Ops Gemm2DPack4LinearTextureA(CommandBuffer, ...) overloads, Ops:3685). */
int aexis_cuda_set_stream(aexis_ctx* ctx, void* cuda_stream);

/* Graphics.ExecuteCommandBuffer + readback fence: wait for enqueued work.
 * Returns AEXIS_E_TIMEOUT (and clears it) when a kernel gave up on a bounded
 * wait since the last sync; the context stays usable. */
int aexis_cuda_sync(aexis_ctx* ctx);

/* No reference counterpart: a self-test of the failure path above. Enqueues
 * one kernel that waits on a device flag nothing sets for limit_cycles
 * (1e3..4e9) of SM clock, then records AEXIS_E_TIMEOUT like any kernel whose
 * bounded barrier wait runs out; the next aexis_cuda_sync reports it. */
int aexis_cuda_selftest_wait(aexis_ctx* ctx, long long limit_cycles);

/* ------------------------------------------------------------------ weights */

/* Session.NewInt8WeightOnlyUpload(AexisQuantizedTensor, n) (Session:12887-
 * 12910) followed by Ops.SetInt8GemmWeights (Ops:706-712).
 * packed: host, ceil(n*k/4) uint32, element (row, col) = byte (idx & 3) of word
 * idx >> 2 with idx = row*k + col, two's complement. scales: host, one per
 * output row, fp32 or fp16 (scale_dtype). The library keeps its own device copy.
 * Errors: NULL arrays -> E_NULL; n, k <= 0 -> E_RANGE. */
int aexis_cuda_weights_q8(aexis_ctx* ctx, const uint32_t* packed, const void* scales,
                          int scale_dtype, int n, int k, aexis_weights** out);

/* Session.NewInt4WeightOnlyUpload(AexisQuantizedTensor, n, k) (Session:12966-
 * 12998) followed by Ops.SetInt4GemmWeights (Ops:730-739).
 * packed: host, ceil(n*k/8) uint32, nibble (idx & 7) of word idx >> 3 (low
 * nibble first), two's complement [-8, 7]. scales: host, n*k/group values;
 * element idx uses scale idx / group. group must divide k (E_SHAPE otherwise,
 * as the reference's "group size must divide the Gemm K dimension"). */
int aexis_cuda_weights_q4(aexis_ctx* ctx, const uint32_t* packed, const void* scales,
                          int scale_dtype, int n, int k, int group, aexis_weights** out);

/* Plain fp16 or fp32 [n, k] table (Ops.SetFp16GemmWeights / the _EmbedW
 * buffer of Ops.EmbedTexture, Ops:10764-10810). Used by aexis_cuda_embed. */
int aexis_cuda_weights_dense(aexis_ctx* ctx, const void* data, int dtype, int n, int k,
                             aexis_weights** out);

/* InnerProductPack.Dispose (Session:357-367): release a weight handle. */
int aexis_cuda_weights_free(aexis_ctx* ctx, aexis_weights* w);

/* Dequantize the whole weight to fp32 [n, k] (device `out`), one
 * AexisGemm2DReadB (HLSL Pack4Matmul:707-734) per element. Used to prove
 * bit-exact unpacking and indexing. */
int aexis_cuda_weights_dequant(aexis_ctx* ctx, const aexis_weights* w, float* out);

/* Host-side quantizers of the float upload paths: Session.NewInt8Weight-
 * OnlyUpload(float[], ...) (Session:12834-12885) and NewInt4WeightOnlyUpload
 * (float[], ...) (Session:12912-12964): per output channel scale maxAbs/127
 * (or /7), values RoundToInt (midpoint to even) and clamped to [-127, 127]
 * (or [-7, 7]). `packed` (ceil(n*k/4) or /8 words) and `scales` (out_ch
 * floats) are host arrays the call fills. For Q4 the effective scale block is
 * per_ch when outputs are contiguous (scaleBlockSize, Session:12956). */
int aexis_quantize_q8_rows(const float* data, int out_ch, int per_ch, int contiguous,
                           uint32_t* packed, float* scales);
int aexis_quantize_q4_rows(const float* data, int out_ch, int per_ch, int contiguous,
                           uint32_t* packed, float* scales);

/* ------------------------------------------------------------------- linear */

/* Ops.Gemm2DPack4LinearTextureA(a, inputPacked, b, c, m, n, k, transB=true,
 * alpha, beta, useC, broadcastTypeC=4, output) (Ops:3649-3683), kernel
 * AexisGemm2DPack4LinearTextureAFromLinear (HLSL Pack4Matmul:1038-1104):
 *   y[r, c] = alpha * (beta * bias[c] + sum_k a[r, k] * W(c, k))
 * a: device [m, lda] of a_dtype; bias: device fp32 [n] or NULL (useC=false);
 * y: device [m, ldy] of y_dtype. Accumulation is fp32.
 * Errors: a/w/y NULL -> E_NULL; m, n, k <= 0 -> E_RANGE; n or k not the
 * weight's shape, lda < k or ldy < n -> E_SHAPE. */
int aexis_cuda_gemm(aexis_ctx* ctx, const void* a, int a_dtype, int lda, int m, int k,
                    const aexis_weights* w, const float* bias, float alpha, float beta,
                    void* y, int y_dtype, int ldy, int n);

/* Ops.Gemm2DPack4LinearTextureA with inputPacked = true (Ops:3649-3683),
 * kernel AexisGemm2DPack4LinearTextureAFromPack4 (HLSL Pack4Matmul:1106-1190,
 * A read as AexisGemm2DPack4LinearTextureAReadPack4, :880-891): the same
 * product as aexis_cuda_gemm with A in a Pack4 texture array of a_width
 * texels, a_height rows and a_slices slices, stored like a CDHW tensor
 * (texel (x, row, slice) at ((slice * a_height + row) * a_width + x) * 4).
 * Element (row, kk) is lane kk & 3 of texel (pack % a_width, row,
 * pack / a_width) with pack = kk >> 2; values past the last slice count as 0.
 * When 4 * a_width >= k the rows are read in place (row stride 4 * a_width);
 * otherwise they are first gathered into a row-major context buffer.
 * The tiled form (Gemm2DPack4TiledTextureAFromPack4, Ops:3782-3826) reads
 * slice 0 only: it is aexis_cuda_gemm_tiled with lda = 4 * a_width.
 * Errors: as aexis_cuda_gemm; a_width, a_slices <= 0 or a_height < m ->
 * E_SHAPE. */
int aexis_cuda_gemm_pack4a(aexis_ctx* ctx, const void* a, int a_dtype, int a_width, int a_height, int a_slices,
                           int m, int k, const aexis_weights* w, const float* bias, float alpha, float beta,
                           void* y, int y_dtype, int ldy, int n);

/* Ops.SetInt8ActivationQuantization (Ops:741-785) with its plan resolved to
 * (scale, zero_point, unsigned): while enabled, aexis_cuda_gemm and
 * aexis_cuda_gemm_tiled fake-quantise every activation as the HLSL
 * AexisQuantizeGemmActivationForInt8 does (Pack4Matmul:792-800),
 *   q = clamp(round(a / scale) + zero_point, -128..127 or 0..255 unsigned),
 *   a' = (q - zero_point) * scale      (round half to even),
 * before the product (the W8A8 mode of Int8W8A8 node plans). The library
 * computes sum (q - zp) * W exactly (integer codes, exact fp16 products, fp32
 * sums) and applies `scale` in the epilogue. enable = 0 restores plain
 * activations. Errors: scale not positive and finite, or |zero_point| > 1024
 * -> E_RANGE. The decoder entry points are not affected. */
int aexis_cuda_set_int8_activations(aexis_ctx* ctx, int enable, float scale, int zero_point, int is_unsigned);
/* Ops.Gemm2DPack4TiledTextureAFromLinear (Ops:3722-3752), the lm_head
 * variant (HLSL Pack4Matmul:2245-2300): bias is added after the sum,
 *   y[r, c] = beta * bias[c] + alpha * sum_k a[r, k] * W(c, k).
 * A tiled Pack4 output texture is row-major with row stride ldy (its
 * tileRowsPerMatrix * width * 4 floats). */
int aexis_cuda_gemm_tiled(aexis_ctx* ctx, const void* a, int a_dtype, int lda, int m, int k,
                          const aexis_weights* w, const float* bias, float alpha, float beta,
                          void* y, int y_dtype, int ldy, int n);

/* --------------------------------------------------------- pointwise layers */

/* Ops.RmsNormPack4LinearMat(input, shape, gamma, affineSize, affine, eps,
 * output) (Ops:8267-8283; COMMON AexisRmsNormPack4LinearMat:4531-4563), per row:
 *   y = x * rsqrt(max(mean(x^2) + eps, 1e-20)) * gamma[clamp(i, 0, affine_size-1)]
 * gamma NULL (or affine_size 0) means no affine. x, y device; ld is the row
 * stride of both. */
int aexis_cuda_rmsnorm(aexis_ctx* ctx, const void* x, int x_dtype, int rows, int width, int ld,
                       const float* gamma, int affine_size, float eps, void* y, int y_dtype);

/* Ops.RotaryEmbedPack4(input, shape[w=embed, h=seq, c=heads], cos, sin,
 * interleaved, output) (Ops:8514-8540; HLSL Pack4PointwiseNorm:414-473).
 * src/out: device fp32 Pack4 CDHW [embed_dim, seq_len, 1, num_heads];
 * cos/sin: device fp32 [seq_len, embed_dim/2]. Rotate-half unless interleaved. */
int aexis_cuda_rope(aexis_ctx* ctx, const float* src, int embed_dim, int seq_len, int num_heads,
                    const float* cos_table, const float* sin_table, int interleaved, float* out);

/* Ops.AppendSequencePack4Cdhw(current, offset, rows, cache) (Ops:6384-6400;
 * HLSL Pack4Elementwise:84-98): copy `rows` rows of `current` (Pack4 CDHW,
 * width texels x rows x slices) into rows offset.. of `cache` (cache_rows
 * rows). Rows beyond the cache are dropped. offset < 0 -> E_RANGE. */
int aexis_cuda_kv_append(aexis_ctx* ctx, const float* current, int width, int rows, int slices,
                         int offset, float* cache, int cache_rows);

/* Ops.ConcatSequencePack4Cdhw(a, b, aHeight, bHeight, output) (Ops:6336-6360;
 * HLSL Pack4Elementwise:64-81); rows past a_rows + b_rows are zeroed. */
int aexis_cuda_kv_concat(aexis_ctx* ctx, const float* past, int past_rows, const float* current,
                         int cur_rows, int width, int slices, float* out, int out_rows);

/* Ops.SdpaAttentionPack4Cdhw(q, k, v, srcLen, dstLen, embedDim, outEmbedDim,
 * numHeads, numGroups, scale, output, mask, causal, causalQueryOffset)
 * (Ops:10147-10200; HLSL Pack4Matmul:420-557). q/out: Pack4 CDHW [embed,
 * src_len, 1, num_heads]; k: [embed, dst_len, 1, num_groups]; v: [out_embed,
 * dst_len, 1, num_groups]; mask: NULL or single-channel Pack4 [mask_w, mask_h]
 * (value in lane 0 of each texel). GQA kv head = head / (num_heads/num_groups).
 * The reference rejects dst_len > 4096; this backend accepts any dst_len. */
int aexis_cuda_sdpa(aexis_ctx* ctx, const float* q, const float* k, const float* v, int src_len,
                    int dst_len, int embed_dim, int out_embed_dim, int num_heads, int num_groups,
                    float scale, const float* mask, int mask_w, int mask_h, int causal,
                    int causal_offset, float* out);

/* Ops.ArgMaxPack4LinearMat(logits, logicalWidth, logicalHeight, tileRows,
 * output) (Ops:9982-10003; HLSL Pack4Matmul:645-686): per row the first index
 * of the maximum (strict >, so ties go to the lowest index; a NaN is never
 * chosen unless it is at index 0). logits: device fp32 [rows, ld];
 * out_idx: device int32 [rows]. */
int aexis_cuda_argmax(aexis_ctx* ctx, const float* logits, int rows, int width, int ld,
                      int32_t* out_idx);

/* The argmax of one vocabulary shard as 64-bit keys, for a cross-GPU max
 * reduction (the vocab-sharded lm_head; no single reference counterpart:
 * AexisArgMaxPack4LinearMat, HLSL Pack4Matmul:645-686, split by columns).
 * keys[r] = (orderable(max value) << 32) | (0xFFFFFFFF - (index_offset + i)),
 * so the maximum key over all shards is the first global index of the
 * maximum, as the single-device scan picks it. keys: device uint64 [rows]. */
int aexis_cuda_argmax_keys(aexis_ctx* ctx, const float* logits, int rows, int width, int ld,
                           int64_t index_offset, uint64_t* keys);

/* The same keys as aexis_cuda_argmax_keys, from the shard's top-k lists of
 * aexis_cuda_topk (top_vals/top_idx: device [rows, k], shard-local indices)
 * instead of a second pass over the logits: the first list entry is the
 * row's largest value at its lowest index (-0 counted as +0, NaN never
 * listed). With index_offset 0 the call also reads logits[r][0], since a NaN
 * there wins the reference's ArgMax. No single reference counterpart (the
 * vocab-sharded lm_head; AexisArgMaxPack4LinearMat, HLSL Pack4Matmul:645-686). */
int aexis_cuda_topk_greedy_keys(aexis_ctx* ctx, const float* logits, int rows, int width, int ld, int k,
                                const float* top_vals, const int32_t* top_idx, int64_t index_offset,
                                uint64_t* keys);
/* The lm_head and the sampler's top-k in one call, for a batch of hidden
 * states: aexis_cuda_gemm_tiled (bias NULL, beta 1) into a context buffer of
 * [m, w->n] fp32 logits, then aexis_cuda_topk and (when greedy_keys is not
 * NULL) aexis_cuda_topk_greedy_keys on them, with the same results
 * (AexisGemm2DPack4TiledTextureAFromLinear, HLSL Pack4Matmul:2245-2275, then
 * the Qwen35Sampler candidate order, Samples/.../Qwen35DecoderSession.cs:
 * 1869-1872; no single reference counterpart).
 * out_vals/out_idx: device [m, top_k] (shard-local indices); greedy_keys:
 * device uint64 [m] with global indices (index_offset added), or NULL.
 * Errors: as aexis_cuda_gemm_tiled; top_k outside 1..64 -> E_RANGE. */
int aexis_cuda_gemm_topk(aexis_ctx* ctx, const void* a, int a_dtype, int lda, int m, int k,
                         const aexis_weights* w, float alpha, int top_k, int64_t index_offset, float* out_vals,
                         int32_t* out_idx, uint64_t* greedy_keys);

/* Rows that aexis_cuda_argmax_static accepts in one call (the size of its
 * fixed key array: 4096 x 8 bytes, held on every GPU that loads the library). */
#define AEXIS_ARGMAX_STATIC_MAX_ROWS 4096

/* The greedy argmax of aexis_cuda_argmax, for callers that cannot allocate
 * device memory. No counterpart in the reference: it exists for hosts that
 * own all device memory through their own allocator (a game engine's
 * graphics-interop path, for instance) or that call from a per-frame callback
 * which must never block, where cudaMalloc / cudaFree may synchronise the
 * device. It needs no context and allocates nothing: its per-row keys live in
 * a fixed array inside the library. The caller passes the logits, the output
 * and a cudaStream_t (NULL = the legacy default stream) of the current device.
 *   - rows must be <= AEXIS_ARGMAX_STATIC_MAX_ROWS, else AEXIS_E_RANGE.
 *   - The first call on a device looks up the array's device address (a
 *     cudaGetSymbolAddress with that device current). Make that first call
 *     before any stream capture.
 *   - Every call on a device shares the one array: calls that overlap on the
 *     GPU (different streams, no ordering between them) race and may return
 *     wrong indices. Calls on one stream are ordered and safe.
 * Same result and tie rule as aexis_cuda_argmax. */
int aexis_cuda_argmax_static(const float* logits, int rows, int width, int ld, int32_t* out_idx,
                             void* cuda_stream);

/* Top-k per row for the sampler (Qwen35Sampler, Samples/.../Qwen35Decoder-
 * Session.cs:1823-1900 sorts the full vocabulary on the CPU): the k largest
 * logits in descending order, equal values by ascending index.
 * out_vals/out_idx: device [rows, k]. 1 <= k <= 64. */
int aexis_cuda_topk(aexis_ctx* ctx, const float* logits, int rows, int width, int ld, int k,
                    float* out_vals, int32_t* out_idx);

/* Qwen35Sampler.Select (Samples/.../Qwen35DecoderSession.cs:1847-1900) for
 * `rows` logit rows on the device. Per row:
 *   s = logits with the repetition penalty on history tokens
 *       (s < 0 ? s * penalty : s / penalty);
 *   temperature <= 0: the first maximum of s (ArgMax, :1894-1900);
 *   else p = (float)(exp((s - max)/T) / sum) with the sum in double; the
 *   top_k most probable (top_k <= 0: the whole vocabulary), then the
 *   smallest prefix whose cumulative reaches top_p (at least one); draw =
 *   uniforms[r] * kept mass; the first token whose cumulative reaches the
 *   draw. top_k 1..64 takes the top-k kernels; any other top_k a radix select
 *   weighted by probability mass (no sort), whose prefix sums are exact in
 *   2^-62 fixed point where the reference sums in fp64 one by one. A sum that is not finite and positive
 *   (a NaN score, no finite score) falls back to ArgMax, as the reference.
 * logits: device fp32 [rows, ld]; history: NULL or a device bitmap
 * [rows][ceil(width/32)] uint32 (bit t % 32 of word t / 32 = token t was
 * emitted, see aexis_cuda_sample_history_add); uniforms: device fp64 [rows],
 * the System.Random.NextDouble draw of each row (may be NULL when greedy);
 * out_idx: device int32 [rows]. Equal probabilities rank by ascending index
 * (the reference's Array.Sort leaves exact ties unordered).
 * Errors: NULL logits/out -> E_NULL; rows, width <= 0, penalty <= 0 or a
 * non-finite temperature / top_p -> E_RANGE; ld < width -> E_SHAPE; when
 * sampling: uniforms NULL -> E_NULL. */
int aexis_cuda_sample(aexis_ctx* ctx, const float* logits, int rows, int width, int ld,
                      const uint32_t* history, float repetition_penalty, float temperature, int top_k,
                      float top_p, const double* uniforms, int32_t* out_idx);
/* Qwen35Sampler.AddHistory (:1840-1844) for every row: sets bit tokens[r] of
 * row r of the history bitmap (tokens: device int32 [rows]; ids outside
 * [0, width) are ignored). */
int aexis_cuda_sample_history_add(aexis_ctx* ctx, uint32_t* history, int rows, int width,
                                  const int32_t* tokens);
/* No reference counterpart (the reference decodes on one device): the merge
 * step of a vocab-sharded lm_head. `gathered` (device) holds, for each of
 * `lists` (1..8) shards in shard order, rows uint64 greedy keys of
 * aexis_cuda_argmax_keys (global indices), then rows x k fp32 values and rows
 * x k int32 shard-local indices of aexis_cuda_topk on the shard, shard s
 * starting at logical row s * shard_rows. Writes per row the greedy id
 * (int64, device), and the k largest (value, global index) pairs under the
 * aexis_cuda_topk order, (-inf, -1) padded: the same results as the
 * single-device calls on the whole vocabulary. */
int aexis_cuda_topk_merge(aexis_ctx* ctx, const int32_t* gathered, int lists, int rows, int k,
                          int shard_rows, int64_t* out_ids, float* out_vals, int32_t* out_idx);

/* No reference counterpart (the reference decodes on one device): the same
 * exchange over peer memory instead of a collective, for ranks that are
 * processes on GPUs of one node joined by NVLink.
 *
 * Every rank owns one receive buffer of aexis_cuda_peer_buffer_bytes(world,
 * rows, k) bytes, made by aexis_cuda_peer_buffer_create (zeroed; out_handle:
 * 64 bytes of CUDA IPC handle). The host hands the handles to the other
 * ranks (any out-of-band channel), and each rank maps the others' buffers
 * with aexis_cuda_peer_buffer_open. Per call (every rank makes the same
 * calls in the same order):
 *   aexis_cuda_topk_push copies this rank's packed result (the
 *   aexis_cuda_topk_merge layout of one shard: rows uint64 greedy keys, rows
 *   x k fp32 values, rows x k int32 shard-local indices; device, 16-byte
 *   aligned) into slot `rank` of every receive buffer (`peers`: host array
 *   of the world buffers as mapped in this process, peers[rank] its own),
 *   then publishes the call's epoch in each buffer's flags;
 *   aexis_cuda_topk_merge_peers waits on this rank's own buffer (`recv`)
 *   until every shard's flag holds the epoch (bounded: AEXIS_E_TIMEOUT from
 *   aexis_cuda_sync when a peer never arrives) and writes what
 *   aexis_cuda_topk_merge writes.
 * The epoch is a counter in the rank's own buffer (the push takes the next
 * one), so the calls carry no host state and can be captured in a CUDA
 * graph. Two parities of slots alternate by epoch, so a rank may push the
 * next call while another still merges the current one.
 * aexis_cuda_peer_buffer_close unmaps an opened buffer (imported = 1) or
 * frees an own one (imported = 0), after every rank is past its last merge. */
int aexis_cuda_peer_buffer_bytes(int world, int rows, int k, size_t* out_bytes);
int aexis_cuda_peer_buffer_create(aexis_ctx* ctx, size_t bytes, void** out_ptr, uint8_t* out_handle);
int aexis_cuda_peer_buffer_open(aexis_ctx* ctx, const uint8_t* handle, void** out_ptr);
int aexis_cuda_peer_buffer_close(aexis_ctx* ctx, void* ptr, int imported);
int aexis_cuda_topk_push(aexis_ctx* ctx, const int32_t* packed, int rows, int k, void* const* peers, int world,
                         int rank);
int aexis_cuda_topk_merge_peers(aexis_ctx* ctx, const void* recv, int world, int rows, int k, int shard_rows,
                                int64_t* out_ids, float* out_vals, int32_t* out_idx);

/* Ops.EmbedTexture (Ops:10764-10810; HLSL BufferTensor AexisEmbedValue:37-62):
 * out[q, p] = W(clamp(words[q], 0, vocab-1), p) (+ bias[p]) for a Q4 (group
 * scales), Q8 (per-token scales) or dense table. words: device int32 [count];
 * bias: device fp32 [dim] or NULL; out: device fp32 [count, dim]. */
int aexis_cuda_embed(aexis_ctx* ctx, const int32_t* words, int count, const aexis_weights* table,
                     const float* bias, float* out);

/* AexisSwishLinearMat (HLSL Pack4Matmul:91-94,205-218): y = x / (1 + exp(-x)). */
int aexis_cuda_swish(aexis_ctx* ctx, const float* x, int count, float* y);

/* Swish on the gate then BinaryOp multiply by the up projection, as one pass
 * (HLSL Pack4Matmul:91-94,118-128): y = silu(gate) * up. */
int aexis_cuda_swiglu(aexis_ctx* ctx, const float* gate, const float* up, int count, float* y);

/* --------------------------------------------- linear-attention decode layers */
/* Ops.ShortConvPack4(weight, mixed, cacheIn, output, cacheOut, groups,
 * kernelSize, sequenceLength, cacheLength) (Ops:12593-12618; COMMON
 * AexisShortConvPack4:623-678; layer AexisShortConvLayer.cs:30-60): causal
 * depthwise Conv1D + SiLU with a streaming cache,
 *   out[t][g]    = silu(sum_j hist(cache_len - kernel + t + 1 + j) * w(g, j))
 *   hist(i)      = i < 0 ? 0 : i < cache_len ? cache_in[i][g] : mixed[i - cache_len][g]
 *   cache_out[i] = hist(seq_len + i)   (the tail of [cache_in; mixed]).
 * weight: device Pack4 CDHW [w=kernel, h=1, c=groups] (element (j, g) at
 * ((g/4)*kernel + j)*4 + (g&3)); mixed/out: device [seq_len][ld];
 * cache_in/cache_out: device [cache_len][ld]; ld = ceil(groups/4)*4.
 * cache_out may be cache_in (updated in place); out may alias no input.
 * Errors: NULL -> E_NULL; groups, kernel_size, seq_len <= 0 or cache_len <
 * kernel_size - 1 -> E_RANGE (as the reference); kernel_size > 16 ->
 * E_UNSUPPORTED; aliasing other than the cache -> E_SHAPE. */
int aexis_cuda_short_conv(aexis_ctx* ctx, const float* weight, const float* mixed, const float* cache_in,
                          float* out, float* cache_out, int groups, int kernel_size, int seq_len,
                          int cache_len);
/* Ops.GatedDeltaRulePack4(aLog, dtBias, b, a, query, key, value, stateIn,
 * output, stateOut, heads, keyDim, valueDim, sequenceLength, tokenIndex,
 * epsilon) (Ops:12620-12657; COMMON AexisGatedDeltaRulePack4:680-753) for the
 * tokens first_token .. first_token + token_count - 1 in one call: the
 * reference's per-token loop of AexisGatedDeltaRuleLayer (AexisGatedDelta-
 * RuleLayer.cs:71-78, ping-pong state) is token_count = seq_len. Per token t
 * and head h:
 *   decay = exp(-exp(a_log[h]) * softplus(a[t][h] + dt_bias[h]))
 *   beta  = sigmoid(b[t][h]);  k^ = k / sqrt(|k|^2 + eps);  q^ likewise
 *   S     = S * decay;  delta = (v - k^ . S) * beta;  S += k^ (x) delta
 *   out   = (q^ . S) / sqrt(key_dim)
 * a_log, dt_bias: device fp32 [heads]; a, b: device fp32 [seq_len][heads];
 * q, k: device Pack4 CDHW [w=key_dim, h=heads, c=seq_len] (element (j, h, t)
 * at ((t/4*heads + h)*key_dim + j)*4 + (t&3)); v, out: CDHW [w=value_dim,
 * h=heads, c=seq_len] (only the lanes of the processed tokens are written);
 * state_in/state_out: device fp32 [heads][key_dim][ceil(value_dim/4)*4],
 * 16-byte aligned; state_out may be state_in (updated in place).
 * Errors: NULL -> E_NULL; sizes <= 0 or tokens outside [0, seq_len) ->
 * E_RANGE; key_dim > 256 -> E_UNSUPPORTED; misaligned state or out aliasing
 * an input -> E_SHAPE. */
int aexis_cuda_gated_delta_rule(aexis_ctx* ctx, const float* a_log, const float* dt_bias, const float* b,
                                const float* a, const float* q, const float* k, const float* v,
                                const float* state_in, float* out, float* state_out, int heads, int key_dim,
                                int value_dim, int seq_len, int first_token, int token_count, float eps);

/* ------------------------------------------------------------------ decoder */

/* Layer kinds of a hybrid stack. Qwen3.5 (Qwen35DecoderSession.cs:167-172:
 * AttentionCacheCount 6, ConvCacheCount 18, GdrCacheCount 18) repeats three
 * linear-attention blocks (ShortConv + GatedDeltaRule) and one full-attention
 * block six times: layer i is full attention when (i + 1) % 4 == 0. */
#define AEXIS_LAYER_FULL_ATTENTION 0
#define AEXIS_LAYER_LINEAR_ATTENTION 1
#define AEXIS_QWEN35_FULL_ATTENTION_INTERVAL 4

/* Shape of the decoder stack driven by Qwen35DecoderSession
 * (Samples/.../Qwen35DecoderSession.cs:167-172 for the reference constants).
 * With layer_types NULL every layer is full attention; otherwise
 * layer_types[l] picks each layer's kind and the lin_* fields give the
 * linear-attention blocks' shape:
 *   xn = RMSNorm(h); [q k v z b a] = in_proj(xn)  (rows in that order:
 *     lin_heads*lin_kdim q, as many k, lin_heads*lin_vdim v and z, lin_heads
 *     b and a)
 *   [q k v] = SiLU(ShortConv([q k v]))  (depthwise, conv_kernel taps over the
 *     previous conv_kernel - 1 tokens and this one; cache of conv_kernel rows)
 *   o = GatedDeltaRule(q, k, v, b, a)   (per head, state [kdim][vdim], eps 1e-6)
 *   y = RMSNorm_per_head(o) * gamma * SiLU(z); h += out_proj(y)
 *   then the same SwiGLU FFN as a full-attention layer. */
typedef struct aexis_decoder_config {
    int32_t n_layers;
    int32_t hidden;
    int32_t n_heads;
    int32_t n_kv_heads;
    int32_t head_dim;
    int32_t ffn;
    int32_t vocab;
    int32_t kv_capacity;   /* KV cache length (positions) */
    int32_t rot_dim;       /* rotated dims per head (rotate-half), even, <= head_dim */
    int32_t bits;          /* 4 or 8: decoder linear weights */
    int32_t group;         /* Q4 group along K (divides hidden and ffn) */
    int32_t lm_bits;       /* 4 or 8: lm_head */
    int32_t lm_group;      /* Q4 group of the lm_head */
    int32_t scale_dtype;   /* AEXIS_F16 or AEXIS_F32: dtype of every weight scale */
    float rope_theta;
    float eps;             /* RMSNorm eps (also the gated per-head norm's) */
    const int32_t* layer_types; /* host [n_layers] of AEXIS_LAYER_*, copied at create; NULL: all full attention */
    int32_t lin_heads;     /* linear attention: heads (q, k, v, z, b, a, GDR state) */
    int32_t lin_kdim;      /* key dim per head: multiple of 4, <= 256 */
    int32_t lin_vdim;      /* value dim per head: multiple of 16, <= 128 */
    int32_t conv_kernel;   /* ShortConv taps, 1..8 */
} aexis_decoder_config;

/* Fills out[0 .. n_layers) with the kinds of a stack whose every
 * `interval`-th layer is full attention (layer i full when (i + 1) %
 * interval == 0, else linear attention); interval AEXIS_QWEN35_FULL_-
 * ATTENTION_INTERVAL gives Qwen3.5's 18 + 6 of 24. interval <= 0 makes
 * every layer full attention. No device work. */
int aexis_cuda_layer_types_interval(int32_t n_layers, int32_t interval, int32_t* out);

/* Qwen35DecoderSession constructor (Qwen35DecoderSession.cs:1748-1766):
 * allocates the weights, fp16 KV cache and the per-step CUDA graph. */
int aexis_cuda_decoder_create(aexis_ctx* ctx, const aexis_decoder_config* cfg,
                              aexis_decoder** out);
int aexis_cuda_decoder_destroy(aexis_decoder* dec);

/* Weight loading (AexisGemmLayer.LoadLayer -> NewInt{4,8}WeightOnlyUpload,
 * AexisGemmLayer.cs:15-160). layer in [0, n_layers) with which: 0 q_proj,
 * 1 k_proj, 2 v_proj, 3 o_proj (full-attention layers), 8 in_proj and
 * 9 out_proj (linear-attention layers), 4 gate_proj, 5 up_proj,
 * 6 down_proj (both); or layer -1, which 7 for the lm_head. Arrays are host
 * arrays in the same packed format as aexis_cuda_weights_q4 / _q8. A `which`
 * of the other layer kind -> E_RANGE. */
int aexis_cuda_decoder_set_linear(aexis_decoder* dec, int layer, int which, const uint32_t* packed,
                                  const void* scales, int scale_dtype);

/* A linear-attention layer's small parameters (host arrays of dtype): conv
 * [channels][conv_kernel] with channels = 2*lin_heads*lin_kdim +
 * lin_heads*lin_vdim in in_proj's q, k, v order (the ShortConv operator's
 * weight = [groups, kernel], Tools/Qwen35NcnnBaseline/reference_ops.py:36-60),
 * a_log and dt_bias [lin_heads] (GatedDeltaRule, reference_ops.py:88-152),
 * gamma [lin_vdim] (the gated norm's gain, shared by the heads).
 * A full-attention layer -> E_RANGE. */
int aexis_cuda_decoder_set_linear_attention(aexis_decoder* dec, int layer, const void* conv, const void* a_log,
                                            const void* dt_bias, const void* gamma, int dtype);

/* RMSNorm gammas (AexisRMSNormLayer.LoadLayer, AexisRMSNormLayer.cs:16-45):
 * which 0 = input norm, 1 = post-attention norm; layer -1 = final norm.
 * gamma: host [hidden] of dtype. */
int aexis_cuda_decoder_set_norm(aexis_decoder* dec, int layer, int which, const void* gamma,
                                int dtype);

/* Token embedding table (AexisEmbedLayer, AexisEmbedLayer.cs:40-180): host
 * [vocab, hidden] of dtype. */
int aexis_cuda_decoder_set_embedding(aexis_decoder* dec, const void* table, int dtype);

/* Qwen35DecoderSession.CreateInitialState (:376-400): position back to 0,
 * every conv and GDR cache zero. */
int aexis_cuda_decoder_reset(aexis_decoder* dec);
int aexis_cuda_decoder_position(const aexis_decoder* dec, int32_t* out_position);

/* RunTokens for a prompt (Qwen35DecoderSession.cs:1254-1269): appends
 * `count` host token ids at the current position and writes the greedy next
 * token (host) after the last one. */
int aexis_cuda_decoder_prefill(aexis_decoder* dec, const int32_t* tokens, int count,
                               int32_t* next_token);

/* One decode step (DecodeCore :469-585 + SelectNextToken :734-809, greedy):
 * host token id in, host greedy token out (the reference's per-token argmax
 * readback). E_RANGE when the KV cache is full. */
int aexis_cuda_decoder_step(aexis_decoder* dec, int32_t token, int32_t* next_token);

/* Qwen35DecoderSession.Generate (:1160-1237), greedy, no EOS stop: prefill
 * `prompt`, then produce max_new tokens into out_tokens (host). */
int aexis_cuda_decoder_generate(aexis_decoder* dec, const int32_t* prompt, int n_prompt,
                                int max_new, int32_t* out_tokens);

/* The fp32 logits of the last step (host [vocab]), for sampling outside the
 * greedy path (Qwen35DecoderSession.ProjectLogits :715-733). */
int aexis_cuda_decoder_logits(aexis_decoder* dec, float* out_logits);

/* ---- decoder state in the reference's layout ------------------------------
 * Qwen35DecoderState (Samples/.../Qwen35DecoderSession.cs:48-100) carries one
 * K and one V texture per attention layer ("cache_k<i>", "cache_v<i>") from
 * step to step (:550-568), plus its SequenceLength / PositionId. These calls
 * move that state across the ABI: a cache texture is a device fp32 Pack4 CDHW
 * tensor [w = head_dim, h = rows, c = n_kv_heads], element (x = dim, y =
 * position, c = kv head) at ((c/4 * rows + y) * head_dim + x) * 4 + (c & 3),
 * the layout aexis_cuda_kv_append writes and aexis_cuda_sdpa reads (k/v with
 * dst_len = the sequence length). The decoders keep fp16 caches, so an
 * import rounds to fp16 (round to nearest even) and a round trip is exact for
 * fp16-representable values. */

/* Write layer `layer`'s K and V caches (device k_out, v_out, each
 * 4 * ceil(n_kv_heads/4) * rows * head_dim floats): positions below the
 * current position hold the cache, the rest of the rows are zero.
 * Errors: rows < position -> E_SHAPE; layer outside [0, n_layers) -> E_RANGE. */
int aexis_cuda_decoder_kv_export(aexis_decoder* dec, int layer, int rows, float* k_out, float* v_out);
/* Load positions [0, length) of layer `layer`'s caches from Pack4 textures of
 * `rows` rows (device). Does not move the position: after importing every
 * layer, call aexis_cuda_decoder_set_position(dec, length). */
int aexis_cuda_decoder_kv_import(aexis_decoder* dec, int layer, const float* k_in, const float* v_in, int rows,
                                 int length);
/* Set the next position (Qwen35DecoderState.PositionId / SequenceLength) to
 * `position` in [0, kv_capacity]: the next token is written at that position
 * and attends positions [0, position]. The conv and GDR caches of a hybrid
 * stack are not touched: import them with the position. */
int aexis_cuda_decoder_set_position(aexis_decoder* dec, int32_t position);

/* A linear-attention layer's recurrent caches as the reference's state holds
 * them (CreateInitialState, Qwen35DecoderSession.cs:376-400): "cache_conv<i>"
 * a Pack4 2D texture [w = channels/4, h = conv_kernel] (device fp32
 * conv_kernel * channels floats, element (tap row, channel) at row *
 * channels + channel, the oldest row first) and "cache_gdr<i>" a Pack4 2D
 * array [w = lin_vdim/4, h = lin_kdim, slice = lin_heads] (lin_heads *
 * lin_kdim * lin_vdim floats, element (head, key row, column) at (head *
 * lin_kdim + row) * lin_vdim + column). Either pointer may be NULL to skip
 * that cache. A full-attention layer -> E_RANGE (its state is the KV cache
 * above; the KV calls take a full-attention layer and return E_RANGE for a
 * linear-attention one). */
int aexis_cuda_decoder_recurrent_export(aexis_decoder* dec, int layer, float* conv_out, float* gdr_out);
int aexis_cuda_decoder_recurrent_import(aexis_decoder* dec, int layer, const float* conv_in, const float* gdr_in);

/* How aexis_cuda_decoder_generate schedules its greedy steps (no reference
 * counterpart: the reference dispatches per layer). mode 0: one CUDA graph
 * per step (every kernel a programmatic dependent of the previous one);
 * mode 1: every emitting step of the call in one persistent cooperative
 * kernel (one CTA per SM, grid barriers between phases, weights streamed
 * ahead through a bulk-copy ring), AEXIS_E_UNSUPPORTED unless the decoder is
 * Q4 group-32 with fp16 scales, head_dim 128, at most 4 query heads per KV
 * head, K dims multiples of 512 and kv_capacity <= 2048; mode -1: 1 where
 * supported, else 0. The default is 0: on B200 the config-3 model decodes at
 * about 1550 tokens/s with graphs and 1400 with the persistent kernel, both
 * bound by about five dependent L2 round trips per layer phase. Both produce
 * the same greedy tokens (fp32 sums in a different order).
 * aexis_cuda_decoder_schedule reports the schedule generate will use (0 or 1). */
int aexis_cuda_decoder_set_schedule(aexis_decoder* dec, int mode);
int aexis_cuda_decoder_schedule(aexis_decoder* dec, int32_t* out_schedule);

/* ---- batched greedy decoding ------------------------------------------------
 * B independent sequences decoded together on one GPU: Qwen35DecoderSession's
 * DecodeCore + SelectNextToken (Qwen35DecoderSession.cs:469-585, 734-809) run
 * for B sequences at once, each with its own context length and KV cache.
 * The reference decodes one sequence per session; a host that serves B
 * sessions replaces B DecodeCore calls per token with one batch step. Every
 * linear reads its weights once per step for all B rows (tensor cores).
 * Requires a Q8 decoder (bits = lm_bits = 8) whose weights are all set: the
 * batch repacks them at creation, so later aexis_cuda_decoder_set_* calls do
 * not reach an existing batch. KV caches are fp16, [layers][B][kv][cap][D]. */
typedef struct aexis_batch aexis_batch;

/* max_batch 1..128 sequences, kv_capacity 1..8192 positions per sequence,
 * max_steps = most tokens one aexis_cuda_batch_generate call may produce. */
int aexis_cuda_batch_create(aexis_decoder* dec, int max_batch, int kv_capacity, int max_steps, aexis_batch** out);
int aexis_cuda_batch_destroy(aexis_batch* batch);

/* Sets `batch` sequences with contexts ctx_lens[i] (host, 0 <= len < capacity)
 * already in their caches: position p < len of layer l holds, for K (kind 0)
 * and V (kind 1) of head h and dim d, the fp16 rounding of
 *   u = (mix64(key ^ idx) >> 40) * 2^-24 - 0.5,
 *   key = mix64(seed ^ mix64(first_seq_id + i)),
 *   idx = ((((l * 2 + kind) * 256 + h) * 65536 + p) * 256 + d),
 * mix64 the splitmix64 finaliser. This stands in for the prefill of a real
 * prompt (synthetic contexts of a serving benchmark); the CPU oracle fills
 * its cache with the same values. Each sequence's next position is len. */
int aexis_cuda_batch_fill_context(aexis_batch* batch, int n, const int32_t* ctx_lens, uint64_t seed,
                                  int64_t first_seq_id);

/* Greedy decoding of `steps` tokens for every sequence: first_tokens[i]
 * (host) is the input of sequence i at its current position; out_tokens
 * (host, may be NULL) receives [steps][n] step-major. Synchronous. E_RANGE
 * when a sequence would pass its capacity. */
int aexis_cuda_batch_generate(aexis_batch* batch, const int32_t* first_tokens, int steps, int32_t* out_tokens);

/* The batch's sequences in the reference's state layout (see the decoder
 * state calls above; one Qwen35DecoderState per sequence). seq in
 * [0, max_batch). Export: rows >= the sequence's position (E_SHAPE), rows
 * past it zero; a sequence beyond the last fill / set_positions exports as
 * empty. Import: positions [0, length) with length < kv_capacity. After the
 * imports, aexis_cuda_batch_set_positions(batch, n, positions) makes
 * sequences 0..n-1 the batch, each continuing at positions[i] (host, each in
 * [0, kv_capacity)), as aexis_cuda_batch_fill_context does for synthetic
 * contexts. */
int aexis_cuda_batch_kv_export(aexis_batch* batch, int seq, int layer, int rows, float* k_out, float* v_out);
int aexis_cuda_batch_kv_import(aexis_batch* batch, int seq, int layer, const float* k_in, const float* v_in, int rows,
                               int length);
int aexis_cuda_batch_set_positions(aexis_batch* batch, int n, const int32_t* positions);

/* Next position of each sequence (host [n]). */
int aexis_cuda_batch_positions(const aexis_batch* batch, int32_t* out);

/* fp32 logits of the last step, host [n][vocab]. */
int aexis_cuda_batch_logits(aexis_batch* batch, float* out_logits);

#ifdef __cplusplus
}
#endif

#endif /* AEXIS_CUDA_H_ */
