// abi.cu -- host side of the libaexis_cuda C ABI (include/aexis_cuda.h):
// argument validation with the reference's error classes, weight handles,
// and dispatch to the kernels. No C++ exception crosses the ABI.
#include <cmath>
#include <cstdarg>
#include <cstring>
#include <algorithm>
#include <new>

#include "aexis_internal.h"

#define AEXIS_API extern "C" __attribute__((visibility("default")))

namespace {
thread_local std::string g_create_error;
}

int aexis_fail(aexis_ctx* ctx, int code, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (ctx) ctx->err = buf;
    else g_create_error = buf;
    return code;
}

int aexis_cuda_check(aexis_ctx* ctx, cudaError_t e, const char* what) {
    if (e == cudaSuccess) return AEXIS_OK;
    return aexis_fail(ctx, AEXIS_E_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int aexis_check_status(aexis_ctx* ctx) {
    int st = 0;
    cudaError_t e = cudaMemcpy(&st, ctx->status, sizeof(int), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return aexis_cuda_check(ctx, e, "status readback");
    if (st == 0) return AEXIS_OK;
    cudaMemset(ctx->status, 0, sizeof(int));
    return aexis_fail(ctx, st, "a kernel gave up on a bounded wait (status %d); the context stays usable", st);
}

int aexis_scratch(aexis_ctx* ctx, size_t bytes, void** out) {
    if (bytes > ctx->scratch_bytes) {
        // The old buffer may still be read by enqueued work: wait before freeing.
        if (ctx->scratch) {
            cudaStreamSynchronize(ctx->stream);
            cudaFree(ctx->scratch);
            ctx->scratch = nullptr;
            ctx->scratch_bytes = 0;
        }
        size_t sz = std::max<size_t>(bytes, 1 << 20);
        cudaError_t e = cudaMalloc(&ctx->scratch, sz);
        if (e != cudaSuccess) return aexis_cuda_check(ctx, e, "scratch cudaMalloc");
        ctx->scratch_bytes = sz;
    }
    *out = ctx->scratch;
    return AEXIS_OK;
}

namespace {

int bind(aexis_ctx* ctx) { return aexis_cuda_check(ctx, cudaSetDevice(ctx->device), "cudaSetDevice"); }

bool valid_dtype(int d) { return d == AEXIS_F32 || d == AEXIS_F16; }

int upload(aexis_ctx* ctx, const void* host, size_t bytes, void** dev, const char* what) {
    cudaError_t e = cudaMalloc(dev, bytes + kWeightPad);
    if (e == cudaSuccess) e = cudaMemset((char*)*dev + bytes, 0, kWeightPad);
    if (e != cudaSuccess) return aexis_cuda_check(ctx, e, what);
    e = cudaMemcpy(*dev, host, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) {
        cudaFree(*dev);
        *dev = nullptr;
        return aexis_cuda_check(ctx, e, what);
    }
    return AEXIS_OK;
}

// Host quantizer shared by the Q8 / Q4 float upload paths
// (AexisGraphSession.NewInt{8,4}WeightOnlyUpload(float[], ...)).
int quantize_rows(int bits, const float* data, int out_ch, int per_ch, int contiguous, uint32_t* packed,
                  float* scales) {
    if (!data || !packed || !scales) return AEXIS_E_NULL;
    if (out_ch <= 0) return AEXIS_E_RANGE;
    if (per_ch <= 0) return AEXIS_E_SHAPE;
    const long long total = (long long)out_ch * per_ch;
    const long long words = std::max<long long>(1, (total + (bits == 4 ? 7 : 3)) / (bits == 4 ? 8 : 4));
    std::memset(packed, 0, sizeof(uint32_t) * words);
    const float qmax = bits == 4 ? 7.0f : 127.0f;
    const int lim = bits == 4 ? 7 : 127;
    for (int oc = 0; oc < out_ch; ++oc) {
        float max_abs = 0.0f;
        for (int vi = 0; vi < per_ch; ++vi) {
            const long long si = contiguous ? (long long)oc * per_ch + vi : (long long)vi * out_ch + oc;
            max_abs = std::max(max_abs, std::fabs(data[si]));
        }
        const float scale = max_abs > 0.0f ? max_abs / qmax : 1.0f;
        scales[oc] = scale;
        for (int vi = 0; vi < per_ch; ++vi) {
            const long long si = contiguous ? (long long)oc * per_ch + vi : (long long)vi * out_ch + oc;
            int q = (int)std::nearbyintf(data[si] / scale);  // midpoint to even, as Mathf.RoundToInt
            q = q < -lim ? -lim : (q > lim ? lim : q);
            if (bits == 4) packed[si >> 3] |= ((uint32_t)q & 0xFu) << ((si & 7) * 4);
            else packed[si >> 2] |= (uint32_t)(uint8_t)(int8_t)q << ((si & 3) * 8);
        }
    }
    return AEXIS_OK;
}

size_t dsize(int dtype) { return dtype == AEXIS_F16 ? 2 : 4; }

// Rows from which a Q8 Gemm takes the tensor-core path (one weight pass)
// instead of one streaming GEMV per row.
constexpr int kTcMinRows = 4;

}  // namespace

// ---------------------------------------------------------------- context
AEXIS_API int aexis_cuda_abi_version(void) { return AEXIS_CUDA_ABI_VERSION; }

AEXIS_API int aexis_cuda_create(int device, aexis_ctx** out) {
    if (!out) return aexis_fail(nullptr, AEXIS_E_NULL, "out is null");
    *out = nullptr;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0)
        return aexis_fail(nullptr, AEXIS_E_CUDA, "no CUDA device: %s", cudaGetErrorString(e));
    if (device < 0 || device >= count)
        return aexis_fail(nullptr, AEXIS_E_RANGE, "device %d out of range [0, %d)", device, count);
    cudaDeviceProp prop;
    e = cudaGetDeviceProperties(&prop, device);
    if (e != cudaSuccess) return aexis_fail(nullptr, AEXIS_E_CUDA, "cudaGetDeviceProperties: %s", cudaGetErrorString(e));
    if (prop.major != 10)
        return aexis_fail(nullptr, AEXIS_E_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a (B200)",
                          device, prop.major, prop.minor);
    aexis_ctx* ctx = new (std::nothrow) aexis_ctx();
    if (!ctx) return aexis_fail(nullptr, AEXIS_E_STATE, "out of host memory");
    ctx->device = device;
    ctx->sm_count = prop.multiProcessorCount;
    e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->own_stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete ctx;
        return aexis_fail(nullptr, AEXIS_E_CUDA, "stream create: %s", cudaGetErrorString(e));
    }
    ctx->stream = ctx->own_stream;
    e = cudaMalloc(&ctx->status, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ctx->status, 0, sizeof(int));
    if (e != cudaSuccess) {
        cudaStreamDestroy(ctx->own_stream);
        delete ctx;
        return aexis_fail(nullptr, AEXIS_E_CUDA, "status alloc: %s", cudaGetErrorString(e));
    }
    *out = ctx;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_destroy(aexis_ctx* ctx) {
    if (!ctx) return AEXIS_E_NULL;
    cudaSetDevice(ctx->device);
    if (ctx->own_stream) cudaStreamSynchronize(ctx->own_stream);
    if (ctx->scratch) cudaFree(ctx->scratch);
    if (ctx->act_q) cudaFree(ctx->act_q);
    if (ctx->samp) cudaFree(ctx->samp);
    if (ctx->pack_a) cudaFree(ctx->pack_a);
    if (ctx->fused) cudaFree(ctx->fused);
    if (ctx->status) cudaFree(ctx->status);
    if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
    delete ctx;
    return AEXIS_OK;
}

AEXIS_API const char* aexis_cuda_last_error(const aexis_ctx* ctx) {
    return ctx ? ctx->err.c_str() : g_create_error.c_str();
}

AEXIS_API int aexis_cuda_set_stream(aexis_ctx* ctx, void* stream) {
    if (!ctx) return AEXIS_E_NULL;
    // NULL is the CUDA legacy default stream, as everywhere in CUDA (torch's
    // default stream handle is 0): work then orders with that stream.
    ctx->stream = (cudaStream_t)stream;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_sync(aexis_ctx* ctx) {
    if (!ctx) return AEXIS_E_NULL;
    int rc = bind(ctx);
    if (rc) return rc;
    rc = aexis_cuda_check(ctx, cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
    if (rc) return rc;
    return aexis_check_status(ctx);
}

AEXIS_API int aexis_cuda_selftest_wait(aexis_ctx* ctx, long long limit_cycles) {
    if (!ctx) return AEXIS_E_NULL;
    if (limit_cycles < 1000 || limit_cycles > 4000000000LL)
        return aexis_fail(ctx, AEXIS_E_RANGE, "limit_cycles %lld outside [1e3, 4e9]", limit_cycles);
    int rc = bind(ctx);
    if (rc) return rc;
    void* flag = nullptr;
    rc = aexis_scratch(ctx, sizeof(int), &flag);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_selftest_wait(reinterpret_cast<int*>(flag), limit_cycles, ctx->status,
                                                      ctx->stream), "self-test launch");
}

// ---------------------------------------------------------------- weights
AEXIS_API int aexis_quantize_q8_rows(const float* data, int out_ch, int per_ch, int contiguous, uint32_t* packed,
                                     float* scales) {
    return quantize_rows(8, data, out_ch, per_ch, contiguous, packed, scales);
}

AEXIS_API int aexis_quantize_q4_rows(const float* data, int out_ch, int per_ch, int contiguous, uint32_t* packed,
                                     float* scales) {
    return quantize_rows(4, data, out_ch, per_ch, contiguous, packed, scales);
}

static int weights_q(aexis_ctx* ctx, int kind, const uint32_t* packed, const void* scales, int scale_dtype, int n,
                     int k, int group, aexis_weights** out) {
    if (!ctx) return AEXIS_E_NULL;
    if (!out) return aexis_fail(ctx, AEXIS_E_NULL, "out is null");
    *out = nullptr;
    if (!packed || !scales)
        return aexis_fail(ctx, AEXIS_E_NULL, "%s Gemm weights and scales must be configured together.",
                          kind == WK_Q4 ? "INT4" : "INT8");
    if (n <= 0 || k <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "n=%d k=%d must be positive", n, k);
    if (!valid_dtype(scale_dtype)) return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "scale dtype %d", scale_dtype);
    const long long total = (long long)n * k;
    if (total > (1LL << 40)) return aexis_fail(ctx, AEXIS_E_RANGE, "weight too large");
    long long nscales;
    if (kind == WK_Q4) {
        if (group <= 0 || k % group != 0)
            return aexis_fail(ctx, AEXIS_E_SHAPE, "Direct Q4 group size must divide the Gemm K dimension.");
        nscales = total / group;
    } else {
        nscales = n;
    }
    int rc = bind(ctx);
    if (rc) return rc;
    aexis_weights* w = new (std::nothrow) aexis_weights();
    if (!w) return aexis_fail(ctx, AEXIS_E_STATE, "out of host memory");
    w->kind = kind;
    w->n = n;
    w->k = k;
    w->group = kind == WK_Q4 ? group : 0;
    w->scale_dtype = scale_dtype;
    const long long words = std::max<long long>(1, (total + (kind == WK_Q4 ? 7 : 3)) / (kind == WK_Q4 ? 8 : 4));
    w->data_bytes = (size_t)words * 4;
    w->scale_bytes = (size_t)nscales * dsize(scale_dtype);
    rc = upload(ctx, packed, w->data_bytes, &w->data, "weight upload");
    if (rc == AEXIS_OK) rc = upload(ctx, scales, w->scale_bytes, &w->scales, "scale upload");
    // A second copy in the tensor-core GEMV's fragment layout.
    if (rc == AEXIS_OK && gemv_mma_eligible(w)) {
        size_t sb = 0;
        const size_t wb = gemv_mma_frag_bytes(w, &sb);
        cudaError_t e = cudaMalloc(&w->frag, wb);
        if (e == cudaSuccess) e = cudaMalloc(&w->frag_scales, sb);
        if (e == cudaSuccess) e = launch_repack_frag(w, ctx->stream);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
        rc = aexis_cuda_check(ctx, e, "fragment repack");
    }
    if (rc) {
        if (w->data) cudaFree(w->data);
        if (w->scales) cudaFree(w->scales);
        if (w->frag) cudaFree(w->frag);
        if (w->frag_scales) cudaFree(w->frag_scales);
        delete w;
        return rc;
    }
    *out = w;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_weights_q8(aexis_ctx* ctx, const uint32_t* packed, const void* scales, int scale_dtype,
                                    int n, int k, aexis_weights** out) {
    return weights_q(ctx, WK_Q8, packed, scales, scale_dtype, n, k, 0, out);
}

AEXIS_API int aexis_cuda_weights_q4(aexis_ctx* ctx, const uint32_t* packed, const void* scales, int scale_dtype,
                                    int n, int k, int group, aexis_weights** out) {
    return weights_q(ctx, WK_Q4, packed, scales, scale_dtype, n, k, group, out);
}

AEXIS_API int aexis_cuda_weights_dense(aexis_ctx* ctx, const void* data, int dtype, int n, int k,
                                       aexis_weights** out) {
    if (!ctx) return AEXIS_E_NULL;
    if (!out || !data) return aexis_fail(ctx, AEXIS_E_NULL, "data/out is null");
    *out = nullptr;
    if (n <= 0 || k <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "n=%d k=%d must be positive", n, k);
    if (!valid_dtype(dtype)) return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "dtype %d", dtype);
    int rc = bind(ctx);
    if (rc) return rc;
    aexis_weights* w = new (std::nothrow) aexis_weights();
    if (!w) return aexis_fail(ctx, AEXIS_E_STATE, "out of host memory");
    w->kind = dtype == AEXIS_F16 ? WK_F16 : WK_F32;
    w->n = n;
    w->k = k;
    w->data_bytes = (size_t)n * k * dsize(dtype);
    rc = upload(ctx, data, w->data_bytes, &w->data, "dense upload");
    if (rc) {
        delete w;
        return rc;
    }
    *out = w;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_weights_free(aexis_ctx* ctx, aexis_weights* w) {
    if (!ctx || !w) return AEXIS_E_NULL;
    bind(ctx);
    cudaStreamSynchronize(ctx->stream);
    if (w->data) cudaFree(w->data);
    if (w->scales) cudaFree(w->scales);
    if (w->tc_tiled) cudaFree(w->tc_tiled);
    if (w->frag) cudaFree(w->frag);
    if (w->frag_scales) cudaFree(w->frag_scales);
    delete w;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_weights_dequant(aexis_ctx* ctx, const aexis_weights* w, float* out) {
    if (!ctx) return AEXIS_E_NULL;
    if (!w || !out) return aexis_fail(ctx, AEXIS_E_NULL, "weights/out is null");
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_dequant(w, out, ctx->stream), "dequant launch");
}

// ----------------------------------------------------------------- linear
static int gemm_common(aexis_ctx* ctx, const void* a, int a_dtype, int lda, int m, int k, const aexis_weights* w,
                       const float* bias, float alpha, float beta, void* y, int y_dtype, int ldy, int n, int epi) {
    if (!ctx) return AEXIS_E_NULL;
    if (!a) return aexis_fail(ctx, AEXIS_E_NULL, "a is null");
    if (!w) return aexis_fail(ctx, AEXIS_E_NULL, "b is null");
    if (!y) return aexis_fail(ctx, AEXIS_E_NULL, "output is null");
    if (m <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "m=%d", m);
    if (n <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "n=%d", n);
    if (k <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "k=%d", k);
    if (w->kind != WK_Q4 && w->kind != WK_Q8)
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "Gemm needs INT4 or INT8 weights");
    if (w->n != n || w->k != k)
        return aexis_fail(ctx, AEXIS_E_SHAPE, "weight is [%d, %d], call asks for n=%d k=%d", w->n, w->k, n, k);
    if (lda < k || ldy < n) return aexis_fail(ctx, AEXIS_E_SHAPE, "lda=%d < k or ldy=%d < n", lda, ldy);
    if (!valid_dtype(a_dtype) || !valid_dtype(y_dtype))
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "dtype a=%d y=%d", a_dtype, y_dtype);
    int rc = bind(ctx);
    if (rc) return rc;
    // W8A8 on the batch-1 tensor-core GEMV: the kernel stages the codes itself
    // (no extra launch). Every other path reads codes written by one more kernel.
    const bool tc_path = m >= kTcMinRows && gemm_tc_supported(w, m, AEXIS_F16);
    const bool fused_codes = ctx->act_quant && !tc_path && gemv_mma_supported(w, a_dtype);
    if (fused_codes) {
        if (epi == EPI_STORE) beta = beta / ctx->act_scale;
        alpha = alpha * ctx->act_scale;
    } else if (ctx->act_quant) {
        // W8A8: the GEMM reads the integer codes q - zp (fp16, exact) instead of
        // the activations and the scale moves into the epilogue:
        //   alpha*(beta*bias + sum (q-zp)*s*W) = (alpha*s)*((beta/s)*bias + sum (q-zp)*W)
        //   beta*bias + alpha*sum (q-zp)*s*W   = beta*bias + (alpha*s)*sum (q-zp)*W
        const size_t need = (size_t)m * k * sizeof(__half);
        if (need > ctx->act_q_bytes) {
            if (ctx->act_q) {
                cudaStreamSynchronize(ctx->stream);
                cudaFree(ctx->act_q);
                ctx->act_q = nullptr;
                ctx->act_q_bytes = 0;
            }
            const size_t sz = std::max<size_t>(need, 1 << 16);
            rc = aexis_cuda_check(ctx, cudaMalloc(&ctx->act_q, sz), "activation code buffer");
            if (rc) return rc;
            ctx->act_q_bytes = sz;
        }
        rc = aexis_cuda_check(ctx, launch_act_quant_i8(a, a_dtype, lda, m, k, ctx->act_scale, ctx->act_zero_point,
                                                       ctx->act_unsigned, (__half*)ctx->act_q, ctx->stream),
                              "activation quantisation launch");
        if (rc) return rc;
        a = ctx->act_q;
        a_dtype = AEXIS_F16;
        lda = k;
        if (epi == EPI_STORE) beta = beta / ctx->act_scale;
        alpha = alpha * ctx->act_scale;
    }
    // Batched Q8: one pass over the weights on the tensor cores.
    if (m >= kTcMinRows && gemm_tc_supported(w, m, a_dtype)) {
        aexis_weights* wm = const_cast<aexis_weights*>(w);
        if (!wm->tc_tiled) {
            cudaError_t e = cudaMalloc(&wm->tc_tiled, gemm_tc_tiled_bytes(w));
            if (e != cudaSuccess) return aexis_cuda_check(ctx, e, "tensor-core weight tiles");
            rc = aexis_cuda_check(ctx, launch_repack_q8(w, wm->tc_tiled, ctx->stream), "weight repack");
            if (rc) return rc;
        }
        void* xt = nullptr;
        rc = aexis_scratch(ctx, gemm_tc_xt_bytes(m, k, a_dtype), &xt);
        if (rc) return rc;
        return aexis_cuda_check(ctx, launch_gemm_tc(w, wm->tc_tiled, a, a_dtype, lda, m, xt, bias, alpha, beta, y,
                                                    y_dtype, ldy, epi == EPI_STORE_TILED, ctx->sm_count, ctx->status,
                                                    ctx->stream), "tensor-core gemm launch");
    }
    GemvArgs g;
    g.status = ctx->status;
    g.a_dtype = a_dtype;
    g.w = w;
    g.bias = bias;
    g.alpha = alpha;
    g.beta = beta;
    g.y_dtype = y_dtype;
    g.epilogue = epi;
    if (fused_codes) {
        g.act_quant = 1;
        g.act_scale = ctx->act_scale;
        g.act_zero_point = ctx->act_zero_point;
        g.act_unsigned = ctx->act_unsigned;
    }
    // Programmatic dependent launch: the GEMV kernels read only the (immutable,
    // library-owned) weights before waiting on the previous kernel of the
    // stream, so their weight streaming overlaps that kernel's tail; every read
    // of x and every write of y comes after the wait.
    g.pdl = true;
    for (int r = 0; r < m; ++r) {
        g.x = (const char*)a + (size_t)r * lda * dsize(a_dtype);
        g.y = (char*)y + (size_t)r * ldy * dsize(y_dtype);
        rc = aexis_cuda_check(ctx, launch_gemv(g, ctx->sm_count, ctx->stream), "gemv launch");
        if (rc) return rc;
    }
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_set_int8_activations(aexis_ctx* ctx, int enable, float scale, int zero_point,
                                             int is_unsigned) {
    if (!ctx) return AEXIS_E_NULL;
    if (!enable) {
        ctx->act_quant = 0;
        ctx->act_scale = 1.0f;
        ctx->act_zero_point = 0;
        ctx->act_unsigned = 0;
        return AEXIS_OK;
    }
    if (!(scale > 0.0f) || !std::isfinite(scale))
        return aexis_fail(ctx, AEXIS_E_RANGE, "activation scale %g must be positive and finite", (double)scale);
    if (zero_point < -1024 || zero_point > 1024)
        return aexis_fail(ctx, AEXIS_E_RANGE, "activation zero point %d outside [-1024, 1024]", zero_point);
    ctx->act_quant = 1;
    ctx->act_scale = scale;
    ctx->act_zero_point = zero_point;
    ctx->act_unsigned = is_unsigned ? 1 : 0;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_gemm(aexis_ctx* ctx, const void* a, int a_dtype, int lda, int m, int k,
                              const aexis_weights* w, const float* bias, float alpha, float beta, void* y,
                              int y_dtype, int ldy, int n) {
    return gemm_common(ctx, a, a_dtype, lda, m, k, w, bias, alpha, beta, y, y_dtype, ldy, n, EPI_STORE);
}

AEXIS_API int aexis_cuda_gemm_tiled(aexis_ctx* ctx, const void* a, int a_dtype, int lda, int m, int k,
                                    const aexis_weights* w, const float* bias, float alpha, float beta, void* y,
                                    int y_dtype, int ldy, int n) {
    return gemm_common(ctx, a, a_dtype, lda, m, k, w, bias, alpha, beta, y, y_dtype, ldy, n, EPI_STORE_TILED);
}

AEXIS_API int aexis_cuda_gemm_pack4a(aexis_ctx* ctx, const void* a, int a_dtype, int a_width, int a_height,
                                     int a_slices, int m, int k, const aexis_weights* w, const float* bias,
                                     float alpha, float beta, void* y, int y_dtype, int ldy, int n) {
    if (!ctx) return AEXIS_E_NULL;
    if (!a) return aexis_fail(ctx, AEXIS_E_NULL, "a is null");
    if (m <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "m=%d", m);
    if (k <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "k=%d", k);
    if (a_width <= 0 || a_slices <= 0 || a_height < m)
        return aexis_fail(ctx, AEXIS_E_SHAPE, "Pack4 input texture %dx%d with %d slices cannot hold %d rows",
                          a_width, a_height, a_slices, m);
    if (!valid_dtype(a_dtype)) return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "dtype a=%d", a_dtype);
    // Every K value in slice 0: rows are row-major with a stride of 4*width.
    if ((long long)a_width * 4 >= k)
        return gemm_common(ctx, a, a_dtype, a_width * 4, m, k, w, bias, alpha, beta, y, y_dtype, ldy, n, EPI_STORE);
    // Validate the GEMM itself before the gather runs.
    if (!w) return aexis_fail(ctx, AEXIS_E_NULL, "b is null");
    if (!y) return aexis_fail(ctx, AEXIS_E_NULL, "output is null");
    if (n <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "n=%d", n);
    if (w->n != n || w->k != k)
        return aexis_fail(ctx, AEXIS_E_SHAPE, "weight is [%d, %d], call asks for n=%d k=%d", w->n, w->k, n, k);
    int rc = bind(ctx);
    if (rc) return rc;
    const size_t need = (size_t)m * k * dsize(a_dtype);
    if (need > ctx->pack_a_bytes) {
        if (ctx->pack_a) {
            cudaStreamSynchronize(ctx->stream);
            cudaFree(ctx->pack_a);
            ctx->pack_a = nullptr;
            ctx->pack_a_bytes = 0;
        }
        const size_t sz = std::max<size_t>(need, 1 << 16);
        rc = aexis_cuda_check(ctx, cudaMalloc(&ctx->pack_a, sz), "Pack4 input buffer");
        if (rc) return rc;
        ctx->pack_a_bytes = sz;
    }
    rc = aexis_cuda_check(ctx, launch_gather_pack4a(a, a_dtype, a_width, a_height, a_slices, m, k, ctx->pack_a,
                                                    ctx->stream), "Pack4 input gather launch");
    if (rc) return rc;
    return gemm_common(ctx, ctx->pack_a, a_dtype, k, m, k, w, bias, alpha, beta, y, y_dtype, ldy, n, EPI_STORE);
}

// ------------------------------------------------------------ lm_head + top-k
namespace {

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

}  // namespace

AEXIS_API int aexis_cuda_gemm_topk(aexis_ctx* ctx, const void* a, int a_dtype, int lda, int m, int k,
                                   const aexis_weights* w, float alpha, int top_k, int64_t index_offset,
                                   float* out_vals, int32_t* out_idx, uint64_t* greedy_keys) {
    if (!ctx) return AEXIS_E_NULL;
    if (!a || !w || !out_vals || !out_idx) return aexis_fail(ctx, AEXIS_E_NULL, "a, b or an output is null");
    if (m <= 0 || k <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "m=%d k=%d", m, k);
    if (top_k < 1 || top_k > 64) return aexis_fail(ctx, AEXIS_E_RANGE, "top_k=%d (1..64)", top_k);
    if (w->kind != WK_Q4 && w->kind != WK_Q8)
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "Gemm needs INT4 or INT8 weights");
    if (w->k != k) return aexis_fail(ctx, AEXIS_E_SHAPE, "weight is [%d, %d], call asks for k=%d", w->n, w->k, k);
    if (lda < k) return aexis_fail(ctx, AEXIS_E_SHAPE, "lda=%d < k", lda);
    if (!valid_dtype(a_dtype)) return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "dtype a=%d", a_dtype);
    int rc = bind(ctx);
    if (rc) return rc;
    const int n = w->n;
    // The logits in a context buffer (row stride n), then the top-k kernels
    // over them and the greedy keys from the top-k lists.
    const size_t need = align256((size_t)m * n * sizeof(float));
    if (need > ctx->fused_bytes) {
        if (ctx->fused) {
            cudaStreamSynchronize(ctx->stream);
            cudaFree(ctx->fused);
            ctx->fused = nullptr;
            ctx->fused_bytes = 0;
        }
        rc = aexis_cuda_check(ctx, cudaMalloc(&ctx->fused, need), "logits buffer");
        if (rc) return rc;
        ctx->fused_bytes = need;
    }
    float* logits = reinterpret_cast<float*>(ctx->fused);
    rc = gemm_common(ctx, a, a_dtype, lda, m, k, w, nullptr, alpha, 1.0f, logits, AEXIS_F32, n, n, EPI_STORE_TILED);
    if (rc) return rc;
    void* tk = nullptr;
    rc = aexis_scratch(ctx, topk_scratch_bytes(m, n, top_k, ctx->sm_count), &tk);
    if (rc) return rc;
    cudaError_t e = launch_topk(logits, m, n, n, top_k, out_vals, out_idx, tk, ctx->sm_count, ctx->stream);
    if (e == cudaSuccess && greedy_keys)
        e = launch_topk_greedy_keys(logits, m, n, out_vals, out_idx, top_k, (long long)index_offset,
                                    reinterpret_cast<unsigned long long*>(greedy_keys), ctx->stream);
    return aexis_cuda_check(ctx, e, "lm_head top-k launch");
}

// ------------------------------------------------------- pointwise layers
AEXIS_API int aexis_cuda_rmsnorm(aexis_ctx* ctx, const void* x, int x_dtype, int rows, int width, int ld,
                                 const float* gamma, int affine_size, float eps, void* y, int y_dtype) {
    if (!ctx) return AEXIS_E_NULL;
    if (!x) return aexis_fail(ctx, AEXIS_E_NULL, "input is null");
    if (!y) return aexis_fail(ctx, AEXIS_E_NULL, "output is null");
    if (rows <= 0 || width <= 0 || ld < width)
        return aexis_fail(ctx, AEXIS_E_STATE, "RmsNormPack4LinearMat requires a one- or two-dimensional logical tensor.");
    if (!valid_dtype(x_dtype) || !valid_dtype(y_dtype)) return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "dtype");
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_rmsnorm(x, x_dtype, rows, width, ld, gamma, gamma ? affine_size : 0, eps, y,
                                                y_dtype, ctx->stream), "rmsnorm launch");
}

AEXIS_API int aexis_cuda_rope(aexis_ctx* ctx, const float* src, int embed_dim, int seq_len, int num_heads,
                              const float* cos_table, const float* sin_table, int interleaved, float* out) {
    if (!ctx) return AEXIS_E_NULL;
    if (!src) return aexis_fail(ctx, AEXIS_E_NULL, "input is null");
    if (!cos_table) return aexis_fail(ctx, AEXIS_E_NULL, "cos is null");
    if (!sin_table) return aexis_fail(ctx, AEXIS_E_NULL, "sin is null");
    if (!out) return aexis_fail(ctx, AEXIS_E_NULL, "output is null");
    if (embed_dim <= 0 || seq_len <= 0 || num_heads <= 0)
        return aexis_fail(ctx, AEXIS_E_RANGE, "shape w=%d h=%d c=%d", embed_dim, seq_len, num_heads);
    if (src == out) return aexis_fail(ctx, AEXIS_E_SHAPE, "in-place RoPE is not supported (pairs are read twice)");
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_rope(src, embed_dim, seq_len, num_heads, cos_table, sin_table, interleaved, out,
                                             ctx->stream), "rope launch");
}

AEXIS_API int aexis_cuda_kv_append(aexis_ctx* ctx, const float* current, int width, int rows, int slices, int offset,
                                   float* cache, int cache_rows) {
    if (!ctx) return AEXIS_E_NULL;
    if (!current) return aexis_fail(ctx, AEXIS_E_NULL, "current is null");
    if (!cache) return aexis_fail(ctx, AEXIS_E_NULL, "output is null");
    if (offset < 0) return aexis_fail(ctx, AEXIS_E_RANGE, "destinationOffset=%d", offset);
    if (rows <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "currentHeight=%d", rows);
    if (width <= 0 || slices <= 0)
        return aexis_fail(ctx, AEXIS_E_STATE, "AppendSequencePack4Cdhw requires matching width/depth textures.");
    if (offset + rows > cache_rows)
        return aexis_fail(ctx, AEXIS_E_STATE, "AppendSequencePack4Cdhw output height is too small.");
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_kv_append(current, width, rows, slices, offset, cache, cache_rows, ctx->stream),
                            "kv append launch");
}

AEXIS_API int aexis_cuda_kv_concat(aexis_ctx* ctx, const float* past, int past_rows, const float* current, int cur_rows,
                                   int width, int slices, float* out, int out_rows) {
    if (!ctx) return AEXIS_E_NULL;
    if (!past) return aexis_fail(ctx, AEXIS_E_NULL, "a is null");
    if (!current) return aexis_fail(ctx, AEXIS_E_NULL, "b is null");
    if (!out) return aexis_fail(ctx, AEXIS_E_NULL, "output is null");
    if (past_rows <= 0 || cur_rows <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "aHeight=%d bHeight=%d", past_rows, cur_rows);
    if (width <= 0 || slices <= 0)
        return aexis_fail(ctx, AEXIS_E_STATE, "ConcatSequencePack4Cdhw requires matching width/depth textures.");
    if (out_rows < past_rows + cur_rows)
        return aexis_fail(ctx, AEXIS_E_STATE, "ConcatSequencePack4Cdhw output height is too small.");
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_kv_concat(past, past_rows, current, cur_rows, width, slices, out, out_rows,
                                                  ctx->stream), "kv concat launch");
}

AEXIS_API int aexis_cuda_sdpa(aexis_ctx* ctx, const float* q, const float* k, const float* v, int src_len, int dst_len,
                              int embed_dim, int out_embed_dim, int num_heads, int num_groups, float scale,
                              const float* mask, int mask_w, int mask_h, int causal, int causal_offset, float* out) {
    if (!ctx) return AEXIS_E_NULL;
    if (!q) return aexis_fail(ctx, AEXIS_E_NULL, "query is null");
    if (!k) return aexis_fail(ctx, AEXIS_E_NULL, "key is null");
    if (!v) return aexis_fail(ctx, AEXIS_E_NULL, "value is null");
    if (!out) return aexis_fail(ctx, AEXIS_E_NULL, "output is null");
    if (src_len <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "srcLen=%d", src_len);
    if (dst_len <= 0 || sdpa_smem_bytes(dst_len) > 200 * 1024)
        return aexis_fail(ctx, AEXIS_E_RANGE, "dstLen=%d (max %d)", dst_len, (int)(200 * 1024 / sizeof(float)));
    if (embed_dim <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "embedDim=%d", embed_dim);
    if (out_embed_dim <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "outEmbedDim=%d", out_embed_dim);
    if (num_heads <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "numHeads=%d", num_heads);
    if (num_groups <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "numGroups=%d", num_groups);
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_sdpa(q, k, v, src_len, dst_len, embed_dim, out_embed_dim, num_heads,
                                             num_groups, scale, mask, mask ? mask_w : 0, mask ? mask_h : 0, causal,
                                             causal_offset, out, ctx->stream), "sdpa launch");
}

AEXIS_API int aexis_cuda_argmax(aexis_ctx* ctx, const float* logits, int rows, int width, int ld, int32_t* out_idx) {
    if (!ctx) return AEXIS_E_NULL;
    if (!logits) return aexis_fail(ctx, AEXIS_E_NULL, "input is null");
    if (!out_idx) return aexis_fail(ctx, AEXIS_E_NULL, "output is null");
    if (width <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "logicalWidth=%d", width);
    if (rows <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "logicalHeight=%d", rows);
    if (ld < width) return aexis_fail(ctx, AEXIS_E_SHAPE, "ld=%d < width", ld);
    int rc = bind(ctx);
    if (rc) return rc;
    void* keys = nullptr;
    rc = aexis_scratch(ctx, sizeof(unsigned long long) * (size_t)rows, &keys);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_argmax(logits, rows, width, ld, out_idx, (unsigned long long*)keys,
                                               ctx->sm_count, ctx->stream), "argmax launch");
}

AEXIS_API int aexis_cuda_argmax_keys(aexis_ctx* ctx, const float* logits, int rows, int width, int ld,
                                     int64_t index_offset, uint64_t* keys) {
    if (!ctx) return AEXIS_E_NULL;
    if (!logits || !keys) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    if (width <= 0 || rows <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "rows=%d width=%d", rows, width);
    if (ld < width) return aexis_fail(ctx, AEXIS_E_SHAPE, "ld=%d < width", ld);
    if (index_offset < 0 || index_offset + width > 0xFFFFFFFFLL)
        return aexis_fail(ctx, AEXIS_E_RANGE, "index_offset=%lld", (long long)index_offset);
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_argmax_keys(logits, rows, width, ld, index_offset,
                                                    (unsigned long long*)keys, ctx->sm_count, ctx->stream),
                            "argmax keys launch");
}

AEXIS_API int aexis_cuda_topk(aexis_ctx* ctx, const float* logits, int rows, int width, int ld, int k, float* out_vals,
                              int32_t* out_idx) {
    if (!ctx) return AEXIS_E_NULL;
    if (!logits || !out_vals || !out_idx) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    if (width <= 0 || rows <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "rows=%d width=%d", rows, width);
    if (k < 1 || k > 64) return aexis_fail(ctx, AEXIS_E_RANGE, "k=%d (1..64)", k);
    if (ld < width) return aexis_fail(ctx, AEXIS_E_SHAPE, "ld=%d < width", ld);
    int rc = bind(ctx);
    if (rc) return rc;
    void* scratch = nullptr;
    rc = aexis_scratch(ctx, topk_scratch_bytes(rows, width, k, ctx->sm_count), &scratch);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_topk(logits, rows, width, ld, k, out_vals, out_idx, scratch, ctx->sm_count,
                                             ctx->stream), "topk launch");
}

AEXIS_API int aexis_cuda_topk_greedy_keys(aexis_ctx* ctx, const float* logits, int rows, int width, int ld, int k,
                                          const float* top_vals, const int32_t* top_idx, int64_t index_offset,
                                          uint64_t* keys) {
    if (!ctx) return AEXIS_E_NULL;
    if (!logits || !top_vals || !top_idx || !keys) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    if (width <= 0 || rows <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "rows=%d width=%d", rows, width);
    if (k < 1 || k > 64) return aexis_fail(ctx, AEXIS_E_RANGE, "k=%d (1..64)", k);
    if (ld < width) return aexis_fail(ctx, AEXIS_E_SHAPE, "ld=%d < width", ld);
    if (index_offset < 0 || index_offset + width > 0x7fffffffLL)
        return aexis_fail(ctx, AEXIS_E_RANGE, "index_offset=%lld", (long long)index_offset);
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_topk_greedy_keys(logits, rows, ld, top_vals, top_idx, k, index_offset,
                                                         reinterpret_cast<unsigned long long*>(keys), ctx->stream),
                            "greedy keys launch");
}

AEXIS_API int aexis_cuda_topk_merge(aexis_ctx* ctx, const int32_t* gathered, int lists, int rows, int k,
                                    int shard_rows, int64_t* out_ids, float* out_vals, int32_t* out_idx) {
    if (!ctx) return AEXIS_E_NULL;
    if (!gathered || !out_ids || !out_vals || !out_idx) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    if (lists < 1 || lists > 8 || rows <= 0 || shard_rows <= 0)
        return aexis_fail(ctx, AEXIS_E_RANGE, "lists=%d (1..8) rows=%d shard_rows=%d", lists, rows, shard_rows);
    if (k < 1 || k > 64) return aexis_fail(ctx, AEXIS_E_RANGE, "k=%d (1..64)", k);
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_topk_shard_merge(gathered, lists, rows, k, shard_rows,
                                                         reinterpret_cast<long long*>(out_ids), out_vals, out_idx,
                                                         ctx->stream), "topk merge launch");
}

AEXIS_API int aexis_cuda_peer_buffer_bytes(int world, int rows, int k, size_t* out_bytes) {
    if (!out_bytes) return AEXIS_E_NULL;
    if (world < 1 || world > kPeerMaxRanks || rows <= 0 || k < 1 || k > 64) return AEXIS_E_RANGE;
    *out_bytes = peer_recv_bytes(world, rows, k);
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_peer_buffer_create(aexis_ctx* ctx, size_t bytes, void** out_ptr, uint8_t* out_handle) {
    if (!ctx) return AEXIS_E_NULL;
    if (!out_ptr || !out_handle) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    if (bytes < kPeerHeaderBytes) return aexis_fail(ctx, AEXIS_E_RANGE, "bytes=%zu", bytes);
    int rc = bind(ctx);
    if (rc) return rc;
    void* p = nullptr;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e == cudaSuccess) e = cudaMemset(p, 0, bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        if (p) cudaFree(p);
        return aexis_cuda_check(ctx, e, "peer buffer create");
    }
    std::memcpy(out_handle, &h, sizeof(h));
    *out_ptr = p;
    return AEXIS_OK;
}

AEXIS_API int aexis_cuda_peer_buffer_open(aexis_ctx* ctx, const uint8_t* handle, void** out_ptr) {
    if (!ctx) return AEXIS_E_NULL;
    if (!handle || !out_ptr) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    int rc = bind(ctx);
    if (rc) return rc;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    return aexis_cuda_check(ctx, cudaIpcOpenMemHandle(out_ptr, h, cudaIpcMemLazyEnablePeerAccess), "peer buffer open");
}

AEXIS_API int aexis_cuda_peer_buffer_close(aexis_ctx* ctx, void* ptr, int imported) {
    if (!ctx) return AEXIS_E_NULL;
    if (!ptr) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    int rc = bind(ctx);
    if (rc) return rc;
    cudaError_t e = cudaStreamSynchronize(ctx->stream);
    if (e == cudaSuccess) e = imported ? cudaIpcCloseMemHandle(ptr) : cudaFree(ptr);
    return aexis_cuda_check(ctx, e, "peer buffer close");
}

AEXIS_API int aexis_cuda_topk_push(aexis_ctx* ctx, const int32_t* packed, int rows, int k, void* const* peers,
                                   int world, int rank) {
    if (!ctx) return AEXIS_E_NULL;
    if (!packed || !peers) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    if (world < 1 || world > kPeerMaxRanks || rank < 0 || rank >= world || rows <= 0 || k < 1 || k > 64)
        return aexis_fail(ctx, AEXIS_E_RANGE, "world=%d rank=%d rows=%d k=%d", world, rank, rows, k);
    if (reinterpret_cast<uintptr_t>(packed) % 16)
        return aexis_fail(ctx, AEXIS_E_SHAPE, "packed must be 16-byte aligned");
    for (int p = 0; p < world; ++p)
        if (!peers[p] || reinterpret_cast<uintptr_t>(peers[p]) % 256)
            return aexis_fail(ctx, AEXIS_E_SHAPE, "peer buffer %d null or not 256-byte aligned", p);
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_topk_peer_push(packed, rows, k, peers, world, rank, ctx->stream),
                            "topk push launch");
}

AEXIS_API int aexis_cuda_topk_merge_peers(aexis_ctx* ctx, const void* recv, int world, int rows, int k,
                                          int shard_rows, int64_t* out_ids, float* out_vals, int32_t* out_idx) {
    if (!ctx) return AEXIS_E_NULL;
    if (!recv || !out_ids || !out_vals || !out_idx) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    if (world < 1 || world > kPeerMaxRanks || rows <= 0 || shard_rows <= 0 || k < 1 || k > 64)
        return aexis_fail(ctx, AEXIS_E_RANGE, "world=%d rows=%d shard_rows=%d k=%d", world, rows, shard_rows, k);
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_topk_peer_merge(recv, world, rows, k, shard_rows,
                                                        reinterpret_cast<long long*>(out_ids), out_vals, out_idx,
                                                        ctx->status, ctx->stream),
                            "topk peer merge launch");
}

AEXIS_API int aexis_cuda_embed(aexis_ctx* ctx, const int32_t* words, int count, const aexis_weights* table,
                               const float* bias, float* out) {
    if (!ctx) return AEXIS_E_NULL;
    if (!words || !table || !out) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    if (count <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "count=%d", count);
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_embed(words, count, table, bias, out, ctx->stream), "embed launch");
}

AEXIS_API int aexis_cuda_swish(aexis_ctx* ctx, const float* x, int count, float* y) {
    if (!ctx) return AEXIS_E_NULL;
    if (!x || !y) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    if (count <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "count=%d", count);
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_swish(x, count, y, ctx->stream), "swish launch");
}

AEXIS_API int aexis_cuda_swiglu(aexis_ctx* ctx, const float* gate, const float* up, int count, float* y) {
    if (!ctx) return AEXIS_E_NULL;
    if (!gate || !up || !y) return aexis_fail(ctx, AEXIS_E_NULL, "null pointer");
    if (count <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "count=%d", count);
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_swiglu(gate, up, count, y, ctx->stream), "swiglu launch");
}

// ------------------------------------------------------ linear-attention decode

AEXIS_API int aexis_cuda_short_conv(aexis_ctx* ctx, const float* weight, const float* mixed, const float* cache_in,
                                    float* out, float* cache_out, int groups, int kernel_size, int seq_len,
                                    int cache_len) {
    if (!ctx) return AEXIS_E_NULL;
    if (!weight || !mixed || !cache_in || !out || !cache_out)
        return aexis_fail(ctx, AEXIS_E_NULL, "ShortConv texture input/output is null.");
    if (groups <= 0 || kernel_size <= 0 || seq_len <= 0 || cache_len < kernel_size - 1)
        return aexis_fail(ctx, AEXIS_E_RANGE, "groups=%d kernel=%d seq=%d cache=%d", groups, kernel_size, seq_len,
                          cache_len);
    if (kernel_size > 16)
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "ShortConv kernel size %d > 16", kernel_size);
    if (out == mixed || out == cache_in || cache_out == mixed || out == cache_out)
        return aexis_fail(ctx, AEXIS_E_SHAPE, "ShortConv output aliases an input (only cache_out == cache_in is allowed)");
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_short_conv(weight, mixed, cache_in, out, cache_out, groups, kernel_size,
                                                   seq_len, cache_len, ctx->stream),
                            "short conv launch");
}

AEXIS_API int aexis_cuda_gated_delta_rule(aexis_ctx* ctx, const float* a_log, const float* dt_bias, const float* b,
                                          const float* a, const float* q, const float* k, const float* v,
                                          const float* state_in, float* out, float* state_out, int heads, int key_dim,
                                          int value_dim, int seq_len, int first_token, int token_count, float eps) {
    if (!ctx) return AEXIS_E_NULL;
    if (!a_log || !dt_bias || !b || !a || !q || !k || !v || !state_in || !out || !state_out)
        return aexis_fail(ctx, AEXIS_E_NULL, "GatedDeltaRule texture input/output is null.");
    if (heads <= 0 || key_dim <= 0 || value_dim <= 0 || seq_len <= 0)
        return aexis_fail(ctx, AEXIS_E_RANGE, "heads=%d keyDim=%d valueDim=%d seq=%d", heads, key_dim, value_dim,
                          seq_len);
    if (first_token < 0 || token_count <= 0 || first_token > seq_len - token_count)
        return aexis_fail(ctx, AEXIS_E_RANGE, "tokens [%d, %d) outside the sequence of %d", first_token,
                          first_token + token_count, seq_len);
    if (key_dim > gdr_max_kdim())
        return aexis_fail(ctx, AEXIS_E_UNSUPPORTED, "GatedDeltaRule key dim %d > %d", key_dim, gdr_max_kdim());
    if ((reinterpret_cast<uintptr_t>(state_in) | reinterpret_cast<uintptr_t>(state_out)) & 15)
        return aexis_fail(ctx, AEXIS_E_SHAPE, "GatedDeltaRule state buffers must be 16-byte aligned");
    if (out == q || out == k || out == v || out == state_out)
        return aexis_fail(ctx, AEXIS_E_SHAPE, "GatedDeltaRule output aliases an input");
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_gated_delta_rule(a_log, dt_bias, b, a, q, k, v, state_in, out, state_out,
                                                         heads, key_dim, value_dim, first_token, token_count, eps,
                                                         ctx->stream),
                            "gated delta rule launch");
}

// ------------------------------------------------------------------ sampler

AEXIS_API int aexis_cuda_sample(aexis_ctx* ctx, const float* logits, int rows, int width, int ld,
                                const uint32_t* history, float repetition_penalty, float temperature, int top_k,
                                float top_p, const double* uniforms, int32_t* out_idx) {
    if (!ctx) return AEXIS_E_NULL;
    if (!logits || !out_idx) return aexis_fail(ctx, AEXIS_E_NULL, "logits or output is null");
    if (rows <= 0 || width <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "rows=%d width=%d", rows, width);
    if (ld < width) return aexis_fail(ctx, AEXIS_E_SHAPE, "LM head logits do not cover the tokenizer vocabulary.");
    if (!(repetition_penalty > 0.0f) || !std::isfinite(repetition_penalty))
        return aexis_fail(ctx, AEXIS_E_RANGE, "repetition penalty %g", (double)repetition_penalty);
    if (!std::isfinite(temperature) || !std::isfinite(top_p))
        return aexis_fail(ctx, AEXIS_E_RANGE, "temperature %g top_p %g", (double)temperature, (double)top_p);
    const bool sample = temperature > 0.0f;
    if (sample && !uniforms) return aexis_fail(ctx, AEXIS_E_NULL, "uniform draws are null");
    int rc = bind(ctx);
    if (rc) return rc;
    const bool penalised = history != nullptr && repetition_penalty != 1.0f;
    const bool full = sample && (top_k <= 0 || top_k > 64);
    const size_t need = sample_scratch_bytes(rows, width, ctx->sm_count, penalised, full);
    if (need > ctx->samp_bytes) {
        if (ctx->samp) {
            cudaStreamSynchronize(ctx->stream);
            cudaFree(ctx->samp);
            ctx->samp = nullptr;
            ctx->samp_bytes = 0;
        }
        rc = aexis_cuda_check(ctx, cudaMalloc(&ctx->samp, need), "sampler scratch");
        if (rc) return rc;
        ctx->samp_bytes = need;
    }
    void* tk = nullptr;
    if (sample && top_k >= 1 && top_k <= 64) {
        rc = aexis_scratch(ctx, topk_scratch_bytes(rows, width, top_k < width ? top_k : width, ctx->sm_count), &tk);
        if (rc) return rc;
    }
    return aexis_cuda_check(ctx, launch_sample(logits, rows, width, ld, history, repetition_penalty, temperature,
                                               top_k, top_p, uniforms, out_idx, ctx->samp, tk, ctx->sm_count,
                                               ctx->stream),
                            "sample launch");
}

AEXIS_API int aexis_cuda_sample_history_add(aexis_ctx* ctx, uint32_t* history, int rows, int width,
                                            const int32_t* tokens) {
    if (!ctx) return AEXIS_E_NULL;
    if (!history || !tokens) return aexis_fail(ctx, AEXIS_E_NULL, "history or tokens is null");
    if (rows <= 0 || width <= 0) return aexis_fail(ctx, AEXIS_E_RANGE, "rows=%d width=%d", rows, width);
    int rc = bind(ctx);
    if (rc) return rc;
    return aexis_cuda_check(ctx, launch_history_add(history, rows, width, tokens, ctx->stream), "history launch");
}
