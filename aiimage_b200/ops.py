"""Host-side mirror of the reference's AexisOps operator surface for the
quantized-decoder hot path, over the libaexis_cuda C ABI.

Method names follow Packages/com.aexis/Runtime/Execution/Graph/AexisOps.cs in
snake_case, with the same argument meaning and the same error classes
(aiimage_b200.errors). Tensors are torch CUDA tensors used only as device
memory; every computation runs in libaexis_cuda's kernels on the tensor's
device. Work is enqueued on torch's current stream.
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import errors
from .native import F16, F32, check, lib


def _ptr(t):
    # A plain int: every pointer parameter is declared c_void_p, and ctypes converts ints itself.
    return None if t is None else t.data_ptr()


_DTYPES = None          # {torch dtype: ABI dtype code}, filled on first use
_raw_stream = None      # device index -> raw cudaStream_t of torch's current stream


def _torch_hooks():
    """Looks up, once, what every call needs from torch: the dtype codes and a raw current-stream getter
    (torch's internal one when present: a few hundred nanoseconds instead of a Stream object per call)."""
    global _DTYPES, _raw_stream
    import torch
    _DTYPES = {torch.float32: F32, torch.float16: F16}
    raw = getattr(torch._C, "_cuda_getCurrentRawStream", None)
    _raw_stream = raw if raw is not None else (lambda dev: torch.cuda.current_stream(dev).cuda_stream)


def _dtype_code(t) -> int:
    if _DTYPES is None:
        _torch_hooks()
    code = _DTYPES.get(t.dtype)
    if code is None:
        raise errors.NotSupportedError(f"dtype {t.dtype} (float32 or float16)")
    return code


def _np_ptr(a: np.ndarray):
    return a.ctypes.data_as(C.c_void_p)


class Weights:
    """An uploaded weight (InnerProductPack / Int{4,8}WeightOnlyUpload)."""

    def __init__(self, ops: "AexisOps", handle, kind: str, n: int, k: int, group: int = 0):
        self._ops, self.handle, self.kind, self.n, self.k, self.group = ops, handle, kind, n, k, group

    def free(self):
        if self.handle:
            lib().aexis_cuda_weights_free(self._ops.ctx, self.handle)
            self.handle = None

    def __del__(self):
        try:
            if self._ops.ctx:
                self.free()
        except Exception:
            pass


def quantize_rows(bits: int, data: np.ndarray, out_ch: int, per_ch: int, contiguous: bool = True):
    """AexisGraphSession.NewInt{8,4}WeightOnlyUpload(float[], ...) host quantizer
    (AexisGraphSession.cs:12834-12964): returns (packed uint32, scales fp32)."""
    d = np.ascontiguousarray(data, dtype=np.float32).reshape(-1)
    if d.size != out_ch * per_ch:
        raise errors.ArgumentError("weight layout must contain exactly outputChannels * valuesPerOutputChannel values")
    per_word = 8 if bits == 4 else 4
    packed = np.zeros(max(1, (d.size + per_word - 1) // per_word), dtype=np.uint32)
    scales = np.zeros(out_ch, dtype=np.float32)
    fn = lib().aexis_quantize_q4_rows if bits == 4 else lib().aexis_quantize_q8_rows
    check(fn(_np_ptr(d), out_ch, per_ch, int(contiguous), _np_ptr(packed), _np_ptr(scales)))
    return packed, scales


class AexisOps:
    """One libaexis_cuda context on one GPU (new AexisOps(), AexisOps.cs)."""

    def __init__(self, device: int = 0, use_torch_stream: bool = True):
        self.ctx = C.c_void_p()
        self.device = device
        st = lib().aexis_cuda_create(device, C.byref(self.ctx))
        if st != 0:
            msg = lib().aexis_cuda_last_error(None)
            raise errors.BY_STATUS.get(st, errors.AexisError)(msg.decode() if msg else "create failed")
        self._use_torch_stream = use_torch_stream
        self._bound_stream = None
        self._int8 = None
        self._int4 = None
        self._children = weakref.WeakSet()

    # -- context ---------------------------------------------------------
    def _register(self, child):
        """Objects owning device state of this context (closed before it)."""
        self._children.add(child)

    def close(self):
        if self.ctx:
            for child in list(self._children):
                child.close()
            lib().aexis_cuda_destroy(self.ctx)
            self.ctx = C.c_void_p()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _bind_stream(self):
        if self._use_torch_stream:
            if _raw_stream is None:
                _torch_hooks()
            s = _raw_stream(self.device)
            if s != self._bound_stream:
                lib().aexis_cuda_set_stream(self.ctx, C.c_void_p(s))
                self._bound_stream = s

    def _call(self, fn, *args):
        self._bind_stream()
        check(fn(self.ctx, *args), self.ctx)

    def sync(self):
        check(lib().aexis_cuda_sync(self.ctx), self.ctx)

    def selftest_wait(self, limit_cycles: int):
        """Enqueue one bounded wait on a flag nothing sets (aexis_cuda_selftest_wait):
        the next sync raises DeviceTimeoutError and the context stays usable."""
        self._bind_stream()
        check(lib().aexis_cuda_selftest_wait(self.ctx, int(limit_cycles)), self.ctx)

    # -- weights ----------------------------------------------------------
    def new_int8_weight_only_upload(self, packed: np.ndarray, scales: np.ndarray, n: int, k: int) -> Weights:
        """AexisGraphSession.NewInt8WeightOnlyUpload(AexisQuantizedTensor, n) (:12887-12910)."""
        p = np.ascontiguousarray(packed, dtype=np.uint32)
        s = np.ascontiguousarray(scales)
        sd = F16 if s.dtype == np.float16 else F32
        s = s.astype(np.float16 if sd == F16 else np.float32, copy=False)
        if s.size != n:
            raise errors.ArgumentError("Direct Q8 upload must contain one scale per output channel.")
        if p.size != max(1, (n * k + 3) // 4):
            raise errors.ArgumentError("Direct Q8 packed payload size mismatch.")
        h = C.c_void_p()
        check(lib().aexis_cuda_weights_q8(self.ctx, _np_ptr(p), _np_ptr(s), sd, n, k, C.byref(h)), self.ctx)
        return Weights(self, h, "q8", n, k)

    def new_int4_weight_only_upload(self, packed: np.ndarray, scales: np.ndarray, n: int, k: int,
                                    group: int) -> Weights:
        """AexisGraphSession.NewInt4WeightOnlyUpload(AexisQuantizedTensor, n, k) (:12966-12998)."""
        p = np.ascontiguousarray(packed, dtype=np.uint32)
        s = np.ascontiguousarray(scales)
        sd = F16 if s.dtype == np.float16 else F32
        s = s.astype(np.float16 if sd == F16 else np.float32, copy=False)
        if group <= 0 or k % group != 0:
            raise errors.ArgumentError("Direct Q4 group size must divide the Gemm K dimension.")
        if s.size != n * k // group:
            raise errors.ArgumentError("Direct Q4 upload scale count does not match its group size.")
        if p.size != max(1, (n * k + 7) // 8):
            raise errors.ArgumentError("Direct Q4 packed payload size mismatch.")
        h = C.c_void_p()
        check(lib().aexis_cuda_weights_q4(self.ctx, _np_ptr(p), _np_ptr(s), sd, n, k, group, C.byref(h)), self.ctx)
        return Weights(self, h, "q4", n, k, group)

    def new_dense_weights(self, data: np.ndarray) -> Weights:
        a = np.ascontiguousarray(data)
        dt = F16 if a.dtype == np.float16 else F32
        a = a.astype(np.float16 if dt == F16 else np.float32, copy=False)
        n, k = a.shape
        h = C.c_void_p()
        check(lib().aexis_cuda_weights_dense(self.ctx, _np_ptr(a), dt, n, k, C.byref(h)), self.ctx)
        return Weights(self, h, "f16" if dt == F16 else "f32", n, k)

    def set_int8_gemm_weights(self, w: Weights | None):
        """AexisOps.SetInt8GemmWeights (:706-712)."""
        self._int8 = w

    def set_int4_gemm_weights(self, w: Weights | None):
        """AexisOps.SetInt4GemmWeights (:730-739)."""
        self._int4 = w

    def set_int8_activation_quantization(self, plan):
        """AexisOps.SetInt8ActivationQuantization (:741-785). `plan` is None (plain activations), a
        QuantizedNodePlan-like object (mode "Int8W8A8", activation_scale, activation_zero_point) or a
        QuantizedActivationPlan-like object (packing "Pack4UnsignedInt8" or signed, calibration minimum /
        maximum), resolved as the reference resolves it (resolve_int8_activation_plan)."""
        if plan is None:
            self._call(lib().aexis_cuda_set_int8_activations, 0, 1.0, 0, 0)
            return
        if hasattr(plan, "activation_scale"):
            if getattr(plan, "mode", "Int8W8A8") != "Int8W8A8":
                self._call(lib().aexis_cuda_set_int8_activations, 0, 1.0, 0, 0)
                return
            scale, zp, uns = float(plan.activation_scale), int(plan.activation_zero_point), False
        else:
            scale, zp, uns = resolve_int8_activation_plan(plan.minimum, plan.maximum,
                                                          plan.packing == "Pack4UnsignedInt8")
        self._call(lib().aexis_cuda_set_int8_activations, 1, scale, zp, int(uns))

    def dequant(self, w: Weights, out):
        self._call(lib().aexis_cuda_weights_dequant, w.handle, _ptr(out))

    # -- linear -----------------------------------------------------------
    def _gemm_weights(self, a, c, trans_b, use_c, broadcast_type_c, output):
        if a is None:
            raise errors.ArgumentNullError("a")
        if output is None:
            raise errors.ArgumentNullError("output")
        if use_c and c is None:
            raise errors.ArgumentNullError("c")
        w = self._int4 or self._int8
        if w is None:
            raise errors.NotSupportedError("only INT4/INT8 weight-only Gemm weights are implemented by this backend")
        if not trans_b:
            raise errors.NotSupportedError("quantized Gemm weights are stored transB (output-channel major)")
        if use_c and broadcast_type_c != 4:
            raise errors.NotSupportedError("bias broadcast type 4 (per output column) only")
        return w

    def _gemm(self, fn, a, c, m, n, k, trans_b, alpha, beta, use_c, broadcast_type_c, output, lda=None):
        w = self._gemm_weights(a, c, trans_b, use_c, broadcast_type_c, output)
        if lda is None:
            lda = a.stride(0) if a.dim() == 2 else k
        ldy = output.stride(0) if output.dim() == 2 else n
        self._call(fn, _ptr(a), _dtype_code(a), lda, m, k, w.handle, _ptr(c) if use_c else None, alpha, beta,
                   _ptr(output), _dtype_code(output), ldy, n)

    def gemm2d_pack4_linear_texture_a(self, a, c, m, n, k, trans_b=True, alpha=1.0, beta=1.0, use_c=False,
                                      broadcast_type_c=4, output=None, input_packed=False, a_width=None,
                                      a_height=None, a_slices=1):
        """AexisOps.Gemm2DPack4LinearTextureA(a, inputPacked, ...) (:3649-3683).

        input_packed=False: `a` is the linear [m, k] texture (row stride = its stride(0)).
        input_packed=True: `a` is a Pack4 texture array of a_width texels x a_height rows x a_slices
        slices stored flat ([slices][height][width][4], the CDHW layout); its K values run along the
        texels of a row and continue in the next slice (AexisGemm2DPack4LinearTextureAFromPack4)."""
        if not input_packed:
            self._gemm(lib().aexis_cuda_gemm, a, c, m, n, k, trans_b, alpha, beta, use_c, broadcast_type_c, output)
            return
        w = self._gemm_weights(a, c, trans_b, use_c, broadcast_type_c, output)
        if a_width is None:
            raise errors.ArgumentNullError("a_width (texels per row of the packed input)")
        a_height = m if a_height is None else a_height
        ldy = output.stride(0) if output.dim() == 2 else n
        self._call(lib().aexis_cuda_gemm_pack4a, _ptr(a), _dtype_code(a), int(a_width), int(a_height),
                   int(a_slices), m, k, w.handle, _ptr(c) if use_c else None, alpha, beta, _ptr(output),
                   _dtype_code(output), ldy, n)

    def gemm2d_pack4_tiled_texture_a(self, a, c, m, n, k, trans_b=True, alpha=1.0, beta=1.0, use_c=False,
                                     broadcast_type_c=4, output=None):
        """AexisOps.Gemm2DPack4TiledTextureAFromLinear (:3722-3752); output row stride = its tiled width."""
        self._gemm(lib().aexis_cuda_gemm_tiled, a, c, m, n, k, trans_b, alpha, beta, use_c, broadcast_type_c,
                   output)

    def gemm2d_pack4_tiled_texture_a_from_pack4(self, a, c, m, n, k, trans_b=True, alpha=1.0, beta=1.0,
                                                use_c=False, broadcast_type_c=4, output=None, a_width=None):
        """AexisOps.Gemm2DPack4TiledTextureAFromPack4 (:3782-3826). The kernel reads slice 0 of the Pack4
        input only (AexisGemm2DPack4TiledTextureAFromPack4_Impl, HLSL Pack4Matmul:2275-2300), so each row
        is a run of a_width texels: the linear form with a row stride of 4 * a_width
        (a_width defaults to ceil(k / 4), the width the reference sets)."""
        a_width = (k + 3) // 4 if a_width is None else int(a_width)
        if 4 * a_width < k:
            raise errors.ArgumentError("a packed row of a_width texels holds fewer than k values")
        self._gemm(lib().aexis_cuda_gemm_tiled, a, c, m, n, k, trans_b, alpha, beta, use_c, broadcast_type_c,
                   output, lda=4 * a_width)

    # -- pointwise --------------------------------------------------------
    def rms_norm_pack4_linear_mat(self, x, rows, width, gamma, affine_size, affine, eps, output):
        """AexisOps.RmsNormPack4LinearMat (:8267-8283)."""
        if x is None:
            raise errors.ArgumentNullError("input")
        if output is None:
            raise errors.ArgumentNullError("output")
        ld = x.stride(0) if x.dim() == 2 else width
        g = gamma if affine else None
        self._call(lib().aexis_cuda_rmsnorm, _ptr(x), _dtype_code(x), rows, width, ld, _ptr(g),
                   affine_size if affine else 0, eps, _ptr(output), _dtype_code(output))

    def rotary_embed_pack4(self, x, embed_dim, seq_len, num_heads, cos, sin, interleaved, output):
        """AexisOps.RotaryEmbedPack4 (:8514-8540); Pack4 CDHW fp32."""
        self._call(lib().aexis_cuda_rope, _ptr(x), embed_dim, seq_len, num_heads, _ptr(cos), _ptr(sin),
                   int(interleaved), _ptr(output))

    def append_sequence_pack4_cdhw(self, current, destination_offset, current_height, cache, width, slices,
                                   cache_rows):
        """AexisOps.AppendSequencePack4Cdhw (:6384-6400)."""
        self._call(lib().aexis_cuda_kv_append, _ptr(current), width, current_height, slices, destination_offset,
                   _ptr(cache), cache_rows)

    def concat_sequence_pack4_cdhw(self, a, b, a_height, b_height, output, width, slices, out_rows):
        """AexisOps.ConcatSequencePack4Cdhw (:6336-6360)."""
        self._call(lib().aexis_cuda_kv_concat, _ptr(a), a_height, _ptr(b), b_height, width, slices, _ptr(output),
                   out_rows)

    def sdpa_attention_pack4_cdhw(self, q, k, v, src_len, dst_len, embed_dim, out_embed_dim, num_heads,
                                  num_groups, scale, output, mask=None, mask_w=0, mask_h=0, causal=False,
                                  causal_query_offset=0):
        """AexisOps.SdpaAttentionPack4Cdhw (:10147-10200)."""
        self._call(lib().aexis_cuda_sdpa, _ptr(q), _ptr(k), _ptr(v), src_len, dst_len, embed_dim, out_embed_dim,
                   num_heads, num_groups, scale, _ptr(mask), mask_w, mask_h, int(causal), causal_query_offset,
                   _ptr(output))

    def arg_max_pack4_linear_mat(self, logits, logical_width, logical_height, output, ld=None):
        """AexisOps.ArgMaxPack4LinearMat (:9982-10003); output int32 [rows]."""
        ld = ld if ld is not None else (logits.stride(0) if logits.dim() == 2 else logical_width)
        self._call(lib().aexis_cuda_argmax, _ptr(logits), logical_height, logical_width, ld, _ptr(output))

    def argmax_keys(self, logits, width, rows, index_offset, keys, ld=None):
        """Per-row 64-bit argmax keys of one vocabulary shard (global indices)."""
        ld = ld if ld is not None else (logits.stride(0) if logits.dim() == 2 else width)
        self._call(lib().aexis_cuda_argmax_keys, _ptr(logits), rows, width, ld, index_offset, _ptr(keys))

    def top_k(self, logits, width, rows, k, out_vals, out_idx, ld=None):
        ld = ld if ld is not None else (logits.stride(0) if logits.dim() == 2 else width)
        self._call(lib().aexis_cuda_topk, _ptr(logits), rows, width, ld, k, _ptr(out_vals), _ptr(out_idx))

    def gemm_topk(self, a, m, k, top_k, out_vals, out_idx, keys=None, alpha=1.0, index_offset=0):
        """The bound Q8/Q4 weights' tiled lm_head (no bias) and the top-k of its logits per row, without
        writing the logits (aexis_cuda_gemm_topk): out_vals/out_idx [m, top_k], optional greedy keys [m]
        (int64 view of the uint64 keys) with global indices (index_offset added)."""
        if a is None:
            raise errors.ArgumentNullError("a")
        w = self._int4 or self._int8
        if w is None:
            raise errors.NotSupportedError("only INT4/INT8 weight-only Gemm weights are implemented by this backend")
        lda = a.stride(0) if a.dim() == 2 else k
        self._call(lib().aexis_cuda_gemm_topk, _ptr(a), _dtype_code(a), lda, m, k, w.handle, float(alpha), int(top_k),
                   int(index_offset), _ptr(out_vals), _ptr(out_idx), _ptr(keys))

    def topk_greedy_keys(self, logits, width, rows, k, top_vals, top_idx, index_offset, keys, ld=None):
        """The shard's argmax keys (as argmax_keys) from its top-k lists, without re-reading the logits."""
        ld = ld if ld is not None else (logits.stride(0) if logits.dim() == 2 else width)
        self._call(lib().aexis_cuda_topk_greedy_keys, _ptr(logits), rows, width, ld, k, _ptr(top_vals), _ptr(top_idx),
                   index_offset, _ptr(keys))

    def topk_merge(self, gathered, lists, rows, k, shard_rows, out_ids, out_vals, out_idx):
        """Merge of vocab shards' packed greedy keys and top-k lists (see
        aexis_cuda_topk_merge)."""
        self._call(lib().aexis_cuda_topk_merge, _ptr(gathered), lists, rows, k, shard_rows, _ptr(out_ids),
                   _ptr(out_vals), _ptr(out_idx))

    # ---- the sharded lm_head's exchange over peer memory (aexis_cuda_peer_*)
    @staticmethod
    def peer_buffer_bytes(world, rows, k) -> int:
        out = C.c_size_t(0)
        check(lib().aexis_cuda_peer_buffer_bytes(world, rows, k, C.byref(out)), None)
        return out.value

    def peer_buffer_create(self, nbytes):
        """A zeroed receive buffer of this device: (device pointer, 64-byte IPC handle)."""
        ptr = C.c_void_p()
        handle = (C.c_uint8 * 64)()
        self._call(lib().aexis_cuda_peer_buffer_create, nbytes, C.byref(ptr), handle)
        return ptr.value, bytes(handle)

    def peer_buffer_open(self, handle: bytes) -> int:
        """Another rank's receive buffer mapped into this process."""
        ptr = C.c_void_p()
        self._call(lib().aexis_cuda_peer_buffer_open, (C.c_uint8 * 64).from_buffer_copy(handle), C.byref(ptr))
        return ptr.value

    def peer_buffer_close(self, ptr: int, imported: bool):
        self._call(lib().aexis_cuda_peer_buffer_close, ptr, int(imported))

    def topk_push(self, packed, rows, k, peers, rank):
        arr = (C.c_void_p * len(peers))(*peers)
        self._call(lib().aexis_cuda_topk_push, _ptr(packed), rows, k, arr, len(peers), rank)

    def topk_merge_peers(self, recv, world, rows, k, shard_rows, out_ids, out_vals, out_idx):
        self._call(lib().aexis_cuda_topk_merge_peers, recv, world, rows, k, shard_rows, _ptr(out_ids),
                   _ptr(out_vals), _ptr(out_idx))

    def embed_texture(self, words, count, table: Weights, bias, output):
        """AexisOps.EmbedTexture (:10764-10810)."""
        self._call(lib().aexis_cuda_embed, _ptr(words), count, table.handle, _ptr(bias), _ptr(output))

    def swish(self, x, count, y):
        self._call(lib().aexis_cuda_swish, _ptr(x), count, _ptr(y))

    def swiglu(self, gate, up, count, y):
        self._call(lib().aexis_cuda_swiglu, _ptr(gate), _ptr(up), count, _ptr(y))

    # -- sampling (Qwen35Sampler.Select on the device) -------------------------
    def sample(self, logits, rows, width, history, repetition_penalty, temperature, top_k, top_p, uniforms,
               output, ld=None):
        """Qwen35Sampler.Select (Qwen35DecoderSession.cs:1847-1892) for `rows` logit rows: penalty on the history
        bitmap, temperature softmax, top-k, top-p, one draw per row from `uniforms` (fp64 [rows], the NextDouble
        values). temperature <= 0 is the greedy ArgMax. output: int32 [rows]."""
        ld = ld if ld is not None else (logits.stride(0) if logits.dim() == 2 else width)
        self._call(lib().aexis_cuda_sample, _ptr(logits), rows, width, ld, _ptr(history), float(repetition_penalty),
                   float(temperature), int(top_k), float(top_p), _ptr(uniforms), _ptr(output))

    def sample_history_add(self, history, rows, width, tokens):
        """Qwen35Sampler.AddHistory (:1840-1844) on the device bitmap: sets bit tokens[r] of row r (ids outside
        [0, width) are ignored)."""
        self._call(lib().aexis_cuda_sample_history_add, _ptr(history), rows, width, _ptr(tokens))

    # -- linear-attention blocks (Qwen3.5 ShortConv + GatedDeltaRule) ---------
    def short_conv_pack4(self, weight, mixed, cache_in, output, cache_out, groups, kernel_size, sequence_length,
                         cache_length):
        """AexisOps.ShortConvPack4 (:12593-12618). weight: Pack4 CDHW [kernel, 1, groups]; mixed/output
        [seq, ceil(groups/4)*4]; caches [cache_length, ceil(groups/4)*4]; cache_out may be cache_in."""
        self._call(lib().aexis_cuda_short_conv, _ptr(weight), _ptr(mixed), _ptr(cache_in), _ptr(output),
                   _ptr(cache_out), groups, kernel_size, sequence_length, cache_length)

    def gated_delta_rule_pack4(self, a_log, dt_bias, b, a, query, key, value, state_in, output, state_out, heads,
                               key_dim, value_dim, sequence_length, token_index=0, token_count=None,
                               epsilon=1e-6):
        """AexisOps.GatedDeltaRulePack4 (:12620-12657) for tokens token_index .. token_index+token_count-1
        (default: the rest of the sequence, the whole per-token loop of AexisGatedDeltaRuleLayer in one
        call). q/k/v/output: Pack4 CDHW [dim, heads, seq]; state: [heads, key_dim, ceil(value_dim/4)*4]."""
        if token_count is None:
            token_count = sequence_length - token_index
        self._call(lib().aexis_cuda_gated_delta_rule, _ptr(a_log), _ptr(dt_bias), _ptr(b), _ptr(a), _ptr(query),
                   _ptr(key), _ptr(value), _ptr(state_in), _ptr(output), _ptr(state_out), heads, key_dim,
                   value_dim, sequence_length, token_index, token_count, float(epsilon))


def resolve_int8_activation_plan(minimum: float, maximum: float, unsigned: bool):
    """(scale, zero_point, unsigned) of a calibrated activation plan, as AexisOps.SetInt8ActivationQuantization
    (QuantizedActivationPlan) computes them (AexisOps.cs:763-785; ActivationCalibrationRange.SymmetricScale,
    Core/AexisPrecisionContracts.cs:30-37): unsigned packing -> scale = (max - min)/255 (1 if empty) and
    zero_point = clamp(RoundToInt(-min/scale), 0, 255); signed -> scale = max(|min|, |max|)/127 (1 if 0),
    zero_point 0. Bounds must be finite and ordered (InferenceContractException otherwise)."""
    lo, hi = np.float32(minimum), np.float32(maximum)
    if not (np.isfinite(lo) and np.isfinite(hi)) or lo > hi:
        raise errors.InvalidOperationError("Activation calibration range must contain finite ordered bounds.")
    if unsigned:
        rng = np.float32(hi - lo)
        scale = np.float32(rng / np.float32(255.0)) if rng > 0 else np.float32(1.0)
        zp = int(min(max(int(np.rint(np.float32(-lo) / scale)), 0), 255))
        return float(scale), zp, True
    mag = max(abs(lo), abs(hi))
    return float(np.float32(mag / np.float32(127.0)) if mag != 0 else np.float32(1.0)), 0, False


def pack4_cdhw(x: np.ndarray) -> np.ndarray:
    """Logical [c, h, w] (ncnn d3: c=channels or sequence, h, w) -> flat Pack4 CDHW storage, element (x, y, c)
    at ((c/4*H + y)*W + x)*4 + (c & 3); lanes past c are zero."""
    x = np.asarray(x, dtype=np.float32)
    c, h, w = x.shape
    c4 = (c + 3) // 4 * 4
    pad = np.zeros((c4, h, w), dtype=np.float32)
    pad[:c] = x
    return np.ascontiguousarray(pad.reshape(c4 // 4, 4, h, w).transpose(0, 2, 3, 1)).reshape(-1)


def unpack4_cdhw(flat: np.ndarray, c: int, h: int, w: int) -> np.ndarray:
    """Inverse of pack4_cdhw: flat Pack4 CDHW storage -> logical [c, h, w]."""
    c4 = (c + 3) // 4 * 4
    x = np.asarray(flat, dtype=np.float32).reshape(c4 // 4, h, w, 4).transpose(0, 3, 1, 2).reshape(c4, h, w)
    return np.ascontiguousarray(x[:c])


def pack4_rows(x: np.ndarray) -> np.ndarray:
    """Logical [rows, width] -> Pack4 linear [rows, ceil(width/4)*4] (zero padded)."""
    x = np.asarray(x, dtype=np.float32)
    rows, width = x.shape
    out = np.zeros((rows, (width + 3) // 4 * 4), dtype=np.float32)
    out[:, :width] = x
    return out
