"""ctypes wrapper for the CPU parity oracle (oracle/aexis_oracle.cpp).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and the
cpu_baseline / ``--impl reference`` legs of bench.py, never by the product
package. Every function takes and returns numpy arrays; fp16 inputs are widened
to fp32 exactly before they reach the C code (the reference computes in fp32).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libaexis_oracle.so")
_lib = None

F32P = np.ctypeslib.ndpointer(dtype=np.float32, flags="C_CONTIGUOUS")
U32P = np.ctypeslib.ndpointer(dtype=np.uint32, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(dtype=np.int32, flags="C_CONTIGUOUS")
U16P = np.ctypeslib.ndpointer(dtype=np.uint16, flags="C_CONTIGUOUS")


def build(force: bool = False) -> str:
    """Compile the oracle with its Makefile (g++ on this host) if needed."""
    src = os.path.join(_HERE, "aexis_oracle.cpp")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        L = C.CDLL(_LIB_PATH)
        vp = C.c_void_p
        L.oracle_quantize_rows.argtypes = [C.c_int, F32P, C.c_int, C.c_int, C.c_int, U32P, F32P]
        L.oracle_dequant.argtypes = [C.c_int, U32P, F32P, C.c_int, C.c_int, C.c_int, F32P]
        for name in ("oracle_gemm", "oracle_gemm_tiled"):
            getattr(L, name).argtypes = [F32P, C.c_int, C.c_int, C.c_int, C.c_int, U32P, F32P,
                                         C.c_int, C.c_int, vp, C.c_float, C.c_float, F32P, C.c_int]
        L.oracle_read_pack4a.argtypes = [F32P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, F32P]
        L.oracle_quantize_activation_int8.argtypes = [F32P, C.c_int, C.c_float, C.c_int, C.c_int, F32P]
        L.oracle_rmsnorm.argtypes = [F32P, C.c_int, C.c_int, C.c_int, vp, C.c_int, C.c_float, F32P, C.c_int]
        L.oracle_rope.argtypes = [F32P, C.c_int, C.c_int, C.c_int, F32P, F32P, C.c_int, F32P]
        L.oracle_append_sequence.argtypes = [F32P, C.c_int, C.c_int, C.c_int, C.c_int, F32P, C.c_int]
        L.oracle_concat_sequence.argtypes = [F32P, C.c_int, F32P, C.c_int, C.c_int, C.c_int, F32P, C.c_int]
        L.oracle_sdpa.argtypes = [F32P, F32P, F32P, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_float, vp, C.c_int, C.c_int, C.c_int, C.c_int, F32P]
        L.oracle_argmax.argtypes = [F32P, C.c_int, C.c_int, C.c_int, I32P]
        L.oracle_topk.argtypes = [F32P, C.c_int, C.c_int, C.c_int, C.c_int, F32P, I32P]
        L.oracle_embed.argtypes = [I32P, C.c_int, C.c_int, vp, vp, C.c_int, vp, C.c_int, C.c_int, vp, F32P]
        L.oracle_swish.argtypes = [F32P, C.c_int, F32P]
        L.oracle_swiglu.argtypes = [F32P, F32P, C.c_int, F32P]
        L.oracle_sample.argtypes = [F32P, C.c_int, C.c_int, C.c_int, vp, C.c_float, C.c_float, C.c_int, C.c_float,
                                    np.ctypeslib.ndpointer(dtype=np.float64, flags="C_CONTIGUOUS"), I32P, vp]
        L.oracle_short_conv.argtypes = [F32P, F32P, F32P, F32P, F32P, C.c_int, C.c_int, C.c_int, C.c_int]
        L.oracle_gated_delta_rule.argtypes = [F32P] * 10 + [C.c_int] * 5 + [C.c_float]
        L.oracle_round_f16.argtypes = [C.c_float]
        L.oracle_round_f16.restype = C.c_float
        L.oracle_f32_to_f16.argtypes = [F32P, C.c_int64, U16P]
        L.oracle_rope_tables.argtypes = [C.c_int, C.c_int, C.c_float, F32P, F32P]
        L.oracle_decoder_create.argtypes = [vp]
        L.oracle_decoder_create.restype = vp
        L.oracle_decoder_destroy.argtypes = [vp]
        L.oracle_decoder_reset.argtypes = [vp]
        L.oracle_decoder_position.argtypes = [vp]
        L.oracle_decoder_set_linear.argtypes = [vp, C.c_int, C.c_int, U32P, F32P]
        L.oracle_decoder_set_norm.argtypes = [vp, C.c_int, C.c_int, F32P]
        L.oracle_decoder_set_embedding.argtypes = [vp, F32P]
        L.oracle_decoder_step.argtypes = [vp, C.c_int, C.c_int, vp, vp]
        L.oracle_decoder_fill_context.argtypes = [vp, C.c_int, C.c_uint64, C.c_int64]
        L.oracle_decoder_kv.argtypes = [vp, C.c_int, C.c_int, F32P]
        L.oracle_decoder_set_linear_attention.argtypes = [vp, C.c_int, F32P, F32P, F32P, F32P]
        L.oracle_decoder_recurrent.argtypes = [vp, C.c_int, vp, vp]
        L.oracle_decoder_fill_context.restype = C.c_int
        L.oracle_num_threads.restype = C.c_int
        _lib = L
    return _lib


def _f32(x) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(x), dtype=np.float32)


def _ptr(x):
    return None if x is None else x.ctypes.data_as(C.c_void_p)


def num_threads() -> int:
    return int(lib().oracle_num_threads())


# ---------------------------------------------------------------- weights
def quantize_rows(bits: int, data, out_ch: int, per_ch: int, contiguous: bool = True):
    """NewInt{8,4}WeightOnlyUpload(float[]): returns (packed uint32, scales fp32)."""
    d = _f32(data).reshape(-1)
    per_word = 8 if bits == 4 else 4
    packed = np.zeros(max(1, (d.size + per_word - 1) // per_word), dtype=np.uint32)
    scales = np.zeros(out_ch, dtype=np.float32)
    lib().oracle_quantize_rows(bits, d, out_ch, per_ch, int(contiguous), packed, scales)
    return packed, scales


def dequant(bits: int, packed, scales, blk: int, n: int, k: int) -> np.ndarray:
    out = np.empty(n * k, dtype=np.float32)
    lib().oracle_dequant(bits, np.ascontiguousarray(packed, dtype=np.uint32), _f32(scales), blk, n, k, out)
    return out.reshape(n, k)


def gemm(a, bits: int, packed, scales, blk: int, n: int, bias=None, alpha: float = 1.0,
         beta: float = 1.0, tiled: bool = False) -> np.ndarray:
    """y[m, n] per AexisGemm2DPack4Linear (tiled=False) or Pack4Tiled (tiled=True)."""
    a = _f32(a)
    if a.ndim == 1:
        a = a.reshape(1, -1)
    m, k = a.shape
    y = np.empty((m, n), dtype=np.float32)
    b = None if bias is None else _f32(bias)
    fn = lib().oracle_gemm_tiled if tiled else lib().oracle_gemm
    fn(a, k, m, k, bits, np.ascontiguousarray(packed, dtype=np.uint32), _f32(scales), blk, n,
       _ptr(b), alpha, beta, y, n)
    return y


def read_pack4a(a_flat, width: int, height: int, slices: int, m: int, k: int) -> np.ndarray:
    """The row-major [m, k] A that AexisGemm2DPack4LinearTextureAFromPack4 reads from a flat Pack4 texture
    array [slices][height][width][4] (see oracle_read_pack4a)."""
    a = _f32(a_flat).reshape(-1)
    assert a.size >= slices * height * width * 4
    out = np.empty((m, k), dtype=np.float32)
    lib().oracle_read_pack4a(a, width, height, slices, m, k, out)
    return out


def quantize_activation_int8(x, scale: float, zp: int = 0, unsigned: bool = False) -> np.ndarray:
    x = _f32(x).reshape(-1)
    out = np.empty_like(x)
    lib().oracle_quantize_activation_int8(x, x.size, scale, zp, int(unsigned), out)
    return out


# ---------------------------------------------------------------- layers
def rmsnorm(x, gamma=None, eps: float = 1e-6, affine_size: int | None = None) -> np.ndarray:
    x = _f32(x)
    if x.ndim == 1:
        x = x.reshape(1, -1)
    rows, w = x.shape
    g = None if gamma is None else _f32(gamma)
    y = np.empty_like(x)
    lib().oracle_rmsnorm(x, rows, w, w, _ptr(g), (affine_size if affine_size is not None else (0 if g is None else g.size)),
                         eps, y, w)
    return y


def rope(src, embed_dim: int, seq_len: int, num_heads: int, cos, sin, interleaved: bool = False):
    src = _f32(src)
    out = np.empty_like(src)
    lib().oracle_rope(src, embed_dim, seq_len, num_heads, _f32(cos), _f32(sin), int(interleaved), out)
    return out


def append_sequence(current, width: int, rows: int, slices: int, offset: int, cache, cache_rows: int):
    cache = _f32(cache).copy()
    lib().oracle_append_sequence(_f32(current), width, rows, slices, offset, cache, cache_rows)
    return cache


def concat_sequence(a, a_rows: int, b, b_rows: int, width: int, slices: int, out_rows: int):
    out = np.empty(slices * out_rows * width * 4, dtype=np.float32)
    lib().oracle_concat_sequence(_f32(a), a_rows, _f32(b), b_rows, width, slices, out, out_rows)
    return out


def sdpa(q, k, v, src_len, dst_len, embed_dim, out_embed_dim, num_heads, num_groups, scale,
         mask=None, mask_w=0, mask_h=0, causal=False, causal_offset=0):
    out = np.zeros(((num_heads + 3) // 4) * src_len * out_embed_dim * 4, dtype=np.float32)
    m = None if mask is None else _f32(mask)
    lib().oracle_sdpa(_f32(q), _f32(k), _f32(v), src_len, dst_len, embed_dim, out_embed_dim,
                      num_heads, num_groups, scale, _ptr(m), mask_w, mask_h, int(causal),
                      causal_offset, out)
    return out


def argmax(logits) -> np.ndarray:
    x = _f32(logits)
    if x.ndim == 1:
        x = x.reshape(1, -1)
    out = np.empty(x.shape[0], dtype=np.int32)
    lib().oracle_argmax(x, x.shape[0], x.shape[1], x.shape[1], out)
    return out


def topk(logits, k: int):
    x = _f32(logits)
    if x.ndim == 1:
        x = x.reshape(1, -1)
    vals = np.empty((x.shape[0], k), dtype=np.float32)
    idx = np.empty((x.shape[0], k), dtype=np.int32)
    lib().oracle_topk(x, x.shape[0], x.shape[1], x.shape[1], k, vals, idx)
    return vals, idx


def embed(words, bits: int, num_output: int, input_dim: int, packed=None, scales=None, blk: int = 0,
          table=None, bias=None) -> np.ndarray:
    w = np.ascontiguousarray(words, dtype=np.int32).reshape(-1)
    out = np.empty((w.size, num_output), dtype=np.float32)
    p = None if packed is None else np.ascontiguousarray(packed, dtype=np.uint32)
    s = None if scales is None else _f32(scales)
    t = None if table is None else _f32(table)
    b = None if bias is None else _f32(bias)
    lib().oracle_embed(w, w.size, bits, _ptr(p), _ptr(s), blk, _ptr(t), input_dim, num_output, _ptr(b), out)
    return out


def swish(x) -> np.ndarray:
    x = _f32(x).reshape(-1)
    y = np.empty_like(x)
    lib().oracle_swish(x, x.size, y)
    return y


def swiglu(gate, up) -> np.ndarray:
    g = _f32(gate).reshape(-1)
    y = np.empty_like(g)
    lib().oracle_swiglu(g, _f32(up).reshape(-1), g.size, y)
    return y


def short_conv(weight, mixed, cache_in, groups: int, kernel: int, seq: int, cache_len: int):
    """AexisShortConvPack4 on flat storage (see oracle_short_conv): weight Pack4 CDHW [kernel, 1, groups],
    mixed [seq, ld], cache_in [cache_len, ld], ld = ceil(groups/4)*4. Returns (out, cache_out)."""
    ld = (groups + 3) // 4 * 4
    out = np.zeros(seq * ld, dtype=np.float32)
    cache_out = np.zeros(max(cache_len, 0) * ld, dtype=np.float32)
    lib().oracle_short_conv(_f32(weight).ravel(), _f32(mixed).ravel(), _f32(cache_in).ravel(), out, cache_out,
                            groups, kernel, seq, cache_len)
    return out, cache_out


def gated_delta_rule(a_log, dt_bias, b, a, q, k, v, state_in, heads: int, kdim: int, vdim: int, seq: int,
                     first: int = 0, count: int | None = None, eps: float = 1e-6, out=None):
    """AexisGatedDeltaRulePack4 per token on flat storage (see oracle_gated_delta_rule): q/k/v Pack4 CDHW
    [dim, heads, seq], state [heads, kdim, ceil(vdim/4)*4]. Returns (out, state_out); `out` (flat CDHW
    [vdim, heads, seq]) is updated in place when given, as the kernel writes only processed tokens' lanes."""
    count = seq - first if count is None else count
    s4 = (seq + 3) // 4 * 4
    out = np.zeros(s4 * heads * vdim, dtype=np.float32) if out is None else _f32(out).ravel().copy()
    state_out = np.zeros(heads * kdim * ((vdim + 3) // 4 * 4), dtype=np.float32)
    lib().oracle_gated_delta_rule(_f32(a_log).ravel(), _f32(dt_bias).ravel(), _f32(b).ravel(), _f32(a).ravel(),
                                  _f32(q).ravel(), _f32(k).ravel(), _f32(v).ravel(), _f32(state_in).ravel(), out,
                                  state_out, heads, kdim, vdim, first, count, eps)
    return out, state_out


def sample(logits, history=None, penalty: float = 1.0, temperature: float = 0.0, top_k: int = 0,
           top_p: float = 1.0, uniforms=None):
    """Qwen35Sampler.Select per row with the given NextDouble draws (see oracle_sample). logits [rows, width];
    history: None or uint32 bitmap [rows, ceil(width/32)]. Returns (token ids, margins)."""
    x = _f32(logits)
    if x.ndim == 1:
        x = x.reshape(1, -1)
    rows, width = x.shape
    u = np.ascontiguousarray(np.zeros(rows) if uniforms is None else uniforms, dtype=np.float64)
    h = None if history is None else np.ascontiguousarray(history, dtype=np.uint32)
    out = np.zeros(rows, dtype=np.int32)
    margin = np.zeros(rows, dtype=np.float64)
    lib().oracle_sample(x, rows, width, width, _ptr(h), penalty, temperature, top_k, top_p, u, out, _ptr(margin))
    return out, margin


def round_f16(x) -> np.ndarray:
    x = _f32(x).reshape(-1)
    out = np.empty(x.size, dtype=np.uint16)
    lib().oracle_f32_to_f16(x, x.size, out)
    return out.view(np.float16).astype(np.float32)


def rope_tables(positions: int, rot_dim: int, theta: float):
    half = rot_dim // 2
    c = np.empty(positions * half, dtype=np.float32)
    s = np.empty(positions * half, dtype=np.float32)
    lib().oracle_rope_tables(positions, rot_dim, theta, c, s)
    return c.reshape(positions, half), s.reshape(positions, half)


# ---------------------------------------------------------------- decoder
class _Cfg(C.Structure):
    _fields_ = ([(n, C.c_int32) for n in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn",
                                          "vocab", "kv_capacity", "rot_dim", "bits", "group", "lm_bits",
                                          "lm_group")] + [("theta", C.c_float), ("eps", C.c_float)]
                + [(n, C.c_int32) for n in ("lin_heads", "lin_kdim", "lin_vdim", "conv_kernel")]
                + [("layer_types", C.POINTER(C.c_int32))])


class OracleDecoder:
    """The synthetic decoder restated on the CPU (see oracle_decoder_step).

    `model` is an aiimage_b200.synth.SyntheticDecoder (reference-format weights
    as numpy arrays); the arrays are borrowed, so the model must outlive this.
    """

    def __init__(self, model):
        cfg = model.cfg
        self._model = model
        kinds = cfg.layer_types()
        self._types = np.ascontiguousarray(kinds, dtype=np.int32)
        self._c = _Cfg(cfg.n_layers, cfg.hidden, cfg.n_heads, cfg.n_kv_heads, cfg.head_dim, cfg.ffn, cfg.vocab,
                       cfg.kv_capacity, cfg.rot_dim, cfg.bits, cfg.group, cfg.lm_bits, cfg.lm_group,
                       cfg.rope_theta, cfg.eps, cfg.lin_heads, cfg.lin_kdim, cfg.lin_vdim, cfg.conv_kernel,
                       self._types.ctypes.data_as(C.POINTER(C.c_int32)))
        L = lib()
        self._h = L.oracle_decoder_create(C.byref(self._c))
        self._keep = []
        for layer in range(cfg.n_layers):
            linear_attention = kinds[layer] == 1
            for which in ((8, 9, 4, 5, 6) if linear_attention else range(7)):
                p, s = model.linear(layer, which)
                s32 = _f32(s)
                self._keep.append(s32)
                L.oracle_decoder_set_linear(self._h, layer, which, p, s32)
            if linear_attention:
                prm = [_f32(x) for x in model.linear_attention(layer)]
                self._keep.extend(prm)
                L.oracle_decoder_set_linear_attention(self._h, layer, *prm)
            for which in range(2):
                g = _f32(model.norm(layer, which))
                self._keep.append(g)
                L.oracle_decoder_set_norm(self._h, layer, which, g)
        p, s = model.linear(-1, 7)
        s32 = _f32(s)
        self._keep.append(s32)
        L.oracle_decoder_set_linear(self._h, -1, 7, p, s32)
        g = _f32(model.norm(-1, 0))
        self._keep.append(g)
        L.oracle_decoder_set_norm(self._h, -1, 0, g)
        e = _f32(model.embedding)
        self._keep.append(e)
        L.oracle_decoder_set_embedding(self._h, e)

    def close(self):
        if self._h:
            lib().oracle_decoder_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def reset(self):
        lib().oracle_decoder_reset(self._h)

    @property
    def position(self) -> int:
        return int(lib().oracle_decoder_position(self._h))

    def fill_context(self, ctx: int, seed: int, seq_id: int):
        """Synthetic context of a batched-decoding sequence (the same values
        aexis_cuda_batch_fill_context writes): positions [0, ctx) filled,
        next position ctx."""
        if lib().oracle_decoder_fill_context(self._h, int(ctx), int(seed) & (2**64 - 1), int(seq_id)) != 0:
            raise ValueError("context must be in [0, kv_capacity)")

    def kv(self, layer: int, kind: int) -> np.ndarray:
        """Layer `layer`'s K (kind 0) or V (kind 1) cache, [kv_heads, capacity, head_dim] fp32."""
        c = self._c
        out = np.empty((c.n_kv_heads, c.kv_capacity, c.head_dim), dtype=np.float32)
        lib().oracle_decoder_kv(self._h, int(layer), int(kind), out)
        return out

    def recurrent(self, layer: int):
        """A linear-attention layer's caches: (conv [conv_kernel, channels], gdr [heads, kdim, vdim]) fp32."""
        c = self._c
        ch = 2 * c.lin_heads * c.lin_kdim + c.lin_heads * c.lin_vdim
        conv = np.empty((c.conv_kernel, ch), dtype=np.float32)
        gdr = np.empty((c.lin_heads, c.lin_kdim, c.lin_vdim), dtype=np.float32)
        lib().oracle_decoder_recurrent(self._h, int(layer), _ptr(conv), _ptr(gdr))
        return conv, gdr

    def step(self, token: int, want_logits: bool = True):
        logits = np.empty(self._c.vocab, dtype=np.float32) if want_logits else None
        margin = np.zeros(1, dtype=np.float32)
        nxt = lib().oracle_decoder_step(self._h, int(token), int(want_logits), _ptr(logits), _ptr(margin))
        if nxt == -2:
            raise RuntimeError("KV capacity exhausted")
        return nxt, logits, float(margin[0])

    def generate(self, prompt, max_new: int):
        """Qwen35DecoderSession.Generate, greedy: returns (tokens, margins);
        the logits of the last step are kept in self.last_logits."""
        prompt = [int(t) for t in prompt]
        for t in prompt[:-1]:
            self.step(t, want_logits=False)
        tok, logits, margin = self.step(prompt[-1])
        out, margins = [tok], [margin]
        while len(out) < max_new:
            tok, logits, margin = self.step(tok)
            out.append(tok)
            margins.append(margin)
        self.last_logits = logits
        return out, margins
