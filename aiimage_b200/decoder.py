"""DecoderSession: the host mirror of Qwen35DecoderSession's greedy decode
(Packages/com.aexis/Samples/AIImageApplicationExample/Runtime/Scripts/
Qwen35DecoderSession.cs: Generate :1160-1237, DecodeCore :469-585,
SelectNextToken :734-809) over libaexis_cuda's fused decoder.
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np

from . import errors
from .native import F16, F32, DecoderConfig, check, lib
from .ops import AexisOps
from .synth import DecoderCfg


def _np(a):
    return a.ctypes.data_as(C.c_void_p)


class DecoderSession:
    """The decoder over a DecoderCfg: every layer full attention, or with
    cfg.full_attention_interval > 0 the hybrid stack of linear-attention
    (ShortConv + Gated Delta Rule) and full-attention layers."""

    def __init__(self, ops: AexisOps, cfg: DecoderCfg, scale_dtype: int = F16):
        self.ops, self.cfg = ops, cfg
        c = cfg
        self.layer_types = c.layer_types()
        self._types = np.ascontiguousarray(self.layer_types, dtype=np.int32)
        hybrid = any(self.layer_types)
        self._cfg = DecoderConfig(c.n_layers, c.hidden, c.n_heads, c.n_kv_heads, c.head_dim, c.ffn, c.vocab,
                                  c.kv_capacity, c.rot_dim, c.bits, c.group, c.lm_bits, c.lm_group, scale_dtype,
                                  c.rope_theta, c.eps,
                                  self._types.ctypes.data_as(C.POINTER(C.c_int32)) if hybrid else None,
                                  c.lin_heads, c.lin_kdim, c.lin_vdim, c.conv_kernel)
        self.h = C.c_void_p()
        check(lib().aexis_cuda_decoder_create(ops.ctx, C.byref(self._cfg), C.byref(self.h)), ops.ctx)
        self._scale_dtype = scale_dtype
        self._batches = weakref.WeakSet()
        ops._register(self)

    def close(self):
        # A decoder lives inside its context: destroy it first (AexisOps.close
        # closes its decoders before the context goes away); its batches go
        # before it.
        for b in list(self._batches):
            b.close()
        if self.h and self.ops.ctx:
            lib().aexis_cuda_decoder_destroy(self.h)
        self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st):
        check(st, self.ops.ctx)

    # -- loading (AexisGemmLayer / AexisRMSNormLayer / AexisEmbedLayer LoadLayer)
    def set_linear(self, layer: int, which: int, packed: np.ndarray, scales: np.ndarray):
        p = np.ascontiguousarray(packed, dtype=np.uint32)
        s = np.ascontiguousarray(scales, dtype=np.float16 if self._scale_dtype == F16 else np.float32)
        self._check(lib().aexis_cuda_decoder_set_linear(self.h, layer, which, _np(p), _np(s), self._scale_dtype))

    def set_norm(self, layer: int, which: int, gamma: np.ndarray):
        g = np.ascontiguousarray(gamma)
        dt = F16 if g.dtype == np.float16 else F32
        g = g.astype(np.float16 if dt == F16 else np.float32, copy=False)
        self._check(lib().aexis_cuda_decoder_set_norm(self.h, layer, which, _np(g), dt))

    def set_linear_attention(self, layer: int, conv: np.ndarray, a_log: np.ndarray, dt_bias: np.ndarray,
                             gamma: np.ndarray):
        """A linear-attention layer's conv [channels, kernel], a_log, dt_bias [lin_heads], gamma [lin_vdim]."""
        dt = F16 if all(np.asarray(x).dtype == np.float16 for x in (conv, a_log, dt_bias, gamma)) else F32
        arrs = [np.ascontiguousarray(x, dtype=np.float16 if dt == F16 else np.float32)
                for x in (conv, a_log, dt_bias, gamma)]
        self._check(lib().aexis_cuda_decoder_set_linear_attention(self.h, int(layer), *[_np(a) for a in arrs], dt))

    def set_embedding(self, table: np.ndarray):
        t = np.ascontiguousarray(table)
        dt = F16 if t.dtype == np.float16 else F32
        t = t.astype(np.float16 if dt == F16 else np.float32, copy=False)
        self._check(lib().aexis_cuda_decoder_set_embedding(self.h, _np(t), dt))

    def load(self, model) -> "DecoderSession":
        """Upload every weight of a SyntheticDecoder (or any object with the
        same linear/norm/embedding accessors)."""
        c = self.cfg
        for layer in range(c.n_layers):
            for which in c.linears(layer):
                self.set_linear(layer, which, *model.linear(layer, which))
            if self.layer_types[layer] == 1:
                self.set_linear_attention(layer, *model.linear_attention(layer))
            for which in range(2):
                self.set_norm(layer, which, model.norm(layer, which))
        self.set_linear(-1, 7, *model.linear(-1, 7))
        self.set_norm(-1, 0, model.norm(-1, 0))
        self.set_embedding(model.embedding)
        return self

    # -- decoding -----------------------------------------------------------
    def reset(self):
        self._check(lib().aexis_cuda_decoder_reset(self.h))

    @property
    def position(self) -> int:
        v = C.c_int32()
        self._check(lib().aexis_cuda_decoder_position(self.h, C.byref(v)))
        return v.value

    def prefill(self, tokens) -> int:
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.zeros(1, dtype=np.int32)
        self._check(lib().aexis_cuda_decoder_prefill(self.h, _np(t), t.size, _np(out)))
        return int(out[0])

    def step(self, token: int) -> int:
        out = np.zeros(1, dtype=np.int32)
        self._check(lib().aexis_cuda_decoder_step(self.h, int(token), _np(out)))
        return int(out[0])

    def generate(self, prompt, max_new: int) -> list[int]:
        """Greedy: prefill `prompt`, return max_new generated token ids."""
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.zeros(max_new, dtype=np.int32)
        self._check(lib().aexis_cuda_decoder_generate(self.h, _np(p), p.size, max_new, _np(out)))
        return [int(x) for x in out]

    def logits(self) -> np.ndarray:
        out = np.empty(self.cfg.vocab, dtype=np.float32)
        self._check(lib().aexis_cuda_decoder_logits(self.h, _np(out)))
        return out

    # -- state in the reference's layout (Qwen35DecoderState) -----------------
    def kv_rows_floats(self, rows: int) -> int:
        """Floats of one Pack4 CDHW cache texture [head_dim, rows, n_kv_heads]."""
        c = self.cfg
        return 4 * ((c.n_kv_heads + 3) // 4) * rows * c.head_dim

    def kv_export(self, layer: int, k_out, v_out, rows: int):
        """Layer `layer`'s K and V caches into device fp32 Pack4 CDHW tensors of `rows` rows
        (aexis_cuda_decoder_kv_export); rows past the position are zero."""
        self.ops._bind_stream()
        self._check(lib().aexis_cuda_decoder_kv_export(self.h, int(layer), int(rows), k_out.data_ptr(),
                                                       v_out.data_ptr()))

    def kv_import(self, layer: int, k_in, v_in, rows: int, length: int):
        """Positions [0, length) of layer `layer`'s caches from Pack4 CDHW tensors (rounded to fp16)."""
        self.ops._bind_stream()
        self._check(lib().aexis_cuda_decoder_kv_import(self.h, int(layer), k_in.data_ptr(), v_in.data_ptr(),
                                                       int(rows), int(length)))

    def set_position(self, position: int):
        self.ops._bind_stream()
        self._check(lib().aexis_cuda_decoder_set_position(self.h, int(position)))

    def recurrent_shapes(self) -> tuple[int, int]:
        """Floats of a linear-attention layer's (conv cache, GDR cache)."""
        c = self.cfg
        return c.conv_kernel * c.conv_channels(), c.lin_heads * c.lin_kdim * c.lin_vdim

    def recurrent_export(self, layer: int, conv_out, gdr_out):
        """A linear-attention layer's caches into device fp32 tensors (either may be None)
        (aexis_cuda_decoder_recurrent_export): conv [conv_kernel, channels], GDR [heads, kdim, vdim]."""
        self.ops._bind_stream()
        self._check(lib().aexis_cuda_decoder_recurrent_export(
            self.h, int(layer), None if conv_out is None else conv_out.data_ptr(),
            None if gdr_out is None else gdr_out.data_ptr()))

    def recurrent_import(self, layer: int, conv_in, gdr_in):
        self.ops._bind_stream()
        self._check(lib().aexis_cuda_decoder_recurrent_import(
            self.h, int(layer), None if conv_in is None else conv_in.data_ptr(),
            None if gdr_in is None else gdr_in.data_ptr()))

    def _state_names(self):
        """(layer, kind, ordinal): the reference numbers each cache kind on its own ("cache_k0".."cache_k5",
        "cache_conv0".."cache_conv17" for Qwen3.5), in layer order."""
        n_full = n_lin = 0
        for layer, kind in enumerate(self.layer_types):
            if kind == 1:
                yield layer, kind, n_lin
                n_lin += 1
            else:
                yield layer, kind, n_full
                n_full += 1

    def export_state(self, rows: int | None = None) -> dict:
        """Qwen35DecoderState as the reference holds it: {"cache_k<i>", "cache_v<i>": Pack4 CDHW fp32
        device tensors of `rows` (default: the position) rows for the i-th full-attention layer,
        "cache_conv<i>", "cache_gdr<i>": the i-th linear-attention layer's caches, "sequence_length": the
        position}."""
        import torch
        pos = self.position
        rows = max(pos, 1) if rows is None else int(rows)
        state = {"sequence_length": pos, "rows": rows}
        dev = f"cuda:{self.ops.device}"
        nc, ng = self.recurrent_shapes()
        for layer, kind, i in self._state_names():
            if kind == 1:
                conv = torch.empty(nc, dtype=torch.float32, device=dev)
                gdr = torch.empty(ng, dtype=torch.float32, device=dev)
                self.recurrent_export(layer, conv, gdr)
                state[f"cache_conv{i}"], state[f"cache_gdr{i}"] = conv, gdr
            else:
                k = torch.empty(self.kv_rows_floats(rows), dtype=torch.float32, device=dev)
                v = torch.empty_like(k)
                self.kv_export(layer, k, v, rows)
                state[f"cache_k{i}"], state[f"cache_v{i}"] = k, v
        return state

    def import_state(self, state: dict):
        """Load a state of export_state's form; decoding continues at its sequence_length."""
        length, rows = int(state["sequence_length"]), int(state["rows"])
        for layer, kind, i in self._state_names():
            if kind == 1:
                self.recurrent_import(layer, state[f"cache_conv{i}"], state[f"cache_gdr{i}"])
            else:
                self.kv_import(layer, state[f"cache_k{i}"], state[f"cache_v{i}"], rows, length)
        self.set_position(length)

    def set_schedule(self, mode: int):
        """How generate runs its greedy steps: 0 (default) one CUDA graph per
        step, 1 one persistent kernel for the whole call, -1 1 where supported."""
        self._check(lib().aexis_cuda_decoder_set_schedule(self.h, int(mode)))

    def schedule(self) -> int:
        out = np.zeros(1, dtype=np.int32)
        self._check(lib().aexis_cuda_decoder_schedule(self.h, _np(out)))
        return int(out[0])


class BatchSession:
    """Batched greedy decoding of B independent sequences over one
    DecoderSession's Q8 weights (aexis_cuda_batch_*): what a host serving B
    Qwen35DecoderSession instances would run, one step for all of them.
    Create it after the decoder's weights are loaded."""

    def __init__(self, dec: DecoderSession, max_batch: int, kv_capacity: int, max_steps: int):
        self.dec = dec
        self.h = C.c_void_p()
        check(lib().aexis_cuda_batch_create(dec.h, max_batch, kv_capacity, max_steps, C.byref(self.h)), dec.ops.ctx)
        self.n = 0
        dec._batches.add(self)

    def close(self):
        if self.h and self.dec.h and self.dec.ops.ctx:
            lib().aexis_cuda_batch_destroy(self.h)
        self.h = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _check(self, st):
        check(st, self.dec.ops.ctx)

    def fill_context(self, ctx_lens, seed: int, first_seq_id: int = 0):
        """Sequences i < len(ctx_lens) get synthetic contexts of ctx_lens[i]
        positions (the values of oracle_decoder_fill_context)."""
        c = np.ascontiguousarray(ctx_lens, dtype=np.int32)
        self._check(lib().aexis_cuda_batch_fill_context(self.h, c.size, _np(c), int(seed) & (2**64 - 1),
                                                        int(first_seq_id)))
        self.n = int(c.size)

    def generate(self, first_tokens, steps: int) -> np.ndarray:
        """Greedy tokens [steps][n]."""
        t = np.ascontiguousarray(first_tokens, dtype=np.int32)
        if self.n and t.size != self.n:  # with no context the library reports the state error
            raise errors.ArgumentOutOfRangeError(f"{t.size} first tokens for {self.n} sequences")
        out = np.zeros((max(steps, 0), max(self.n, 1)), dtype=np.int32)
        self._check(lib().aexis_cuda_batch_generate(self.h, _np(t), int(steps), _np(out)))
        return out

    def generate_device(self, first_tokens, steps: int):
        """As generate, without copying the tokens back (timing runs)."""
        t = np.ascontiguousarray(first_tokens, dtype=np.int32)
        self._check(lib().aexis_cuda_batch_generate(self.h, _np(t), int(steps), None))

    def kv_export(self, seq: int, layer: int, k_out, v_out, rows: int):
        """Sequence `seq`'s layer-`layer` K and V caches as Pack4 CDHW fp32 device tensors of `rows` rows."""
        self.dec.ops._bind_stream()
        self._check(lib().aexis_cuda_batch_kv_export(self.h, int(seq), int(layer), int(rows), k_out.data_ptr(),
                                                     v_out.data_ptr()))

    def kv_import(self, seq: int, layer: int, k_in, v_in, rows: int, length: int):
        self.dec.ops._bind_stream()
        self._check(lib().aexis_cuda_batch_kv_import(self.h, int(seq), int(layer), k_in.data_ptr(), v_in.data_ptr(),
                                                     int(rows), int(length)))

    def set_positions(self, positions):
        """Sequences 0..len(positions)-1 become the batch, each continuing at positions[i]."""
        p = np.ascontiguousarray(positions, dtype=np.int32)
        self.dec.ops._bind_stream()
        self._check(lib().aexis_cuda_batch_set_positions(self.h, p.size, _np(p)))
        self.n = int(p.size)

    @property
    def positions(self) -> np.ndarray:
        out = np.zeros(self.n, dtype=np.int32)
        self._check(lib().aexis_cuda_batch_positions(self.h, _np(out)))
        return out

    def logits(self) -> np.ndarray:
        out = np.empty((self.n, self.dec.cfg.vocab), dtype=np.float32)
        self._check(lib().aexis_cuda_batch_logits(self.h, _np(out)))
        return out


__all__ = ["DecoderSession", "BatchSession", "errors"]
