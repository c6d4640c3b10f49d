"""ctypes binding of libaexis_cuda.so (the C ABI in include/aexis_cuda.h).

The library is the product: there is no CPU or eager-PyTorch fallback. If the
shared library is missing, every entry point raises instead of computing.
"""
from __future__ import annotations

import ctypes as C
import os
import re

from . import errors

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libaexis_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "aexis_cuda.h")

F32, F16 = 0, 1

vp = C.c_void_p
i32 = C.c_int
f32 = C.c_float


class DecoderConfig(C.Structure):
    """aexis_decoder_config (field order is the ABI)."""
    _fields_ = ([(n, C.c_int32) for n in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab",
                                          "kv_capacity", "rot_dim", "bits", "group", "lm_bits", "lm_group",
                                          "scale_dtype")] + [("rope_theta", C.c_float), ("eps", C.c_float)]
                + [("layer_types", C.POINTER(C.c_int32))]
                + [(n, C.c_int32) for n in ("lin_heads", "lin_kdim", "lin_vdim", "conv_kernel")])


# name -> (restype, argtypes)
SIGNATURES = {
    "aexis_cuda_abi_version": (i32, []),
    "aexis_cuda_create": (i32, [i32, C.POINTER(vp)]),
    "aexis_cuda_destroy": (i32, [vp]),
    "aexis_cuda_last_error": (C.c_char_p, [vp]),
    "aexis_cuda_set_stream": (i32, [vp, vp]),
    "aexis_cuda_sync": (i32, [vp]),
    "aexis_cuda_weights_q8": (i32, [vp, vp, vp, i32, i32, i32, C.POINTER(vp)]),
    "aexis_cuda_weights_q4": (i32, [vp, vp, vp, i32, i32, i32, i32, C.POINTER(vp)]),
    "aexis_cuda_weights_dense": (i32, [vp, vp, i32, i32, i32, C.POINTER(vp)]),
    "aexis_cuda_weights_free": (i32, [vp, vp]),
    "aexis_cuda_weights_dequant": (i32, [vp, vp, vp]),
    "aexis_quantize_q8_rows": (i32, [vp, i32, i32, i32, vp, vp]),
    "aexis_quantize_q4_rows": (i32, [vp, i32, i32, i32, vp, vp]),
    "aexis_cuda_set_int8_activations": (i32, [vp, i32, f32, i32, i32]),
    "aexis_cuda_gemm": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, f32, f32, vp, i32, i32, i32]),
    "aexis_cuda_gemm_tiled": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, f32, f32, vp, i32, i32, i32]),
    "aexis_cuda_gemm_pack4a": (i32, [vp, vp, i32, i32, i32, i32, i32, i32, vp, vp, f32, f32, vp, i32, i32, i32]),
    "aexis_cuda_rmsnorm": (i32, [vp, vp, i32, i32, i32, i32, vp, i32, f32, vp, i32]),
    "aexis_cuda_rope": (i32, [vp, vp, i32, i32, i32, vp, vp, i32, vp]),
    "aexis_cuda_kv_append": (i32, [vp, vp, i32, i32, i32, i32, vp, i32]),
    "aexis_cuda_kv_concat": (i32, [vp, vp, i32, vp, i32, i32, i32, vp, i32]),
    "aexis_cuda_sdpa": (i32, [vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, f32, vp, i32, i32, i32, i32, vp]),
    "aexis_cuda_argmax": (i32, [vp, vp, i32, i32, i32, vp]),
    "aexis_cuda_argmax_static": (i32, [vp, i32, i32, i32, vp, vp]),
    "aexis_cuda_argmax_keys": (i32, [vp, vp, i32, i32, i32, C.c_int64, vp]),
    "aexis_cuda_topk": (i32, [vp, vp, i32, i32, i32, i32, vp, vp]),
    "aexis_cuda_gemm_topk": (i32, [vp, vp, i32, i32, i32, i32, vp, f32, i32, C.c_int64, vp, vp, vp]),
    "aexis_cuda_topk_merge": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, vp]),
    "aexis_cuda_peer_buffer_bytes": (i32, [i32, i32, i32, C.POINTER(C.c_size_t)]),
    "aexis_cuda_peer_buffer_create": (i32, [vp, C.c_size_t, C.POINTER(vp), vp]),
    "aexis_cuda_peer_buffer_open": (i32, [vp, vp, C.POINTER(vp)]),
    "aexis_cuda_peer_buffer_close": (i32, [vp, vp, i32]),
    "aexis_cuda_topk_push": (i32, [vp, vp, i32, i32, C.POINTER(vp), i32, i32]),
    "aexis_cuda_topk_merge_peers": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, vp]),
    "aexis_cuda_embed": (i32, [vp, vp, i32, vp, vp, vp]),
    "aexis_cuda_swish": (i32, [vp, vp, i32, vp]),
    "aexis_cuda_swiglu": (i32, [vp, vp, vp, i32, vp]),
    "aexis_cuda_topk_greedy_keys": (i32, [vp, vp, i32, i32, i32, i32, vp, vp, C.c_int64, vp]),
    "aexis_cuda_sample": (i32, [vp, vp, i32, i32, i32, vp, f32, f32, i32, f32, vp, vp]),
    "aexis_cuda_sample_history_add": (i32, [vp, vp, i32, i32, vp]),
    "aexis_cuda_short_conv": (i32, [vp, vp, vp, vp, vp, vp, i32, i32, i32, i32]),
    "aexis_cuda_gated_delta_rule": (i32, [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, f32]),
    "aexis_cuda_decoder_create": (i32, [vp, C.POINTER(DecoderConfig), C.POINTER(vp)]),
    "aexis_cuda_decoder_destroy": (i32, [vp]),
    "aexis_cuda_decoder_set_linear": (i32, [vp, i32, i32, vp, vp, i32]),
    "aexis_cuda_decoder_set_norm": (i32, [vp, i32, i32, vp, i32]),
    "aexis_cuda_decoder_set_embedding": (i32, [vp, vp, i32]),
    "aexis_cuda_decoder_reset": (i32, [vp]),
    "aexis_cuda_decoder_position": (i32, [vp, C.POINTER(C.c_int32)]),
    "aexis_cuda_decoder_prefill": (i32, [vp, vp, i32, vp]),
    "aexis_cuda_decoder_step": (i32, [vp, C.c_int32, vp]),
    "aexis_cuda_decoder_generate": (i32, [vp, vp, i32, i32, vp]),
    "aexis_cuda_decoder_logits": (i32, [vp, vp]),
    "aexis_cuda_decoder_set_schedule": (i32, [vp, i32]),
    "aexis_cuda_decoder_kv_export": (i32, [vp, i32, i32, vp, vp]),
    "aexis_cuda_decoder_kv_import": (i32, [vp, i32, vp, vp, i32, i32]),
    "aexis_cuda_decoder_set_position": (i32, [vp, C.c_int32]),
    "aexis_cuda_layer_types_interval": (i32, [i32, i32, vp]),
    "aexis_cuda_decoder_set_linear_attention": (i32, [vp, i32, vp, vp, vp, vp, i32]),
    "aexis_cuda_decoder_recurrent_export": (i32, [vp, i32, vp, vp]),
    "aexis_cuda_decoder_recurrent_import": (i32, [vp, i32, vp, vp]),
    "aexis_cuda_batch_kv_export": (i32, [vp, i32, i32, i32, vp, vp]),
    "aexis_cuda_batch_kv_import": (i32, [vp, i32, i32, vp, vp, i32, i32]),
    "aexis_cuda_batch_set_positions": (i32, [vp, i32, vp]),
    "aexis_cuda_decoder_schedule": (i32, [vp, vp]),
    "aexis_cuda_selftest_wait": (i32, [vp, C.c_longlong]),
    "aexis_cuda_batch_create": (i32, [vp, i32, i32, i32, C.POINTER(vp)]),
    "aexis_cuda_batch_destroy": (i32, [vp]),
    "aexis_cuda_batch_fill_context": (i32, [vp, i32, vp, C.c_uint64, C.c_int64]),
    "aexis_cuda_batch_generate": (i32, [vp, vp, i32, vp]),
    "aexis_cuda_batch_positions": (i32, [vp, vp]),
    "aexis_cuda_batch_logits": (i32, [vp, vp]),
}

_lib = None


def declared_functions() -> list[str]:
    """Entry points declared in include/aexis_cuda.h (parsed from the header)."""
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(aexis_(?:cuda_|quantize_)\w+)\s*\(", text)))


def header_constant(name: str) -> int:
    """An integer #define or enum value of include/aexis_cuda.h (e.g. AEXIS_E_RANGE)."""
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    m = re.search(r"#define\s+" + name + r"\s+(-?\d+)\b", text) or re.search(r"\b" + name + r"\s*=\s*(-?\d+)\b",
                                                                                text)
    if not m:
        raise KeyError(name)
    return int(m.group(1))


def lib():
    """Load the library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"libaexis_cuda.so is missing ({LIB_PATH}); build it with "
                               "aiimage_b200.build.build_native() -- there is no CPU fallback")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def check(status: int, ctx=None) -> None:
    """Raise the exception class of a non-zero status with the context message."""
    if status == 0:
        return
    msg = lib().aexis_cuda_last_error(ctx)
    text = msg.decode() if msg else ""
    raise errors.BY_STATUS.get(status, errors.AexisError)(f"status {status}: {text}")
