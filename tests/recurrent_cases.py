"""Shared inputs of the linear-attention (ShortConv / GatedDeltaRule) tests.

Golden cases come from tests/golden/recurrent_ops.npz, written by
tests/golden/make_recurrent_golden.py from the reference's own fp32 NumPy
operators (Tools/Qwen35NcnnBaseline/reference_ops.py:36-152). These helpers
turn their logical arrays into the storage layouts of the C ABI.
"""
import os

import numpy as np

from aiimage_b200.ops import pack4_cdhw, pack4_rows, unpack4_cdhw

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "recurrent_ops.npz")


def golden_cases(prefix: str) -> dict:
    z = np.load(GOLDEN)
    cases = {}
    for key in z.files:
        name, field = key.split("/")
        if name.startswith(prefix):
            cases.setdefault(name, {})[field] = z[key]
    return cases


def short_conv_storage(weight, mixed, state_in, cache_len):
    """Logical weight [groups, kernel], mixed [seq, groups], state [cache, groups] (None = zeros) ->
    (weight Pack4 CDHW [kernel, 1, groups], mixed rows, cache rows, groups, kernel, seq, cache_len)."""
    groups, kernel = weight.shape
    seq = mixed.shape[0]
    if state_in is None:
        state_in = np.zeros((cache_len, groups), np.float32)
    # ncnn MemoryData [w=kernel, h=1, c=groups]: logical [c=groups, h=1, w=kernel].
    w = pack4_cdhw(weight.reshape(groups, 1, kernel))
    return w, pack4_rows(mixed), pack4_rows(state_in), groups, kernel, seq, cache_len


def unpack_rows(flat, rows, width):
    ld = (width + 3) // 4 * 4
    return np.asarray(flat, np.float32).reshape(rows, ld)[:, :width]


def pad_state(state):
    """[heads, kdim, vdim] -> [heads, kdim, ceil(vdim/4)*4] (zero columns)."""
    h, kd, vd = state.shape
    out = np.zeros((h, kd, (vd + 3) // 4 * 4), np.float32)
    out[:, :, :vd] = state
    return out


def gdr_storage(case):
    """Golden/logical GDR case -> dict of flat storage arrays and sizes."""
    seq, heads, kdim = case["q"].shape
    vdim = case["v"].shape[2]
    return dict(
        a_log=case["a_log"].astype(np.float32), dt_bias=case["dt_bias"].astype(np.float32),
        b=np.ascontiguousarray(case["b"], np.float32).ravel(), a=np.ascontiguousarray(case["a"], np.float32).ravel(),
        q=pack4_cdhw(case["q"]), k=pack4_cdhw(case["k"]), v=pack4_cdhw(case["v"]),
        state=pad_state(case["state_in"]).ravel(), heads=heads, kdim=kdim, vdim=vdim, seq=seq)


def gdr_out_logical(flat, seq, heads, vdim):
    return unpack4_cdhw(flat, seq, heads, vdim)


def gdr_state_logical(flat, heads, kdim, vdim):
    return np.asarray(flat, np.float32).reshape(heads, kdim, (vdim + 3) // 4 * 4)[:, :, :vdim]


def random_gdr(rng, seq, heads, kdim, vdim, state_sigma=0.05):
    """Seeded logical inputs with the reference test's distributions (test_reference_ops.py:51-59)."""
    return dict(
        a_log=rng.normal(-1.0, 0.2, heads).astype(np.float32), dt_bias=rng.normal(0, 0.2, heads).astype(np.float32),
        b=rng.normal(0, 0.4, (seq, heads)).astype(np.float32), a=rng.normal(0, 0.4, (seq, heads)).astype(np.float32),
        q=rng.normal(0, 0.5, (seq, heads, kdim)).astype(np.float32),
        k=rng.normal(0, 0.5, (seq, heads, kdim)).astype(np.float32),
        v=rng.normal(0, 0.5, (seq, heads, vdim)).astype(np.float32),
        state_in=rng.normal(0, state_sigma, (heads, kdim, vdim)).astype(np.float32))
