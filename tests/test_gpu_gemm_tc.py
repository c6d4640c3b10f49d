"""Batched Q8 GEMM on the tensor cores (tcgen05) against the CPU oracle.

aexis_cuda_gemm takes this path for Q8 weights with m >= 4 rows and K a
multiple of 64. fp16 activations are multiplied exactly; fp32 activations are
split into fp16 hi + lo rows (about 22 bits). Same tolerance as the GEMV:
|gpu - ref| <= 1e-2 |ref| + 1e-3 max|ref|, norm-wise error <= 2e-3.
"""
import numpy as np
import pytest

from aiimage_b200 import synth
from test_gpu_gemv import assert_gemv_close

pytestmark = pytest.mark.gpu


def run_batched(ops, w, x, n, out_dtype, bias=None, alpha=1.0, beta=1.0, tiled=False):
    import torch
    xt = torch.from_numpy(x).cuda()
    m = x.shape[0]
    y = torch.zeros((m, n), dtype=out_dtype, device="cuda")
    b = None if bias is None else torch.from_numpy(bias).cuda()
    ops.set_int4_gemm_weights(None)
    ops.set_int8_gemm_weights(w)
    fn = ops.gemm2d_pack4_tiled_texture_a if tiled else ops.gemm2d_pack4_linear_texture_a
    fn(xt, b, m, n, w.k, True, alpha, beta, b is not None, 4, y)
    torch.cuda.synchronize()
    ops.sync()  # also reports a bounded-wait timeout, if any
    return y.float().cpu().numpy()


@pytest.mark.parametrize("m,n,k,act", [
    (8, 256, 64, "f16"),       # one tile, one k-block
    (32, 3584, 1024, "f32"),   # config 4 shape (fp32 activations, hi/lo split)
    (256, 4096, 1024, "f16"),  # config 5 batch with a smaller vocabulary slice
    (5, 1000, 3584, "f32"),    # ragged N (partial tile), long K
    (100, 640, 128, "f16"),
    (256, 38000, 1024, "f16"),  # 297 slabs over the SMs: 2-3 per CTA, single-slab tail tiles
    (128, 384, 256, "f32"),     # hi/lo split at the full MMA width (nb = 256)
    (7, 1001, 128, "f16"),      # odd row stride: direct stores instead of staged bulk copies
    (40, 1003, 192, "f32"),
    (150, 76000, 128, "f16"),   # nb = 160: one slab per tile, four tiles per CTA (both TMEM buffers twice)
    (64, 151936, 128, "f16"),   # nb = 64: two slabs per tile, four tiles per CTA
])
def test_tc_gemm_matches_oracle(ops, oracle, m, n, k, act):
    import torch
    p, s = synth.q8_weights(n, k, seed=7, tag=(n, k))
    w = ops.new_int8_weight_only_upload(p, s, n, k)
    x = synth.activations(k, seed=7, tag=(m, k), m=m)
    if act == "f32":
        x = (x.astype(np.float32) * 0.37).astype(np.float32)
    got = run_batched(ops, w, x, n, torch.float32)
    ref = oracle.gemm(x.astype(np.float32), 8, p, s.astype(np.float32), 0, n)
    assert_gemv_close(got, ref)


@pytest.mark.parametrize("tiled,act", [(False, "f16"), (True, "f16"), (False, "f32"), (True, "f32")])
def test_tc_gemm_bias_alpha_beta_f16_out(ops, oracle, tiled, act):
    import torch
    m, n, k = 16, 768, 256
    p, s = synth.q8_weights(n, k, seed=8)
    w = ops.new_int8_weight_only_upload(p, s.astype(np.float32), n, k)
    x = synth.activations(k, seed=8, m=m)
    if act == "f32":
        x = (x.astype(np.float32) * 0.37).astype(np.float32)
    bias = np.random.default_rng(8).standard_normal(n).astype(np.float32)
    got = run_batched(ops, w, x, n, torch.float16, bias=bias, alpha=0.75, beta=1.5, tiled=tiled)
    ref = oracle.gemm(x.astype(np.float32), 8, p, s.astype(np.float32), 0, n, bias=bias, alpha=0.75, beta=1.5,
                      tiled=tiled)
    assert_gemv_close(got, ref)


def test_config5_lm_head_rows_and_argmax(ops, oracle):
    """BASELINE config 5 on one GPU: 151936 x 1024 Q8 lm_head, 256 fp16 hidden
    states. Eight of the 256 rows are checked against the oracle (logits and
    greedy ids)."""
    import torch
    n, k, m = 151936, 1024, 256
    p, s = synth.q8_weights(n, k, seed=5, tag=(n, k))
    w = ops.new_int8_weight_only_upload(p, s, n, k)
    x = synth.activations(k, seed=5, tag=(m, k), m=m)
    got = run_batched(ops, w, x, n, torch.float32)
    rows = np.array([0, 1, 37, 100, 128, 200, 254, 255])
    ref = oracle.gemm(x[rows].astype(np.float32), 8, p, s.astype(np.float32), 0, n)
    assert_gemv_close(got[rows], ref)
    assert np.array_equal(np.argmax(got[rows], axis=1), oracle.argmax(ref))
