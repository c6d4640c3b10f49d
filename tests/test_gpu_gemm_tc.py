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


def _unfused_topk(ops, w, x, k, offset):
    """Reference for aexis_cuda_gemm_topk: the tiled lm_head to fp32 logits, then the top-k and greedy-key calls."""
    import torch
    m, n = x.shape[0], w.n
    logits = torch.empty((m, n), dtype=torch.float32, device="cuda")
    ops.set_int4_gemm_weights(None)
    ops.set_int8_gemm_weights(w)
    ops.gemm2d_pack4_tiled_texture_a(x, None, m, n, w.k, True, 1.0, 1.0, False, 4, logits)
    vals = torch.empty((m, k), dtype=torch.float32, device="cuda")
    idx = torch.empty((m, k), dtype=torch.int32, device="cuda")
    keys = torch.empty(m, dtype=torch.int64, device="cuda")
    ops.top_k(logits, n, m, k, vals, idx)
    ops.topk_greedy_keys(logits, n, m, k, vals, idx, offset, keys)
    return vals, idx, keys


@pytest.mark.parametrize("n,m,act,k,offset", [
    (151936, 256, "f16", 50, 0),      # BASELINE config 5 on one GPU
    (18992, 256, "f16", 50, 132944),  # the last of eight vocab shards (global indices)
    (37984, 37, "f32", 64, 37984),    # fp32 activations (hi/lo split), ragged m
    (75968, 5, "f16", 1, 0),          # k = 1: the greedy token alone
    (4097, 128, "f16", 20, 0),        # a partial last slab
    (3000, 16, "f16", 50, 0),         # narrow rows: the exact top-k path
])
def test_fused_lm_head_topk_matches_unfused(ops, n, m, act, k, offset):
    """aexis_cuda_gemm_topk: the same values, indices and greedy keys, bit for bit, as the logits written
    by the tiled GEMM followed by aexis_cuda_topk and aexis_cuda_topk_greedy_keys. Adversarial rows: all
    logits equal (x = 0: ties go by index), all NaN (nothing selectable, (-inf, -1) padding, the greedy
    key of a NaN at index 0), huge activations, and a row equal to another."""
    import torch
    p, s = synth.q8_weights(n, 1024, seed=n % 97, tag=(n, 1024))
    w = ops.new_int8_weight_only_upload(p, s, n, 1024)
    x = synth.activations(1024, seed=n % 89, tag=(m, 1024), m=m).astype(np.float32)
    x[0] = 0.0
    if m > 3:
        x[1] = np.nan
        x[2] *= 1000.0
        x[3] = x[4 % m]
    xt = torch.from_numpy(x if act == "f32" else x.astype(np.float16)).cuda()
    rv, ri, rk = _unfused_topk(ops, w, xt, k, offset)
    vals = torch.full((m, k), 7.0, dtype=torch.float32, device="cuda")
    idx = torch.full((m, k), -7, dtype=torch.int32, device="cuda")
    keys = torch.zeros(m, dtype=torch.int64, device="cuda")
    ops.set_int8_gemm_weights(w)
    for _ in range(2):  # twice: the second call reuses the sample and the buffers
        ops.gemm_topk(xt, m, 1024, k, vals, idx, keys, 1.0, offset)
        torch.cuda.synchronize()
        ops.sync()
        assert torch.equal(vals, rv) and torch.equal(idx, ri) and torch.equal(keys, rk)
    assert idx[0].tolist() == list(range(k))  # the plateau: lowest indices first
    if m > 3:
        assert (idx[1] == -1).all() and torch.isinf(vals[1]).all()
        if offset == 0:
            assert int(keys[1]) & 0xFFFFFFFF == 0xFFFFFFFF  # a NaN at global index 0 is the greedy pick
        else:
            assert int(keys[1]) == 0  # a shard past index 0 has nothing selectable in an all-NaN row
        assert torch.equal(idx[3], idx[4 % m])
