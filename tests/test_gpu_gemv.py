"""GPU parity of the dequant GEMV (libaexis_cuda) against the CPU oracle.

Tolerance (the north-star bar for fp16/fp32 accumulation): every output within
1e-2 relative, |gpu - ref| <= 1e-2 * |ref| + 1e-3 * max|ref|, plus a norm-wise
relative error <= 2e-3. Unpacking and indexing are checked bit-exact through
aexis_cuda_weights_dequant.
"""
import numpy as np
import pytest

from aiimage_b200 import errors, synth

pytestmark = pytest.mark.gpu

RTOL, ATOL_REL, NORM_TOL = 1e-2, 1e-3, 2e-3


def assert_gemv_close(got, ref):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    scale = np.abs(ref).max()
    err = np.abs(got - ref)
    bad = err > RTOL * np.abs(ref) + ATOL_REL * scale
    assert not bad.any(), f"{bad.sum()} outputs off; worst {err.max():.3g} at {int(err.argmax())} (scale {scale:.3g})"
    assert np.linalg.norm(got - ref) <= NORM_TOL * np.linalg.norm(ref)


def run_gemv(ops, w, x16, n, dtype_out, bias=None, alpha=1.0, beta=1.0, tiled=False, x_f32=False):
    import torch
    x = torch.from_numpy(x16.astype(np.float32) if x_f32 else x16).cuda()
    m = x.shape[0]
    y = torch.zeros((m, n), dtype=dtype_out, device="cuda")
    b = None if bias is None else torch.from_numpy(bias).cuda()
    ops.set_int4_gemm_weights(w if w.kind == "q4" else None)
    ops.set_int8_gemm_weights(w if w.kind == "q8" else None)
    fn = ops.gemm2d_pack4_tiled_texture_a if tiled else ops.gemm2d_pack4_linear_texture_a
    fn(x, b, m, n, w.k, True, alpha, beta, b is not None, 4, y)
    torch.cuda.synchronize()
    return y.float().cpu().numpy()


def test_config1_q8_gemv(ops, oracle):
    """Q8 K=1024 N=3584, fp16 per-row scales, fp16 x and y, seed 0."""
    k, n = 1024, 3584
    p, s = synth.q8_weights(n, k, seed=0)
    x = synth.activations(k, seed=0)
    w = ops.new_int8_weight_only_upload(p, s, n, k)
    import torch
    got = run_gemv(ops, w, x, n, torch.float16)
    ref = oracle.gemm(x.astype(np.float32), 8, p, s.astype(np.float32), 0, n)
    assert_gemv_close(got, ref)


@pytest.mark.parametrize("k,n", synth.Q4_SWEEP)
def test_config2_q4_sweep(ops, oracle, k, n):
    """Q4 group 32, fp16 scales, every sweep shape."""
    import torch
    p, s = synth.q4_weights(n, k, 32, seed=1, tag=(k, n))
    x = synth.activations(k, seed=1, tag=(k, n))
    w = ops.new_int4_weight_only_upload(p, s, n, k, 32)
    got = run_gemv(ops, w, x, n, torch.float16)
    ref = oracle.gemm(x.astype(np.float32), 4, p, s.astype(np.float32), 32, n)
    assert_gemv_close(got, ref)


@pytest.mark.parametrize("bits,k,n,group,sdt", [
    (4, 1024, 256, 16, np.float32),   # reference-native mobile Q4: group 16, fp32 scales
    (4, 2048, 96, 64, np.float16),    # group 64 (scale per two chunks)
    (4, 1024, 72, 1024, np.float32),  # per-row Q4 (float upload path, scaleBlockSize = K)
    (4, 3584, 40, 3584, np.float16),  # per-row, K not a power of two
    (8, 3584, 128, 0, np.float32),    # Q8, K spans several tiles
    (8, 4096, 24, 0, np.float16),
])
def test_fast_kernel_formats(ops, oracle, bits, k, n, group, sdt):
    import torch
    if bits == 4:
        p, s = synth.q4_weights(n, k, group, seed=2, tag=(k, n, group))
        s = s.astype(sdt)
        w = ops.new_int4_weight_only_upload(p, s, n, k, group)
    else:
        p, s = synth.q8_weights(n, k, seed=2, tag=(k, n))
        s = s.astype(sdt)
        w = ops.new_int8_weight_only_upload(p, s, n, k)
    x = synth.activations(k, seed=2, tag=(k,))
    got = run_gemv(ops, w, x, n, torch.float32)
    ref = oracle.gemm(x.astype(np.float32), bits, p, s.astype(np.float32), group, n)
    assert_gemv_close(got, ref)


@pytest.mark.parametrize("k,n", [(1024, 20000), (3584, 19000), (1024, 4100), (1024, 48)])
def test_q4_fp16_int8_path_wide_range_groups(ops, oracle, k, n):
    """fp16 activations on Q4 group-32 weights with N >= 8 x 16 x 148 rows run
    on int8 MMAs with each group as 23-bit fixed point (exact within 2^11 of
    the group maximum); smaller N on the fp16 MMAs. Groups with outliers up to
    2000 times the rest, an all-zero group, subnormals, tiny groups and a
    group of large values up to the fp16 maximum: every row within 3e-5 of
    sum|w s x| of the exact result (the size of fp32 accumulation error), and
    the north-star tolerance. N off the 16-row tile; K = 3584 splits tiles
    over warps."""
    import torch
    p, s = synth.q4_weights(n, k, 32, seed=7, tag=(k, n))
    x = synth.activations(k, seed=7, tag=(k, n)).astype(np.float32)[0]
    x[5] = 1900.0
    x[32 * 3 + 7] = -1024.5
    x[64:96] = 0.0
    x[300] = 3e-6          # fp16 subnormal
    x[301] = -6e-8
    x[32 * 20:32 * 21] = np.clip(x[32 * 20:32 * 21] * 20000.0, -65504.0, 65504.0)
    x[32 * 20 + 1] = 65504.0  # fp16 max in a group of large values
    x[32 * 21:32 * 22] *= 1e-3
    x16 = x.astype(np.float16)
    w = ops.new_int4_weight_only_upload(p, s, n, k, 32)
    got = run_gemv(ops, w, x16.reshape(1, -1), n, torch.float32)[0].astype(np.float64)
    ref = oracle.gemm(x16.reshape(1, -1).astype(np.float32), 4, p, s.astype(np.float32), 32, n)[0].astype(np.float64)
    wq = synth.unpack_q4(p, n, k).astype(np.float64) * np.repeat(s.astype(np.float64).reshape(n, k // 32), 32, 1)
    absum = np.abs(wq * x16.astype(np.float64)[None, :]).sum(1)
    err = np.abs(got - ref)
    assert (err <= 3e-5 * absum).all(), f"worst row {int((err / absum).argmax())}: {(err / absum).max():.3g}"
    assert_gemv_close(got[None, :], ref[None, :])


def test_q4_fp16_nonfinite_activation_gives_nonfinite_rows(ops):
    """An Inf in a group of fp16 activations makes the rows non-finite (the
    reference's fp32 sum would too), not a silently finite number."""
    import torch
    k, n = 1024, 64
    p, s = synth.q4_weights(n, k, 32, seed=8, tag=(k, n))
    x = synth.activations(k, seed=8, tag=(k, n))
    x[0, 40] = np.float16(np.inf)
    w = ops.new_int4_weight_only_upload(p, s, n, k, 32)
    got = run_gemv(ops, w, x, n, torch.float32)[0]
    assert not np.isfinite(got).any()


@pytest.mark.parametrize("bits,k,n,group", [(4, 100, 37, 10), (4, 48, 33, 16), (8, 40, 19, 0), (8, 7, 5, 0),
                                            (4, 5, 3, 5)])
def test_generic_kernel_odd_shapes(ops, oracle, bits, k, n, group):
    """Shapes the streaming kernel cannot take (rows not 16-byte aligned, odd K)
    go through the exact flat-index kernel."""
    import torch
    r = np.random.default_rng(k * 131 + n)
    words = (n * k + (7 if bits == 4 else 3)) // (8 if bits == 4 else 4)
    p = r.integers(0, 2 ** 32, size=words, dtype=np.uint64).astype(np.uint32)
    s = r.uniform(0.002, 0.02, size=(n * k // group) if bits == 4 else n).astype(np.float32)
    w = (ops.new_int4_weight_only_upload(p, s, n, k, group) if bits == 4
         else ops.new_int8_weight_only_upload(p, s, n, k))
    x = synth.activations(k, seed=3, tag=(k,))
    got = run_gemv(ops, w, x, n, torch.float32)
    ref = oracle.gemm(x.astype(np.float32), bits, p, s, group, n)
    assert_gemv_close(got, ref)


@pytest.mark.parametrize("bits,k,n,group,sdt", [(4, 1024, 512, 32, np.float16), (4, 1024, 64, 16, np.float32),
                                                (8, 1024, 300, 0, np.float16), (4, 100, 37, 10, np.float32),
                                                (8, 7, 5, 0, np.float32)])
def test_dequant_bit_exact(ops, oracle, bits, k, n, group, sdt):
    """Every element of AexisGemm2DReadB, bit for bit."""
    import torch
    r = np.random.default_rng(n)
    words = (n * k + (7 if bits == 4 else 3)) // (8 if bits == 4 else 4)
    p = r.integers(0, 2 ** 32, size=words, dtype=np.uint64).astype(np.uint32)
    s = r.uniform(0.002, 0.02, size=(n * k // group) if bits == 4 else n).astype(sdt)
    w = (ops.new_int4_weight_only_upload(p, s, n, k, group) if bits == 4
         else ops.new_int8_weight_only_upload(p, s, n, k))
    out = torch.empty(n * k, dtype=torch.float32, device="cuda")
    ops.dequant(w, out)
    got = out.cpu().numpy().reshape(n, k)
    ref = oracle.dequant(bits, p, s.astype(np.float32), group, n, k)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


@pytest.mark.parametrize("tiled", [False, True])
def test_bias_alpha_beta_rows_and_strides(ops, oracle, tiled):
    """m > 1 with Pack4 row strides, fp32 in/out, bias seeded (linear) or added
    after (tiled), alpha/beta."""
    import torch
    k, n, m = 1024, 250, 3
    p, s = synth.q4_weights(n, k, 32, seed=4)
    w = ops.new_int4_weight_only_upload(p, s, n, k, 32)
    x = synth.activations(k, seed=4, m=m).astype(np.float32)
    bias = np.random.default_rng(4).standard_normal(n).astype(np.float32)
    ld = (n + 3) // 4 * 4 + 4
    xa = torch.zeros((m, k + 12), dtype=torch.float32, device="cuda")
    xa[:, :k] = torch.from_numpy(x).cuda()
    y = torch.zeros((m, ld), dtype=torch.float32, device="cuda")
    b = torch.from_numpy(bias).cuda()
    ops.set_int8_gemm_weights(None)
    ops.set_int4_gemm_weights(w)
    fn = ops.gemm2d_pack4_tiled_texture_a if tiled else ops.gemm2d_pack4_linear_texture_a
    fn(xa, b, m, n, k, True, 0.5, 2.0, True, 4, y)
    torch.cuda.synchronize()
    got = y[:, :n].cpu().numpy()
    ref = oracle.gemm(x, 4, p, s.astype(np.float32), 32, n, bias=bias, alpha=0.5, beta=2.0, tiled=tiled)
    assert_gemv_close(got, ref)
    assert torch.count_nonzero(y[:, n:]).item() == 0  # padding lanes untouched


def test_reference_gemm_known_answer_on_gpu(ops):
    """NcnnInt8WeightOnlyGpuTests.AssertGemmKernel through the GPU path (1e-5)."""
    import torch
    from aiimage_b200.ops import quantize_rows
    inp = np.array([1, -1, 0.5, 2], dtype=np.float32)
    wts = np.array([1, -0.5, 0.25, 2, 0.5, 1, -1, 0.25], dtype=np.float32)
    bias = np.array([0.1, -0.2], dtype=np.float32)
    p, s = quantize_rows(8, wts, 2, 4)
    w = ops.new_int8_weight_only_upload(p, s, 2, 4)
    got = run_gemv(ops, w, inp.reshape(1, 4), 2, torch.float32, bias=bias, x_f32=True)[0]
    f = np.float32
    for oc in range(2):
        q = np.clip(np.rint(wts[oc * 4:oc * 4 + 4] / s[oc]), -127, 127)
        exp = f(bias[oc]) + f(np.sum(inp * q.astype(np.float32) * s[oc], dtype=np.float32))
        assert abs(got[oc] - exp) <= 1e-5


def test_argument_errors(ops):
    import torch
    p, s = synth.q4_weights(64, 64, 32, seed=5)
    w = ops.new_int4_weight_only_upload(p, s, 64, 64, 32)
    ops.set_int8_gemm_weights(None)
    ops.set_int4_gemm_weights(w)
    x = torch.zeros((1, 64), dtype=torch.float16, device="cuda")
    y = torch.zeros((1, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(errors.ArgumentError):
        ops.gemm2d_pack4_linear_texture_a(x, None, 1, 32, 64, output=y)  # n differs from the weight
    with pytest.raises(errors.ArgumentOutOfRangeError):
        ops.gemm2d_pack4_linear_texture_a(x, None, 0, 64, 64, output=y)
    with pytest.raises(errors.ArgumentNullError):
        ops.gemm2d_pack4_linear_texture_a(x, None, 1, 64, 64, use_c=True, output=y)
    with pytest.raises(errors.ArgumentError):
        ops.new_int4_weight_only_upload(p, s, 64, 64, 48)  # group does not divide K
    with pytest.raises(errors.ArgumentError):
        ops.new_int8_weight_only_upload(p, s[:10], 64, 64)


# inputPacked = true (AexisGemm2DPack4LinearTextureAFromPack4): A in a Pack4 texture array
# [slices][height][width][4]. Cases: several slices with m > 1, a ragged last slice (K not a
# multiple of 4*width), texture taller than m, slices beyond K (unused), too few slices (the
# missing K values count as 0), a single slice read in place, and the tensor-core path (Q8, m >= 4).
@pytest.mark.parametrize("bits,k,n,m,width,height,slices,a_f32", [
    (4, 1024, 512, 3, 128, 3, 2, False),     # two slices, exactly full
    (4, 1024, 3072, 2, 96, 5, 3, True),      # ragged last slice, taller texture, fp32 A
    (8, 1024, 3584, 5, 64, 5, 4, False),     # Q8 tensor-core GEMM (m >= 4) behind the gather
    (8, 4096, 96, 2, 200, 2, 6, True),       # more slices than K needs
    (4, 512, 256, 2, 32, 2, 2, False),       # too few slices: K values 256.. read as 0
    (8, 1024, 256, 3, 256, 4, 1, True),      # one slice: read in place, row stride 4 * width
])
def test_gemm_input_packed_pack4_array(ops, oracle, bits, k, n, m, width, height, slices, a_f32):
    import torch
    if bits == 4:
        p, s = synth.q4_weights(n, k, 32, seed=9, tag=(k, n, m))
        w = ops.new_int4_weight_only_upload(p, s, n, k, 32)
        blk = 32
    else:
        p, s = synth.q8_weights(n, k, seed=9, tag=(k, n, m))
        w = ops.new_int8_weight_only_upload(p, s, n, k)
        blk = 0
    rng = np.random.default_rng([k, n, m, width])
    flat = rng.standard_normal(slices * height * width * 4).astype(np.float16)
    bias = rng.standard_normal(n).astype(np.float32)
    a_ref = oracle.read_pack4a(flat.astype(np.float32), width, height, slices, m, k)
    ref = oracle.gemm(a_ref, bits, p, s.astype(np.float32), blk, n, bias=bias, alpha=0.75, beta=0.5)
    a = torch.from_numpy(flat.astype(np.float32) if a_f32 else flat).cuda()
    y = torch.zeros((m, n), dtype=torch.float32, device="cuda")
    b = torch.from_numpy(bias).cuda()
    ops.set_int4_gemm_weights(w if bits == 4 else None)
    ops.set_int8_gemm_weights(w if bits == 8 else None)
    ops.gemm2d_pack4_linear_texture_a(a, b, m, n, k, True, 0.75, 0.5, True, 4, y, input_packed=True,
                                      a_width=width, a_height=height, a_slices=slices)
    torch.cuda.synchronize()
    assert_gemv_close(y.cpu().numpy(), ref)
    if 4 * width < k:
        # The gather must give the same numbers as the linear path on the gathered rows.
        y2 = torch.zeros_like(y)
        a_lin = torch.from_numpy(a_ref.astype(np.float32 if a_f32 else np.float16)).cuda()
        ops.gemm2d_pack4_linear_texture_a(a_lin, b, m, n, k, True, 0.75, 0.5, True, 4, y2)
        torch.cuda.synchronize()
        assert torch.equal(y, y2)


def test_gemm_input_packed_errors(ops):
    import torch
    p, s = synth.q4_weights(64, 256, 32, seed=1)
    w = ops.new_int4_weight_only_upload(p, s, 64, 256, 32)
    ops.set_int4_gemm_weights(w)
    ops.set_int8_gemm_weights(None)
    a = torch.zeros(4096, device="cuda")
    y = torch.zeros((2, 64), device="cuda")
    with pytest.raises(errors.ArgumentError):  # texture shorter than m
        ops.gemm2d_pack4_linear_texture_a(a, None, 2, 64, 256, output=y, input_packed=True, a_width=16,
                                          a_height=1, a_slices=4)
    with pytest.raises(errors.ArgumentError):  # no slices
        ops.gemm2d_pack4_linear_texture_a(a, None, 2, 64, 256, output=y, input_packed=True, a_width=16,
                                          a_height=2, a_slices=0)
    with pytest.raises(errors.ArgumentNullError):
        ops.gemm2d_pack4_linear_texture_a(a, None, 2, 64, 256, output=y, input_packed=True)
    with pytest.raises(errors.ArgumentError):  # weight shape mismatch is caught before the gather
        ops.gemm2d_pack4_linear_texture_a(a, None, 2, 64, 512, output=y, input_packed=True, a_width=16,
                                          a_height=2, a_slices=8)


def test_tiled_from_pack4_matches_tiled_from_linear(ops, oracle):
    """Gemm2DPack4TiledTextureAFromPack4 reads slice 0 of a texture ceil(k/4) (or more) texels wide."""
    import torch
    k, n, m, width = 1000, 300, 3, 260
    p, s = synth.q8_weights(n, k, seed=12)
    w = ops.new_int8_weight_only_upload(p, s, n, k)
    ops.set_int8_gemm_weights(w)
    ops.set_int4_gemm_weights(None)
    rng = np.random.default_rng(12)
    flat = rng.standard_normal(m * width * 4).astype(np.float32)
    bias = rng.standard_normal(n).astype(np.float32)
    ref = oracle.gemm(oracle.read_pack4a(flat, width, m, 1, m, k), 8, p, s.astype(np.float32), 0, n, bias=bias,
                      alpha=1.5, beta=0.25, tiled=True)
    y = torch.zeros((m, n), device="cuda")
    ops.gemm2d_pack4_tiled_texture_a_from_pack4(torch.from_numpy(flat).cuda(), torch.from_numpy(bias).cuda(), m, n,
                                                k, True, 1.5, 0.25, True, 4, y, a_width=width)
    torch.cuda.synchronize()
    assert_gemv_close(y.cpu().numpy(), ref)
