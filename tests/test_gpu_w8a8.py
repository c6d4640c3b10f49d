"""GPU parity of the W8A8 activation fake-quantisation (aexis_cuda_set_int8_activations,
the Int8W8A8 mode of AexisOps.SetInt8ActivationQuantization, AexisOps.cs:741-785;
HLSL AexisQuantizeGemmActivationForInt8, Pack4Matmul:792-800) through the GEMM
entry points, against the oracle's fake-quantised GEMM.

The codes (q - zp) reach the kernels as exact fp16 integers, so the products are
exact and only the fp32 summation order differs from the reference's: outputs
within the GEMV tolerance of test_gpu_gemv (1e-2 relative + 1e-3 of the largest
output, 2e-3 norm-wise)."""
import types

import numpy as np
import pytest

from aiimage_b200 import errors, synth
from test_gpu_gemv import assert_gemv_close, run_gemv

pytestmark = pytest.mark.gpu


def plan(scale, zp=0):
    return types.SimpleNamespace(mode="Int8W8A8", activation_scale=scale, activation_zero_point=zp)


@pytest.fixture
def w8a8(ops):
    yield ops
    ops.set_int8_activation_quantization(None)


def test_w8a8_known_answer(w8a8):
    """NcnnInt8WeightOnlyGpuTests.AssertGemmW8A8Kernel: activations fake-quantised at scale 0.5 become
    [1, -1, 0.5, 1.5]; y = bias + dot with the dequantised weights, within 1e-5."""
    import torch
    from aiimage_b200.ops import quantize_rows
    ops = w8a8
    inp = np.array([1.1, -0.9, 0.3, 1.7], dtype=np.float32)
    wts = np.array([1, -0.5, 0.25, 2, 0.5, 1, -1, 0.25], dtype=np.float32)
    bias = np.array([0.1, -0.2], dtype=np.float32)
    p, s = quantize_rows(8, wts, 2, 4)
    w = ops.new_int8_weight_only_upload(p, s, 2, 4)
    ops.set_int8_activation_quantization(plan(0.5))
    got = run_gemv(ops, w, inp.reshape(1, 4), 2, torch.float32, bias=bias, x_f32=True)[0]
    qin = np.array([1.0, -1.0, 0.5, 1.5], dtype=np.float32)
    for oc in range(2):
        q = np.clip(np.rint(wts[oc * 4:oc * 4 + 4] / s[oc]), -127, 127)
        exp = np.float32(bias[oc]) + np.float32(np.sum(qin * q.astype(np.float32) * s[oc], dtype=np.float32))
        assert abs(got[oc] - exp) <= 1e-5


@pytest.mark.parametrize("bits,m,k,n,x_f32,tiled", [
    (8, 1, 1024, 3584, False, False),     # config-1 GEMV shape
    (8, 1, 1024, 3584, True, True),       # fp32 activations, lm_head (tiled) epilogue
    (4, 1, 1024, 3072, False, False),     # Q4 g32, fp16-MMA path
    (4, 1, 1024, 19000, False, False),    # Q4 g32, int8-MMA path (large N)
    (8, 3, 1024, 512, True, False),       # several rows through the GEMV
    (8, 32, 1024, 3584, False, False),    # tcgen05 batched GEMM
    (8, 256, 1024, 4096, True, True),     # tcgen05, lm_head epilogue, fp32 activations
    (8, 1, 96, 50, True, False),          # odd shape: codes from the separate kernel, generic GEMV
    (4, 2, 160, 72, False, True),
])
@pytest.mark.parametrize("mode", ["signed", "unsigned", "zero_point"])
def test_w8a8_gemm_against_oracle(w8a8, oracle, bits, m, k, n, x_f32, tiled, mode):
    import torch
    from aiimage_b200.ops import resolve_int8_activation_plan
    ops = w8a8
    rng = np.random.default_rng(bits * 1000 + m + n)
    x = rng.standard_normal((m, k)).astype(np.float16)
    xf = x.astype(np.float32)
    if mode == "unsigned":
        scale, zp, uns = resolve_int8_activation_plan(float(xf.min()), float(xf.max()) * 0.8, True)
        ops.set_int8_activation_quantization(types.SimpleNamespace(minimum=float(xf.min()),
                                                                   maximum=float(xf.max()) * 0.8,
                                                                   packing="Pack4UnsignedInt8"))
    elif mode == "signed":
        scale, zp, uns = resolve_int8_activation_plan(float(xf.min()), float(xf.max()), False)
        ops.set_int8_activation_quantization(types.SimpleNamespace(minimum=float(xf.min()), maximum=float(xf.max()),
                                                                   packing="Pack4Int8"))
    else:
        scale, zp, uns = 0.03, 5, False
        ops.set_int8_activation_quantization(plan(scale, zp))
    if bits == 8:
        p, s = synth.q8_weights(n, k, seed=3, tag=(k, n))
        w = ops.new_int8_weight_only_upload(p, s, n, k)
        blk = 0
    else:
        p, s = synth.q4_weights(n, k, 32, seed=3, tag=(k, n))
        w = ops.new_int4_weight_only_upload(p, s, n, k, 32)
        blk = 32
    bias = rng.normal(0, 0.5, n).astype(np.float32)
    got = run_gemv(ops, w, x, n, torch.float32, bias=bias, alpha=0.75, beta=1.25, tiled=tiled, x_f32=x_f32)
    xq = oracle.quantize_activation_int8(xf, scale, zp, uns).reshape(m, k)
    ref = oracle.gemm(xq, bits, p, s.astype(np.float32), blk, n, bias=bias, alpha=0.75, beta=1.25, tiled=tiled)
    for r in range(m):
        assert_gemv_close(got[r], ref[r])
    # Fake quantisation changes the result: the plain GEMM differs beyond the tolerance somewhere.
    ops.set_int8_activation_quantization(None)
    plain = run_gemv(ops, w, x, n, torch.float32, bias=bias, alpha=0.75, beta=1.25, tiled=tiled, x_f32=x_f32)
    assert np.abs(plain - got).max() > 1e-3 * np.abs(ref).max()


def test_w8a8_argument_errors(w8a8):
    ops = w8a8
    with pytest.raises(errors.ArgumentOutOfRangeError):
        ops.set_int8_activation_quantization(plan(0.0))
    with pytest.raises(errors.ArgumentOutOfRangeError):
        ops.set_int8_activation_quantization(plan(float("inf")))
    with pytest.raises(errors.ArgumentOutOfRangeError):
        ops.set_int8_activation_quantization(plan(0.1, 2000))
    with pytest.raises(errors.InvalidOperationError):
        ops.set_int8_activation_quantization(types.SimpleNamespace(minimum=1.0, maximum=-1.0, packing="Pack4Int8"))
    # A node plan of another mode leaves the activations unquantised (plan.mode != Int8W8A8).
    ops.set_int8_activation_quantization(types.SimpleNamespace(mode="WeightOnlyInt8", activation_scale=0.5,
                                                               activation_zero_point=0))
