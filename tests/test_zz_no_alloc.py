"""aexis_cuda_argmax_static: the greedy argmax for callers that cannot
allocate device memory (hosts whose engine owns all device memory, or
callbacks that must not block on cudaMalloc / cudaFree). It keeps its keys in
a fixed array inside the library instead of the context's scratch buffer.

Checked against an independent NumPy restatement of the reference's scan
(AexisArgMaxPack4LinearMat, HLSL Pack4Matmul:645-686: first index of the
maximum by strict >, -0 equal to +0, a NaN never wins unless it sits at index
0, where the scan starts) and against the context entry point.

This file is collected last so that a run stopping at its first failure has
already run every other test; it passes alone in a fresh process as well.
"""
import ctypes as C

import numpy as np
import pytest

from aiimage_b200 import native

pytestmark = pytest.mark.gpu

MAX_ROWS = native.header_constant("AEXIS_ARGMAX_STATIC_MAX_ROWS")
E_RANGE = native.header_constant("AEXIS_E_RANGE")
E_SHAPE = native.header_constant("AEXIS_E_SHAPE")


def reference_scan(x: np.ndarray) -> np.ndarray:
    """Per row: best = x[0]; for i >= 1, take i when x[i] > best (a NaN compares false)."""
    out = np.zeros(x.shape[0], dtype=np.int32)
    for r, row in enumerate(x):
        if np.isnan(row[0]):
            continue  # nothing compares greater than NaN: index 0 stays
        finite = np.where(np.isnan(row), -np.inf, row)
        best = finite.max()
        if best == row[0] or (best == 0 and row[0] == 0):
            continue
        out[r] = int(np.flatnonzero(finite == best)[0])
    return out


def _static_argmax(logits, rows, width, ld, out, stream):
    return native.lib().aexis_cuda_argmax_static(C.c_void_p(logits.data_ptr()), rows, width, ld,
                                                  C.c_void_p(out.data_ptr()), C.c_void_p(stream))


def test_static_argmax_matches_reference_scan_twice_in_a_row(ops):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    r = np.random.default_rng(42)
    for call in range(2):  # the second call must not see the first call's keys
        rows, width, ld = (7, 151936, 151936) if call == 0 else (5, 5000, 5003)  # ld > width on the second
        x = np.full((rows, ld), 1e30, dtype=np.float32)  # padding past width must be ignored
        x[:, :width] = r.standard_normal((rows, width)).astype(np.float32)
        x[0, 17] = x[0, 4000] = x[0, :width].max() + 1.0  # tie: the lowest index wins
        x[1, :width] = -np.abs(x[1, :width]) - 100.0  # much smaller values than a previous call left
        x[2, 0] = np.nan  # NaN at index 0 wins the scan
        x[3, 5] = np.nan
        x[3, 9] = x[3, :width][~np.isnan(x[3, :width])].max() + 2.0  # a NaN elsewhere never wins
        x[4, :width] = -0.0
        x[4, 3] = 0.0  # +0 after -0 at index 0: equal, index 0 stays
        xt = torch.from_numpy(x).cuda()
        ref = torch.zeros(rows, dtype=torch.int32, device="cuda")
        got = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        ops.arg_max_pack4_linear_mat(xt, width, rows, ref, ld=ld)
        assert _static_argmax(xt, rows, width, ld, got, stream) == 0
        torch.cuda.synchronize()
        want = reference_scan(x[:, :width])
        assert got.cpu().numpy().tolist() == want.tolist(), (call, got.tolist(), want.tolist())
        assert torch.equal(got, ref)
        assert got[0].item() == 17 and got[2].item() == 0 and got[3].item() == 9 and got[4].item() == 0


def test_static_argmax_full_array_and_argument_errors():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    lib = native.lib()
    r = np.random.default_rng(7)
    x = r.standard_normal((MAX_ROWS, 64)).astype(np.float32)
    xt = torch.from_numpy(x).cuda()
    out = torch.zeros(MAX_ROWS + 1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    assert _static_argmax(xt, MAX_ROWS, 64, 64, out, stream) == 0  # exactly the array's size
    torch.cuda.synchronize()
    assert out[:MAX_ROWS].cpu().numpy().tolist() == reference_scan(x).tolist()
    p = lambda t: C.c_void_p(t.data_ptr())
    assert lib.aexis_cuda_argmax_static(p(xt), MAX_ROWS + 1, 64, 64, p(out), None) == E_RANGE
    assert lib.aexis_cuda_argmax_static(p(xt), 4, 64, 63, p(out), None) == E_SHAPE
