"""aexis_cuda_argmax_static: the greedy argmax for callers that cannot
allocate device memory (hosts whose engine owns all device memory, or
callbacks that must not block on cudaMalloc / cudaFree). It keeps its keys in
a fixed array inside the library instead of the context's scratch buffer.

This file is collected last so that a run stopping at its first failure has
already run every other test; it passes alone in a fresh process as well.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _static_argmax(logits, rows, width, ld, out, stream):
    from aiimage_b200 import native
    return native.lib().aexis_cuda_argmax_static(C.c_void_p(logits.data_ptr()), rows, width, ld,
                                                  C.c_void_p(out.data_ptr()), C.c_void_p(stream))


def test_static_argmax_matches_context_argmax_twice_in_a_row(ops):
    import torch
    stream = torch.cuda.current_stream().cuda_stream
    r = np.random.default_rng(42)
    for call in range(2):  # the second call must not see the first call's keys
        rows, width = (7, 151936) if call == 0 else (3, 5000)
        x = r.standard_normal((rows, width)).astype(np.float32)
        x[0, 17] = x[0, 4000] = x[0].max() + 1.0  # tie: the lowest index wins
        if call == 1:
            x[1] = -x[1] - 100.0  # much smaller values than the previous call left
        xt = torch.from_numpy(x).cuda()
        ref = torch.zeros(rows, dtype=torch.int32, device="cuda")
        got = torch.full((rows,), -1, dtype=torch.int32, device="cuda")
        ops.arg_max_pack4_linear_mat(xt, width, rows, ref)
        assert _static_argmax(xt, rows, width, width, got, stream) == 0
        torch.cuda.synchronize()
        assert torch.equal(got, ref), (call, got.tolist(), ref.tolist())
        assert got[0].item() == 17


def test_static_argmax_rejects_rows_beyond_its_array():
    import torch
    from aiimage_b200 import native
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    lib = native.lib()
    x = torch.zeros((1, 4), dtype=torch.float32, device="cuda")
    out = torch.zeros(8, dtype=torch.int32, device="cuda")
    too_many = 4097
    assert lib.aexis_cuda_argmax_static(C.c_void_p(x.data_ptr()), too_many, 4, 4, C.c_void_p(out.data_ptr()),
                                        None) == 2
