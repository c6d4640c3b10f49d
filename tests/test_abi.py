"""CPU-only checks of the C ABI: the library loads, exports every entry point
include/aexis_cuda.h declares, and rejects bad arguments with status codes
(no kernel is launched here)."""
import ctypes as C
import subprocess

import numpy as np
import pytest

from aiimage_b200 import native


def test_library_exports_every_declared_symbol():
    declared = native.declared_functions()
    assert len(declared) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", native.LIB_PATH], capture_output=True, text=True,
                         check=True).stdout
    exported = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    missing = [f for f in declared if f not in exported]
    assert not missing, missing
    # Nothing but the ABI is exported (internal symbols stay hidden).
    extra = sorted(s for s in exported if s.startswith("aexis") and s not in declared)
    assert not extra, extra


def test_binding_table_covers_header():
    assert sorted(native.SIGNATURES) == native.declared_functions()
    lib = native.lib()
    assert lib.aexis_cuda_abi_version() == 1


def test_null_context_is_rejected_everywhere():
    lib = native.lib()
    null = None
    assert lib.aexis_cuda_destroy(null) == 1
    assert lib.aexis_cuda_sync(null) == 1
    assert lib.aexis_cuda_gemm(null, None, 0, 1, 1, 1, None, None, 1.0, 1.0, None, 0, 1, 1) == 1
    assert lib.aexis_cuda_rmsnorm(null, None, 0, 1, 1, 1, None, 0, 1e-6, None, 0) == 1
    assert lib.aexis_cuda_sdpa(null, None, None, None, 1, 1, 1, 1, 1, 1, 1.0, None, 0, 0, 0, 0, None) == 1
    assert lib.aexis_cuda_argmax(null, None, 1, 1, 1, None) == 1
    assert lib.aexis_cuda_decoder_step(null, 0, None) == 1
    assert lib.aexis_cuda_decoder_destroy(null) == 1
    assert lib.aexis_cuda_weights_free(null, None) == 1


def test_host_quantizer_argument_errors():
    lib = native.lib()
    d = np.zeros(8, dtype=np.float32)
    p = np.zeros(2, dtype=np.uint32)
    s = np.zeros(2, dtype=np.float32)
    ptr = lambda a: a.ctypes.data_as(C.c_void_p)
    assert lib.aexis_quantize_q8_rows(None, 2, 4, 1, ptr(p), ptr(s)) == 1
    assert lib.aexis_quantize_q8_rows(ptr(d), 0, 4, 1, ptr(p), ptr(s)) == 2
    assert lib.aexis_quantize_q8_rows(ptr(d), 2, 0, 1, ptr(p), ptr(s)) == 3
    assert lib.aexis_quantize_q4_rows(ptr(d), 2, 4, 1, ptr(p), ptr(s)) == 0


def test_create_without_a_gpu_reports_cuda_error():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present; covered by the gpu tests")
    ctx = C.c_void_p()
    st = native.lib().aexis_cuda_create(0, C.byref(ctx))
    assert st in (2, 6)
    assert not ctx.value
    assert native.lib().aexis_cuda_last_error(None)
