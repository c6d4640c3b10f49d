"""GPU parity of the linear-attention decode kernels (k_recurrent.cu) through the
C ABI: aexis_cuda_short_conv (AexisShortConvPack4) and aexis_cuda_gated_delta_rule
(AexisGatedDeltaRulePack4), against the reference's NumPy gold outputs
(tests/golden/recurrent_ops.npz) and the CPU oracle at Qwen3.5 shapes.

Tolerances: ShortConv is a short fp32 sum and one SiLU: 1e-6 relative + 1e-6
absolute. The Gated Delta Rule sums its dot products over key rows in a
different order (per-thread partials, then a shuffle tree) and folds the key
norm after the sum: outputs and states within 1e-5 relative + 1e-5 of the
tensor's largest magnitude, per token over up to 64 recurrent steps."""
import numpy as np
import pytest

from aiimage_b200 import errors
from recurrent_cases import (gdr_out_logical, gdr_state_logical, gdr_storage, golden_cases, random_gdr,
                             short_conv_storage, unpack_rows)

pytestmark = pytest.mark.gpu


def cuda(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


def close(got, ref, rel=1e-5):
    ref = np.asarray(ref, np.float32)
    tol = rel * np.abs(ref) + rel * max(float(np.abs(ref).max()), 1e-6)
    err = np.abs(np.asarray(got, np.float32) - ref)
    assert (err <= tol).all(), f"max err {err.max()} at {np.unravel_index(err.argmax(), err.shape)}"


def run_short_conv(ops, w, mixed, cache, groups, kernel, seq, cache_len, in_place=False):
    import torch
    ld = (groups + 3) // 4 * 4
    out = torch.full((seq * ld,), 7.0, dtype=torch.float32, device="cuda")
    cache_in = cuda(cache)
    cache_out = cache_in if in_place else torch.zeros(max(cache_len, 1) * ld, dtype=torch.float32, device="cuda")
    ops.short_conv_pack4(cuda(w), cuda(mixed), cache_in, out, cache_out, groups, kernel, seq, cache_len)
    return host(out), host(cache_out).ravel()[:cache_len * ld]


@pytest.mark.parametrize("name", sorted(golden_cases("sc_")))
def test_short_conv_reference_gold(ops, oracle, name):
    case = golden_cases("sc_")[name]
    w, mixed, cache, groups, kernel, seq, cl = short_conv_storage(case["weight"], case["mixed"],
                                                                  case.get("state_in"), int(case["cache_length"]))
    out, cache_out = run_short_conv(ops, w, mixed, cache, groups, kernel, seq, cl)
    np.testing.assert_allclose(unpack_rows(out, seq, groups), case["out"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(unpack_rows(cache_out, cl, groups), case["state_out"])
    ref_out, ref_cache = oracle.short_conv(w, mixed, cache, groups, kernel, seq, cl)
    # Pack4 padding lanes (channels past `groups`) are left as they were, as the HLSL leaves them.
    np.testing.assert_allclose(unpack_rows(out, seq, groups), unpack_rows(ref_out, seq, groups), rtol=1e-6,
                               atol=1e-6)
    np.testing.assert_array_equal(unpack_rows(cache_out, cl, groups), unpack_rows(ref_cache, cl, groups))


@pytest.mark.parametrize("seq,cache_len,in_place", [(1, 4, True), (1, 3, False), (33, 4, False), (5, 9, True)])
def test_short_conv_qwen35_shape(ops, oracle, seq, cache_len, in_place):
    """Qwen3.5 linear-attention conv: 6144 channels (q, k, v of 16 heads x 128), kernel 4; decode (one
    token, cache updated in place) and prefill forms."""
    rng = np.random.default_rng(seq * 100 + cache_len)
    groups, kernel = 6144, 4
    weight = rng.normal(0, 0.3, (groups, kernel)).astype(np.float32)
    mixed = rng.normal(0, 1.0, (seq, groups)).astype(np.float32)
    state = rng.normal(0, 1.0, (cache_len, groups)).astype(np.float32)
    w, m, c, g, k, s, cl = short_conv_storage(weight, mixed, state, cache_len)
    out, cache_out = run_short_conv(ops, w, m, c, g, k, s, cl, in_place=in_place)
    ref_out, ref_cache = oracle.short_conv(w, m, c, g, k, s, cl)
    np.testing.assert_allclose(out, ref_out, rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(cache_out, ref_cache.ravel())


def run_gdr(ops, s, first=0, count=None, state=None, out=None, in_place=False):
    import torch
    seq, heads, kdim, vdim = s["seq"], s["heads"], s["kdim"], s["vdim"]
    s4 = (seq + 3) // 4 * 4
    out_t = cuda(np.zeros(s4 * heads * vdim, np.float32) if out is None else out)
    st_in = cuda(s["state"] if state is None else state)
    st_out = st_in if in_place else torch.zeros_like(st_in)
    ops.gated_delta_rule_pack4(cuda(s["a_log"]), cuda(s["dt_bias"]), cuda(s["b"]), cuda(s["a"]), cuda(s["q"]),
                               cuda(s["k"]), cuda(s["v"]), st_in, out_t, st_out, heads, kdim, vdim, seq,
                               token_index=first, token_count=count)
    return host(out_t), host(st_out)


@pytest.mark.parametrize("name", sorted(golden_cases("gdr_")))
def test_gated_delta_rule_reference_gold(ops, oracle, name):
    case = golden_cases("gdr_")[name]
    s = gdr_storage(case)
    out, state = run_gdr(ops, s)
    close(gdr_out_logical(out, s["seq"], s["heads"], s["vdim"]), case["out"])
    close(gdr_state_logical(state, s["heads"], s["kdim"], s["vdim"]), case["state_out"])
    ref_out, ref_state = oracle.gated_delta_rule(s["a_log"], s["dt_bias"], s["b"], s["a"], s["q"], s["k"], s["v"],
                                                 s["state"], s["heads"], s["kdim"], s["vdim"], s["seq"])
    close(out, ref_out)
    close(state, ref_state)


@pytest.mark.parametrize("seq,heads,kdim,vdim", [(1, 16, 128, 128), (64, 16, 128, 128), (5, 3, 256, 36),
                                                 (9, 2, 48, 24), (2, 4, 200, 130)])
def test_gated_delta_rule_against_oracle(ops, oracle, seq, heads, kdim, vdim):
    """Qwen3.5-0.8B's linear attention (16 heads, key/value dims 128): one decode token and a 64-token
    prefill in one call; plus ragged dims (every row-per-thread template, value dims not a multiple of 16 or 4)."""
    s = gdr_storage(random_gdr(np.random.default_rng(seq * 7 + kdim), seq, heads, kdim, vdim))
    out, state = run_gdr(ops, s)
    ref_out, ref_state = oracle.gated_delta_rule(s["a_log"], s["dt_bias"], s["b"], s["a"], s["q"], s["k"], s["v"],
                                                 s["state"], heads, kdim, vdim, seq)
    close(out, ref_out)
    close(state, ref_state)


def test_gated_delta_rule_per_token_calls_equal_one_call(ops):
    """The reference's layer loop (one GatedDeltaRulePack4 per token, ping-pong states) and one call over the
    sequence give identical bits; the state may also be updated in place."""
    s = gdr_storage(random_gdr(np.random.default_rng(4), 6, 16, 128, 128))
    full_out, full_state = run_gdr(ops, s)
    out, state = None, None
    for t in range(s["seq"]):
        out, state = run_gdr(ops, s, first=t, count=1, state=state, out=out, in_place=(t % 2 == 1))
    np.testing.assert_array_equal(out, full_out)
    np.testing.assert_array_equal(state, full_state)


def test_recurrent_argument_errors(ops):
    import torch
    f = torch.zeros(4096, dtype=torch.float32, device="cuda")
    with pytest.raises(errors.ArgumentNullError):
        ops.short_conv_pack4(None, f, f, f, f, 4, 4, 1, 4)
    with pytest.raises(errors.ArgumentOutOfRangeError):
        ops.short_conv_pack4(f, f[1024:], f[2048:], f[3072:], f[2048:], 4, 4, 1, 2)   # cache < kernel - 1
    with pytest.raises(errors.NotSupportedError):
        ops.short_conv_pack4(f, f[1024:], f[2048:], f[3072:], f[2048:], 4, 17, 1, 16)
    with pytest.raises(errors.ArgumentError):
        ops.short_conv_pack4(f, f[1024:], f[2048:], f[1024:], f[2048:], 4, 4, 1, 4)  # out aliases mixed
    v = [f[i * 256:] for i in range(10)]
    with pytest.raises(errors.ArgumentNullError):
        ops.gated_delta_rule_pack4(None, *v[1:], 1, 4, 4, 1)
    with pytest.raises(errors.ArgumentOutOfRangeError):
        ops.gated_delta_rule_pack4(*v, 1, 4, 4, 2, token_index=1, token_count=2)
    with pytest.raises(errors.NotSupportedError):
        ops.gated_delta_rule_pack4(*v, 1, 257, 4, 1)
    with pytest.raises(errors.ArgumentError):
        ops.gated_delta_rule_pack4(*v[:7], f[1:], v[8], v[9], 1, 4, 4, 1)          # misaligned state
    ops.sync()
