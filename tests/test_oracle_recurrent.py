"""Pins the oracle's ShortConv and GatedDeltaRule (restatements of the HLSL
kernels AexisShortConvPack4 / AexisGatedDeltaRulePack4, AexisCommon.compute:
623-753) against the reference's own fp32 NumPy operators
(Tools/Qwen35NcnnBaseline/reference_ops.py:36-152), whose outputs are stored
in tests/golden/recurrent_ops.npz, and restates the reference's operator
tests (Tools/Qwen35NcnnBaseline/tests/test_reference_ops.py) on the oracle."""
import numpy as np
import pytest

from recurrent_cases import (gdr_out_logical, gdr_state_logical, gdr_storage, golden_cases, random_gdr,
                             short_conv_storage, unpack_rows)


@pytest.mark.parametrize("name", sorted(golden_cases("sc_")))
def test_short_conv_oracle_matches_reference_gold(oracle, name):
    case = golden_cases("sc_")[name]
    cache_len = int(case["cache_length"])
    w, mixed, cache, groups, kernel, seq, cl = short_conv_storage(case["weight"], case["mixed"],
                                                                  case.get("state_in"), cache_len)
    out, cache_out = oracle.short_conv(w, mixed, cache, groups, kernel, seq, cl)
    # The reference's own tolerance between its prefill and decode forms (test_reference_ops.py:22).
    np.testing.assert_allclose(unpack_rows(out, seq, groups), case["out"], rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(unpack_rows(cache_out, cl, groups), case["state_out"])


@pytest.mark.parametrize("name", sorted(golden_cases("gdr_")))
def test_gated_delta_rule_oracle_matches_reference_gold(oracle, name):
    case = golden_cases("gdr_")[name]
    s = gdr_storage(case)
    out, state = oracle.gated_delta_rule(s["a_log"], s["dt_bias"], s["b"], s["a"], s["q"], s["k"], s["v"],
                                         s["state"], s["heads"], s["kdim"], s["vdim"], s["seq"])
    np.testing.assert_allclose(gdr_out_logical(out, s["seq"], s["heads"], s["vdim"]), case["out"],
                               rtol=1e-5, atol=2e-6)
    np.testing.assert_allclose(gdr_state_logical(state, s["heads"], s["kdim"], s["vdim"]), case["state_out"],
                               rtol=1e-5, atol=2e-6)
    # Columns past vdim (Pack4 padding) stay zero when they start at zero.
    pad = np.asarray(state).reshape(s["heads"], s["kdim"], -1)[:, :, s["vdim"]:]
    assert not pad.any()


def test_gated_delta_rule_oracle_token_by_token_equals_prefill(oracle):
    """GatedDeltaRuleTests.test_prefill_matches_token_decode and test_cache_continuity
    (test_reference_ops.py:62-81), restated on the oracle's per-token dispatch."""
    s = gdr_storage(random_gdr(np.random.default_rng(21), 7, 2, 16, 12))
    full_out, full_state = oracle.gated_delta_rule(s["a_log"], s["dt_bias"], s["b"], s["a"], s["q"], s["k"], s["v"],
                                                   s["state"], s["heads"], s["kdim"], s["vdim"], s["seq"])
    out, state = None, s["state"]
    for t in range(s["seq"]):
        out, state = oracle.gated_delta_rule(s["a_log"], s["dt_bias"], s["b"], s["a"], s["q"], s["k"], s["v"],
                                             state, s["heads"], s["kdim"], s["vdim"], s["seq"], first=t, count=1,
                                             out=out)
    np.testing.assert_array_equal(out, full_out)
    np.testing.assert_array_equal(state, full_state)


def test_short_conv_oracle_decode_equals_prefill(oracle):
    """ShortConvTests.test_prefill_matches_token_decode_for_ncnn_cache (test_reference_ops.py:16-24)."""
    rng = np.random.default_rng(7)
    weight = rng.normal(0, 0.2, (6, 4)).astype(np.float32)
    values = rng.normal(0, 0.5, (9, 6)).astype(np.float32)
    w, mixed, cache, groups, kernel, seq, cl = short_conv_storage(weight, values, None, 4)
    full_out, full_cache = oracle.short_conv(w, mixed, cache, groups, kernel, seq, cl)
    rows = []
    for t in range(seq):
        o, cache = oracle.short_conv(w, mixed[t:t + 1], cache, groups, kernel, 1, cl)
        rows.append(unpack_rows(o, 1, groups))
    np.testing.assert_allclose(np.concatenate(rows), unpack_rows(full_out, seq, groups), rtol=0, atol=0)
    np.testing.assert_array_equal(cache, full_cache)
