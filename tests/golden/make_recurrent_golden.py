"""Generates tests/golden/recurrent_ops.npz from the reference's own gold operators.

The reference ships fp32 NumPy implementations of the two linear-attention
operators of Qwen3.5 (Tools/Qwen35NcnnBaseline/reference_ops.py:36-152:
`short_conv`, `gated_delta_rule`) and tests them in
Tools/Qwen35NcnnBaseline/tests/test_reference_ops.py. This script imports that
module from a reference checkout (argument or $AEXIS_REFERENCE; it is not
needed at test time), runs it on seeded inputs and stores inputs and outputs
in logical layouts:
  short_conv: weight [groups, kernel], mixed [seq, groups], state [cache, groups]
  gdr:        a_log/dt_bias [heads], a/b [seq, heads], q/k [seq, heads, kdim],
              v [seq, heads, vdim], state [heads, kdim, vdim], out [seq, heads, vdim]
Cases "sc_ref" and "gdr_ref" use the reference test's own seeds and shapes
(ShortConvTests.setUp: default_rng(7); GatedDeltaRuleTests.setUp:
default_rng(11)); the others add ragged widths, explicit initial states, the
minimal (kernel-1) cache and one Qwen3.5-sized head (128 x 128).

Run from the repository root:
  python tests/golden/make_recurrent_golden.py <reference checkout>
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def main(ref_root: str) -> None:
    sys.path.insert(0, os.path.join(ref_root, "Tools", "Qwen35NcnnBaseline"))
    from reference_ops import gated_delta_rule, short_conv

    out = {}

    def sc_case(name, weight, mixed, state, cache_length):
        o, s = short_conv(weight, mixed, state, cache_length=cache_length)
        out[f"{name}/weight"] = weight
        out[f"{name}/mixed"] = mixed
        if state is not None:
            out[f"{name}/state_in"] = state
        out[f"{name}/cache_length"] = np.int32(cache_length)
        out[f"{name}/out"] = o
        out[f"{name}/state_out"] = s

    # ShortConvTests.setUp (test_reference_ops.py:11-14), prefill from no state.
    rng = np.random.default_rng(7)
    weight = rng.normal(0, 0.2, (6, 4)).astype(np.float32)
    values = rng.normal(0, 0.5, (9, 6)).astype(np.float32)
    sc_case("sc_ref", weight, values, None, 4)
    # Same weights, one token with the minimal (kernel - 1) cache from a prefill of 8 tokens.
    _, st = short_conv(weight, values[:8], None, cache_length=3)
    sc_case("sc_ref_decode_min", weight, values[8:], st, 3)
    # Ragged width (37 channels), explicit ncnn-sized cache.
    rng = np.random.default_rng(3)
    sc_case("sc_wide", rng.normal(0, 0.3, (37, 4)).astype(np.float32),
            rng.normal(0, 0.5, (5, 37)).astype(np.float32), rng.normal(0, 0.5, (4, 37)).astype(np.float32), 4)
    # Kernel 3, two tokens, minimal cache.
    rng = np.random.default_rng(4)
    sc_case("sc_k3", rng.normal(0, 0.3, (10, 3)).astype(np.float32),
            rng.normal(0, 0.5, (2, 10)).astype(np.float32), rng.normal(0, 0.5, (2, 10)).astype(np.float32), 2)

    def gdr_case(name, rng, seq, heads, kdim, vdim, state_sigma):
        args = (
            rng.normal(-1.0, 0.2, heads).astype(np.float32),
            rng.normal(0, 0.2, heads).astype(np.float32),
            rng.normal(0, 0.4, (seq, heads)).astype(np.float32),
            rng.normal(0, 0.4, (seq, heads)).astype(np.float32),
            rng.normal(0, 0.5, (seq, heads, kdim)).astype(np.float32),
            rng.normal(0, 0.5, (seq, heads, kdim)).astype(np.float32),
            rng.normal(0, 0.5, (seq, heads, vdim)).astype(np.float32),
        )
        state = None if state_sigma == 0 else rng.normal(0, state_sigma, (heads, kdim, vdim)).astype(np.float32)
        o, s = gated_delta_rule(*args, state)
        for key, val in zip(("a_log", "dt_bias", "b", "a", "q", "k", "v"), args):
            out[f"{name}/{key}"] = val
        out[f"{name}/state_in"] = np.zeros((heads, kdim, vdim), np.float32) if state is None else state
        out[f"{name}/out"] = o
        out[f"{name}/state_out"] = s

    # GatedDeltaRuleTests.setUp (test_reference_ops.py:49-60): seq 8, 3 heads, kdim 5, vdim 4, zero state.
    gdr_case("gdr_ref", np.random.default_rng(11), 8, 3, 5, 4, 0.0)
    gdr_case("gdr_state", np.random.default_rng(5), 6, 2, 32, 20, 0.1)
    gdr_case("gdr_odd", np.random.default_rng(13), 3, 2, 7, 6, 0.2)
    gdr_case("gdr_qwen_head", np.random.default_rng(9), 2, 1, 128, 128, 0.05)

    path = os.path.join(HERE, "recurrent_ops.npz")
    np.savez_compressed(path, **out)
    print(path, os.path.getsize(path), "bytes,", len(out), "arrays")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ["AEXIS_REFERENCE"])
