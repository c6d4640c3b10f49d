"""The reference's own known-answer tests, restated against the CPU oracle.

These pin the oracle before any GPU result is compared with it. Sources
(paths under Packages/com.aexis/Samples/AIImageApplicationExample/Editor/):
  NcnnInt8WeightOnlyTests.cs:51-86      int8 packing known answer
  NcnnInt8WeightOnlyGpuTests.cs:67-192  Gemm Q8 + bias (and W8A8) vs DotDequantized
  Qwen35Q8ArchiveTests.cs:14-123        argmax 13 of 17, tiled Pack4 34 of 37
  NcnnLinearCmdPack4GoldenTests.cs:96-176,248-367,722-728,1130-1257
                                        SDPA mask+causal, KV concat + causal offset
"""
import math

import numpy as np
import pytest


def create_values(count, scale, period):
    """CreateValues (NcnnLinearCmdPack4GoldenTests.cs:722-728), fp32 like C#."""
    i = np.arange(count, dtype=np.int64)
    return (((i * 7) % period - period // 2).astype(np.float32) * np.float32(scale)).astype(np.float32)


def planar_to_pack4(planar, w, h, c):
    """FillPack4FromBufferCDHW: planar [c][h][w] -> Pack4 CDHW."""
    slices = (c + 3) // 4
    out = np.zeros(slices * h * w * 4, dtype=np.float32)
    p = planar.reshape(c, h, w)
    for ch in range(c):
        for y in range(h):
            for x in range(w):
                out[(((ch // 4) * h + y) * w + x) * 4 + (ch & 3)] = p[ch, y, x]
    return out


def pack4_to_planar(packed, w, h, c):
    out = np.zeros((c, h, w), dtype=np.float32)
    for ch in range(c):
        for y in range(h):
            for x in range(w):
                out[ch, y, x] = packed[(((ch // 4) * h + y) * w + x) * 4 + (ch & 3)]
    return out.reshape(-1)


def reference_sdpa_with_cache(q, k, v, qlen, klen, embed, heads, scale, causal, offset, mask=None):
    """ReferenceSdpa / ReferenceSdpaWithCache (GoldenTests.cs:1130-1230), fp32."""
    f = np.float32
    out = np.zeros(heads * qlen * embed, dtype=np.float32)
    idx = lambda w, h, x, y, c: (c * h + y) * w + x  # Index(w, h, 1, c, x, y, 0, c)
    for head in range(heads):
        for row in range(qlen):
            scores = np.zeros(klen, dtype=np.float32)
            for col in range(klen):
                s = f(0)
                for i in range(embed):
                    s = f(s + f(q[idx(embed, qlen, i, row, head)] * k[idx(embed, klen, i, col, head)]))
                if causal and col > row + offset:
                    s = f(-1e20)
                else:
                    s = f(s * f(scale))
                    if mask is not None:
                        s = f(s + mask[col + row * klen])
                scores[col] = s
            mx = scores.max()
            e = np.exp((scores - mx).astype(np.float64)).astype(np.float32)
            tot = f(e.sum(dtype=np.float32))
            for ox in range(embed):
                acc = f(0)
                for col in range(klen):
                    acc = f(acc + f(f(e[col] / tot) * v[idx(embed, klen, ox, col, head)]))
                out[idx(embed, qlen, ox, row, head)] = acc
    return out


def test_int8_packing_known_answer(oracle):
    """NcnnInt8WeightOnlyTests.WeightPacker_UsesPerOutputChannelSymmetricInt8WithoutFloatExpansion."""
    src = np.array([-2, -1, 0, 1, 0.25, -0.5, 0.75, -1], dtype=np.float32)
    packed, scales = oracle.quantize_rows(8, src, 2, 4, True)
    assert abs(scales[0] - 2 / 127) <= 1e-7 and abs(scales[1] - 1 / 127) <= 1e-7
    b = packed.view(np.uint8)
    assert list(b[:4]) == [(-127) & 0xFF, (-64) & 0xFF, 0, 64]
    assert list(b[4:8]) == [32, (-64) & 0xFF, 95, (-127) & 0xFF]


def test_product_quantizer_matches_known_answer_and_oracle(oracle):
    """The library's host quantizer (aexis_quantize_q{8,4}_rows) is bit-exact
    with the oracle, including the known answer and midpoint-to-even ties."""
    from aiimage_b200.ops import quantize_rows
    src = np.array([-2, -1, 0, 1, 0.25, -0.5, 0.75, -1], dtype=np.float32)
    p, s = quantize_rows(8, src, 2, 4)
    po, so = oracle.quantize_rows(8, src, 2, 4, True)
    assert np.array_equal(p, po) and np.array_equal(s, so)
    r = np.random.default_rng(5)
    for bits in (4, 8):
        for contiguous in (True, False):
            data = (r.standard_normal(37 * 24) * 3).astype(np.float32)
            data[::7] = np.round(data[::7] * 2) / 2  # exact .5 multiples exercise the tie rule
            data[:24] = 0.0  # an all-zero channel takes scale 1
            p, s = quantize_rows(bits, data, 37, 24, contiguous)
            po, so = oracle.quantize_rows(bits, data, 37, 24, contiguous)
            assert np.array_equal(p, po), (bits, contiguous)
            assert np.array_equal(s, so), (bits, contiguous)


def test_round_to_int_is_midpoint_to_even(oracle):
    # 2.5 -> 2, 3.5 -> 4, -0.5 -> 0, -1.5 -> -2 (Mathf.RoundToInt = Math.Round).
    data = np.array([2.5, 3.5, -0.5, -1.5, 127.0], dtype=np.float32)  # scale = 127/127 = 1
    packed, scales = oracle.quantize_rows(8, data, 1, 5, True)
    assert scales[0] == 1.0
    assert list(packed.view(np.int8)[:5]) == [2, 4, 0, -2, 127]


def dot_dequantized(inp, weights, oc, per):
    """DotDequantized (NcnnInt8WeightOnlyGpuTests.cs:167-181), fp32."""
    f = np.float32
    start = oc * per
    max_abs = max(abs(float(x)) for x in weights[start:start + per])
    scale = f(max_abs / f(127)) if max_abs > 0 else f(1)
    total = f(0)
    for i in range(per):
        q = int(np.clip(np.rint(f(weights[start + i] / scale)), -127, 127))
        total = f(total + f(f(inp[i] * f(q)) * scale))
    return total


def test_gemm_q8_bias_known_answer(oracle):
    """NcnnInt8WeightOnlyGpuTests.AssertGemmKernel: 1e-5 absolute."""
    inp = np.array([1, -1, 0.5, 2], dtype=np.float32)
    w = np.array([1, -0.5, 0.25, 2, 0.5, 1, -1, 0.25], dtype=np.float32)
    bias = np.array([0.1, -0.2], dtype=np.float32)
    packed, scales = oracle.quantize_rows(8, w, 2, 4, True)
    y = oracle.gemm(inp, 8, packed, scales, 0, 2, bias=bias, alpha=1.0, beta=1.0)[0]
    for oc in range(2):
        assert abs(y[oc] - (bias[oc] + dot_dequantized(inp, w, oc, 4))) <= 1e-5


def test_gemm_w8a8_known_answer(oracle):
    """NcnnInt8WeightOnlyGpuTests.AssertGemmW8A8Kernel: activations fake-quantised at scale 0.5."""
    inp = np.array([1.1, -0.9, 0.3, 1.7], dtype=np.float32)
    w = np.array([1, -0.5, 0.25, 2, 0.5, 1, -1, 0.25], dtype=np.float32)
    bias = np.array([0.1, -0.2], dtype=np.float32)
    qin = oracle.quantize_activation_int8(inp, 0.5)
    assert list(qin) == [1.0, -1.0, 0.5, 1.5]
    packed, scales = oracle.quantize_rows(8, w, 2, 4, True)
    y = oracle.gemm(qin, 8, packed, scales, 0, 2, bias=bias)[0]
    for oc in range(2):
        assert abs(y[oc] - (bias[oc] + dot_dequantized(qin, w, oc, 4))) <= 1e-5


def test_argmax_known_answers(oracle):
    """Qwen35Q8ArchiveTests: 13 of 17 (values -i), tiled Pack4 34 of 37."""
    v = -np.arange(17, dtype=np.float32)
    v[13] = 100
    assert oracle.argmax(v)[0] == 13
    packs = (37 + 3) // 4
    tiled = np.zeros(packs * 4, dtype=np.float32)
    for p in range(packs):
        tiled[p * 4:p * 4 + 4] = [-(p * 4 + 1), -(p * 4 + 2), -(p * 4 + 3), -(p * 4 + 4)]
    tiled[34] = 100
    assert oracle.argmax(tiled[:37].copy())[0] == 34


def test_argmax_first_max_wins(oracle):
    v = np.array([1, 3, 3, 2, 3], dtype=np.float32)
    assert oracle.argmax(v)[0] == 1
    assert oracle.argmax(np.array([np.nan, 5, 6], dtype=np.float32))[0] == 0
    assert oracle.argmax(np.array([1, np.nan, 6], dtype=np.float32))[0] == 2


def test_sdpa_mask_and_causal_golden(oracle):
    """CommandBufferPack4_SdpaMaskAndCausalMatchFp32Oracle (3e-4)."""
    seq, embed, heads = 3, 3, 2
    q = create_values(heads * seq * embed, 0.07, 3)
    k = create_values(heads * seq * embed, 0.05, 5)
    v = create_values(heads * seq * embed, 0.11, 7)
    mask = np.array([0, -0.25, -1.5, 0, 0, -0.5, 0.1, 0, 0], dtype=np.float32)
    scale = 1.0 / math.sqrt(embed)
    expected = reference_sdpa_with_cache(q, k, v, seq, seq, embed, heads, scale, True, 0, mask)
    mask_p4 = planar_to_pack4(mask, seq, seq, 1)
    out = oracle.sdpa(planar_to_pack4(q, embed, seq, heads), planar_to_pack4(k, embed, seq, heads),
                      planar_to_pack4(v, embed, seq, heads), seq, seq, embed, embed, heads, heads, scale,
                      mask=mask_p4, mask_w=seq, mask_h=seq, causal=True)
    got = pack4_to_planar(out, embed, seq, heads)
    assert np.max(np.abs(got - expected)) <= 3e-4


def test_sdpa_kv_cache_concat_causal_offset_golden(oracle):
    """CommandBufferPack4_SdpaKvCacheConcatAndCausalOffsetMatchFp32Oracle (3e-4 / 1e-5)."""
    past, cur, embed, heads = 3, 2, 3, 5
    total = past + cur
    q = create_values(heads * cur * embed, 0.07, 3)
    pk = create_values(heads * past * embed, 0.05, 5)
    ck = create_values(heads * cur * embed, 0.04, 11)
    pv = create_values(heads * past * embed, 0.11, 7)
    cv = create_values(heads * cur * embed, 0.09, 13)

    def concat_ref(a, b):
        out = np.zeros(embed * total * heads, dtype=np.float32)
        for c in range(heads):
            for y in range(total):
                for x in range(embed):
                    out[(c * total + y) * embed + x] = (a[(c * past + y) * embed + x] if y < past
                                                        else b[(c * cur + y - past) * embed + x])
        return out

    ek, ev = concat_ref(pk, ck), concat_ref(pv, cv)
    scale = 1.0 / math.sqrt(embed)
    expected = reference_sdpa_with_cache(q, ek, ev, cur, total, embed, heads, scale, True, past)
    w = embed
    kc = oracle.concat_sequence(planar_to_pack4(pk, w, past, heads), past, planar_to_pack4(ck, w, cur, heads), cur,
                                w, (heads + 3) // 4, total)
    vc = oracle.concat_sequence(planar_to_pack4(pv, w, past, heads), past, planar_to_pack4(cv, w, cur, heads), cur,
                                w, (heads + 3) // 4, total)
    assert np.max(np.abs(pack4_to_planar(kc, w, total, heads) - ek)) <= 1e-5
    assert np.max(np.abs(pack4_to_planar(vc, w, total, heads) - ev)) <= 1e-5
    out = oracle.sdpa(planar_to_pack4(q, w, cur, heads), kc, vc, cur, total, embed, embed, heads, heads, scale,
                      causal=True, causal_offset=past)
    assert np.max(np.abs(pack4_to_planar(out, w, cur, heads) - expected)) <= 3e-4


def test_rmsnorm_formula(oracle):
    x = np.random.default_rng(1).standard_normal((3, 37)).astype(np.float32)
    g = np.random.default_rng(2).standard_normal(37).astype(np.float32)
    y = oracle.rmsnorm(x, g, eps=1e-6)
    ref = x / np.sqrt(np.maximum((x.astype(np.float64) ** 2).mean(1, keepdims=True) + 1e-6, 1e-20)) * g
    assert np.allclose(y, ref, rtol=1e-5, atol=1e-6)
    # affine_size 1 broadcasts gamma[0] (the clamp in the kernel).
    y1 = oracle.rmsnorm(x, g, eps=1e-6, affine_size=1)
    assert np.allclose(y1, y / g * g[0], rtol=1e-5, atol=1e-6)


def test_rope_rotate_half_and_interleaved(oracle):
    E, L, H = 8, 3, 5
    src_planar = np.random.default_rng(3).standard_normal(H * L * E).astype(np.float32)
    cos, sin = oracle.rope_tables(L, E, 1e4)
    out = pack4_to_planar(oracle.rope(planar_to_pack4(src_planar, E, L, H), E, L, H, cos, sin, False), E, L, H)
    x = src_planar.reshape(H, L, E)
    half = E // 2
    ref = np.concatenate([x[..., :half] * cos - x[..., half:] * sin, x[..., :half] * sin + x[..., half:] * cos], -1)
    assert np.allclose(out.reshape(H, L, E), ref, atol=1e-6)
    out_i = pack4_to_planar(oracle.rope(planar_to_pack4(src_planar, E, L, H), E, L, H, cos, sin, True), E, L, H)
    ev, od = x[..., 0::2], x[..., 1::2]
    ref_i = np.empty_like(x)
    ref_i[..., 0::2] = ev * cos - od * sin
    ref_i[..., 1::2] = ev * sin + od * cos
    assert np.allclose(out_i.reshape(H, L, E), ref_i, atol=1e-6)


def test_fp16_rounding_matches_ieee(oracle):
    r = np.random.default_rng(4)
    vals = np.concatenate([r.standard_normal(20000).astype(np.float32) * 10.0 ** r.integers(-9, 5, 20000),
                           np.array([65504, 65519.99, 65520, 1e-8, 2.98e-8, 2.99e-8, -0.0, np.inf, -np.inf],
                                    dtype=np.float32)]).astype(np.float32)
    got = oracle.round_f16(vals)
    ref = vals.astype(np.float16).astype(np.float32)
    assert np.array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_dequant_indexing_matches_numpy_unpack(oracle):
    """AexisGemm2DReadB indexing against an independent numpy unpack."""
    from aiimage_b200 import synth
    n, k = 24, 64
    p4, s4 = synth.q4_weights(n, k, 16, seed=9)
    deq = oracle.dequant(4, p4, s4.astype(np.float32), 16, n, k)
    q = synth.unpack_q4(p4, n, k).astype(np.float32)
    ref = q * np.repeat(s4.astype(np.float32).reshape(n, k // 16), 16, axis=1)
    assert np.array_equal(deq, ref)
    p8, s8 = synth.q8_weights(n, k, seed=9)
    deq8 = oracle.dequant(8, p8, s8.astype(np.float32), 0, n, k)
    assert np.array_equal(deq8, synth.unpack_q8(p8, n, k).astype(np.float32) * s8.astype(np.float32)[:, None])


def test_sweep_byte_counts_match_baseline():
    """The algorithmic byte counts behind roofline.achieved (BASELINE config 2 / 1)."""
    from aiimage_b200 import synth
    expected = {(1024, 3072): 1777664, (1024, 512): 297984, (1024, 3584): 2073600, (3584, 1024): 2073600,
                (1024, 151936): 87821056}
    for (k, n), b in expected.items():
        assert synth.gemv_bytes(4, n, k, 32) == b
    assert synth.gemv_bytes(8, 3584, 1024) == 3686400
