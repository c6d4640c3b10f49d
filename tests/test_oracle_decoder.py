"""The decoder oracle on a tiny model: determinism, prefill/step equivalence,
and agreement with a decoder built from the single-op oracles."""
import math

import numpy as np
import pytest

from aiimage_b200 import synth


@pytest.fixture(scope="module")
def tiny():
    return synth.SyntheticDecoder(synth.TINY, seed=11)


def test_oracle_decoder_is_deterministic(oracle, tiny):
    a = oracle.OracleDecoder(tiny)
    toks1, m1 = a.generate(tiny.prompt(8), 12)
    a.reset()
    toks2, m2 = a.generate(tiny.prompt(8), 12)
    assert toks1 == toks2 and m1 == m2
    assert a.position == 8 + 12 - 1


def test_oracle_decoder_matches_composed_ops(oracle, tiny):
    """One step of oracle_decoder_step equals the same layers composed from the
    single-op oracles in numpy (embed, RMSNorm, Gemm, RoPE, SDPA, SwiGLU)."""
    c = tiny.cfg
    dec = oracle.OracleDecoder(tiny)
    prompt = tiny.prompt(5)
    for t in prompt[:-1]:
        dec.step(int(t), want_logits=False)
    _, logits, _ = dec.step(int(prompt[-1]))

    D, NH, KVH = c.head_dim, c.n_heads, c.n_kv_heads
    cos, sin = oracle.rope_tables(c.kv_capacity, c.rot_dim, c.rope_theta)
    kc = np.zeros((c.n_layers, KVH, len(prompt), D), dtype=np.float32)
    vc = np.zeros_like(kc)

    def lin(layer, which, x):
        p, s = tiny.linear(layer, which)
        n, k = (c.shapes()[which] if layer >= 0 else (c.vocab, c.hidden))
        bits = c.bits if layer >= 0 else c.lm_bits
        grp = (c.group if layer >= 0 else c.lm_group) if bits == 4 else 0
        return oracle.gemm(x, bits, p, s.astype(np.float32), grp, n)[0]

    def rope(x, pos):
        x = x.reshape(-1, D).copy()
        half = c.rot_dim // 2
        x0, x1 = x[:, :half].copy(), x[:, half:c.rot_dim].copy()
        x[:, :half] = x0 * cos[pos] - x1 * sin[pos]
        x[:, half:c.rot_dim] = x0 * sin[pos] + x1 * cos[pos]
        return x

    for pos, tok in enumerate(prompt):
        h = tiny.embedding[tok].astype(np.float32)
        for l in range(c.n_layers):
            xn = oracle.rmsnorm(h, tiny.norm(l, 0).astype(np.float32), eps=c.eps)[0]
            q = rope(lin(l, 0, xn), pos)
            k = rope(lin(l, 1, xn), pos)
            v = lin(l, 2, xn).reshape(KVH, D)
            kc[l, :, pos] = oracle.round_f16(k).reshape(KVH, D)
            vc[l, :, pos] = oracle.round_f16(v).reshape(KVH, D)
            att = np.zeros((NH, D), dtype=np.float32)
            for hh in range(NH):
                kh = hh // (NH // KVH)
                s = (kc[l, kh, :pos + 1] @ q[hh]) / math.sqrt(D)
                p = np.exp(s - s.max())
                att[hh] = (p / p.sum()) @ vc[l, kh, :pos + 1]
            h = h + lin(l, 3, att.reshape(-1))
            xn = oracle.rmsnorm(h, tiny.norm(l, 1).astype(np.float32), eps=c.eps)[0]
            act = oracle.swiglu(lin(l, 4, xn), lin(l, 5, xn))
            h = h + lin(l, 6, act)
    xf = oracle.rmsnorm(h, tiny.norm(-1, 0).astype(np.float32), eps=c.eps)[0]
    ref = lin(-1, 7, xf)
    assert np.allclose(logits, ref, rtol=1e-4, atol=1e-5 * np.abs(ref).max())
    assert int(np.argmax(ref)) == int(np.argmax(logits))


def test_oracle_decoder_capacity(oracle):
    cfg = synth.DecoderCfg(**{**synth.TINY.as_dict(), "kv_capacity": 4, "n_layers": 1})
    m = synth.SyntheticDecoder(cfg, seed=1)
    dec = oracle.OracleDecoder(m)
    for t in range(4):
        dec.step(t)
    with pytest.raises(RuntimeError):
        dec.step(0)
