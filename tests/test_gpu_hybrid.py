"""The hybrid Qwen3.5 decoder (Qwen35DecoderSession.cs:167-172: three
linear-attention blocks, ShortConv + Gated Delta Rule, before each
full-attention block) against the CPU oracle's restatement of the same stack:
greedy tokens, logits at every step, the conv/GDR caches in the reference's
layout, and a state round trip into a fresh decoder."""
import json
import os

import numpy as np
import pytest

from aiimage_b200 import errors, synth

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decoder_greedy.json")
STEPS = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decoder_steps.npz")
TOL = 1e-3          # logits within TOL * max|logit| of the oracle's
STATE_TOL = 2e-3    # recurrent caches within STATE_TOL * max|cache|
CASE = "qwen35_08b_hybrid_q4_selective"


def tiny(**over):
    return synth.DecoderCfg(**{**synth.TINY_HYBRID.as_dict(), **over})


def session(ops, model):
    from aiimage_b200.decoder import DecoderSession
    return DecoderSession(ops, model.cfg).load(model)


@pytest.mark.parametrize("over", [
    {},                                                         # [lin, full, lin, full], kdim 64, vdim 32
    dict(bits=8, group=0, lm_bits=8, lm_group=0),               # Q8 weights
    dict(lin_kdim=32, lin_vdim=64, lin_heads=2, conv_kernel=3),  # four-CTA clusters, three conv taps
    dict(n_layers=4, full_attention_interval=4, lin_kdim=128, lin_vdim=128, lin_heads=2),  # Qwen3.5 order, 8-CTA
])
def test_tiny_hybrid_teacher_forced_against_oracle(ops, oracle, over):
    """Feed the same tokens to both decoders; at every step the logits agree
    within TOL of their scale and the greedy token is the oracle's wherever
    its top-1/top-2 margin exceeds twice that."""
    cfg = tiny(**over)
    model = synth.SyntheticDecoder(cfg, seed=71, norm_mean=1.0, balanced_q4=True)
    prompt = model.prompt(13)
    odec = oracle.OracleDecoder(model)
    sess = session(ops, model)
    for t in prompt[:-1]:
        odec.step(int(t), want_logits=False)
    tok = int(prompt[-1])
    got = sess.prefill(prompt)
    decided = 0
    for s in range(40):
        if s:
            got = sess.step(tok)
        ref_tok, ref, margin = odec.step(tok)
        logits = sess.logits()
        scale = np.abs(ref).max()
        err = np.max(np.abs(logits - ref))
        assert err <= TOL * scale, (s, err, scale)
        if margin > 2 * TOL * scale:
            decided += 1
            assert got == ref_tok, (s, got, ref_tok)
        tok = ref_tok  # teacher forcing: both continue from the oracle's token
    assert decided >= 30
    assert sess.position == len(prompt) + 39


def test_tiny_hybrid_generate_matches_oracle(ops, oracle):
    """aexis_cuda_decoder_generate (greedy tokens fed back on the device) against the oracle's greedy path:
    identical up to the first step whose top-1/top-2 margin is a near-tie (below 2 TOL of the logit scale),
    where a flip is a rounding question; the paths diverge after it."""
    model = synth.SyntheticDecoder(synth.TINY_HYBRID, seed=72, norm_mean=1.0, balanced_q4=True)
    prompt = model.prompt(11)
    odec = oracle.OracleDecoder(model)
    for t in prompt[:-1]:
        odec.step(int(t), want_logits=False)
    ref, near_tie, tok = [], [], int(prompt[-1])
    for _ in range(48):
        tok, logits, margin = odec.step(tok)
        ref.append(tok)
        near_tie.append(margin <= 2 * TOL * np.abs(logits).max())
    sess = session(ops, model)
    got = sess.generate(prompt, 48)
    first = next((i for i, (a, b) in enumerate(zip(got, ref)) if a != b), None)
    assert first is None or near_tie[first], (first, got[first], ref[first])
    assert len(set(ref)) >= 16
    # reset() zeroes the recurrent caches (CreateInitialState): the same call gives the same tokens.
    sess.reset()
    assert sess.generate(prompt, 48) == got


def test_hybrid_recurrent_state_layout_and_round_trip(ops, oracle):
    """After a prompt the conv/GDR caches equal the oracle's (reference texture layouts);
    a fresh decoder loaded from export_state continues exactly as the original."""
    import torch
    from aiimage_b200.decoder import DecoderSession
    cfg = synth.TINY_HYBRID
    model = synth.SyntheticDecoder(cfg, seed=73, norm_mean=1.0, balanced_q4=True)
    prompt = model.prompt(17)
    a = session(ops, model)
    nxt = a.prefill(prompt)
    odec = oracle.OracleDecoder(model)
    for t in prompt:
        odec.step(int(t), want_logits=False)
    state = a.export_state()
    kinds = cfg.layer_types()
    lin_layers = [i for i, k in enumerate(kinds) if k == 1]
    full_layers = [i for i, k in enumerate(kinds) if k == 0]
    assert sorted(k for k in state if k.startswith("cache_conv")) == [f"cache_conv{i}" for i in range(len(lin_layers))]
    assert sorted(k for k in state if k.startswith("cache_k")) == [f"cache_k{i}" for i in range(len(full_layers))]
    for i, layer in enumerate(lin_layers):
        conv_ref, gdr_ref = odec.recurrent(layer)
        conv = state[f"cache_conv{i}"].cpu().numpy().reshape(conv_ref.shape)
        gdr = state[f"cache_gdr{i}"].cpu().numpy().reshape(gdr_ref.shape)
        assert np.max(np.abs(conv - conv_ref)) <= STATE_TOL * np.abs(conv_ref).max(), layer
        assert np.max(np.abs(gdr - gdr_ref)) <= STATE_TOL * np.abs(gdr_ref).max(), layer
        # The conv cache holds the last conv_kernel in_proj rows: its newest row is nonzero.
        assert np.abs(conv[-1]).max() > 0
    b = DecoderSession(ops, cfg).load(model)
    b.import_state(state)
    assert b.position == len(prompt)
    again = b.export_state()
    for key in state:
        if key.startswith("cache_"):
            assert torch.equal(state[key], again[key]), key
    ta, tb = [nxt], [nxt]
    for _ in range(10):
        ta.append(a.step(ta[-1]))
        tb.append(b.step(tb[-1]))
    assert ta == tb
    assert np.array_equal(a.logits(), b.logits())
    # Re-importing rewinds the first decoder, recurrent caches included.
    a.import_state(state)
    assert [a.step(nxt)] == tb[1:2]


def test_hybrid_argument_errors(ops):
    import torch
    from aiimage_b200.decoder import BatchSession, DecoderSession
    cfg = synth.TINY_HYBRID
    model = synth.SyntheticDecoder(cfg, seed=74)
    d = DecoderSession(ops, cfg)
    p, s = model.linear(0, 8)
    with pytest.raises(errors.ArgumentOutOfRangeError):
        d.set_linear(0, 0, p, s)        # q_proj does not exist in a linear-attention layer
    with pytest.raises(errors.ArgumentOutOfRangeError):
        d.set_linear(1, 8, p, s)        # in_proj does not exist in a full-attention layer
    with pytest.raises(errors.ArgumentOutOfRangeError):
        d.set_linear_attention(1, *model.linear_attention(0))
    with pytest.raises(errors.InvalidOperationError):
        d.prefill(model.prompt(2))      # weights incomplete
    d.load(model)
    d.prefill(model.prompt(4))
    buf = torch.zeros(d.kv_rows_floats(8), device="cuda")
    with pytest.raises(errors.ArgumentOutOfRangeError):
        d.kv_export(0, buf, buf, 8)     # layer 0 is linear attention: no KV cache
    with pytest.raises(errors.ArgumentOutOfRangeError):
        d.recurrent_export(1, buf, None)
    with pytest.raises(errors.NotSupportedError):
        d.set_schedule(1)               # the persistent loop runs full-attention stacks only
    with pytest.raises(errors.NotSupportedError):
        BatchSession(d, max_batch=2, kv_capacity=32, max_steps=2)
    for bad in (dict(lin_vdim=24), dict(lin_vdim=256), dict(lin_kdim=260), dict(conv_kernel=9)):
        with pytest.raises((errors.NotSupportedError, errors.ArgumentError)):
            DecoderSession(ops, tiny(**bad))


def _golden():
    return json.load(open(GOLDEN))[CASE]


def test_qwen35_hybrid_golden_tokens(ops):
    """The full-size hybrid stack (24 layers: 18 linear-attention, 6
    full-attention; Q4 g32, vocab 151936): 64 greedy tokens identical to the
    oracle's, written offline into tests/golden/decoder_greedy.json."""
    gold = _golden()
    assert gold["distinct"] >= 16
    model = synth.SyntheticDecoder(getattr(synth, gold["cfg"]), seed=gold["seed"], norm_mean=gold["norm_mean"],
                                   balanced_q4=gold["balanced_q4"])
    prompt = model.prompt(gold["prompt_len"], seed=gold["prompt_seed"])
    sess = session(ops, model)
    assert sess.generate(prompt, gold["max_new"]) == gold["tokens"]
    ref = np.array(gold["last_top20_logits"], dtype=np.float32)
    got = sess.logits()[np.array(gold["last_top20_ids"])]
    assert np.max(np.abs(got - ref)) <= TOL * np.abs(ref).max()


def test_qwen35_hybrid_golden_teacher_forced_logits(ops):
    """Every step of the full-size hybrid golden: the oracle's 20 largest
    logits within TOL of the scale, and the greedy token wherever the margin
    decides it."""
    gold = _golden()
    steps = np.load(STEPS)
    ids, vals = steps[CASE + ".ids"], steps[CASE + ".logits"]
    model = synth.SyntheticDecoder(getattr(synth, gold["cfg"]), seed=gold["seed"], norm_mean=gold["norm_mean"],
                                   balanced_q4=gold["balanced_q4"])
    prompt = model.prompt(gold["prompt_len"], seed=gold["prompt_seed"])
    sess = session(ops, model)
    toks = gold["tokens"]
    got = sess.prefill(prompt)
    exact = decided = 0
    for s in range(gold["max_new"]):
        if s:
            got = sess.step(toks[s - 1])
        logits = sess.logits()
        scale = gold["logit_scale"][s]
        err = np.max(np.abs(logits[ids[s]] - vals[s]))
        assert err <= TOL * scale, (s, err, scale)
        if gold["margins"][s] > 2 * TOL * scale:
            decided += 1
            assert got == toks[s], (s, got, toks[s])
        exact += got == toks[s]
    assert exact >= decided and exact >= gold["max_new"] - 2, (exact, decided)
