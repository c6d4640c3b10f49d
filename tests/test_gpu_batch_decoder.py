"""Batched greedy decoding (aexis_cuda_batch_*) against the CPU oracle, one
oracle decoder per sequence.

Each sequence starts from a synthetic context of its own length (the values
of oracle_decoder_fill_context), then decodes greedily. The oracle is run
with the GPU's tokens as inputs (teacher forcing), so one near-tie cannot
derail the rest of the comparison: at every step the GPU token must be the
oracle's argmax, or tie with it within 1e-3 of the logit scale. The last
step's logits must agree within 1e-3 of the logit scale.
"""
import numpy as np
import pytest

from aiimage_b200 import synth

pytestmark = pytest.mark.gpu

TOL = 1e-3


def q8(cfg: synth.DecoderCfg, **over) -> synth.DecoderCfg:
    d = cfg.as_dict()
    d.update(bits=8, group=0, lm_bits=8, lm_group=0)
    d.update(over)
    return synth.DecoderCfg(**d)


def check_against_oracle(oracle, model, ctx_lens, seed, first, got, last_logits, seqs=None):
    """got: [steps][n] GPU tokens; last_logits: [n][vocab] of the last step."""
    steps, n = got.shape
    exact = 0
    for i in (range(n) if seqs is None else seqs):
        dec = oracle.OracleDecoder(model)
        dec.fill_context(int(ctx_lens[i]), seed, i)
        tok = int(first[i])
        for s in range(steps):
            nxt, logits, _ = dec.step(tok)
            g = int(got[s, i])
            scale = float(np.abs(logits).max())
            assert 0 <= g < model.cfg.vocab
            if g == nxt:
                exact += 1
            else:
                assert logits[nxt] - logits[g] <= TOL * scale, (i, s, g, nxt, logits[nxt] - logits[g])
            tok = g
        scale = float(np.abs(logits).max())
        assert np.max(np.abs(last_logits[i] - logits)) <= TOL * scale, i
    return exact


def test_batch_matches_oracle_per_sequence(ops, oracle):
    from aiimage_b200.decoder import BatchSession, DecoderSession
    cfg = q8(synth.TINY, kv_capacity=320)
    model = synth.SyntheticDecoder(cfg, seed=41)
    dec = DecoderSession(ops, cfg).load(model)
    ctx_lens = np.array([0, 1, 37, 128, 130, 257], dtype=np.int32)  # 0-3 attention splits, ragged
    seed = 0x5EED
    first = np.random.default_rng(7).integers(0, cfg.vocab, size=ctx_lens.size).astype(np.int32)
    batch = BatchSession(dec, max_batch=8, kv_capacity=300, max_steps=16)
    batch.fill_context(ctx_lens, seed)
    got = batch.generate(first, 12)
    assert got.shape == (12, ctx_lens.size)
    assert np.array_equal(batch.positions, ctx_lens + 12)
    exact = check_against_oracle(oracle, model, ctx_lens, seed, first, got, batch.logits())
    assert exact >= got.size - 1
    # A second call continues every sequence from where it stopped.
    more = batch.generate(got[-1], 3)
    assert more.shape == (3, ctx_lens.size)
    assert np.array_equal(batch.positions, ctx_lens + 15)


def test_batch_errors(ops):
    from aiimage_b200 import errors
    from aiimage_b200.decoder import BatchSession, DecoderSession
    model4 = synth.SyntheticDecoder(synth.TINY, seed=3)
    dec4 = DecoderSession(ops, synth.TINY).load(model4)
    with pytest.raises(errors.NotSupportedError):
        BatchSession(dec4, 4, 128, 4)  # Q4 decoders decode one sequence at a time
    cfg = q8(synth.TINY)
    dec = DecoderSession(ops, cfg)
    with pytest.raises(errors.InvalidOperationError):
        BatchSession(dec, 4, 128, 4)  # weights not loaded yet
    dec.load(synth.SyntheticDecoder(cfg, seed=4))
    with pytest.raises(errors.ArgumentOutOfRangeError):
        BatchSession(dec, 0, 128, 4)
    b = BatchSession(dec, 4, 128, 4)
    with pytest.raises(errors.InvalidOperationError):
        b.generate([1], 1)  # no context yet
    with pytest.raises(errors.ArgumentOutOfRangeError):
        b.fill_context([5, 128], seed=1)  # a context must leave room for a token
    with pytest.raises(errors.ArgumentOutOfRangeError):
        b.fill_context([1] * 5, seed=1)  # more sequences than max_batch
    b.fill_context([120, 3], seed=1)
    with pytest.raises(errors.ArgumentOutOfRangeError):
        b.generate([1, 2], 9)  # 120 + 9 > 128
    with pytest.raises(errors.ArgumentOutOfRangeError):
        b.generate([1, 2], 5)  # more steps than max_steps
    assert b.generate([1, 2], 4).shape == (4, 2)


def test_config4_batch_against_oracle(ops, oracle):
    """BASELINE config 4 on one GPU: the Q8 0.8B-shaped decoder, 32 sequences
    with contexts U[256, 4096] (seeded), a few greedy steps. Two sequences
    (the shortest and the longest context) are replayed on the oracle."""
    from aiimage_b200.decoder import BatchSession, DecoderSession
    cfg = q8(synth.QWEN35_08B_Q8, kv_capacity=256)
    model = synth.SyntheticDecoder(cfg, seed=4)
    dec = DecoderSession(ops, cfg).load(model)
    rng = np.random.default_rng([4, 256, 4096])
    ctx_lens = rng.integers(256, 4097, size=32).astype(np.int32)
    first = rng.integers(0, cfg.vocab, size=32).astype(np.int32)
    seed = 4
    batch = BatchSession(dec, max_batch=32, kv_capacity=4096 + 8, max_steps=8)
    batch.fill_context(ctx_lens, seed)
    got = batch.generate(first, 3)
    assert np.array_equal(batch.positions, ctx_lens + 3)
    import copy
    omodel = copy.copy(model)  # same weights, an oracle cache as long as the batch's
    omodel.cfg = q8(synth.QWEN35_08B_Q8, kv_capacity=4096 + 8)
    pick = [int(np.argmin(ctx_lens)), int(np.argmax(ctx_lens))]
    check_against_oracle(oracle, omodel, ctx_lens, seed, first, got, batch.logits(), seqs=pick)


@pytest.mark.parametrize("hpg", [4, 2])
def test_batch_tensor_core_attention_against_oracle(ops, oracle, hpg):
    """head_dim 128 takes the tensor-core attention (swizzled caches, online
    softmax over each CTA's chunks, the split merge in the O projection's
    prep): contexts that end inside, at and just past 64-position chunks,
    nine sequences (not a multiple of 16), every sequence checked."""
    from aiimage_b200.decoder import BatchSession, DecoderSession
    heads = 4 if hpg == 4 else 8
    cfg = q8(synth.TINY, n_layers=2, hidden=512, n_heads=heads, n_kv_heads=heads // hpg, head_dim=128, ffn=1024,
             vocab=4000, kv_capacity=1024, rot_dim=128)
    model = synth.SyntheticDecoder(cfg, seed=51 + hpg)
    dec = DecoderSession(ops, cfg).load(model)
    ctx_lens = np.array([0, 1, 62, 63, 64, 127, 129, 300, 700], dtype=np.int32)
    seed = 0xA77
    first = np.random.default_rng(8).integers(0, cfg.vocab, size=ctx_lens.size).astype(np.int32)
    batch = BatchSession(dec, max_batch=12, kv_capacity=1000, max_steps=8)
    batch.fill_context(ctx_lens, seed)
    got = batch.generate(first, 6)
    assert np.array_equal(batch.positions, ctx_lens + 6)
    exact = check_against_oracle(oracle, model, ctx_lens, seed, first, got, batch.logits())
    assert exact >= got.size - 1
