"""Decoder KV state in the reference's Pack4 CDHW layout (Qwen35DecoderState's
cache_k<i> / cache_v<i> textures, Qwen35DecoderSession.cs:48-100, 550-568):
export from the fused decoders, import into fresh ones, and the exported
textures as inputs of the ops-level attention (aexis_cuda_sdpa)."""
import numpy as np
import pytest

from aiimage_b200 import errors, synth
from aiimage_b200.ops import pack4_cdhw, unpack4_cdhw

pytestmark = pytest.mark.gpu


def q8(cfg, **over):
    d = cfg.as_dict()
    d.update(bits=8, group=0, lm_bits=8, lm_group=0)
    d.update(over)
    return synth.DecoderCfg(**d)


def cache_to_pack4(cache, rows):
    """Oracle cache [kvh, cap, D] -> flat Pack4 CDHW [w=D, h=rows, c=kvh] (positions past rows dropped)."""
    kvh, cap, D = cache.shape
    return pack4_cdhw(cache[:, :rows, :])


def test_decoder_state_export_import_and_sdpa(ops, oracle):
    import torch
    from aiimage_b200.decoder import DecoderSession
    cfg = synth.TINY
    model = synth.SyntheticDecoder(cfg, seed=61)
    prompt = model.prompt(21)
    a = DecoderSession(ops, cfg).load(model)
    nxt = a.prefill(prompt)
    pos = a.position
    assert pos == 21
    rows = 29
    state = a.export_state(rows)
    assert state["sequence_length"] == pos
    # Against the oracle's fp16 cache after the same prompt.
    odec = oracle.OracleDecoder(model)
    for t in prompt:
        odec.step(int(t), want_logits=False)
    for layer in range(cfg.n_layers):
        for kind, name in ((0, "cache_k"), (1, "cache_v")):
            got = state[f"{name}{layer}"].cpu().numpy()
            ref = cache_to_pack4(odec.kv(layer, kind), rows)
            scale = np.abs(ref).max()
            assert np.max(np.abs(got - ref)) <= 2e-3 * scale, (layer, name)
            logical = unpack4_cdhw(got, cfg.n_kv_heads, rows, cfg.head_dim)
            assert not logical[:, pos:, :].any()  # rows past the position are zero
    # Textures of exactly `position` rows are valid SDPA inputs (dst_len =
    # position, GQA): the GPU op over them equals the oracle's SDPA over the
    # oracle's cache.
    exact = a.export_state()
    assert exact["rows"] == pos
    rng = np.random.default_rng(6)
    q = pack4_cdhw(rng.standard_normal((cfg.n_heads, 1, cfg.head_dim)).astype(np.float32))
    out = torch.zeros(q.size, dtype=torch.float32, device="cuda")
    qd = torch.from_numpy(q).cuda()
    scale = 1.0 / np.sqrt(cfg.head_dim)
    for layer in range(cfg.n_layers):
        ops.sdpa_attention_pack4_cdhw(qd, exact[f"cache_k{layer}"], exact[f"cache_v{layer}"], 1, pos, cfg.head_dim,
                                      cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, scale, out)
        torch.cuda.synchronize()
        ref = oracle.sdpa(q, cache_to_pack4(odec.kv(layer, 0), pos), cache_to_pack4(odec.kv(layer, 1), pos), 1, pos,
                          cfg.head_dim, cfg.head_dim, cfg.n_heads, cfg.n_kv_heads, scale)
        assert np.max(np.abs(out.cpu().numpy() - ref)) <= 3e-4 * max(1.0, np.abs(ref).max())
    # Round trip: a fresh decoder seeded from the state continues exactly as the original.
    b = DecoderSession(ops, cfg).load(model)
    b.import_state(state)
    assert b.position == pos
    again = b.export_state(rows)
    for key in state:
        if key.startswith("cache_"):
            assert torch.equal(state[key], again[key]), key
    ta, tb = [nxt], [nxt]
    for _ in range(8):
        ta.append(a.step(ta[-1]))
        tb.append(b.step(tb[-1]))
    assert ta == tb
    assert np.array_equal(a.logits(), b.logits())
    # A state taken mid-way and re-imported into the first decoder rewinds it.
    a.import_state(state)
    assert a.position == pos
    assert [a.step(nxt)] == tb[1:2]


def test_decoder_state_errors(ops):
    import torch
    from aiimage_b200.decoder import DecoderSession
    cfg = synth.TINY
    model = synth.SyntheticDecoder(cfg, seed=62)
    d = DecoderSession(ops, cfg).load(model)
    d.prefill(model.prompt(10))
    buf = torch.zeros(d.kv_rows_floats(16), device="cuda")
    with pytest.raises(errors.ArgumentError):
        d.kv_export(0, buf, buf, 9)  # fewer rows than the sequence
    with pytest.raises(errors.ArgumentOutOfRangeError):
        d.kv_export(cfg.n_layers, buf, buf, 16)
    with pytest.raises(errors.ArgumentOutOfRangeError):
        d.kv_import(0, buf, buf, 16, 17)  # length beyond the texture
    with pytest.raises(errors.ArgumentOutOfRangeError):
        d.set_position(cfg.kv_capacity + 1)


@pytest.mark.parametrize("head_dim", [64, 128])
def test_batch_state_export_import(ops, oracle, head_dim):
    """head_dim 128 takes the tensor-core attention with swizzled cache rows; 64 the plain layout."""
    import torch
    from aiimage_b200.decoder import BatchSession, DecoderSession
    if head_dim == 64:
        cfg = q8(synth.TINY, kv_capacity=160)
    else:
        cfg = q8(synth.TINY, n_layers=2, hidden=512, n_heads=4, n_kv_heads=1, head_dim=128, ffn=1024, vocab=4000,
                 kv_capacity=160, rot_dim=128)
    model = synth.SyntheticDecoder(cfg, seed=63)
    dec = DecoderSession(ops, cfg).load(model)
    ctx = np.array([5, 64, 130, 0, 77], dtype=np.int32)
    seed = 0x51A7E
    src = BatchSession(dec, max_batch=8, kv_capacity=150, max_steps=8)
    src.fill_context(ctx, seed)
    dst = BatchSession(dec, max_batch=8, kv_capacity=150, max_steps=8)
    rows = 140
    nf = dec.kv_rows_floats(rows)
    k = torch.empty(nf, device="cuda")
    v = torch.empty_like(k)
    for i, n in enumerate(ctx):
        o = oracle.OracleDecoder(model)
        o.fill_context(int(n), seed, i)
        for layer in range(cfg.n_layers):
            src.kv_export(i, layer, k, v, rows)
            torch.cuda.synchronize()
            assert np.array_equal(k.cpu().numpy(), cache_to_pack4(o.kv(layer, 0)[:, :rows], rows)), (i, layer)
            assert np.array_equal(v.cpu().numpy(), cache_to_pack4(o.kv(layer, 1)[:, :rows], rows)), (i, layer)
            dst.kv_import(i, layer, k, v, rows, int(n))
    dst.set_positions(ctx)
    assert np.array_equal(dst.positions, ctx)
    first = np.random.default_rng(3).integers(0, cfg.vocab, size=ctx.size).astype(np.int32)
    got_src = src.generate(first, 6)
    got_dst = dst.generate(first, 6)
    assert np.array_equal(got_src, got_dst)
    # The batched GEMMs split K over CTAs and add with fp32 atomics, so two
    # runs agree to rounding, not bit for bit: after six steps through fp16
    # caches the logits have been seen to differ by up to 7e-5 of their
    # scale, so the bound is the decoder tests' 1e-3.
    ls, ld = src.logits(), dst.logits()
    assert np.max(np.abs(ls - ld)) <= 1e-3 * np.abs(ls).max()
    # After decoding, both hold the same (longer) state: the imported context
    # bit for bit, the decoded positions to rounding. Those rows come from
    # the same atomics-ordered projections (and, after the first step, from
    # attention over slightly different rows), so they are held to 2e-3 of
    # the rows' scale rather than per element: an element near zero can
    # differ by more than 2e-3 of itself.
    k2, v2 = torch.empty_like(k), torch.empty_like(k)
    for i in range(ctx.size):
        src.kv_export(i, 1, k, v, rows)
        dst.kv_export(i, 1, k2, v2, rows)
        for a, b in ((k, k2), (v, v2)):
            la = unpack4_cdhw(a.cpu().numpy(), cfg.n_kv_heads, rows, cfg.head_dim)
            lb = unpack4_cdhw(b.cpu().numpy(), cfg.n_kv_heads, rows, cfg.head_dim)
            n = int(ctx[i])
            assert np.array_equal(la[:, :n], lb[:, :n])
            dec_a, dec_b = la[:, n:n + 6], lb[:, n:n + 6]
            assert np.max(np.abs(dec_a - dec_b)) <= 2e-3 * np.abs(dec_a).max(), (i, np.max(np.abs(dec_a - dec_b)))
    with pytest.raises(errors.ArgumentOutOfRangeError):
        dst.kv_import(0, 0, k, v, rows, 150)  # no room left for a token
    with pytest.raises(errors.ArgumentOutOfRangeError):
        dst.set_positions([150])
