"""GPU parity of the pointwise / attention / selection kernels against the oracle
and the reference's own golden cases (Pack4 layouts at the ABI)."""
import math

import numpy as np
import pytest

from test_oracle_pins import create_values, pack4_to_planar, planar_to_pack4, reference_sdpa_with_cache

pytestmark = pytest.mark.gpu


def cuda(a):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    import torch
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("dtype", ["f32", "f16"])
def test_rmsnorm(ops, oracle, dtype):
    import torch
    x = np.random.default_rng(1).standard_normal((3, 1024)).astype(np.float32)
    if dtype == "f16":
        x = x.astype(np.float16).astype(np.float32)
    g = np.random.default_rng(2).standard_normal(1024).astype(np.float32) * 0.02
    xt = cuda(x.astype(np.float16) if dtype == "f16" else x)
    y = torch.zeros((3, 1024), dtype=torch.float32, device="cuda")
    ops.rms_norm_pack4_linear_mat(xt, 3, 1024, cuda(g), 1024, True, 1e-6, y)
    assert np.allclose(host(y), oracle.rmsnorm(x, g, eps=1e-6), rtol=2e-6, atol=1e-9)
    ops.rms_norm_pack4_linear_mat(xt, 3, 1024, cuda(g), 1, True, 1e-6, y)
    assert np.allclose(host(y), oracle.rmsnorm(x, g, eps=1e-6, affine_size=1), rtol=2e-6, atol=1e-9)
    ops.rms_norm_pack4_linear_mat(xt, 3, 1024, None, 0, False, 1e-6, y)
    assert np.allclose(host(y), oracle.rmsnorm(x, None, eps=1e-6), rtol=2e-6, atol=1e-9)


@pytest.mark.parametrize("interleaved", [False, True])
def test_rope(ops, oracle, interleaved):
    import torch
    E, L, H = 128, 3, 10
    src = np.random.default_rng(3).standard_normal(((H + 3) // 4) * L * E * 4).astype(np.float32)
    cos, sin = oracle.rope_tables(L, E, 1e6)
    out = torch.zeros(src.size, dtype=torch.float32, device="cuda")
    ops.rotary_embed_pack4(cuda(src), E, L, H, cuda(cos), cuda(sin), interleaved, out)
    ref = oracle.rope(src, E, L, H, cos, sin, interleaved)
    got = host(out)
    valid = pack4_to_planar(ref, E, L, H)
    assert np.array_equal(pack4_to_planar(got, E, L, H), valid)


def test_kv_append_and_concat_bit_exact(ops, oracle):
    import torch
    W, slices, cap = 128, 1, 16
    cur = np.random.default_rng(4).standard_normal(slices * 2 * W * 4).astype(np.float32)
    cache0 = np.random.default_rng(5).standard_normal(slices * cap * W * 4).astype(np.float32)
    cache = cuda(cache0.copy())
    ops.append_sequence_pack4_cdhw(cuda(cur), 5, 2, cache, W, slices, cap)
    assert np.array_equal(host(cache), oracle.append_sequence(cur, W, 2, slices, 5, cache0, cap))
    a = np.random.default_rng(6).standard_normal(2 * 3 * W * 4).astype(np.float32)
    b = np.random.default_rng(7).standard_normal(2 * 2 * W * 4).astype(np.float32)
    out = torch.full((2 * 7 * W * 4,), 9.0, dtype=torch.float32, device="cuda")
    ops.concat_sequence_pack4_cdhw(cuda(a), cuda(b), 3, 2, out, W, 2, 7)
    assert np.array_equal(host(out), oracle.concat_sequence(a, 3, b, 2, W, 2, 7))
    from aiimage_b200 import errors
    with pytest.raises(errors.InvalidOperationError):
        ops.append_sequence_pack4_cdhw(cuda(cur), 15, 2, cache, W, slices, cap)
    with pytest.raises(errors.ArgumentOutOfRangeError):
        ops.append_sequence_pack4_cdhw(cuda(cur), -1, 2, cache, W, slices, cap)


def test_sdpa_reference_golden_cases(ops):
    """The two SDPA golden tests of NcnnLinearCmdPack4GoldenTests (3e-4)."""
    import torch
    seq, embed, heads = 3, 3, 2
    q = create_values(heads * seq * embed, 0.07, 3)
    k = create_values(heads * seq * embed, 0.05, 5)
    v = create_values(heads * seq * embed, 0.11, 7)
    mask = np.array([0, -0.25, -1.5, 0, 0, -0.5, 0.1, 0, 0], dtype=np.float32)
    scale = 1.0 / math.sqrt(embed)
    exp = reference_sdpa_with_cache(q, k, v, seq, seq, embed, heads, scale, True, 0, mask)
    out = torch.zeros(seq * embed * 4, dtype=torch.float32, device="cuda")
    ops.sdpa_attention_pack4_cdhw(cuda(planar_to_pack4(q, embed, seq, heads)), cuda(planar_to_pack4(k, embed, seq, heads)),
                                  cuda(planar_to_pack4(v, embed, seq, heads)), seq, seq, embed, embed, heads, heads,
                                  scale, out, mask=cuda(planar_to_pack4(mask, seq, seq, 1)), mask_w=seq, mask_h=seq,
                                  causal=True)
    assert np.max(np.abs(pack4_to_planar(host(out), embed, seq, heads) - exp)) <= 3e-4

    past, cur, heads = 3, 2, 5
    total = past + cur
    q = create_values(heads * cur * embed, 0.07, 3)
    pk = create_values(heads * past * embed, 0.05, 5)
    ck = create_values(heads * cur * embed, 0.04, 11)
    pv = create_values(heads * past * embed, 0.11, 7)
    cv = create_values(heads * cur * embed, 0.09, 13)
    sl = (heads + 3) // 4
    kc = torch.zeros(sl * total * embed * 4, dtype=torch.float32, device="cuda")
    vc = torch.zeros_like(kc)
    ops.concat_sequence_pack4_cdhw(cuda(planar_to_pack4(pk, embed, past, heads)), cuda(planar_to_pack4(ck, embed, cur, heads)),
                                   past, cur, kc, embed, sl, total)
    ops.concat_sequence_pack4_cdhw(cuda(planar_to_pack4(pv, embed, past, heads)), cuda(planar_to_pack4(cv, embed, cur, heads)),
                                   past, cur, vc, embed, sl, total)
    out = torch.zeros(sl * cur * embed * 4, dtype=torch.float32, device="cuda")
    ops.sdpa_attention_pack4_cdhw(cuda(planar_to_pack4(q, embed, cur, heads)), kc, vc, cur, total, embed, embed, heads,
                                  heads, scale, out, causal=True, causal_query_offset=past)

    def cat(a, b):
        x = np.concatenate([a.reshape(heads, past, embed), b.reshape(heads, cur, embed)], 1)
        return x.reshape(-1)

    ek, ev = cat(pk, ck), cat(pv, cv)
    assert np.max(np.abs(pack4_to_planar(host(kc), embed, total, heads) - ek)) <= 1e-5
    exp = reference_sdpa_with_cache(q, ek, ev, cur, total, embed, heads, scale, True, past)
    assert np.max(np.abs(pack4_to_planar(host(out), embed, cur, heads) - exp)) <= 3e-4


def test_sdpa_gqa_beyond_reference_cap(ops, oracle):
    """GQA 8/2 heads, head_dim 128, 5000 keys (past the reference's 4096 cap)."""
    import torch
    src, dst, E, H, G = 2, 5000, 128, 8, 2
    r = np.random.default_rng(8)
    q = r.standard_normal(2 * src * E * 4).astype(np.float32)
    k = r.standard_normal(1 * dst * E * 4).astype(np.float32)
    v = r.standard_normal(1 * dst * E * 4).astype(np.float32)
    out = torch.zeros(2 * src * E * 4, dtype=torch.float32, device="cuda")
    scale = 1 / math.sqrt(E)
    ops.sdpa_attention_pack4_cdhw(cuda(q), cuda(k), cuda(v), src, dst, E, E, H, G, scale, out, causal=True,
                                  causal_query_offset=dst - src)
    ref = oracle.sdpa(q, k, v, src, dst, E, E, H, G, scale, causal=True, causal_offset=dst - src)
    got = pack4_to_planar(host(out), E, src, H)
    exp = pack4_to_planar(ref, E, src, H)
    assert np.allclose(got, exp, rtol=1e-4, atol=1e-5)


def test_argmax_known_answers_and_ties(ops, oracle):
    import torch
    out = torch.zeros(8, dtype=torch.int32, device="cuda")
    v = -np.arange(17, dtype=np.float32)
    v[13] = 100
    ops.arg_max_pack4_linear_mat(cuda(v), 17, 1, out)
    assert host(out)[0] == 13
    packs = 10
    tiled = np.zeros(packs * 4, dtype=np.float32)
    for p in range(packs):
        tiled[p * 4:p * 4 + 4] = [-(p * 4 + 1), -(p * 4 + 2), -(p * 4 + 3), -(p * 4 + 4)]
    tiled[34] = 100
    ops.arg_max_pack4_linear_mat(cuda(tiled), 37, 1, out, ld=40)
    assert host(out)[0] == 34
    cases = [np.array([1, 3, 3, 2, 3], np.float32), np.array([np.nan, 5, 6], np.float32),
             np.array([1, np.nan, 6], np.float32), np.array([-0.0, 0.0, -1], np.float32),
             np.array([-np.inf, -np.inf], np.float32)]
    for c in cases:
        ops.arg_max_pack4_linear_mat(cuda(c), c.size, 1, out)
        assert host(out)[0] == oracle.argmax(c)[0], c
    r = np.random.default_rng(9)
    big = r.standard_normal((4, 151936)).astype(np.float32)
    big[1, 1000] = big[1, 77] = big[1].max() + 1  # tie -> lowest index
    ops.arg_max_pack4_linear_mat(cuda(big), 151936, 4, out)
    assert np.array_equal(host(out)[:4], oracle.argmax(big))


def test_topk(ops, oracle):
    import torch
    r = np.random.default_rng(10)
    x = r.standard_normal((5, 20000)).astype(np.float32)
    x[0, 50:60] = 9.0     # ties ordered by index
    x[1, :] = 1.0         # one plateau far larger than the candidate buffer
    x[2, ::2] = -0.0      # signed zeros count as equal
    x[3, 7000:] = 3.0     # a plateau of 13000 ranked after nothing
    x[4] *= 1e-30         # tiny values (one exponent bin)
    k = 50
    vals = torch.zeros((5, k), dtype=torch.float32, device="cuda")
    idx = torch.zeros((5, k), dtype=torch.int32, device="cuda")
    ops.top_k(cuda(x), 20000, 5, k, vals, idx)
    rv, ri = oracle.topk(x, k)
    assert np.array_equal(host(idx), ri)
    assert np.array_equal(host(vals), rv)
    # Fewer values than k: the rest is padded with (-inf, -1).
    small = r.standard_normal((2, 30)).astype(np.float32)
    ops.top_k(cuda(small), 30, 2, k, vals[:2], idx[:2], ld=30)
    sv, si = oracle.topk(small, 30)
    assert np.array_equal(host(idx)[:2, :30], si) and np.all(host(idx)[:2, 30:] == -1)
    assert np.all(np.isneginf(host(vals)[:2, 30:]))


def _wide_topk_rows(width: int, seed: int) -> np.ndarray:
    """Rows built to defeat a sampled threshold: every case must fall back to
    the exact per-row path or survive the candidate filter unchanged."""
    r = np.random.default_rng(seed)
    x = r.standard_normal((12, width)).astype(np.float32)
    samples = (np.arange(4096, dtype=np.int64) * width) // 4096
    off = np.setdiff1d(np.arange(width), samples)
    x[1, :] = 1.0                                   # one plateau: candidate overflow
    x[2, :] = -1.0                                  # large values only between samples
    x[2, r.choice(off, 1000, replace=False)] = 5.0
    x[3] *= 0.01                                    # 20 large values on sample positions:
    x[3, samples[r.choice(4096, 20, replace=False)]] = 10.0  # fewer than k above t
    x[4, ::2] = np.nan                              # half NaN
    x[5, :] = np.nan                                # 30 selectable values: padding
    x[5, r.choice(width, 30, replace=False)] = r.standard_normal(30)
    x[6, :] = -np.inf                               # -inf is selectable, by index
    x[6, r.choice(width, 10, replace=False)] = 1.0
    x[7] = np.sort(x[7])                            # ascending along the index
    x[8] = np.round(x[8] * 2) / 2                   # few levels: ties at t
    x[9, :] = 0.0                                   # signed zeros plus 100 positives
    x[9, ::3] = -0.0
    x[9, r.choice(width, 100, replace=False)] = 2.0
    x[10, -1] = 100.0                               # the row's last element wins
    x[11, 1:] = x[11, 0]                            # tie at every index
    return x


@pytest.mark.parametrize("width,ld", [(151936, 151936), (40001, 40004), (40001, 40001), (32768, 32768)])
def test_topk_wide_rows(ops, oracle, width, ld):
    """The sampled path (width >= 32768, 16-byte rows) and the exact path
    behind it against the oracle; ld == width odd takes the exact path."""
    import torch
    x = _wide_topk_rows(width, 12 + width)
    rows, k = x.shape[0], 50
    buf = np.full((rows, ld), 7.0, dtype=np.float32)  # ld padding never read
    buf[:, :width] = x
    vals = torch.zeros((rows, k), dtype=torch.float32, device="cuda")
    idx = torch.zeros((rows, k), dtype=torch.int32, device="cuda")
    ops.top_k(cuda(buf), width, rows, k, vals, idx, ld=ld)
    rv, ri = oracle.topk(x, k)
    assert np.array_equal(host(idx), ri)
    assert np.array_equal(host(vals), rv)


@pytest.mark.parametrize("k", [1, 7, 64])
def test_topk_k_range(ops, oracle, k):
    import torch
    x = np.random.default_rng(13 + k).standard_normal((3, 151936)).astype(np.float32)
    vals = torch.zeros((3, k), dtype=torch.float32, device="cuda")
    idx = torch.zeros((3, k), dtype=torch.int32, device="cuda")
    ops.top_k(cuda(x), 151936, 3, k, vals, idx)
    rv, ri = oracle.topk(x, k)
    assert np.array_equal(host(idx), ri) and np.array_equal(host(vals), rv)


def test_topk_config5_shape(ops, oracle):
    """256 rows x 151936 logits, k = 50 (the config-5 sampler input)."""
    import torch
    x = np.random.default_rng(11).standard_normal((256, 151936)).astype(np.float32)
    vals = torch.zeros((256, 50), dtype=torch.float32, device="cuda")
    idx = torch.zeros((256, 50), dtype=torch.int32, device="cuda")
    ops.top_k(cuda(x), 151936, 256, 50, vals, idx)
    rv, ri = oracle.topk(x, 50)
    assert np.array_equal(host(idx), ri)


@pytest.mark.parametrize("kind", ["q4", "q8", "f16", "f32"])
def test_embed(ops, oracle, kind):
    import torch
    from aiimage_b200 import synth
    V, Dm = 300, 64
    words = np.array([0, 5, 299, 400, -3, 17], dtype=np.int32)  # out-of-range ids clamp
    bias = np.random.default_rng(11).standard_normal(Dm).astype(np.float32)
    out = torch.zeros((words.size, Dm), dtype=torch.float32, device="cuda")
    if kind == "q4":
        p, s = synth.q4_weights(V, Dm, 16, seed=12)
        t = ops.new_int4_weight_only_upload(p, s, V, Dm, 16)
        ref = oracle.embed(words, 4, Dm, V, packed=p, scales=s.astype(np.float32), blk=16, bias=bias)
    elif kind == "q8":
        p, s = synth.q8_weights(V, Dm, seed=12)
        t = ops.new_int8_weight_only_upload(p, s, V, Dm)
        ref = oracle.embed(words, 8, Dm, V, packed=p, scales=s.astype(np.float32), bias=bias)
    else:
        tab = np.random.default_rng(13).standard_normal((V, Dm)).astype(np.float16 if kind == "f16" else np.float32)
        t = ops.new_dense_weights(tab)
        ref = oracle.embed(words, 32, Dm, V, table=tab.astype(np.float32), bias=bias)
    ops.embed_texture(cuda(words), words.size, t, cuda(bias), out)
    assert np.array_equal(host(out), ref)


def test_swish_and_swiglu(ops, oracle):
    import torch
    x = (np.random.default_rng(14).standard_normal(4096) * 4).astype(np.float32)
    u = np.random.default_rng(15).standard_normal(4096).astype(np.float32)
    y = torch.zeros(4096, dtype=torch.float32, device="cuda")
    ops.swish(cuda(x), 4096, y)
    assert np.allclose(host(y), oracle.swish(x), rtol=2e-6, atol=1e-7)
    ops.swiglu(cuda(x), cuda(u), 4096, y)
    assert np.allclose(host(y), oracle.swiglu(x, u), rtol=2e-6, atol=1e-7)


def test_bounded_wait_timeout_leaves_context_usable(ops):
    """The failure path of every bounded barrier wait: a kernel waits on a
    flag nothing sets, gives up after ~1 ms of SM clock, records
    AEXIS_E_TIMEOUT; sync reports it once and the context keeps working."""
    import torch
    from aiimage_b200 import errors
    ops.sync()
    ops.selftest_wait(2_000_000)
    with pytest.raises(errors.DeviceTimeoutError):
        ops.sync()
    ops.sync()  # the status word was cleared by the report
    x = torch.tensor([[0.5, 3.0, -1.0, 3.0]], dtype=torch.float32, device="cuda")
    out = torch.empty(1, dtype=torch.int32, device="cuda")
    ops.arg_max_pack4_linear_mat(x, 4, 1, out)
    ops.sync()
    assert int(out.item()) == 1
    with pytest.raises(errors.ArgumentOutOfRangeError):
        ops.selftest_wait(10)


@pytest.mark.parametrize("world", [2, 3, 8])
def test_topk_shard_merge_matches_full_vocab(ops, oracle, world):
    """aexis_cuda_topk_merge over `world` simulated vocab shards (each through
    argmax_keys and top_k, packed as the sharded lm_head packs them) gives
    the greedy ids and top-k of the full-vocabulary calls and the oracle:
    ties across shards, a tie at the k-th place, a row of -inf, a shard of
    fewer than k values (the last one when the vocab does not divide)."""
    import torch
    from aiimage_b200 import sharded
    rows, vocab, k = 7, 20003, 50
    x = np.random.default_rng(30 + world).standard_normal((rows, vocab)).astype(np.float32)
    per = (vocab + world - 1) // world
    x[0, 5] = x[0, vocab - 3] = x[0].max() + 1         # greedy tie across shards: lowest index
    x[1, 100:160] = 9.0                                 # 60 equal values straddling a boundary for small shards
    x[2, :] = -np.inf                                   # -inf values are selectable, by index
    x[3, per - 1] = x[3, per] = x[3].max() + 2          # tie at a shard boundary
    x[4, ::7] = np.nan                                  # NaN never selected
    xc = cuda(x)
    w = sharded.packed_words(rows, k)
    gathered = torch.zeros(world * w, dtype=torch.int32, device="cuda")
    for r in range(world):
        lo, hi = sharded.shard_range(vocab, world, r)
        keys, vals, idx = sharded.pack_views(gathered[r * w:(r + 1) * w], rows, k)
        part = xc[:, lo:hi]
        ops.argmax_keys(part, hi - lo, rows, lo, keys, ld=vocab)
        ops.top_k(part, hi - lo, rows, k, vals, idx, ld=vocab)
    ids = torch.zeros(rows, dtype=torch.int64, device="cuda")
    mv = torch.zeros((rows, k), dtype=torch.float32, device="cuda")
    mi = torch.zeros((rows, k), dtype=torch.int32, device="cuda")
    ops.topk_merge(gathered, world, rows, k, per, ids, mv, mi)
    fv = torch.zeros((rows, k), dtype=torch.float32, device="cuda")
    fi = torch.zeros((rows, k), dtype=torch.int32, device="cuda")
    ops.top_k(xc, vocab, rows, k, fv, fi)
    assert np.array_equal(host(mi), host(fi)) and np.array_equal(host(mv), host(fv))
    rv, ri = oracle.topk(x, k)
    assert np.array_equal(host(mi), ri)
    full_keys = torch.zeros(rows, dtype=torch.int64, device="cuda")
    ops.argmax_keys(xc, vocab, rows, 0, full_keys)
    assert np.array_equal(host(ids), host(sharded.keys_to_ids(full_keys)))


@pytest.mark.parametrize("world", [2, 3, 8])
def test_topk_peer_exchange_matches_gathered_merge(ops, world):
    """The sharded lm_head's exchange over peer memory with `world` ranks
    simulated on one GPU (one receive buffer per rank; each rank's
    aexis_cuda_topk_push writes every buffer, then each rank's
    aexis_cuda_topk_merge_peers reads its own): every rank merges exactly
    what aexis_cuda_topk_merge gives on the all-gathered buffers, over two
    calls (both slot parities, other data in the second). The pushes finish
    before any merge starts, so no kernel waits on another. An odd row count
    leaves a packed result that is not a whole number of 16-byte units. When
    one rank skips a push, the others' merges give up (AEXIS_E_TIMEOUT,
    about a second) and the context keeps working."""
    import torch
    from aiimage_b200 import errors, sharded
    rows, vocab, k = 7, 20003, 50
    per = (vocab + world - 1) // world
    w = sharded.packed_words(rows, k)
    assert w % 4 != 0
    recv = [ops.peer_buffer_create(ops.peer_buffer_bytes(world, rows, k))[0] for _ in range(world)]
    try:
        for call in (1, 2):
            x = np.random.default_rng(40 + 10 * world + call).standard_normal((rows, vocab)).astype(np.float32)
            x[0, 5] = x[0, vocab - 3] = x[0].max() + 1  # greedy tie across shards
            x[1, per - 1] = x[1, per] = x[1].max() + 2  # tie at a shard boundary
            xc = cuda(x)
            bufs = [torch.zeros(w, dtype=torch.int32, device="cuda") for _ in range(world)]
            for r in range(world):
                lo, hi = sharded.shard_range(vocab, world, r)
                keys, vals, idx = sharded.pack_views(bufs[r], rows, k)
                ops.argmax_keys(xc[:, lo:hi], hi - lo, rows, lo, keys, ld=vocab)
                ops.top_k(xc[:, lo:hi], hi - lo, rows, k, vals, idx, ld=vocab)
            for r in range(world):
                ops.topk_push(bufs[r], rows, k, recv, r)
            ref = [torch.zeros(rows, dtype=torch.int64, device="cuda"),
                   torch.zeros((rows, k), dtype=torch.float32, device="cuda"),
                   torch.zeros((rows, k), dtype=torch.int32, device="cuda")]
            ops.topk_merge(torch.cat(bufs), world, rows, k, per, *ref)
            for r in range(world):
                got = [torch.full_like(t, -7) for t in ref]
                ops.topk_merge_peers(recv[r], world, rows, k, per, *got)
                for g, e in zip(got, ref):
                    assert np.array_equal(host(g), host(e)), (call, r)
        ops.sync()
        for r in range(1, world):  # rank 0 does not push the third call
            ops.topk_push(bufs[r], rows, k, recv, r)
        got = [torch.zeros_like(t) for t in ref]
        ops.topk_merge_peers(recv[1], world, rows, k, per, *got)
        with pytest.raises(errors.DeviceTimeoutError):
            ops.sync()
        ops.sync()
    finally:
        for p in recv:
            ops.peer_buffer_close(p, False)


@pytest.mark.parametrize("world", [1, 3, 8])
def test_topk_greedy_keys_match_argmax_keys(ops, world):
    """aexis_cuda_topk_greedy_keys (the shard's argmax key from its top-k list) against aexis_cuda_argmax_keys
    (a pass over the logits) on every shard: a NaN at global index 0 (wins) and at a shard's local 0 (does not),
    a row of NaN, -0 before +0 at the maximum, ties, a row of -inf, shards narrower than k."""
    import torch
    from aiimage_b200 import sharded
    rows, vocab, k = 9, 300 if world == 8 else 20003, 50
    x = np.random.default_rng(40 + world).standard_normal((rows, vocab)).astype(np.float32)
    per = (vocab + world - 1) // world
    x[0, 0] = np.nan                                    # NaN at global index 0: ArgMax keeps index 0
    x[1, per if world > 1 else 1] = np.nan              # NaN at the second shard's first element: never wins
    x[2, :] = np.nan
    x[3, :] = -1.0
    x[3, 10], x[3, 20] = -0.0, 0.0                      # -0 first: equal to +0, the lower index wins
    x[4, 7] = x[4, vocab - 2] = x[4].max() + 3          # tie across shards
    x[5, :] = -np.inf
    x[6, ::3] = np.nan
    xc = cuda(x)
    ids_a, ids_b = [], []
    for r in range(world):
        lo, hi = sharded.shard_range(vocab, world, r)
        part = xc[:, lo:hi]
        ka = torch.zeros(rows, dtype=torch.int64, device="cuda")
        kb = torch.zeros(rows, dtype=torch.int64, device="cuda")
        kk = min(k, hi - lo)
        vals = torch.zeros((rows, kk), dtype=torch.float32, device="cuda")
        idx = torch.zeros((rows, kk), dtype=torch.int32, device="cuda")
        ops.argmax_keys(part, hi - lo, rows, lo, ka, ld=vocab)
        ops.top_k(part, hi - lo, rows, kk, vals, idx, ld=vocab)
        ops.topk_greedy_keys(part, hi - lo, rows, kk, vals, idx, lo, kb, ld=vocab)
        a, b = host(ka).view(np.uint64), host(kb).view(np.uint64)
        # Equal keys wherever the shard row holds a non-NaN value or global index 0; a shard row of NaN
        # only (which can never win) gives key 0 here.
        all_nan = np.isnan(x[:, lo:hi]).all(axis=1) & (lo > 0)
        np.testing.assert_array_equal(a[~all_nan], b[~all_nan])
        ids_a.append(a)
        ids_b.append(b)
    best_a = np.max(np.stack(ids_a), axis=0)
    best_b = np.max(np.stack(ids_b), axis=0)
    tok = lambda key: np.where(key == 0, 0, (0xFFFFFFFF - (key & np.uint64(0xFFFFFFFF))).astype(np.int64))
    np.testing.assert_array_equal(tok(best_a), tok(best_b))
    assert tok(best_b)[0] == 0 and tok(best_b)[2] == 0 and tok(best_b)[3] == 10 and tok(best_b)[5] == 0
