"""GPU parity of the device sampler (aexis_cuda_sample: Qwen35Sampler.Select,
Qwen35DecoderSession.cs:1847-1900) against the oracle's restatement, with the
same uniform draws.

Greedy selections are bit-exact. A sampled token is a step function of the
draw: the GPU's float softmax (CUDA expf, per-segment sums merged in fp64)
and the oracle's (libm expf, one fp64 sum) agree to about 1e-7 relative, so
the tokens must be equal wherever the oracle's draw lies more than 1e-5 of the
kept mass from a cumulative boundary (and the nucleus cut more than 1e-5 from
top_p); rows closer than that are skipped and counted."""
import numpy as np
import pytest

from aiimage_b200 import errors

pytestmark = pytest.mark.gpu


def cuda(a, dtype=None):
    import torch
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t.cuda() if dtype is None else t.to(dtype).cuda()


def run(ops, logits, history, pen, temp, top_k, top_p, u):
    import torch
    rows, width = logits.shape
    out = torch.full((rows,), -7, dtype=torch.int32, device="cuda")
    h = None if history is None else cuda(history.view(np.int32))
    uu = None if u is None else cuda(np.asarray(u, np.float64))
    ops.sample(cuda(logits), rows, width, h, pen, temp, top_k, top_p, uu, out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def make_case(seed, rows, width, scale, hist_per_row):
    rng = np.random.default_rng(seed)
    logits = (rng.standard_normal((rows, width)) * scale).astype(np.float32)
    hist = np.zeros((rows, (width + 31) // 32), dtype=np.uint32)
    for r in range(rows):
        # Half the history on each row's current top scores, so the penalty changes the ranking.
        top = np.argpartition(-logits[r], hist_per_row // 2)[:hist_per_row // 2]
        for t in np.concatenate([top, rng.integers(0, width, hist_per_row - len(top))]):
            hist[r, t // 32] |= np.uint32(1 << int(t % 32))
    return logits, hist, rng.random(rows)


@pytest.mark.parametrize("rows,width", [(1, 151936), (8, 151936), (3, 1000), (5, 40), (2, 151935)])
def test_greedy_bit_exact(ops, oracle, rows, width):
    logits, hist, _ = make_case(rows * 7 + width, rows, width, 3.0, 64)
    logits[0, width // 3] = logits[0].max() + 1.0           # a clear maximum
    logits[-1, 1] = logits[-1, 5] = logits[-1].max() + 2.0  # a tie: the first index wins
    for h, pen in ((None, 1.0), (hist, 1.1), (hist, 3.0)):
        got = run(ops, logits, h, pen, 0.0, 0, 1.0, None)
        ref, _ = oracle.sample(logits, h, pen)
        np.testing.assert_array_equal(got, ref)


@pytest.mark.parametrize("temp,top_k,top_p,pen", [
    (0.3, 50, 0.8, 1.1),     # Qwen35SamplingConfig defaults
    (1.0, 64, 1.0, 1.0),     # top-k only
    (0.7, 20, 0.95, 1.3),
    (2.0, 1, 0.5, 1.1),      # a single candidate
    (0.5, 50, 0.0, 1.1),     # top_p 0 keeps one token
])
@pytest.mark.parametrize("rows,width,scale", [(1, 151936, 4.0), (16, 151936, 4.0), (7, 3000, 2.0), (4, 64, 1.0),
                                              (3, 1001, 2.0)])   # an odd row stride: the scalar prep path
def test_sampling_matches_oracle(ops, oracle, temp, top_k, top_p, pen, rows, width, scale):
    logits, hist, u = make_case(int(temp * 100) + top_k + rows + width, rows, width, scale, 40)
    got = run(ops, logits, hist, pen, temp, top_k, top_p, u)
    ref, margin = oracle.sample(logits, hist, pen, temp, top_k, top_p, u)
    sure = margin > 1e-5
    assert sure.sum() >= max(1, rows - 2)
    np.testing.assert_array_equal(got[sure], ref[sure])


def test_sampling_config5_batch_and_draw_sweep(ops, oracle):
    """256 rows of the config-5 vocabulary with the default config, and one row under 64 draws (every part of
    its cumulative distribution)."""
    logits, hist, u = make_case(5, 256, 151936, 4.0, 100)
    got = run(ops, logits, hist, 1.1, 0.3, 50, 0.8, u)
    ref, margin = oracle.sample(logits, hist, 1.1, 0.3, 50, 0.8, u)
    sure = margin > 1e-5
    assert sure.sum() >= 250
    np.testing.assert_array_equal(got[sure], ref[sure])
    one = np.repeat(logits[:1], 64, axis=0)
    hist1 = np.repeat(hist[:1], 64, axis=0)
    u = (np.arange(64) + 0.5) / 64
    got = run(ops, one, hist1, 1.1, 1.0, 64, 1.0, u)
    ref, margin = oracle.sample(one, hist1, 1.1, 1.0, 64, 1.0, u)
    sure = margin > 1e-5
    np.testing.assert_array_equal(got[sure], ref[sure])
    assert len(set(got.tolist())) > 8


def test_nan_and_inf_rows(ops, oracle):
    logits, hist, u = make_case(9, 4, 5000, 2.0, 10)
    logits[0, 17] = np.nan               # NaN poisons the sum: ArgMax fallback
    logits[1, :] = -np.inf               # no finite score: ArgMax -> 0
    logits[2, ::2] = -np.inf             # half the row impossible
    logits[3, 0] = np.nan                # NaN at index 0 wins ArgMax
    for temp in (0.0, 0.8):
        got = run(ops, logits, hist, 1.1, temp, 50, 0.9, u)
        ref, margin = oracle.sample(logits, hist, 1.1, temp, 50, 0.9, u)
        sure = margin > 1e-5
        np.testing.assert_array_equal(got[sure], ref[sure])
        assert got[1] == 0 and got[3] == 0


def test_history_add_and_device_sampler(ops, oracle):
    import torch
    from aiimage_b200.sampler import DeviceSampler, DotNetRandom, SamplingConfig
    vocab = 151936
    s = DeviceSampler(ops, vocab, SamplingConfig(), rows=4, seeds=[1, 2, 3, 4])
    toks = torch.tensor([5, 151935, -1, 40000], dtype=torch.int32, device="cuda")
    s.add_history(toks)
    s.add_history(toks)
    h = s.history.cpu().numpy().view(np.uint32)
    assert h[0, 0] == 1 << 5 and h[1, 151935 // 32] == 1 << (151935 % 32) and not h[2].any()
    assert h[3, 40000 // 32] == 1 << (40000 % 32) and int(np.count_nonzero(h)) == 3
    rng = np.random.default_rng(3)
    logits = (rng.standard_normal((4, vocab)) * 4).astype(np.float32)
    rngs = [DotNetRandom(x) for x in (1, 2, 3, 4)]
    for step in range(3):
        got = s.select(torch.from_numpy(logits).cuda()).cpu().numpy()
        u = np.array([r.next_double() for r in rngs])
        ref, margin = oracle.sample(logits, h, 1.1, 0.3, 50, 0.8, u)
        sure = margin > 1e-5
        np.testing.assert_array_equal(got[sure], ref[sure])
        logits = np.roll(logits, 1, axis=1)


WHOLE_MARGIN = 1e-6


def draw_bracket_ok(logits, hist, pen, temp, top_k, top_p, u, tok, tol=2e-6):
    """Independent float64 check of one sampled token: in descending order of
    probability (ties by index), the token's cumulative interval must contain
    the draw u * kept within `tol`, for some nucleus cut within `tol` of top_p
    (float rounding decides cuts and draws that close to a boundary)."""
    x = logits.astype(np.float32).copy()
    if hist is not None:
        bits = np.unpackbits(hist.view(np.uint8), bitorder="little")[: x.size].astype(bool)
        x[bits] = np.where(x[bits] < 0, x[bits] * np.float32(pen), x[bits] / np.float32(pen))
    p = np.exp((x.astype(np.float64) - x.max()) / temp)
    p /= p.sum()
    order = np.lexsort((np.arange(p.size), -p))
    cum = np.cumsum(p[order])
    keep = p.size if top_k <= 0 else min(top_k, p.size)
    k_lo = k_hi = keep
    if top_p < 1:
        k_lo = min(keep, int(np.searchsorted(cum, top_p - tol)) + 1)
        k_hi = min(keep, int(np.searchsorted(cum, top_p + tol)) + 1)
    r = int(np.flatnonzero(order == tok)[0])
    x_lo, x_hi = u * cum[k_lo - 1] - tol, u * cum[k_hi - 1] + tol
    lo = cum[r - 1] if r else 0.0
    return r < k_hi and lo <= x_hi and x_lo <= cum[r]


@pytest.mark.parametrize("temp,top_k,top_p,pen", [
    (0.3, 0, 0.8, 1.1),      # whole vocabulary with the default temperature and nucleus
    (1.0, 0, 1.0, 1.0),      # whole vocabulary, no nucleus: the draw walks the full distribution
    (2.0, 0, 0.95, 1.1),     # a flat distribution: a nucleus of thousands of tokens
    (0.7, -3, 0.9, 1.3),     # top_k <= 0 means the whole vocabulary, as in the reference
    (0.8, 100, 0.97, 1.1),   # more candidates than the top-k kernels keep
    (1.5, 5000, 1.0, 1.0),   # top-k only, thousands of candidates
    (0.5, 0, 0.0, 1.1),      # top_p 0 keeps one token
])
@pytest.mark.parametrize("rows,width,scale", [(1, 151936, 4.0), (5, 151936, 2.0), (6, 3001, 1.0)])
def test_whole_vocabulary_sampling_matches_oracle(ops, oracle, temp, top_k, top_p, pen, rows, width, scale):
    """top_k <= 0 and top_k > 64 (the radix-select path) against the oracle's
    full sort of every probability, same draws: equal tokens wherever the
    oracle's draw and nucleus cut lie more than WHOLE_MARGIN of the kept mass
    from a boundary, and for every row a float64 check that the token's
    cumulative interval holds the draw. (Over the whole vocabulary a token's
    probability is often below 1e-5, and so are those distances.)"""
    logits, hist, u = make_case(int(temp * 10) + abs(top_k) + rows + width, rows, width, scale, 40)
    got = run(ops, logits, hist, pen, temp, top_k, top_p, u)
    ref, margin = oracle.sample(logits, hist, pen, temp, top_k, top_p, u)
    sure = margin > WHOLE_MARGIN
    np.testing.assert_array_equal(got[sure], ref[sure])
    for r in range(rows):
        assert draw_bracket_ok(logits[r], hist[r], pen, temp, top_k, top_p, u[r], int(got[r])), r


def test_whole_vocabulary_draw_sweep_and_ties(ops, oracle):
    """One row under 64 draws spread over its whole distribution (top_k 0,
    top_p 1); then rows of exactly equal scores, where every token has the
    same probability and the draw picks by index (equal probabilities rank by
    ascending index), and a row with half its scores at -inf."""
    logits, hist, _ = make_case(77, 1, 151936, 1.5, 30)
    one = np.repeat(logits, 64, axis=0)
    h1 = np.repeat(hist, 64, axis=0)
    u = (np.arange(64) + 0.5) / 64
    got = run(ops, one, h1, 1.1, 1.0, 0, 1.0, u)
    ref, margin = oracle.sample(one, h1, 1.1, 1.0, 0, 1.0, u)
    sure = margin > WHOLE_MARGIN
    assert sure.sum() >= 48
    np.testing.assert_array_equal(got[sure], ref[sure])
    for r in range(64):
        assert draw_bracket_ok(one[r], h1[r], 1.1, 1.0, 0, 1.0, u[r], int(got[r])), r
    assert len(set(got.tolist())) > 32
    flat = np.zeros((8, 5000), dtype=np.float32)
    flat[7, ::2] = -np.inf
    uf = np.array([0.0, 0.1, 0.25, 0.5, 0.75, 0.9, 0.999, 0.5])
    got = run(ops, flat, None, 1.0, 1.0, 0, 1.0, uf)
    ref, _ = oracle.sample(flat, None, 1.0, 1.0, 0, 1.0, uf)
    np.testing.assert_array_equal(got, ref)
    got = run(ops, flat, None, 1.0, 1.0, 0, 0.3, uf)
    ref, _ = oracle.sample(flat, None, 1.0, 1.0, 0, 0.3, uf)
    np.testing.assert_array_equal(got, ref)


def test_sample_argument_errors(ops):
    import torch
    x = torch.zeros((2, 100), dtype=torch.float32, device="cuda")
    out = torch.zeros(2, dtype=torch.int32, device="cuda")
    u = torch.zeros(2, dtype=torch.float64, device="cuda")
    with pytest.raises(errors.ArgumentNullError):
        ops.sample(x, 2, 100, None, 1.0, 0.5, 10, 1.0, None, out)  # sampling needs draws
    with pytest.raises(errors.ArgumentOutOfRangeError):
        ops.sample(x, 2, 100, None, 0.0, 0.5, 10, 1.0, u, out)     # penalty must be positive
    with pytest.raises(errors.ArgumentError):
        ops.sample(x, 2, 100, None, 1.0, 0.5, 10, 1.0, u, out, ld=50)
    ops.sample(x, 2, 100, None, 1.0, 0.0, 0, 1.0, None, out)       # greedy needs neither
    torch.cuda.synchronize()
