"""Host side of the device sampler (no GPU): the System.Random restatement that
supplies Qwen35Sampler's draws, and the oracle's restatement of
Qwen35Sampler.Select (Qwen35DecoderSession.cs:1847-1900) on hand-worked cases.

No reference test pins Select or the random stream, so the cases below are
worked out by hand from the C# source. The first draws of System.Random(0)
(0.7262432699679598, 0.8173253595909687) are the values widely published for
.NET's seeded generator; they are a sanity check of the restatement, not a
fixture produced by the reference."""
import math

import numpy as np
import pytest

from aiimage_b200.sampler import DotNetRandom, SamplingConfig


def test_dotnet_random_first_draws_and_range():
    r = DotNetRandom(0)
    assert r.next_double() == 0.7262432699679598
    assert r.next_double() == 0.8173253595909687
    for seed in (1, 20260718, -5, 2**31 - 1, -2**31):
        r = DotNetRandom(seed)
        u = [r.next_double() for _ in range(2000)]
        assert all(0.0 <= v < 1.0 for v in u)
        assert abs(np.mean(u) - 0.5) < 0.05
    a, b = DotNetRandom(7), DotNetRandom(7)
    assert [a.next_double() for _ in range(100)] == [b.next_double() for _ in range(100)]
    assert DotNetRandom(7).next_double() != DotNetRandom(8).next_double()


def test_sampling_config_defaults():
    c = SamplingConfig()
    assert (c.do_sample, c.temperature, c.top_p, c.top_k, c.repetition_penalty, c.seed) == \
        (True, 0.3, 0.8, 50, 1.1, 20260718)
    g = SamplingConfig.greedy()
    assert (g.do_sample, g.temperature, g.top_p, g.top_k, g.repetition_penalty) == (False, 0.0, 1.0, 0, 1.0)


def bitmap(rows_tokens, width):
    h = np.zeros((len(rows_tokens), (width + 31) // 32), dtype=np.uint32)
    for r, toks in enumerate(rows_tokens):
        for t in toks:
            h[r, t // 32] |= np.uint32(1 << (t % 32))
    return h


def test_oracle_select_hand_worked(oracle):
    # p = [1, 2, 4] / 7 at T = 1: descending order is tokens 2, 1, 0 with cumulative 4/7, 6/7, 1.
    logits = np.array([[0.0, math.log(2.0), math.log(4.0)]], dtype=np.float32)
    draw = lambda u, **kw: int(oracle.sample(logits, temperature=1.0, top_k=3, uniforms=[u], **kw)[0][0])
    assert draw(0.5) == 2
    assert draw(0.6) == 1
    assert draw(0.9) == 0
    # Top-k 2 keeps 6/7 of the mass: the draw scales to it (0.9 * 6/7 = 0.771 > 4/7 -> token 1).
    assert int(oracle.sample(logits, temperature=1.0, top_k=2, uniforms=[0.9])[0][0]) == 1
    # Top-p 0.5: the first token already reaches it, so only token 2 is kept.
    assert draw(0.99, top_p=0.5) == 2
    # Top-p 0.6 keeps two tokens (4/7 < 0.6 <= 6/7).
    assert draw(0.9, top_p=0.6) == 1
    # Greedy (temperature 0) and the repetition penalty: ln4 / 2 = ln2 ties token 1, first index wins.
    assert int(oracle.sample(logits)[0][0]) == 2
    assert int(oracle.sample(logits, history=bitmap([[2]], 3), penalty=2.0)[0][0]) == 1
    # A negative score is multiplied by the penalty.
    neg = np.array([[-1.0, -1.5]], dtype=np.float32)
    assert int(oracle.sample(neg, history=bitmap([[0]], 2), penalty=2.0)[0][0]) == 1
    # A NaN poisons the softmax sum: the sampler falls back to ArgMax.
    nan = np.array([[1.0, np.nan, 3.0]], dtype=np.float32)
    assert int(oracle.sample(nan, temperature=1.0, top_k=3, uniforms=[0.99])[0][0]) == 2


def test_oracle_select_margin_flags_boundaries(oracle):
    logits = np.array([[0.0, math.log(2.0), math.log(4.0)]], dtype=np.float32)
    _, m = oracle.sample(logits, temperature=1.0, top_k=3, uniforms=[4.0 / 7.0])
    assert m[0] < 1e-6
    _, m = oracle.sample(logits, temperature=1.0, top_k=3, uniforms=[0.3])
    assert m[0] > 0.1
