"""Seeded synthetic inputs with the shapes and value distributions of the
measured configurations (there are no real weights or datasets on the box).

Generator: numpy's PCG64 (np.random.default_rng) with a per-tensor seed
sequence [seed, tag...], so every tensor is reproducible on its own and in any
order. Packed formats are the reference's (AexisGemm2DReadB, HLSL
Pack4Matmul:707-734): Q4 eight nibbles per uint32, low nibble first, along K
of each output row; Q8 four int8 per uint32.
"""
from __future__ import annotations

from dataclasses import dataclass, asdict

import numpy as np


def rng(seed: int, *tag: int) -> np.random.Generator:
    return np.random.default_rng([int(seed), *[int(t) for t in tag]])


def q4_weights(n: int, k: int, group: int, seed: int, tag=(0,), scale_lo=0.002, scale_hi=0.02,
               balanced: bool = False):
    """Symmetric int4 uniform in [-8, 7] packed two per byte along K; one fp16
    scale per `group` consecutive K values (config 2).

    balanced=True draws codes uniform in [-7, 7] instead, the range the
    reference's own quantizer emits (maxAbs/7, clamp to [-7, 7]). The [-8, 7]
    draw has mean -1/2, so every output row carries a bias of -scale/2 times
    the sum of its inputs; through a 24-layer residual stack with unit norm
    gains that common mode feeds itself and the greedy path collapses onto
    one token. The balanced draw has mean zero."""
    assert (n * k) % 8 == 0 and k % group == 0
    r = rng(seed, 4, *tag)
    if balanced:
        q = (r.integers(-7, 8, size=n * k, dtype=np.int8).astype(np.uint8) & 0xF).reshape(-1, 2)
        packed = (q[:, 0] | (q[:, 1] << 4)).astype(np.uint8).view(np.uint32)
    else:
        packed = r.integers(0, 256, size=n * k // 2, dtype=np.uint8).view(np.uint32)
    scales = r.uniform(scale_lo, scale_hi, size=n * k // group).astype(np.float16)
    return packed, scales


def q8_weights(n: int, k: int, seed: int, tag=(0,), scale_lo=0.001, scale_hi=0.01):
    """int8 uniform in [-127, 127]; one fp16 scale per output row (config 1)."""
    assert (n * k) % 4 == 0
    r = rng(seed, 8, *tag)
    packed = r.integers(-127, 128, size=n * k, dtype=np.int8).view(np.uint32)
    scales = r.uniform(scale_lo, scale_hi, size=n).astype(np.float16)
    return packed, scales


def activations(k: int, seed: int, tag=(0,), m: int = 1) -> np.ndarray:
    """fp16 activations drawn from N(0, 1)."""
    return rng(seed, 1, *tag).standard_normal((m, k), dtype=np.float32).astype(np.float16)


def unpack_q4(packed: np.ndarray, n: int, k: int) -> np.ndarray:
    b = np.ascontiguousarray(packed).view(np.uint8)
    lo = (b & 0xF).astype(np.int8)
    hi = (b >> 4).astype(np.int8)
    q = np.empty(b.size * 2, dtype=np.int8)
    q[0::2], q[1::2] = lo, hi
    q = np.where(q >= 8, q - 16, q).astype(np.int8)
    return q[: n * k].reshape(n, k)


def unpack_q8(packed: np.ndarray, n: int, k: int) -> np.ndarray:
    return np.ascontiguousarray(packed).view(np.int8)[: n * k].reshape(n, k)


# Configuration 2 of the measured sweep: (K, N) shapes at M = 1.
Q4_SWEEP = [(1024, 3072), (1024, 512), (1024, 3584), (3584, 1024), (1024, 151936)]


def gemv_bytes(bits: int, n: int, k: int, group: int = 32, scale_bytes: int = 2, act_bytes: int = 2,
               out_bytes: int = 2) -> int:
    """Algorithmic bytes of one GEMV: weights + scales + activation in + output,
    each counted once."""
    w = n * k * bits // 8
    s = (n * k // group if bits == 4 else n) * scale_bytes
    return w + s + k * act_bytes + n * out_bytes


@dataclass
class DecoderCfg:
    n_layers: int = 24
    hidden: int = 1024
    n_heads: int = 8
    n_kv_heads: int = 2
    head_dim: int = 128
    ffn: int = 3584
    vocab: int = 151936
    kv_capacity: int = 2048
    rot_dim: int = 128
    bits: int = 4
    group: int = 32
    lm_bits: int = 4
    lm_group: int = 32
    rope_theta: float = 1e6
    eps: float = 1e-6
    # Hybrid stacks: 0 makes every layer full attention; n > 0 makes layer i
    # full attention when (i + 1) % n == 0 and a linear-attention block
    # (ShortConv + Gated Delta Rule) otherwise. Qwen3.5: 4, i.e. three linear
    # blocks before each full-attention block, 18 + 6 of 24
    # (Qwen35DecoderSession.cs:167-172).
    full_attention_interval: int = 0
    lin_heads: int = 16      # linear attention: heads of q, k, v, z, b and a
    lin_kdim: int = 128      # per-head key dim (the GDR state's rows)
    lin_vdim: int = 128      # per-head value dim (the GDR state's columns)
    conv_kernel: int = 4     # ShortConv taps (cache rows)

    def shapes(self):
        qd, kvd = self.n_heads * self.head_dim, self.n_kv_heads * self.head_dim
        return [(qd, self.hidden), (kvd, self.hidden), (kvd, self.hidden), (self.hidden, qd),
                (self.ffn, self.hidden), (self.ffn, self.hidden), (self.hidden, self.ffn)]

    def layer_types(self) -> list[int]:
        """Per layer 0 (full attention) or 1 (linear attention)."""
        n = self.full_attention_interval
        return [0 if n <= 0 or (i + 1) % n == 0 else 1 for i in range(self.n_layers)]

    def conv_channels(self) -> int:
        """ShortConv channels: q, k and v of every linear-attention head."""
        return 2 * self.lin_heads * self.lin_kdim + self.lin_heads * self.lin_vdim

    def lin_shapes(self):
        """{which: (rows, k)} of a linear-attention layer: 8 in_proj with rows [q k v z b a], 9 out_proj, then
        the FFN's 4, 5, 6."""
        nv = self.lin_heads * self.lin_vdim
        sh = self.shapes()
        return {8: (self.conv_channels() + nv + 2 * self.lin_heads, self.hidden), 9: (self.hidden, nv),
                4: sh[4], 5: sh[5], 6: sh[6]}

    def linears(self, layer: int) -> tuple:
        """The `which` ids a layer loads."""
        return (8, 9, 4, 5, 6) if self.layer_types()[layer] == 1 else tuple(range(7))

    def as_dict(self):
        return asdict(self)


# The synthetic Qwen3.5-0.8B-shaped decoder of configuration 3 (Q4 g32).
QWEN35_08B_Q4 = DecoderCfg()
# Its Q8 per-row variant (configuration 4's weights).
QWEN35_08B_Q8 = DecoderCfg(bits=8, group=0, lm_bits=8, lm_group=0)
# A small model of the same structure for quick parity checks.
TINY = DecoderCfg(n_layers=2, hidden=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=512, vocab=1000,
                  kv_capacity=96, rot_dim=64, group=32, lm_group=32)
# The hybrid Qwen3.5-0.8B layout: 18 linear-attention blocks (16 heads,
# key/value dims 128, conv kernel 4) and 6 full-attention blocks.
QWEN35_08B_HYBRID_Q4 = DecoderCfg(full_attention_interval=4)
QWEN35_08B_HYBRID_Q8 = DecoderCfg(full_attention_interval=4, bits=8, group=0, lm_bits=8, lm_group=0)
# A small hybrid stack [linear, full, linear, full] with kdim != vdim.
TINY_HYBRID = DecoderCfg(n_layers=4, hidden=256, n_heads=4, n_kv_heads=2, head_dim=64, ffn=512, vocab=1000,
                         kv_capacity=96, rot_dim=64, group=32, lm_group=32, full_attention_interval=2,
                         lin_heads=4, lin_kdim=64, lin_vdim=32, conv_kernel=4)


class SyntheticDecoder:
    """Random-init weights of a DecoderCfg in the reference's packed formats.

    linear(layer, which) -> (packed uint32, scales fp16) with which 0..6 =
    q, k, v, o, gate, up, down (layer -1, which 7 = lm_head). Norm and
    embedding weights are fp16 drawn from N(0, 0.02) (the measured configs).

    norm_mean shifts the norm gains to N(norm_mean, 0.02). With the measured
    configs' gains near zero every layer's output is tiny next to the
    residual, attention scores are about 0.01 and the softmax is nearly
    uniform, so the greedy path barely depends on the context. Gains near 1
    (norm_mean=1, as a trained model has) give selective attention and
    context-dependent tokens: a parity check on such a model fails on errors
    in late-position attention or RoPE that the measured model hides.
    balanced_q4 draws the Q4 codes from [-7, 7] (see q4_weights), which such
    a model needs to keep its greedy path from collapsing.
    """

    def __init__(self, cfg: DecoderCfg, seed: int = 3, norm_mean: float = 0.0, balanced_q4: bool = False):
        self.cfg, self.seed, self.norm_mean, self.balanced_q4 = cfg, seed, float(norm_mean), bool(balanced_q4)
        self._lin = {}
        self._norm = {}
        self._lat = {}
        c = cfg
        kinds = c.layer_types()
        for layer in range(c.n_layers):
            shapes = c.lin_shapes() if kinds[layer] == 1 else dict(enumerate(c.shapes()))
            for which, (n, k) in shapes.items():
                self._lin[(layer, which)] = self._make(c.bits, c.group, n, k, (layer, which))
            for which in range(2):
                self._norm[(layer, which)] = self._gain(c.hidden, (100, layer, which))
            if kinds[layer] == 1:
                self._lat[layer] = self._linear_attention_params(layer)
        self._lin[(-1, 7)] = self._make(c.lm_bits, c.lm_group, c.vocab, c.hidden, (999, 7))
        self._norm[(-1, 0)] = self._gain(c.hidden, (100, 999, 0))
        self.embedding = self._normal(c.vocab * c.hidden, (200,)).reshape(c.vocab, c.hidden)

    def _make(self, bits, group, n, k, tag):
        if bits == 4:
            return q4_weights(n, k, group, self.seed, tag, balanced=self.balanced_q4)
        return q8_weights(n, k, self.seed, tag)

    def _normal(self, count, tag):
        return (rng(self.seed, 7, *tag).standard_normal(count, dtype=np.float32) * 0.02).astype(np.float16)

    def _gain(self, count, tag):
        g = rng(self.seed, 7, *tag).standard_normal(count, dtype=np.float32) * 0.02
        return (g + np.float32(self.norm_mean)).astype(np.float16)

    def _linear_attention_params(self, layer):
        """fp16 (conv [channels, kernel] ~ U(-1/2, 1/2), the Conv1d default bound 1/sqrt(kernel) for kernel 4;
        a_log = log(U(0.05, 2)), so the per-token decay exp(-exp(a_log) * softplus(a + dt_bias)) ranges from
        nearly 1 to nearly 0 over the heads; dt_bias ~ N(0, 1/2); gamma ~ N(norm_mean, 0.02) like the other
        gains)."""
        c = self.cfg
        r = rng(self.seed, 9, layer)
        conv = r.uniform(-0.5, 0.5, size=(c.conv_channels(), c.conv_kernel)).astype(np.float16)
        a_log = np.log(r.uniform(0.05, 2.0, size=c.lin_heads)).astype(np.float16)
        dt_bias = (r.standard_normal(c.lin_heads) * 0.5).astype(np.float16)
        gamma = self._gain(c.lin_vdim, (110, layer))
        return conv, a_log, dt_bias, gamma

    def linear(self, layer: int, which: int):
        return self._lin[(layer, which)]

    def linear_attention(self, layer: int):
        """A linear-attention layer's (conv [channels, kernel], a_log [heads], dt_bias [heads], gamma [vdim])."""
        return self._lat[layer]

    def norm(self, layer: int, which: int):
        return self._norm[(layer, which)]

    def prompt(self, length: int, seed: int | None = None) -> np.ndarray:
        """Uniform random token ids."""
        return rng(self.seed if seed is None else seed, 300).integers(0, self.cfg.vocab, size=length).astype(np.int32)

    def weight_bytes_per_token(self) -> int:
        """Algorithmic bytes one greedy token reads: every linear weight and
        scale once, norms, one embedding row (KV traffic is added per step)."""
        c = self.cfg
        tot = 0
        for layer in range(c.n_layers):
            for which in c.linears(layer):
                p, s = self.linear(layer, which)
                tot += p.nbytes + s.nbytes
            tot += 2 * c.hidden * 4
        p, s = self.linear(-1, 7)
        return tot + p.nbytes + s.nbytes + c.hidden * 4 + c.hidden * 2
