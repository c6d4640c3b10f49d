"""Device-side token sampling: the host mirror of Qwen35Sampler
(Packages/com.aexis/Samples/AIImageApplicationExample/Runtime/Scripts/
Qwen35DecoderSession.cs:1823-1900) over libaexis_cuda's aexis_cuda_sample.

The reference keeps a history set, copies each step's logits to the host and
sorts the whole vocabulary there. Here the history is a device bitmap, the
selection runs in three kernels on the logits where they are, and the host
only supplies one uniform draw per row from the same random stream the
reference uses (System.Random seeded with Qwen35SamplingConfig.Seed).
"""
from __future__ import annotations

import dataclasses

import numpy as np

_MBIG = 2147483647
_MSEED = 161803398


def _i32(x: int) -> int:
    return ((x + 2**31) % 2**32) - 2**31


class DotNetRandom:
    """System.Random(int seed) of .NET (the seeded, compatible generator: Knuth's subtractive method with a
    55-entry table, as published in the .NET runtime's Random implementation and Numerical Recipes' ran3).
    Only NextDouble is needed: Qwen35Sampler.Select draws one value per sampling call (:1886).
    C# int arithmetic wraps at 32 bits; the seeding does the same here."""

    def __init__(self, seed: int):
        seed = _i32(int(seed))
        subtraction = _MBIG if seed == -2**31 else abs(seed)
        mj = _i32(_MSEED - subtraction)
        table = [0] * 56
        table[55] = mj
        mk = 1
        for i in range(1, 55):
            ii = (21 * i) % 55
            table[ii] = mk
            mk = _i32(mj - mk)
            if mk < 0:
                mk += _MBIG
            mj = table[ii]
        for _ in range(4):
            for i in range(1, 56):
                table[i] = _i32(table[i] - table[1 + (i + 30) % 55])
                if table[i] < 0:
                    table[i] += _MBIG
        self._t = table
        self._inext = 0
        self._inextp = 21

    def _internal_sample(self) -> int:
        a = self._inext + 1
        if a >= 56:
            a = 1
        b = self._inextp + 1
        if b >= 56:
            b = 1
        ret = _i32(self._t[a] - self._t[b])
        if ret == _MBIG:
            ret -= 1
        if ret < 0:
            ret += _MBIG
        self._t[a] = ret
        self._inext, self._inextp = a, b
        return ret

    def next_double(self) -> float:
        return self._internal_sample() * (1.0 / _MBIG)


@dataclasses.dataclass
class SamplingConfig:
    """Qwen35SamplingConfig (Qwen35DecoderSession.cs:136-149), same defaults."""
    do_sample: bool = True
    temperature: float = 0.3
    top_p: float = 0.8
    top_k: int = 50
    repetition_penalty: float = 1.1
    seed: int = 20260718

    @staticmethod
    def greedy() -> "SamplingConfig":
        return SamplingConfig(do_sample=False, temperature=0.0, top_p=1.0, top_k=0, repetition_penalty=1.0)


class DeviceSampler:
    """Qwen35Sampler for `rows` independent sessions sharing one config: each row has its own history and its
    own System.Random stream (seeded with config.seed, or `seeds[r]`).

    One difference from the reference: the reference takes its draw only when it reaches the draw (not on the
    greedy fallback of a non-finite softmax sum); here every sampling call takes one draw per row."""

    def __init__(self, ops, vocab: int, config: SamplingConfig | None = None, rows: int = 1, seeds=None):
        import torch
        if vocab <= 0:
            from . import errors
            raise errors.ArgumentOutOfRangeError("vocabularySize")
        self.ops, self.vocab, self.rows = ops, vocab, rows
        self.config = config or SamplingConfig()
        seeds = [self.config.seed] * rows if seeds is None else list(seeds)
        self._rng = [DotNetRandom(s) for s in seeds]
        self._words = (vocab + 31) // 32
        self.history = torch.zeros((rows, self._words), dtype=torch.int32, device="cuda")
        self._u = torch.zeros(rows, dtype=torch.float64, device="cuda")
        self.out = torch.zeros(rows, dtype=torch.int32, device="cuda")

    @property
    def can_use_texture_argmax(self) -> bool:
        """Qwen35Sampler.CanUseTextureArgMax (:1838-1840): plain greedy argmax suffices."""
        c = self.config
        return (not c.do_sample or c.temperature <= 0.0) and abs(c.repetition_penalty - 1.0) < 1e-6

    def add_history(self, tokens) -> None:
        """Qwen35Sampler.AddHistory for every row: tokens is a device int32 [rows] tensor."""
        self.ops.sample_history_add(self.history, self.rows, self.vocab, tokens)

    def select(self, logits, ld: int | None = None):
        """Qwen35Sampler.Select for every row of the device fp32 logits [rows, >= vocab]; returns the device
        int32 [rows] token ids (no host synchronisation)."""
        c = self.config
        sample = c.do_sample and c.temperature > 0.0
        if sample:
            # A pageable source: the copy has consumed it when copy_ returns, so the next call may draw again.
            self._u.copy_(torch_tensor([r.next_double() for r in self._rng]))
        self.ops.sample(logits, self.rows, self.vocab, self.history, c.repetition_penalty,
                        c.temperature if sample else 0.0, c.top_k, c.top_p, self._u if sample else None, self.out,
                        ld=ld)
        return self.out


def torch_tensor(values):
    import torch
    return torch.tensor(np.asarray(values, dtype=np.float64))
