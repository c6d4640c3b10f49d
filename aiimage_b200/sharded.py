"""Vocabulary-sharded lm_head with greedy argmax and top-k.

Rank r of G holds the contiguous lm_head rows [r*V/G, (r+1)*V/G) as a Q8 weight
handle. One call:
  1. logits of the shard, [M, V/G] fp32, on the tensor cores (aexis_cuda_gemm);
  2. per row the shard's argmax as a 64-bit key carrying the GLOBAL index
     (aexis_cuda_argmax_keys) and the shard's top-k (aexis_cuda_topk, indices
     shifted by the shard offset);
  3. one all-reduce MAX over the keys and one all-gather of the top-k lists
     (NCCL over NVLink; gloo in the CPU tests), then a deterministic merge.
Every logit is computed by exactly one rank with the same kernel and the same
K order whatever G is, and the key's tie rule (lowest global index) matches
the single-device scan (AexisArgMaxPack4LinearMat, HLSL Pack4Matmul:645-686),
so the token ids are bit-identical for every G.
"""
from __future__ import annotations

import torch

_SIGN = -(1 << 63)  # int64 bit 63


def shard_range(vocab: int, world: int, rank: int):
    per = (vocab + world - 1) // world
    lo = min(vocab, rank * per)
    return lo, min(vocab, lo + per)


def keys_to_ids(keys: torch.Tensor) -> torch.Tensor:
    """Global index from a 64-bit key (int64 view of the uint64 key)."""
    return (0xFFFFFFFF - (keys & 0xFFFFFFFF)).to(torch.int64)


def reduce_keys(keys: torch.Tensor, group=None) -> torch.Tensor:
    """All-reduce MAX of uint64 keys held in an int64 tensor: flipping bit 63
    maps unsigned order onto signed order and back."""
    import torch.distributed as dist
    k = keys ^ _SIGN
    dist.all_reduce(k, op=dist.ReduceOp.MAX, group=group)
    return k ^ _SIGN


def merge_topk(vals: torch.Tensor, idx: torch.Tensor, k: int, group=None):
    """All-gather the per-shard top-k (values, global indices) and keep the k
    largest per row, equal values ordered by ascending index."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    vs = [torch.empty_like(vals) for _ in range(world)]
    ix = [torch.empty_like(idx) for _ in range(world)]
    dist.all_gather(vs, vals.contiguous(), group=group)
    dist.all_gather(ix, idx.contiguous(), group=group)
    v = torch.cat(vs, dim=1)
    i = torch.cat(ix, dim=1)
    return topk_merge_local(v, i, k)


def topk_merge_local(v: torch.Tensor, i: torch.Tensor, k: int):
    # Stable sorts: by index ascending, then by value descending.
    o1 = torch.argsort(i, dim=1, stable=True)
    v1, i1 = torch.gather(v, 1, o1), torch.gather(i, 1, o1)
    o2 = torch.argsort(v1, dim=1, descending=True, stable=True)
    return torch.gather(v1, 1, o2)[:, :k], torch.gather(i1, 1, o2)[:, :k]


class ShardedLmHead:
    """One rank's shard of the lm_head (see module docstring)."""

    def __init__(self, ops, packed, scales, vocab: int, hidden: int, world: int = 1, rank: int = 0, group=None):
        self.ops, self.vocab, self.hidden, self.group = ops, vocab, hidden, group
        self.lo, self.hi = shard_range(vocab, world, rank)
        self.n = self.hi - self.lo
        import numpy as np
        p8 = np.ascontiguousarray(packed).view(np.int8).reshape(vocab, hidden)[self.lo:self.hi]
        self.w = ops.new_int8_weight_only_upload(np.ascontiguousarray(p8).view(np.uint32),
                                                 np.ascontiguousarray(scales[self.lo:self.hi]), self.n, hidden)
        self.world = world

    def shard_logits(self, x: torch.Tensor, out: torch.Tensor | None = None) -> torch.Tensor:
        m = x.shape[0]
        if out is None:
            out = torch.empty((m, self.n), dtype=torch.float32, device=x.device)
        self.ops.set_int4_gemm_weights(None)
        self.ops.set_int8_gemm_weights(self.w)
        self.ops.gemm2d_pack4_tiled_texture_a(x, None, m, self.n, self.hidden, True, 1.0, 1.0, False, 4, out)
        return out

    def forward(self, x: torch.Tensor, k: int = 50, logits: torch.Tensor | None = None):
        """Greedy ids [M] (int64) and the global top-k (values [M,k], ids [M,k])."""
        m = x.shape[0]
        logits = self.shard_logits(x, logits)
        keys = torch.empty(m, dtype=torch.int64, device=x.device)
        self.ops.argmax_keys(logits, self.n, m, self.lo, keys)
        vals = torch.empty((m, k), dtype=torch.float32, device=x.device)
        idx = torch.empty((m, k), dtype=torch.int32, device=x.device)
        self.ops.top_k(logits, self.n, m, k, vals, idx)
        gidx = idx.to(torch.int64) + self.lo
        if self.world > 1:
            keys = reduce_keys(keys, self.group)
            vals, gidx = merge_topk(vals, gidx, k, self.group)
        return keys_to_ids(keys), vals, gidx
