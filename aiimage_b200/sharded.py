"""Vocabulary-sharded lm_head with greedy argmax and top-k.

Rank r of G holds the contiguous lm_head rows [r*V/G, (r+1)*V/G) as a Q8 weight
handle. One call:
  1-2. per row the shard's top-k and, from its first entry, the shard's
     argmax as a 64-bit key carrying the GLOBAL index, in one
     aexis_cuda_gemm_topk: the [M, V/G] logits on the tensor cores, then the
     top-k and the greedy keys from the top-k lists (aexis_cuda_gemm_tiled +
     aexis_cuda_topk + aexis_cuda_topk_greedy_keys in one call);
  3. the keys and the top-k lists packed into one buffer, one all-gather of
     those buffers (NCCL over NVLink; gloo in the CPU tests), then one merge
     kernel (aexis_cuda_topk_merge): the largest key, and the k largest
     (value, global index) keys of the shards' sorted lists.
Every logit is computed by exactly one rank with the same kernel and the same
K order whatever G is, and the key's tie rule (lowest global index) matches
the single-device scan (AexisArgMaxPack4LinearMat, HLSL Pack4Matmul:645-686),
so the token ids are bit-identical for every G.
"""
from __future__ import annotations

import torch

def shard_range(vocab: int, world: int, rank: int):
    per = (vocab + world - 1) // world
    lo = min(vocab, rank * per)
    return lo, min(vocab, lo + per)


def keys_to_ids(keys: torch.Tensor) -> torch.Tensor:
    """Global index from a 64-bit key (int64 view of the uint64 key)."""
    return (0xFFFFFFFF - (keys & 0xFFFFFFFF)).to(torch.int64)


def packed_words(rows: int, k: int) -> int:
    """32-bit words of one shard's packed result: rows uint64 greedy keys,
    rows x k fp32 top-k values, rows x k int32 shard-local indices."""
    return 2 * rows + 2 * rows * k


def pack_views(buf: torch.Tensor, rows: int, k: int):
    """(keys int64 [rows], vals fp32 [rows, k], idx int32 [rows, k]) views of
    one shard's packed buffer (int32 [packed_words])."""
    keys = buf[: 2 * rows].view(torch.int64)
    vals = buf[2 * rows: 2 * rows + rows * k].view(torch.float32).view(rows, k)
    idx = buf[2 * rows + rows * k:].view(rows, k)
    return keys, vals, idx


def exchange(buf: torch.Tensor, group=None) -> torch.Tensor:
    """All-gather of every rank's packed buffer into one tensor [world * W],
    rank order: one NCCL all-gather over NVLink (gloo in the CPU tests)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if dist.get_backend(group) == "nccl":
        out = torch.empty(world * buf.numel(), dtype=buf.dtype, device=buf.device)
        dist.all_gather_into_tensor(out, buf, group=group)
        return out
    parts = [torch.empty_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf, group=group)
    return torch.cat(parts)


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

    def shard_topk(self, x: torch.Tensor, k: int, keys, vals, idx):
        """The shard's top-k (shard-local indices) and greedy keys (global indices), fused with its GEMM."""
        self.ops.set_int4_gemm_weights(None)
        self.ops.set_int8_gemm_weights(self.w)
        self.ops.gemm_topk(x, x.shape[0], self.hidden, k, vals, idx, keys, 1.0, self.lo)

    def forward(self, x: torch.Tensor, k: int = 50, logits: torch.Tensor | None = None):
        """Greedy ids [M] (int64) and the global top-k (values [M,k], ids [M,k]).
        `logits` is accepted for compatibility and not used (nothing is materialised)."""
        m = x.shape[0]
        if self.world == 1:
            keys = torch.empty(m, dtype=torch.int64, device=x.device)
            vals = torch.empty((m, k), dtype=torch.float32, device=x.device)
            idx = torch.empty((m, k), dtype=torch.int32, device=x.device)
            self.shard_topk(x, k, keys, vals, idx)
            return keys_to_ids(keys), vals, idx.to(torch.int64)
        # The shard's keys and top-k straight into one packed buffer, one
        # all-gather, one merge kernel.
        buf = torch.empty(packed_words(m, k), dtype=torch.int32, device=x.device)
        keys, vals, idx = pack_views(buf, m, k)
        self.shard_topk(x, k, keys, vals, idx)
        return self.merge(buf, m, k)

    def merge(self, buf: torch.Tensor, m: int, k: int):
        """The exchange step alone: all-gather every rank's packed buffer, then the merge kernel."""
        gathered = exchange(buf, self.group)
        ids = torch.empty(m, dtype=torch.int64, device=buf.device)
        out_v = torch.empty((m, k), dtype=torch.float32, device=buf.device)
        out_i = torch.empty((m, k), dtype=torch.int32, device=buf.device)
        per = (self.vocab + self.world - 1) // self.world
        self.ops.topk_merge(gathered, self.world, m, k, per, ids, out_v, out_i)
        return ids, out_v, out_i.to(torch.int64)
