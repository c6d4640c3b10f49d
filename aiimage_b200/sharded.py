"""Vocabulary-sharded lm_head with greedy argmax and top-k.

Rank r of G holds the contiguous lm_head rows [r*V/G, (r+1)*V/G) as a Q8 weight
handle. One call:
  1-2. per row the shard's top-k and, from its first entry, the shard's
     argmax as a 64-bit key carrying the GLOBAL index, in one
     aexis_cuda_gemm_topk: the [M, V/G] logits on the tensor cores, then the
     top-k and the greedy keys from the top-k lists (aexis_cuda_gemm_tiled +
     aexis_cuda_topk + aexis_cuda_topk_greedy_keys in one call);
  3. the keys and the top-k lists packed into one buffer, exchanged between
     the ranks, then one merge kernel: the largest key, and the k largest
     (value, global index) keys of the shards' sorted lists. With NCCL ranks
     (one process per GPU of a node) the exchange goes over peer memory: each
     rank's push kernel writes its buffer into every rank's receive buffer
     over NVLink and releases an epoch flag, and the merge kernel waits for
     all flags (aexis_cuda_topk_push / aexis_cuda_topk_merge_peers, buffers
     mapped through CUDA IPC handles). exchange="collective" (and gloo, in
     the CPU tests) uses one all-gather and aexis_cuda_topk_merge instead.
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


class PeerExchange:
    """Every rank's packed result through peer memory: one receive buffer per
    rank (aexis_cuda_peer_buffer_create), the others' buffers mapped here by
    their IPC handles (all-gathered once through torch.distributed), then per
    call a push of this rank's buffer into every receive buffer and a merge
    that waits for the call's epoch in this rank's own buffer (the epoch is a
    device counter: a call can be captured in a CUDA graph)."""

    def __init__(self, ops, rows: int, k: int, world: int, rank: int, group=None):
        import torch.distributed as dist
        self.ops, self.rows, self.k, self.world, self.rank, self.group = ops, rows, k, world, rank, group
        self.own, handle = ops.peer_buffer_create(ops.peer_buffer_bytes(world, rows, k))
        handles = [None] * world
        dist.all_gather_object(handles, handle, group=group)
        self.peers = [self.own if r == rank else ops.peer_buffer_open(h) for r, h in enumerate(handles)]
        dist.barrier(group=group)  # every buffer mapped everywhere before the first push

    def merge(self, buf: torch.Tensor, shard_rows: int, ids, vals, idx):
        self.ops.topk_push(buf, self.rows, self.k, self.peers, self.rank)
        self.ops.topk_merge_peers(self.own, self.world, self.rows, self.k, shard_rows, ids, vals, idx)

    def close(self):
        """Unmap the others' buffers and free this one, once every rank is past its last merge."""
        import torch.distributed as dist
        self.ops.sync()
        dist.barrier(group=self.group)
        for r, p in enumerate(self.peers):
            if r != self.rank:
                self.ops.peer_buffer_close(p, True)
        dist.barrier(group=self.group)
        self.ops.peer_buffer_close(self.own, False)
        self.peers = []


class ShardedLmHead:
    """One rank's shard of the lm_head (see module docstring)."""

    def __init__(self, ops, packed, scales, vocab: int, hidden: int, world: int = 1, rank: int = 0, group=None,
                 exchange: str = "auto"):
        if exchange not in ("auto", "peer", "collective"):
            raise ValueError(f"exchange={exchange!r} (auto, peer or collective)")
        self.ops, self.vocab, self.hidden, self.group = ops, vocab, hidden, group
        self.rank, self.exchange_mode, self._peer = rank, exchange, None
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

    def uses_peer_exchange(self) -> bool:
        """Whether merge goes over peer memory (NCCL ranks, exchange "auto" or "peer")."""
        if self.world == 1 or self.exchange_mode == "collective":
            return False
        import torch.distributed as dist
        return dist.get_backend(self.group) == "nccl"

    def merge(self, buf: torch.Tensor, m: int, k: int):
        """The exchange step alone: every rank's packed buffer to every rank, then the merge kernel."""
        ids = torch.empty(m, dtype=torch.int64, device=buf.device)
        out_v = torch.empty((m, k), dtype=torch.float32, device=buf.device)
        out_i = torch.empty((m, k), dtype=torch.int32, device=buf.device)
        self.merge_into(buf, m, k, ids, out_v, out_i)
        return ids, out_v, out_i.to(torch.int64)

    def merge_into(self, buf: torch.Tensor, m: int, k: int, ids, out_v, out_i):
        """merge into caller-owned outputs (ids int64 [m], values fp32 [m, k],
        global indices int32 [m, k]). The peer path allocates nothing once its
        buffers exist for (m, k), so a call can be captured in a CUDA graph."""
        per = (self.vocab + self.world - 1) // self.world
        if self.uses_peer_exchange():
            if self._peer is None or (self._peer.rows, self._peer.k) != (m, k):
                if self._peer is not None:
                    self._peer.close()
                self._peer = PeerExchange(self.ops, m, k, self.world, self.rank, self.group)
            self._peer.merge(buf, per, ids, out_v, out_i)
        else:
            gathered = exchange(buf, self.group)
            self.ops.topk_merge(gathered, self.world, m, k, per, ids, out_v, out_i)

    def close(self):
        """Release the peer exchange's buffers (collective: every rank calls it)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None
