"""The vocab-sharded lm_head exchange (config 5) on CPU: world size 2 over
gloo. Each rank holds half of the logits and packs its argmax keys (global
indices) and its top-k (shard-local indices) into one buffer; one all-gather
of the buffers, then the merge (restated here on the host; the device kernel
is tested against full-vocabulary kernels in test_gpu_ops.py) must give the
full-vocabulary oracle's greedy ids and top-k (ties included)."""
import os
import socket

import numpy as np
import pytest


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ukey(v: float, idx: int) -> int:
    """The 64-bit greedy key of aexis_argmax_key (unsigned)."""
    b = int(np.float32(0.0 if v == 0 else v).view(np.uint32))
    if v != v:
        hi = 0xFFFFFFFF if idx == 0 else 0
    else:
        hi = (~b & 0xFFFFFFFF) if (b & 0x80000000) else (b | 0x80000000)
    return (hi << 32) | (0xFFFFFFFF - idx)


def _signed(u: int) -> int:
    return u - (1 << 64) if u >= (1 << 63) else u


def _logits():
    r = np.random.default_rng(123)
    x = r.standard_normal((6, 1001)).astype(np.float32)
    x[0, 3] = x[0, 700] = x[0].max() + 1  # tie across shards -> lowest index
    x[1, 510] = x[1, 520] = x[1].max() + 1  # tie inside shard 1
    x[2, :] = -5.0
    x[2, 900] = 7.0
    x[3, 40:60] = 9.0  # a plateau straddling ranks is not needed; 20 equal values in shard 0
    return x


def _reference_merge(gathered, world, rows, k, per):
    """The merge aexis_cuda_topk_merge performs on the device, restated on
    the host: the largest unsigned key per row, and the k largest (value,
    global index) pairs (value descending, index ascending)."""
    import torch
    from aiimage_b200 import sharded
    w = sharded.packed_words(rows, k)
    ids, vals, idx = [], [], []
    for row in range(rows):
        best, cand = None, []
        for r in range(world):
            keys, v, i = sharded.pack_views(gathered[r * w:(r + 1) * w], rows, k)
            u = int(keys[row]) & ((1 << 64) - 1)
            best = u if best is None else max(best, u)
            cand += [(float(v[row, j]), r * per + int(i[row, j])) for j in range(k) if int(i[row, j]) >= 0]
        cand.sort(key=lambda t: (-t[0], t[1]))
        cand = cand[:k] + [(float("-inf"), -1)] * (k - len(cand[:k]))
        ids.append(int(sharded.keys_to_ids(torch.tensor([_signed(best)]))[0]))
        vals.append([c[0] for c in cand])
        idx.append([c[1] for c in cand])
    return ids, vals, idx


def _worker(rank, world, port, out):
    import torch
    import torch.distributed as dist
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    import oracle as O
    from aiimage_b200 import sharded
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    x = _logits()
    rows, k = x.shape[0], 10
    lo, hi = sharded.shard_range(x.shape[1], world, rank)
    part = x[:, lo:hi]
    # This rank's packed buffer: keys in unsigned key order (as the kernel
    # computes them), then its top-k with shard-local indices.
    buf = torch.zeros(sharded.packed_words(rows, k), dtype=torch.int32)
    keys, vals, idx = sharded.pack_views(buf, rows, k)
    keys[:] = torch.tensor([_signed(max(_ukey(float(v), lo + i) for i, v in enumerate(row))) for row in part],
                           dtype=torch.int64)
    v, i = O.topk(part, k)
    vals[:] = torch.from_numpy(v)
    idx[:] = torch.from_numpy(i)
    gathered = sharded.exchange(buf)
    if rank == 0:
        per = (x.shape[1] + world - 1) // world
        ids, mv, mi = _reference_merge(gathered, world, rows, k, per)
        out["ids"] = ids
        out["vals"] = mv
        out["idx"] = mi
    dist.destroy_process_group()


def test_sharded_exchange_matches_full_vocab():
    import multiprocessing as mp
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    import oracle as O
    ctx = mp.get_context("spawn")
    with ctx.Manager() as mgr:
        out = mgr.dict()
        port = _free_port()
        procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        res = dict(out)
    x = _logits()
    assert res["ids"] == O.argmax(x).tolist()
    assert res["ids"][0] == 3 and res["ids"][1] == 510
    v, i = O.topk(x, 10)
    assert np.array_equal(np.array(res["idx"]), i)
    assert np.array_equal(np.array(res["vals"], dtype=np.float32), v)


def test_key_order_matches_scan():
    vals = [1.0, -0.0, 0.0, -3.0, 2.5, 2.5]
    keys = [_signed(_ukey(v, i)) for i, v in enumerate(vals)]
    from aiimage_b200 import sharded
    import torch
    best = _signed(max(_ukey(v, i) for i, v in enumerate(vals)))
    assert int(sharded.keys_to_ids(torch.tensor([best]))[0]) == 4
    assert max(_ukey(v, i) for i, v in enumerate(vals)) == _ukey(2.5, 4)
