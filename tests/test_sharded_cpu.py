"""The vocab-sharded lm_head exchange (config 5) on CPU: world size 2 over
gloo. Each rank holds half of the logits, packs its argmax keys with global
indices and its top-k, and the all-reduce / all-gather merge must give the
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
    lo, hi = sharded.shard_range(x.shape[1], world, rank)
    part = x[:, lo:hi]
    # Each shard's maximum is taken in unsigned key order, as the kernel does.
    keys = torch.tensor([_signed(max(_ukey(float(v), lo + i) for i, v in enumerate(row))) for row in part],
                        dtype=torch.int64)
    vals, idx = O.topk(part, 10)
    ids = sharded.keys_to_ids(sharded.reduce_keys(keys))
    mv, mi = sharded.merge_topk(torch.from_numpy(vals), torch.from_numpy(idx.astype(np.int64)) + lo, 10)
    if rank == 0:
        out["ids"] = ids.tolist()
        out["vals"] = mv.numpy().tolist()
        out["idx"] = mi.numpy().tolist()
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
    best = max(k ^ (-(1 << 63)) for k in keys) ^ (-(1 << 63))
    assert int(sharded.keys_to_ids(torch.tensor([best]))[0]) == 4
    assert max(_ukey(v, i) for i, v in enumerate(vals)) == _ukey(2.5, 4)
