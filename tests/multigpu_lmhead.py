"""One rank of tests/test_gpu_multi.py (launched through torch.distributed.run,
one process per GPU): the vocab-sharded lm_head over `world` GPUs with the
peer-memory exchange and with the collective one, against one GPU holding
the whole vocabulary. Exits non-zero on any mismatch."""
import datetime
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from aiimage_b200 import synth  # noqa: E402
from aiimage_b200.ops import AexisOps  # noqa: E402
from aiimage_b200.sharded import ShardedLmHead  # noqa: E402


def main():
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    ops = AexisOps(local)
    vocab, hidden, k = 20011, 256, 50
    p, s = synth.q8_weights(vocab, hidden, seed=7, tag=(vocab, hidden))
    peer = ShardedLmHead(ops, p, s, vocab, hidden, world, rank)
    coll = ShardedLmHead(ops, p, s, vocab, hidden, world, rank, exchange="collective")
    whole = ShardedLmHead(ops, p, s, vocab, hidden, 1, 0)
    assert peer.uses_peer_exchange() and not coll.uses_peer_exchange()
    bad = 0
    # Five calls over two batch shapes: both slot parities, and a new exchange when the shape changes.
    for call, m in enumerate((19, 19, 19, 8, 8)):
        x = torch.from_numpy(synth.activations(hidden, seed=11 + call, tag=(m, hidden), m=m)).cuda()
        got_p = peer.forward(x, k)
        got_c = coll.forward(x, k)
        ref = whole.forward(x, k)
        for a, b, c in zip(got_p, got_c, ref):
            if not (torch.equal(a, c) and torch.equal(b, c)):
                bad += 1
                print(f"rank {rank} call {call}: mismatch", flush=True)
    peer.close()
    for h in (peer, coll, whole):
        h.w.free()
    ops.close()
    dist.barrier()
    dist.destroy_process_group()
    if bad:
        sys.exit(1)
    print(f"OK rank {rank} of {world}", flush=True)


if __name__ == "__main__":
    main()
