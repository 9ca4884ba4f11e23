"""The multi-GPU path's host logic on two gloo ranks (CPU): each rank takes its contiguous shard of the batch of
independent sequences, runs it (here: on the oracle, standing in for its GPU), and the shards together equal the
whole batch; the bench's max-over-ranks reduction picks the slowest rank. No collective touches the data path
except the final gather this test does to check the result."""
import os

import numpy as np
import torch.multiprocessing as mp


def _rank(rank, world, port, q):
    import sys
    here = os.path.dirname(os.path.abspath(__file__))
    sys.path[:0] = [os.path.join(os.path.dirname(here), "anvil-compiler_b200"), os.path.dirname(here), here]
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import anvil
        from anvil.driver import CudaParams
        from graphs import random_case
        from oracle import interp
        import bench
        m, c, x, want = random_case(5, batch=6)
        cm = anvil.compile(m, consts=c, prove=False, params=CudaParams(devices=tuple(range(world))))
        shards = cm._shards(6)
        _, lo, hi = shards[rank]
        mine = interp.run(m, {k: v[lo:hi] for k, v in x.items()}, c, batch=True)
        out = torch.tensor(mine.outputs[0])
        parts = [torch.zeros((hi_ - lo_,) + tuple(out.shape[1:]), dtype=out.dtype) for _, lo_, hi_ in shards]
        dist.all_gather(parts, out)
        whole = torch.cat(parts).numpy()
        slowest = bench._max_over_ranks(dist, float(rank + 1))
        q.put((rank, bool(np.array_equal(whole, want.outputs[0])), slowest))
    finally:
        dist.destroy_process_group()


def test_two_rank_shards_reassemble_the_batch():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29500 + os.getpid() % 1000
    ps = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=180) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert [r[1] for r in res] == [True, True]
    assert [r[2] for r in res] == [2.0, 2.0]
