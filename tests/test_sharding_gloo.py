"""Multi-rank host logic of the batch x head sharding, on CPU with world-size-2
gloo process groups: shards partition the batch, the timing reduction returns
the max over ranks, and attention computed per shard (float64 oracle) equals
the unsharded result - the units are independent, so no collective is needed."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from conftest import PKG, REPO


def test_shard_batches_partition():
    import sharding
    for B in (1, 7, 8, 64):
        for world in (1, 2, 3, 8):
            ranges = [sharding.shard_batches(B, world, r) for r in range(world)]
            covered = [b for (b0, b1) in ranges for b in range(b0, b1)]
            assert covered == list(range(B))
            sizes = [b1 - b0 for b0, b1 in ranges]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sharding.shard_batches(8, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_dir):
    import sys
    for p in (REPO, PKG, os.path.join(REPO, "oracle"), os.path.join(REPO, "tests")):
        sys.path.insert(0, p)
    import datetime
    import torch.distributed as dist
    import oracle
    import sharding
    from conftest import seeded_normal
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        # timing reduction: rank r reports 10 + r
        mx = sharding.max_over_ranks(10.0 + rank)
        B, L, H, D = 4, 48, 2, 16
        q, k, v = (seeded_normal(s, (B, L, H, D)) for s in (1, 2, 3))
        b0, b1 = sharding.shard_batches(B, world, rank)
        o, lse = oracle.attn_fwd(q[b0:b1], k[b0:b1], v[b0:b1])
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"), o=o, lse=lse, b0=b0, b1=b1, mx=mx)
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_sharded_attention_and_timing(tmp_path):
    import sys
    for p in (REPO, PKG, os.path.join(REPO, "oracle")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import oracle
    from conftest import seeded_normal
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    B, L, H, D = 4, 48, 2, 16
    q, k, v = (seeded_normal(s, (B, L, H, D)) for s in (1, 2, 3))
    o_full, lse_full = oracle.attn_fwd(q, k, v)
    for r in range(world):
        z = np.load(os.path.join(tmp_path, f"rank{r}.npz"))
        assert float(z["mx"]) == 10.0 + world - 1
        b0, b1 = int(z["b0"]), int(z["b1"])
        np.testing.assert_array_equal(z["o"], o_full[b0:b1])
        np.testing.assert_array_equal(z["lse"], lse_full[b0 * H:b1 * H])
