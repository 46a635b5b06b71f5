"""Host logic of the data-parallel denoise training step, on CPU: the bucketed
gradient all-reduce averages every gradient over world-size-2 gloo ranks
(buckets split at the byte limit, a tensor larger than the limit alone in its
bucket, views written in place), also when buckets are reduced as their
gradients become ready (in bucket order whatever the readiness order, the
rest flushed by finish()), and the synthetic denoise data has the stated
shapes, ranges and per-seed determinism."""
import os
import socket

import numpy as np
import torch.multiprocessing as mp

from conftest import PKG, REPO

SHAPES = [(3, 5), (17,), (64, 33), (2, 2, 2), (1000,), (7, 9)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _grads(rank):
    import torch
    g = torch.Generator().manual_seed(100 + rank)
    return [torch.randn(s, generator=g) for s in SHAPES]


def _worker(rank, world, port, out_dir, bucket_bytes):
    import sys
    for p in (REPO, PKG):
        sys.path.insert(0, p)
    import datetime
    import torch
    import torch.distributed as dist
    import denoise
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    try:
        grads = _grads(rank)
        storage = [g.clone() for g in grads]       # the "gradient buffers"
        views = [s.view(-1) for s in storage]      # what the trainer hands over
        red = denoise.GradAllReduce(views, bucket_bytes=bucket_bytes)
        red()
        red()  # averaging twice leaves equal buffers unchanged
        nb = [[v.numel() for v in b] for b in red.buckets]
        assert all(s.data_ptr() == v.data_ptr() for s, v in zip(storage, views))
        # overlapped form: gradients become ready in forward order (the last
        # bucket's first), one never does; unknown keys are ignored
        storage2 = [g.clone() for g in grads]
        keys = ["g%d" % i for i in range(len(storage2))]
        red2 = denoise.GradAllReduce([s.view(-1) for s in storage2], bucket_bytes=bucket_bytes,
                                     keys=keys)
        launched = []
        orig = red2._launch
        red2._launch = lambda b: (launched.append(b), orig(b))
        red2.begin()
        red2.ready("not a gradient")
        for k in keys[1:]:
            red2.ready(k)
        before_finish = list(launched)
        red2.finish()
        assert launched == list(range(len(red2.buckets)))
        # grads[0] sits in the last bucket, which only finish() reduces
        assert len(before_finish) == len(red2.buckets) - 1
        # in place: the gradients are slices of one arena per bucket (what
        # for_tensors builds around the trainer's parameters)
        plan = denoise.plan_buckets([g.numel() * 4 for g in grads], bucket_bytes)
        arenas, slices = [], [None] * len(grads)
        for idx in plan:
            arena = torch.zeros(sum(grads[i].numel() for i in idx))
            off = 0
            for i in idx:
                slices[i] = arena[off:off + grads[i].numel()]
                slices[i].copy_(grads[i].view(-1))
                off += grads[i].numel()
            arenas.append(arena)
        red3 = denoise.GradAllReduce(slices, group=None, arenas=arenas, plan=plan)
        red3()
        assert all(f.data_ptr() == a.data_ptr() for f, a in zip(red3.flat, arenas))
        np.savez(os.path.join(out_dir, f"rank{rank}.npz"),
                 *[s.numpy() for s in storage], *[s.numpy() for s in storage2],
                 *[s.view(g.shape).numpy() for s, g in zip(slices, grads)],
                 buckets=np.array(repr(nb)))
    finally:
        dist.destroy_process_group()


def _run(tmp_path, bucket_bytes):
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path), bucket_bytes))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    want = [(a.numpy().astype(np.float64) + b.numpy()) / 2 for a, b in zip(_grads(0), _grads(1))]
    outs = [np.load(os.path.join(tmp_path, f"rank{r}.npz")) for r in range(world)]
    for r in range(world):
        for i, w in enumerate(want):
            np.testing.assert_allclose(outs[r][f"arr_{i}"], w, rtol=1e-6, atol=1e-6)
            np.testing.assert_allclose(outs[r][f"arr_{len(want) + i}"], w, rtol=1e-6, atol=1e-6)
            np.testing.assert_allclose(outs[r][f"arr_{2 * len(want) + i}"], w, rtol=1e-6, atol=1e-6)
    np.testing.assert_array_equal(outs[0]["arr_3"], outs[1]["arr_3"])
    return eval(str(outs[0]["buckets"]))


def test_grad_all_reduce_averages_in_buckets(tmp_path):
    # 512 B buckets: the 1000-float tensor (4000 B) is alone; reverse order
    buckets = _run(tmp_path, 512)
    assert buckets[0] == [63] and buckets[1] == [1000]
    assert sum(sum(b) for b in buckets) == sum(int(np.prod(s)) for s in SHAPES)
    for b in buckets:
        assert len(b) == 1 or 4 * sum(b) <= 512


def test_grad_all_reduce_single_bucket(tmp_path):
    buckets = _run(tmp_path, 1 << 20)
    assert len(buckets) == 1 and buckets[0][0] == 63


def test_denoise_batch_shapes_and_determinism():
    import sys
    sys.path.insert(0, PKG)
    import denoise
    lift = denoise.embedding(32, 5)
    x1, t1 = denoise.denoise_batch(np.random.default_rng(5), 3, 64, lift)
    x2, t2 = denoise.denoise_batch(np.random.default_rng(5), 3, 64, lift)
    assert x1.shape == t1.shape == (3, 64, 32) and x1.dtype == np.float32
    np.testing.assert_array_equal(x1, x2)
    np.testing.assert_array_equal(t1, t2)
    # the clean target is an affine lift of one scalar signal per position
    w, b = lift
    sig = (t1 - b) / w
    np.testing.assert_allclose(sig, np.repeat(sig[..., :1], 32, axis=2), atol=1e-4)
    assert np.abs(sig).max() <= 4.0
    noise = x1 - t1
    assert abs(noise.std() - 0.1) < 0.01 and abs(noise.mean()) < 0.01
    x3, _ = denoise.denoise_batch(np.random.default_rng(6), 3, 64, lift)
    assert not np.array_equal(x1, x3)


def test_plan_buckets_reverse_order_and_small_tail_buckets():
    import denoise
    sizes = [100, 100, 100, 100, 100, 100]
    # reverse order, buckets of at most 250 B: [5, 4], [3, 2], [1, 0]
    assert denoise.plan_buckets(sizes, 250) == [[5, 4], [3, 2], [1, 0]]
    # the last 200 B in order (gradients 1 and 0, finished last) get 100 B buckets
    assert denoise.plan_buckets(sizes, 250, tail_bytes=200, tail_bucket_bytes=100) == \
        [[5, 4], [3, 2], [1], [0]]
    # a gradient larger than the bucket size gets a bucket of its own
    assert denoise.plan_buckets([10, 500, 10], 100) == [[2], [1], [0]]
