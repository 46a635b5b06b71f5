"""The denoise training step on one GPU: a two-layer denoise transformer
(tests/main_denoise.py:27-54 stacked) forward + MSE + backward against torch
float64 with the same weights (loss within 1e-4, every parameter gradient and
the input gradient within 1e-3 norm-wise); the trainer reduces the loss on the
synthetic denoise data; a checkpoint restores parameters, Adam moments and
step count exactly; two NCCL ranks with half the batch each take the same
steps as one rank with the whole batch (needs two GPUs)."""
import math
import os
import socket

import numpy as np
import pytest

from conftest import PKG, REPO, rel_err

torch = pytest.importorskip("torch")
F32_TOL = 1e-3


@pytest.fixture(scope="module")
def dn():
    import denoise
    return denoise


@pytest.fixture(autouse=True)
def _default_math():
    """Trainers set the thread's float32 math mode; put the default back."""
    yield
    if torch.cuda.is_available():
        import PureAttention as pa
        pa.set_float32_math("split3")


def _h(t):
    return np.asarray(t.to_host(), dtype=np.float64).reshape(t.shape())


def _g(t):
    return np.asarray(t.grad_to_host(), dtype=np.float64).reshape(t.shape())


def _ref_layer(x, P, H):
    """float64 torch restatement of one denoise layer; P = its 14 parameters
    in TransformerLayer.parameters() order."""
    wi, bi, wo, bo, g1, c1, w1, b1, w2, b2, g2, c2, g3, c3 = P
    B, L, E = x.shape
    D = E // H

    def ln(v, g, c):
        mu = v.mean(-1, keepdim=True)
        var = ((v - mu) ** 2).mean(-1, keepdim=True)
        return (v - mu) / torch.sqrt(var + 1e-5) * g + c

    xn = ln(x, g1, c1)
    qkv = xn @ wi + bi
    q, k, v = (qkv[..., i * E:(i + 1) * E].reshape(B, L, H, D).transpose(1, 2) for i in range(3))
    s = q @ k.transpose(-1, -2) / math.sqrt(D)
    o = (torch.softmax(s, -1) @ v).transpose(1, 2).reshape(B, L, E)
    x = x + (o @ wo + bo)
    h = torch.relu(ln(x, g2, c2) @ w1 + b1) @ w2 + b2
    return ln(x + h, g3, c3)


@pytest.mark.gpu
@pytest.mark.parametrize("math_mode,tol", [("split3", F32_TOL), ("bf16", 3e-2)])
def test_two_layer_denoise_model_matches_float64(dn, math_mode, tol):
    """split3: every gradient within 1e-3 of float64; bf16 products: within
    3e-2 (operands rounded to 8 mantissa bits, fp32 accumulation)."""
    import PureAttention as pa
    B, L, E, H, F = 2, 160, 128, 4, 256
    pa.set_float32_math(math_mode)
    pa.set_seed(77)
    model = dn.DenoiseTransformer(2, E, H, F)
    params = model.parameters()
    assert len(params) == 28
    # non-trivial LayerNorm affine parameters and biases
    rng = np.random.default_rng(8)
    for p in params:
        if p.shape()[0] == 1:
            n = p.shape()[1]
            base = 1.0 if np.allclose(_h(p), 1.0) else 0.0
            p.to_device((base + 0.1 * rng.standard_normal(n)).astype(np.float32).tolist())
    lift = dn.embedding(E, 5)
    xn, tn = dn.denoise_batch(np.random.default_rng(5), B, L, lift)
    X = pa.Tensor([B, L, E], True)
    X.to_device(xn.ravel().tolist())
    T = pa.Tensor([B, L, E], False)
    T.to_device(tn.ravel().tolist())
    loss = pa.MSE()(model.forward(X), T)
    loss.backward()
    assert pa.device_status() == 0

    tp = [torch.tensor(_h(p), dtype=torch.float64, requires_grad=True) for p in params]
    tx = torch.tensor(xn, dtype=torch.float64, requires_grad=True)
    y = tx
    for i in range(2):
        y = _ref_layer(y, tp[14 * i:14 * (i + 1)], H)
    tl = torch.mean((y - torch.tensor(tn, dtype=torch.float64)) ** 2)
    tl.backward()
    assert abs(_h(loss)[0] - tl.item()) < (1e-4 if math_mode == "split3" else 1e-2) * tl.item()
    errs = {"dX": rel_err(_g(X), tx.grad.numpy())}
    for i, (p, q) in enumerate(zip(params, tp)):
        errs["p%d%s" % (i, p.shape())] = rel_err(_g(p), q.grad.numpy())
    print("denoise model (%s) relative errors:" % math_mode, errs)
    for name, e in errs.items():
        assert e < tol, (name, e)


def _pinned(a):
    return torch.from_numpy(a).pin_memory()


SMALL = dict(layers=2, embed=128, heads=4, ffn=256, seq=256, batch=4)


@pytest.mark.gpu
@pytest.mark.parametrize("math_mode", ["split3", "bf16"])
def test_trainer_reduces_denoise_loss(dn, math_mode):
    tr = dn.DenoiseTrainer(lr=1e-3, math=math_mode, **SMALL)
    lift = dn.embedding(SMALL["embed"], 5)
    rng = np.random.default_rng(5)
    data = [tuple(_pinned(a) for a in dn.denoise_batch(rng, SMALL["batch"], SMALL["seq"], lift))
            for _ in range(4)]
    losses = [tr.step(*data[i % 4]) for i in range(60)]
    import PureAttention as pa
    assert pa.device_status() == 0
    assert all(np.isfinite(losses))
    first, last = np.mean(losses[:4]), np.mean(losses[-4:])
    print("denoise loss: first %.4f last %.4f" % (first, last))
    assert last < 0.5 * first


@pytest.mark.gpu
def test_checkpoint_restores_training_state(dn, tmp_path):
    lift = dn.embedding(SMALL["embed"], 5)
    rng = np.random.default_rng(9)
    data = [tuple(_pinned(a) for a in dn.denoise_batch(rng, SMALL["batch"], SMALL["seq"], lift))
            for _ in range(3)]
    a = dn.DenoiseTrainer(lr=1e-3, seed=5, **SMALL)
    for i in range(3):
        a.step(*data[i])
    path = os.path.join(tmp_path, "ckpt.npz")
    a.save(path)
    la = [a.step(*data[i]) for i in range(3)]
    b = dn.DenoiseTrainer(lr=1e-3, seed=6, **SMALL)  # different initial weights
    b.restore(path)
    assert b.opt.step_count == 3
    lb = [b.step(*data[i]) for i in range(3)]
    assert la[0] == lb[0]  # the forward pass of restored weights is bit-identical
    np.testing.assert_allclose(lb, la, rtol=1e-4)
    with pytest.raises(ValueError):
        dn.DenoiseTrainer(lr=1e-3, **dict(SMALL, layers=1)).restore(path)


@pytest.mark.gpu
def test_pipelined_train_loop_matches_step_by_step(dn):
    """train() (copies one step ahead on a side stream, losses read one step
    behind) takes the same steps as step() called per batch."""
    lift = dn.embedding(SMALL["embed"], 5)
    rng = np.random.default_rng(12)
    data = [tuple(_pinned(a) for a in dn.denoise_batch(rng, SMALL["batch"], SMALL["seq"], lift))
            for _ in range(3)]
    seq = [data[i % 3] for i in range(5)]
    a = dn.DenoiseTrainer(lr=1e-3, **SMALL)
    la = [a.step(*b) for b in seq]
    b = dn.DenoiseTrainer(lr=1e-3, **SMALL)
    lb = b.train(seq)
    assert len(lb) == 5 and lb[0] == la[0]
    np.testing.assert_allclose(lb, la, rtol=1e-4)
    assert b.train(seq[:1])[0] > 0 and len(b.train([])) == 0


@pytest.mark.gpu
def test_graph_replay_takes_the_eager_steps(dn):
    """On one GPU the trainer captures its forward + backward into a CUDA graph
    once per input buffer and math mode and replays it: the same losses as a
    trainer launching every kernel (graph=False) - the first one bit for bit -
    also after the math mode changes (a new capture)."""
    lift = dn.embedding(SMALL["embed"], 5)
    rng = np.random.default_rng(21)
    data = [tuple(_pinned(a) for a in dn.denoise_batch(rng, SMALL["batch"], SMALL["seq"], lift))
            for _ in range(2)]
    a = dn.DenoiseTrainer(lr=1e-3, graph=False, **SMALL)
    b = dn.DenoiseTrainer(lr=1e-3, **SMALL)
    assert b.graph and not a.graph
    la = [a.step(*data[i % 2]) for i in range(4)]
    lb = [b.step(*data[i % 2]) for i in range(4)]
    assert len(b._graphs) == 1
    assert lb[0] == la[0]
    np.testing.assert_allclose(lb, la, rtol=1e-5)
    a.math = b.math = "bf16"
    la2 = [a.step(*data[i % 2]) for i in range(2)]
    lb2 = [b.step(*data[i % 2]) for i in range(2)]
    assert len(b._graphs) == 1 and list(b._graphs)[0][1] == "bf16"
    np.testing.assert_allclose(lb2, la2, rtol=1e-4)
    assert b.train(data)[1] > 0 and len(b._graphs) == 2  # the second input buffer


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _dp_worker(rank, world, port, out_dir):
    import sys
    for p in (REPO, PKG):
        sys.path.insert(0, p)
    import datetime
    import torch as th
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_DEBUG="WARN")
    th.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=th.device("cuda", rank))
    try:
        import denoise as d
        cfg = dict(SMALL, batch=SMALL["batch"] // world)
        tr = d.DenoiseTrainer(lr=1e-3, **cfg)
        x, t = d.denoise_batch(np.random.default_rng(11), SMALL["batch"], SMALL["seq"],
                               d.embedding(SMALL["embed"], 5))
        n = cfg["batch"]
        xs, ts = (th.from_numpy(np.ascontiguousarray(a[rank * n:(rank + 1) * n])).pin_memory()
                  for a in (x, t))
        tr.step(xs, ts)
        th.cuda.synchronize()
        grads = [d.grad_view(p).cpu().numpy() for p in tr.params]  # averaged over the ranks
        for _ in range(2):
            tr.step(xs, ts)
        th.cuda.synchronize()
        np.savez(os.path.join(out_dir, "dp%d.npz" % rank),
                 *[d.device_view(p).cpu().numpy() for p in tr.params], *grads)
        tr.release_graphs()  # its graph holds NCCL calls: dropped before the group
    finally:
        dist.destroy_process_group()


@pytest.mark.gpu
def test_two_rank_data_parallel_matches_one_rank(dn, tmp_path):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_dp_worker, args=(r, world, port, str(tmp_path)))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    tr = dn.DenoiseTrainer(lr=1e-3, **SMALL)
    x, t = dn.denoise_batch(np.random.default_rng(11), SMALL["batch"], SMALL["seq"],
                            dn.embedding(SMALL["embed"], 5))
    tr.step(_pinned(x), _pinned(t))
    ref = [dn.grad_view(p).cpu().numpy().astype(np.float64) for p in tr.params]
    outs = [np.load(os.path.join(tmp_path, "dp%d.npz" % r)) for r in range(world)]
    n = len(ref)
    # replicas stay identical (same averaged gradients, same Adam steps)
    for i in range(2 * n):
        np.testing.assert_array_equal(outs[0]["arr_%d" % i], outs[1]["arr_%d" % i])
    # the averaged half-batch gradients equal the whole-batch gradient: norm-wise
    # over all parameters, and per tensor where the gradient is not ~0 (the key
    # bias has a zero gradient in exact arithmetic: softmax ignores a constant
    # shift of the scores)
    dp = [outs[0]["arr_%d" % (n + i)] for i in range(n)]
    cat = lambda gs: np.concatenate([g.ravel() for g in gs])
    assert rel_err(cat(dp), cat(ref)) < 1e-4
    top = max(np.linalg.norm(g) for g in ref)
    for i, (a, b) in enumerate(zip(dp, ref)):
        if np.linalg.norm(b) > 1e-3 * top:
            assert rel_err(a, b) < 1e-3, i


@pytest.mark.gpu
@pytest.mark.parametrize("graph", [False, True])
def test_gradient_arenas_reduce_in_place(dn, graph):
    """GradAllReduce.for_tensors moves every parameter's gradient into one flat
    arena per bucket (the first layers' gradients, finished last, in small tail
    buckets) and all-reduces each arena in place. With a one-rank NCCL group
    the average is the identity, so a trainer whose gradients live in the
    arenas takes the same steps as one without a reducer, launched eagerly or
    replayed as a CUDA graph that holds the all-reduces - up to the last bits
    that differ between any two runs (the split-K weight-gradient GEMMs and
    the dQ reductions add their parts in no fixed order)."""
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_free_port()))
    dist.init_process_group("nccl", rank=0, world_size=1, device_id=torch.device("cuda", 0))
    try:
        x, t = dn.denoise_batch(np.random.default_rng(13), SMALL["batch"], SMALL["seq"],
                                dn.embedding(SMALL["embed"], 5))
        x, t = _pinned(x), _pinned(t)
        a = dn.DenoiseTrainer(lr=1e-3, graph=graph, **SMALL)
        b = dn.DenoiseTrainer(lr=1e-3, graph=graph, **SMALL)
        assert a.reducer is None and b.reducer is None  # one rank: no reducer by default
        b.reducer = dn.GradAllReduce.for_tensors(b.params, bucket_bytes=1 << 16,
                                                 tail_bytes=1 << 16, tail_bucket_bytes=1 << 14)
        spans = [(f.data_ptr(), f.data_ptr() + 4 * f.numel()) for f in b.reducer.flat]
        for p in b.params:
            ptr = dn.grad_view(p).data_ptr()
            assert any(lo <= ptr < hi for lo, hi in spans)
            assert ptr % 256 == 0
        assert len(b.reducer.buckets) > 2
        for _ in range(2):
            la, lb = a.step(x, t), b.step(x, t)
            assert abs(la - lb) <= 1e-6 * abs(la)
        assert len(b._graphs) == (1 if graph else 0)  # graph: the NCCL buckets captured too
        # The key slice of each in-projection bias has a gradient that is zero in
        # exact arithmetic (softmax ignores a constant added to a query's scores),
        # so it holds rounding noise, which Adam turns into steps of +-lr: it is
        # left out of the comparison.
        E, per_layer = SMALL["embed"], len(a.params) // SMALL["layers"]
        for i, (p, q) in enumerate(zip(a.params, b.params)):
            hp, hq, gp, gq = _h(p), _h(q), _g(p), _g(q)
            if i % per_layer == 1:  # MultiheadAttention.in_proj_bias [1, 3E]: q, k, v slices
                keep = np.r_[0:E, 2 * E:3 * E]
                hp, hq, gp, gq = hp[..., keep], hq[..., keep], gp[..., keep], gq[..., keep]
            assert rel_err(hq, hp) < 1e-5, i
            if np.linalg.norm(gp) > 0:
                assert rel_err(gq, gp) < 1e-4, i
    finally:
        for name in ("a", "b"):
            if name in locals():
                locals()[name].release_graphs()  # graphs holding NCCL calls go first
        dist.destroy_process_group()
