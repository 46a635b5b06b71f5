"""The host operator layer (PureAttention module over the C ABI) against
float64 references: Tensor round trips, the reverse-topological backward on
a graph with fan-out, Linear / ReLU / MSE / Adam against torch float64, and
the pre-LayerNorm multi-head-attention block (B=8, L=1024, E=512, H=8, fp32)
forward + backward against the float64 oracle, every gradient within 1e-3."""
import numpy as np
import pytest

from conftest import rel_err, seeded_normal

torch = pytest.importorskip("torch")
F32_TOL = 1e-3


@pytest.fixture(scope="module")
def pa():
    import PureAttention
    PureAttention.set_seed(1234)
    return PureAttention


def _t(pa, x, requires_grad=False):
    x = np.ascontiguousarray(x, dtype=np.float32)
    t = pa.Tensor(list(x.shape), requires_grad)
    t.to_device(x.ravel().tolist())
    return t


def _h(t):
    return np.asarray(t.to_host(), dtype=np.float64).reshape(t.shape())


def _g(t):
    return np.asarray(t.grad_to_host(), dtype=np.float64).reshape(t.shape())


@pytest.mark.gpu
def test_tensor_round_trip_and_zero_grads(pa):
    x = seeded_normal(1, (3, 5))
    t = _t(pa, x, True)
    np.testing.assert_array_equal(_h(t), x)
    np.testing.assert_array_equal(_g(t), np.zeros((3, 5)))
    with pytest.raises(Exception):
        t.to_device([1.0])
    with pytest.raises(RuntimeError):
        pa.Tensor([2], False).backward()


@pytest.mark.gpu
def test_fan_out_gradients_accumulate_once(pa):
    """y = x W;  z = y + y (same-shape add);  loss = mse(z, t). The shared y
    must receive both contributions before its matmul node runs."""
    x = seeded_normal(2, (64, 32))
    t = seeded_normal(3, (64, 16))
    lin = pa.Linear(32, 16)
    w = _h(lin.weight)
    X = _t(pa, x, True)
    y = lin.forward(X)
    z = pa.add(y, y)
    loss = pa.MSE()(z, _t(pa, t))
    loss.backward()
    tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    tw = torch.tensor(w, dtype=torch.float64, requires_grad=True)
    tb = torch.zeros(16, dtype=torch.float64, requires_grad=True)
    ty = tx @ tw + tb
    tl = torch.mean((ty + ty - torch.tensor(t, dtype=torch.float64)) ** 2)
    tl.backward()
    assert abs(_h(loss)[0] - tl.item()) < 1e-5 * abs(tl.item())
    assert rel_err(_g(X), tx.grad.numpy()) < 1e-4
    assert rel_err(_g(lin.weight), tw.grad.numpy()) < 1e-4
    assert rel_err(_g(lin.bias).ravel(), tb.grad.numpy()) < 1e-4


@pytest.mark.gpu
def test_fused_add_layer_norm_matches_unfused_graph(pa):
    """LayerNorm.forward_add(x, r) gives (x + r, LN(x + r)) with the same values
    and the same gradients for x, r, gamma, beta as pa.add followed by
    LayerNorm.forward, when both the sum and the norm feed the loss."""
    x, r, t1, t2 = (seeded_normal(40 + i, (6, 24, 32)) for i in range(4))
    ln = pa.LayerNorm(32)
    g0 = 1.0 + 0.1 * seeded_normal(44, (1, 32))
    b0 = 0.1 * seeded_normal(45, (1, 32))
    outs = []
    for fused in (True, False):
        ln.gamma.to_device(g0.astype(np.float32).ravel().tolist())
        ln.beta.to_device(b0.astype(np.float32).ravel().tolist())
        for p in ln.parameters():
            p.zero_grad()
        X, R = _t(pa, x, True), _t(pa, r, True)
        if fused:
            s, y = ln.forward_add(X, R)
        else:
            s = pa.add(X, R)
            y = ln.forward(s)
        loss = pa.add(pa.MSE()(s, _t(pa, t1)), pa.MSE()(y, _t(pa, t2)))
        loss.backward()
        outs.append([_h(s), _h(y), _h(loss), _g(X), _g(R), _g(ln.gamma), _g(ln.beta)])
    for a, b in zip(*outs):
        assert rel_err(a, b) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["out_only", "sum_only", "same_input", "chained"])
def test_fused_add_layer_norm_gradient_paths_match_torch(pa, case):
    """The Add+LayerNorm node against torch float64 on each path its backward
    takes: only the norm feeds the loss (no gradient reaches the sum
    directly), only the sum does (no LayerNorm backward), x + x (one
    buffer receives both addends' gradient), and two chained blocks with an
    intermediate gradient read back (a gradient written once, never zeroed)."""
    import torch.nn.functional as F
    x, r, t = (seeded_normal(60 + i, (4, 16, 32)) for i in range(3))
    g0 = (1.0 + 0.1 * seeded_normal(63, (32,))).astype(np.float32)
    b0 = (0.1 * seeded_normal(64, (32,))).astype(np.float32)
    ln, ln2 = pa.LayerNorm(32), pa.LayerNorm(32)
    for m in (ln, ln2):
        m.gamma.to_device(g0.tolist())
        m.beta.to_device(b0.tolist())
    X = _t(pa, x, True)
    R = X if case == "same_input" else _t(pa, r, True)
    s, y = ln.forward_add(X, R)
    T = _t(pa, t)
    if case == "sum_only":
        loss = pa.MSE()(s, T)
    elif case == "chained":
        s2, y2 = ln2.forward_add(s, y)
        loss = pa.MSE()(y2, T)
    else:
        loss = pa.MSE()(y, T)
    loss.backward()
    tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    tr = tx if case == "same_input" else torch.tensor(r, dtype=torch.float64, requires_grad=True)
    tg = torch.tensor(g0, dtype=torch.float64, requires_grad=True)
    tb = torch.tensor(b0, dtype=torch.float64, requires_grad=True)
    ts = tx + tr
    ts.retain_grad()
    ty = F.layer_norm(ts, (32,), tg, tb, 1e-5)
    tt = torch.tensor(t, dtype=torch.float64)
    if case == "sum_only":
        tl = torch.mean((ts - tt) ** 2)
    elif case == "chained":
        ty.retain_grad()
        tl = torch.mean((F.layer_norm(ts + ty, (32,), tg, tb, 1e-5) - tt) ** 2)
    else:
        tl = torch.mean((ty - tt) ** 2)
    tl.backward()
    assert abs(_h(loss)[0] - tl.item()) < 1e-5 * abs(tl.item())
    assert rel_err(_g(X), tx.grad.numpy()) < 1e-4
    if case != "same_input":
        assert rel_err(_g(R), tr.grad.numpy()) < 1e-4
    if case == "sum_only":
        assert not _g(ln.gamma).any() and not _g(ln.beta).any()
    elif case == "chained":
        # y's gradient was written once by the second block's node and is readable
        assert rel_err(_g(y), ty.grad.numpy()) < 1e-4
        for a, b, want in ((ln.gamma, ln2.gamma, tg), (ln.beta, ln2.beta, tb)):
            assert rel_err(_g(a).ravel() + _g(b).ravel(), want.grad.numpy()) < 1e-4
    else:
        assert rel_err(_g(ln.gamma).ravel(), tg.grad.numpy()) < 1e-4
        assert rel_err(_g(ln.beta).ravel(), tb.grad.numpy()) < 1e-4
    # the sum's gradient is never formed by the fused node: it reads as zero
    # unless a consumer of the sum wrote it (the second block, or the loss)
    if case in ("out_only", "same_input"):
        assert not _g(s).any()


@pytest.mark.gpu
def test_backward_leaf_hook_reports_final_gradients(pa):
    """backward(seed, hook) calls hook(t) once per gradient-requiring leaf
    (every parameter of a denoise layer and the input), after the last node
    that writes its gradient: a copy taken in the hook, on the operators'
    stream, equals the gradient after the whole backward."""
    import denoise as dn
    model = dn.DenoiseTransformer(1, 128, 4, 256)  # head dim 32
    params = model.parameters()
    X = _t(pa, seeded_normal(50, (2, 48, 128)), True)
    loss = pa.MSE()(model.forward(X), _t(pa, seeded_normal(51, (2, 48, 128))))
    ptr = lambda t: t.grad_view().__cuda_array_interface__["data"][0]
    snaps, calls = {}, []

    def hook(t):
        calls.append(ptr(t))
        snaps[ptr(t)] = torch.as_tensor(t.grad_view(), device="cuda").clone()

    loss.backward(True, hook)
    torch.cuda.synchronize()
    leaves = params + [X]
    assert sorted(calls) == sorted(ptr(t) for t in leaves)
    for t in leaves:
        np.testing.assert_array_equal(snaps[ptr(t)].cpu().numpy(), _g(t).astype(np.float32))


@pytest.mark.gpu
def test_mlp_relu_mse_adam_matches_torch(pa):
    x = seeded_normal(4, (128, 24))
    t = seeded_normal(5, (128, 8))
    l1, act, l2 = pa.Linear(24, 32), pa.ReLU(), pa.Linear(32, 8)
    params = l1.parameters() + l2.parameters()
    init = [_h(p) for p in params]
    tp = [torch.tensor(v, dtype=torch.float64, requires_grad=True) for v in init]
    opt = pa.Adam(params, lr=1e-2)
    topt = torch.optim.Adam(tp, lr=1e-2, betas=(0.9, 0.999), eps=1e-8)
    X, T = _t(pa, x), _t(pa, t)
    tx, tt = torch.tensor(x, dtype=torch.float64), torch.tensor(t, dtype=torch.float64)
    for _ in range(3):
        opt.zero_grad()
        loss = pa.MSE()(l2.forward(act.forward(l1.forward(X))), T)
        loss.backward()
        opt.step()
        topt.zero_grad()
        tl = torch.mean(((torch.relu(tx @ tp[0] + tp[1]) @ tp[2] + tp[3]) - tt) ** 2)
        tl.backward()
        topt.step()
        assert abs(_h(loss)[0] - tl.item()) < 1e-4 * abs(tl.item())
    for p, q in zip(params, tp):
        assert rel_err(_h(p), q.detach().numpy()) < 1e-4


def _xavier(seed, fan_in, fan_out, shape):
    rng = np.random.default_rng(seed)
    a = np.sqrt(6.0 / (fan_in + fan_out))
    return rng.uniform(-a, a, size=shape).astype(np.float32)


@pytest.mark.gpu
def test_pre_ln_mha_block_matches_oracle(pa):
    """One pre-LN multi-head-attention block (LN -> MHA(q=k=v) -> residual add
    -> MSE), B=8, L=1024, E=512, H=8, fp32; gradients for X and all weights."""
    import oracle
    B, L, E, H = 8, 1024, 512, 8
    D = E // H
    M = B * L
    x = seeded_normal(2, (B, L, E))
    tgt = seeded_normal(3, (B, L, E))
    w_in = _xavier(10, E, 3 * E, (E, 3 * E))
    w_out = _xavier(11, E, E, (E, E))
    ln = pa.LayerNorm(E)
    mha = pa.MultiheadAttention(E, H)
    in_w, in_b, out_w, out_b = mha.parameters()
    in_w.to_device(w_in.ravel().tolist())
    out_w.to_device(w_out.ravel().tolist())
    X = _t(pa, x, True)
    xn = ln.forward(X)
    attn = mha.forward(xn, xn, xn)
    out = pa.add(X, attn)
    loss = pa.MSE()(out, _t(pa, tgt))
    loss.backward()
    assert pa.device_status() == 0

    # float64 oracle of the same block
    x2 = x.reshape(M, E).astype(np.float64)
    g1, b1 = np.ones(E), np.zeros(E)
    y1, mu, rs = oracle.layer_norm_fwd(x2, g1, b1)
    qkv = y1 @ w_in.astype(np.float64)
    q, k, v = (qkv[:, i * E:(i + 1) * E].reshape(B, L, H, D) for i in range(3))
    o, lse = oracle.attn_fwd(q, k, v)
    o2 = o.reshape(M, E)
    a = o2 @ w_out.astype(np.float64)
    res = x2 + a
    n = res.size
    ref_loss = np.mean((res - tgt.reshape(M, E)) ** 2)
    dres = 2.0 / n * (res - tgt.reshape(M, E))
    dw_out = o2.T @ dres
    db_out = dres.sum(0)
    do = (dres @ w_out.T.astype(np.float64)).reshape(B, L, H, D)
    dq, dk, dv, _ = oracle.attn_bwd(q, k, v, o, do, lse)
    dqkv = np.concatenate([g.reshape(M, E) for g in (dq, dk, dv)], axis=1)
    dw_in = y1.T @ dqkv
    db_in = dqkv.sum(0)
    dy1 = dqkv @ w_in.T.astype(np.float64)
    dx_ln, dg1, db1 = oracle.layer_norm_bwd(dy1, x2, mu, rs, g1)
    dx = dres + dx_ln

    assert abs(_h(loss)[0] - ref_loss) < 1e-4 * ref_loss
    assert rel_err(_h(out).reshape(M, E), res) < 1e-5
    errs = {
        "dX": rel_err(_g(X).reshape(M, E), dx),
        "d in_proj_weight": rel_err(_g(in_w), dw_in),
        "d in_proj_bias": rel_err(_g(in_b).ravel(), db_in),
        "d out_proj_weight": rel_err(_g(out_w), dw_out),
        "d out_proj_bias": rel_err(_g(out_b).ravel(), db_out),
        "d gamma": rel_err(_g(ln.gamma).ravel(), dg1),
        "d beta": rel_err(_g(ln.beta).ravel(), db1),
    }
    print("pre-LN block relative errors:", errs)
    for name, e in errs.items():
        assert e < F32_TOL, (name, e)


@pytest.mark.gpu
@pytest.mark.parametrize("same", [True, False])
def test_flash_attention_node_with_one_tensor_in_several_roles(pa, same):
    """flash_attention(x, x, x) (self-attention on x itself) gives x the sum of
    its three gradients, as torch does; with three tensors each gets its own
    (fp32 tensors, split3 products: within 1e-3 of float64)."""
    import torch.nn.functional as F
    N, L, E, H = 2, 96, 64, 2
    x, k2, v2, t = (seeded_normal(90 + i, (N, L, E), 0.5) for i in range(4))
    X = _t(pa, x, True)
    K = X if same else _t(pa, k2, True)
    V = X if same else _t(pa, v2, True)
    o = pa.flash_attention(X, K, V, H)
    loss = pa.MSE()(o, _t(pa, t))
    loss.backward()
    tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    tk = tx if same else torch.tensor(k2, dtype=torch.float64, requires_grad=True)
    tv = tx if same else torch.tensor(v2, dtype=torch.float64, requires_grad=True)
    sp = lambda a: a.view(N, L, H, E // H).transpose(1, 2)
    to = F.scaled_dot_product_attention(sp(tx), sp(tk), sp(tv)).transpose(1, 2).reshape(N, L, E)
    tl = torch.mean((to - torch.tensor(t, dtype=torch.float64)) ** 2)
    tl.backward()
    assert rel_err(_h(o), to.detach().numpy()) < F32_TOL
    assert rel_err(_g(X), tx.grad.numpy()) < F32_TOL
    if not same:
        assert rel_err(_g(K), tk.grad.numpy()) < F32_TOL
        assert rel_err(_g(V), tv.grad.numpy()) < F32_TOL


@pytest.mark.gpu
def test_input_shared_by_two_projections_gets_both_gradients(pa):
    """x feeds two Linear layers: the first projection backward writes x's
    gradient outright (nothing had written it), the second adds to it - the
    sum of both, as torch gives."""
    x, t = seeded_normal(95, (128, 48)), seeded_normal(96, (128, 32))
    l1, l2 = pa.Linear(48, 32), pa.Linear(48, 32, True)
    w1, w2 = _h(l1.weight), _h(l2.weight)
    X = _t(pa, x, True)
    loss = pa.MSE()(pa.add(l1.forward(X), l2.forward(X)), _t(pa, t))
    loss.backward()
    tx = torch.tensor(x, dtype=torch.float64, requires_grad=True)
    tw1, tw2 = (torch.tensor(w, dtype=torch.float64, requires_grad=True) for w in (w1, w2))
    ty = tx @ tw1 + torch.relu(tx @ tw2)
    tl = torch.mean((ty - torch.tensor(t, dtype=torch.float64)) ** 2)
    tl.backward()
    assert abs(_h(loss)[0] - tl.item()) < 1e-5 * abs(tl.item())
    assert rel_err(_g(X), tx.grad.numpy()) < 1e-4
    assert rel_err(_g(l1.weight), tw1.grad.numpy()) < 1e-4
    assert rel_err(_g(l2.weight), tw2.grad.numpy()) < 1e-4
