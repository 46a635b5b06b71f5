"""Parity of the attention block's non-attention kernels (through the C ABI)
with the float64 oracle: the matmul forward and both gradients, LayerNorm
forward and backward, bias add / bias grad / grad accumulate / residual add,
and the last-dimension split and its adjoint.

Tolerances (fp32 path): GEMMs 1e-4 norm-wise (bf16 hi/lo split products),
LayerNorm 1e-5 (y, dgamma, dbeta) and 1e-4 (dX), elementwise 1e-6. In the
bf16 math mode the GEMMs are checked against the oracle on bf16-rounded
operands (exact products, fp32 accumulation): 1e-5."""
import numpy as np
import pytest

from conftest import rel_err, seeded_normal

torch = pytest.importorskip("torch")
GEMM_TOL = 1e-4  # 10x under the fp32 path budget of 1e-3; dW at M=8192 measures 2.9e-5


def _cu(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


def _np(t):
    torch.cuda.synchronize()
    return t.cpu().numpy().astype(np.float64)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [
    (256, 192, 320),
    (100, 70, 50),        # ragged: partial tiles, K < 64, N % 4 != 0
    (8192, 1536, 512),    # pre-LN block in-projection
    (8192, 512, 512),     # out-projection
])
def test_matmul_forward_matches_oracle(M, N, K):
    import oracle
    import pa_capi
    a = seeded_normal(M + 1, (M, K))
    b = seeded_normal(N + 2, (K, N))
    c = torch.full((M, N), float("nan"), device="cuda")
    pa_capi.matmul(_cu(a), _cu(b), c, M, N, K)
    assert pa_capi.device_status() == 0
    assert rel_err(_np(c), oracle.matmul(a, b)) < GEMM_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(256, 192, 320), (100, 70, 50), (8192, 512, 1536)])
def test_matmul_grad_x_accumulates_like_oracle(M, N, K):
    import oracle
    import pa_capi
    dy = seeded_normal(M + 3, (M, K))
    w = seeded_normal(N + 4, (N, K))
    dx0 = seeded_normal(M + 5, (M, N))
    dx = _cu(dx0)
    pa_capi.matmul_grad_x(_cu(dy), _cu(w), dx, M, N, K)
    assert rel_err(_np(dx), oracle.matmul_grad_x(dy, w, dx0)) < GEMM_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(256, 192, 320), (100, 70, 50), (8192, 512, 1536)])
def test_matmul_grad_w_accumulates_like_oracle(M, N, K):
    import oracle
    import pa_capi
    x = seeded_normal(M + 6, (M, N))
    dy = seeded_normal(M + 7, (M, K))
    dw0 = seeded_normal(N + 8, (N, K))
    dw = _cu(dw0)
    pa_capi.matmul_grad_w(_cu(x), _cu(dy), dw, M, N, K)
    assert rel_err(_np(dw), oracle.matmul_grad_w(x, dy, dw0)) < GEMM_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("M,N", [(8192, 512), (37, 128), (16384, 1024), (5, 12)])
def test_layer_norm_matches_oracle(M, N):
    import oracle
    import pa_capi
    x = seeded_normal(M, (M, N))
    gamma = 1.0 + 0.1 * seeded_normal(N, (N,))
    beta = 0.1 * seeded_normal(N + 1, (N,))
    dy = seeded_normal(M + 9, (M, N))
    y = torch.empty(M, N, device="cuda")
    mean = torch.empty(M, device="cuda")
    rstd = torch.empty(M, device="cuda")
    pa_capi.layer_norm_fwd(_cu(x), _cu(gamma), _cu(beta), y, mean, rstd)
    oy, om, ors = oracle.layer_norm_fwd(x, gamma, beta)
    assert rel_err(_np(y), oy) < 1e-5
    assert rel_err(_np(mean), om) < 1e-5
    assert rel_err(_np(rstd), ors) < 1e-5
    dx = torch.full((M, N), float("nan"), device="cuda")
    dg0 = seeded_normal(3, (N,))
    db0 = seeded_normal(4, (N,))
    dg, db = _cu(dg0), _cu(db0)
    ws = torch.empty(pa_capi.layer_norm_bwd_workspace_size(M, N), dtype=torch.uint8, device="cuda")
    pa_capi.layer_norm_bwd(_cu(dy), _cu(x), mean, rstd, _cu(gamma), dx, dg, db, ws)
    odx, odg, odb = oracle.layer_norm_bwd(dy, x, _np(mean), _np(rstd), gamma)
    assert rel_err(_np(dx), odx) < 1e-4
    assert rel_err(_np(dg), dg0 + odg) < 1e-5
    assert rel_err(_np(db), db0 + odb) < 1e-5
    # accumulating form: dx += dL/dx (the residual branch's gradient kept)
    dx0 = seeded_normal(5, (M, N))
    dxa = _cu(dx0)
    pa_capi.layer_norm_bwd(_cu(dy), _cu(x), mean, rstd, _cu(gamma), dxa, None, None, None,
                           accumulate=True)
    assert rel_err(_np(dxa), dx0 + odx) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("M,N", [(8192, 1024), (37, 128), (5, 12)])
def test_add_layer_norm_matches_oracle(M, N):
    """sum = x + r exactly (one fp32 add per element), y = LayerNorm(sum) as the
    oracle's forward of the sum, and identical to the unfused kernel on it."""
    import oracle
    import pa_capi
    x = seeded_normal(M + 20, (M, N))
    r = seeded_normal(M + 21, (M, N))
    gamma = 1.0 + 0.1 * seeded_normal(N + 22, (N,))
    beta = 0.1 * seeded_normal(N + 23, (N,))
    s = torch.empty(M, N, device="cuda")
    y = torch.empty(M, N, device="cuda")
    mean = torch.empty(M, device="cuda")
    rstd = torch.empty(M, device="cuda")
    pa_capi.add_layer_norm_fwd(_cu(x), _cu(r), s, _cu(gamma), _cu(beta), y, mean, rstd)
    want_s = (x.astype(np.float32) + r.astype(np.float32)).astype(np.float64)
    np.testing.assert_array_equal(_np(s), want_s)
    oy, om, ors = oracle.layer_norm_fwd(want_s, gamma, beta)
    assert rel_err(_np(y), oy) < 1e-5
    assert rel_err(_np(mean), om) < 1e-5
    assert rel_err(_np(rstd), ors) < 1e-5
    y2, m2, r2 = torch.empty_like(y), torch.empty_like(mean), torch.empty_like(rstd)
    pa_capi.layer_norm_fwd(s, _cu(gamma), _cu(beta), y2, m2, r2)
    np.testing.assert_array_equal(_np(y), _np(y2))
    np.testing.assert_array_equal(_np(mean), _np(m2))


@pytest.mark.gpu
@pytest.mark.parametrize("M,N", [(16384, 1024), (37, 128), (5, 12)])
def test_add_layer_norm_bwd_matches_oracle(M, N):
    """pa_add_layer_norm_bwd: G = LN_bwd(dy) + dsum written to both addends'
    gradients (overwritten or accumulated per flag), dgamma / dbeta as the
    plain LayerNorm backward's bits; dx and dr may be one buffer (x + x)."""
    import oracle
    import pa_capi
    x, r = seeded_normal(M + 30, (M, N)), seeded_normal(M + 31, (M, N))
    gamma = 1.0 + 0.1 * seeded_normal(N + 32, (N,))
    beta = 0.1 * seeded_normal(N + 33, (N,))
    dy, dsum = seeded_normal(M + 34, (M, N)), seeded_normal(M + 35, (M, N))
    s, y = torch.empty(M, N, device="cuda"), torch.empty(M, N, device="cuda")
    mean, rstd = torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
    pa_capi.add_layer_norm_fwd(_cu(x), _cu(r), s, _cu(gamma), _cu(beta), y, mean, rstd)
    odx, odg, odb = oracle.layer_norm_bwd(dy, _np(s), _np(mean), _np(rstd), gamma)
    G = odx + dsum
    ws = torch.empty(pa_capi.layer_norm_bwd_workspace_size(M, N), dtype=torch.uint8, device="cuda")
    dx0, dr0 = seeded_normal(M + 36, (M, N)), seeded_normal(M + 37, (M, N))
    dg0, db0 = seeded_normal(38, (N,)), seeded_normal(39, (N,))
    dx = torch.full((M, N), float("nan"), device="cuda")  # overwritten
    dr = _cu(dr0)                                         # accumulated
    dg, db = _cu(dg0), _cu(db0)
    pa_capi.add_layer_norm_bwd(_cu(dy), _cu(dsum), s, mean, rstd, _cu(gamma), dx, dr, dg, db, ws,
                               acc_dx=False, acc_dr=True)
    assert pa_capi.device_status() == 0
    assert rel_err(_np(dx), G) < 1e-4
    assert rel_err(_np(dr), dr0 + G) < 1e-4
    # parameter gradients: the same bits as the plain LayerNorm backward
    dg2, db2 = _cu(dg0), _cu(db0)
    pa_capi.layer_norm_bwd(_cu(dy), s, mean, rstd, _cu(gamma), None, dg2, db2, ws)
    assert torch.equal(dg, dg2) and torch.equal(db, db2)
    # without dsum, and x + x: one buffer receives both addends' gradient
    both = _cu(dx0)
    pa_capi.add_layer_norm_bwd(_cu(dy), None, s, mean, rstd, _cu(gamma), both, both, None, None, None,
                               acc_dx=True, acc_dr=True)
    assert rel_err(_np(both), dx0 + 2 * odx) < 1e-4
    fresh = torch.full((M, N), float("nan"), device="cuda")
    pa_capi.add_layer_norm_bwd(_cu(dy), None, s, mean, rstd, _cu(gamma), fresh, fresh, None, None, None,
                               acc_dx=False, acc_dr=True)
    assert rel_err(_np(fresh), 2 * odx) < 1e-4
    assert pa_capi.device_status() == 0


@pytest.mark.gpu
def test_layer_norm_backward_is_deterministic():
    import pa_capi
    M, N = 4096, 512
    x, dy = _cu(seeded_normal(1, (M, N))), _cu(seeded_normal(2, (M, N)))
    g, b = torch.ones(N, device="cuda"), torch.zeros(N, device="cuda")
    y, mean, rstd = torch.empty(M, N, device="cuda"), torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
    pa_capi.layer_norm_fwd(x, g, b, y, mean, rstd)
    ws = torch.empty(pa_capi.layer_norm_bwd_workspace_size(M, N), dtype=torch.uint8, device="cuda")
    outs = []
    for _ in range(2):
        dx, dg, db = torch.empty(M, N, device="cuda"), torch.zeros(N, device="cuda"), torch.zeros(N, device="cuda")
        pa_capi.layer_norm_bwd(dy, x, mean, rstd, g, dx, dg, db, ws)
        outs.append([_np(t) for t in (dx, dg, db)])
    for a, b_ in zip(*outs):
        np.testing.assert_array_equal(a, b_)


@pytest.mark.gpu
def test_elementwise_kernels_match_oracle():
    import oracle
    import pa_capi
    M, N = 1000, 300
    a = seeded_normal(11, (M, N))
    bias = seeded_normal(12, (N,))
    out = torch.empty(M, N, device="cuda")
    pa_capi.bias_add(_cu(a), _cu(bias), out, M, N)
    assert rel_err(_np(out), oracle.bias_add(a, bias)) < 1e-7
    b = seeded_normal(13, (M, N))
    pa_capi.add(_cu(a), _cu(b), out, M * N)
    assert rel_err(_np(out), a + b) < 1e-7
    dst = _cu(b)
    pa_capi.grad_accumulate(_cu(a), dst, M * N)
    assert rel_err(_np(dst), a + b) < 1e-7
    db0 = seeded_normal(14, (N,))
    db = _cu(db0)
    pa_capi.bias_grad(_cu(a), db, M, N)
    assert rel_err(_np(db), oracle.bias_grad(a, db0)) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("M,N", [(16384, 1024), (16384, 4096), (8192, 1536), (300, 12), (77, 130)])
def test_bias_grad_large_and_ragged(M, N):
    """Column sums in one pass, or with a workspace split over many CTAs (two
    stages; one pass for small or unaligned shapes); accumulated into db;
    deterministic."""
    import oracle
    import pa_capi
    a = seeded_normal(M + N, (M, N))
    db0 = seeded_normal(15, (N,))
    ws = torch.empty(pa_capi.bias_grad_workspace_size(M, N), dtype=torch.uint8, device="cuda")
    for w in (None, ws):  # one pass / two stages over the GPU
        outs = []
        for _ in range(2):
            db = _cu(db0)
            pa_capi.bias_grad(_cu(a), db, M, N, workspace=w)
            outs.append(_np(db))
        assert rel_err(outs[0], oracle.bias_grad(a, db0)) < 1e-6
        np.testing.assert_array_equal(outs[0], outs[1])


@pytest.mark.gpu
@pytest.mark.parametrize("n,offset", [(16384 * 1024, 0), (16384 * 1024 + 3, 1), (5, 0), (1000, 0)])
def test_mse_forward_matches_float64(n, offset):
    """loss = mean((p - t)^2): with a workspace a two-stage reduction over the
    GPU, without one a single CTA; both deterministic. An odd length and a
    4-byte offset take the scalar path."""
    import ctypes
    import pa_capi
    p = seeded_normal(21, (n + offset,))
    t = seeded_normal(22, (n + offset,))
    pd, td = _cu(p), _cu(t)
    want = np.mean((p[offset:].astype(np.float64) - t[offset:]) ** 2)
    lib = pa_capi.load()
    ws = torch.empty(lib.pa_mse_fwd_workspace_size(n), dtype=torch.uint8, device="cuda")
    args = (ctypes.c_void_p(pd.data_ptr() + 4 * offset), ctypes.c_void_p(td.data_ptr() + 4 * offset))
    for with_ws in (True, False):
        if not with_ws and n > 4 * 1024 * 1024:
            continue  # the one-CTA form is for small losses
        got = []
        for _ in range(2):
            loss = torch.full((1,), float("nan"), device="cuda")
            if with_ws:
                st = lib.pa_mse_fwd_ws(*args, ctypes.c_void_p(loss.data_ptr()), n, ws.data_ptr(),
                                       ws.numel(), None)
            else:
                st = lib.pa_mse_fwd(*args, ctypes.c_void_p(loss.data_ptr()), n, None)
            assert st == 0
            got.append(float(loss.item()))
        assert abs(got[0] - want) < 1e-6 * want
        assert got[0] == got[1]


@pytest.mark.gpu
def test_split_and_concat_grad_match_oracle():
    import oracle
    import pa_capi
    rows, parts, w = 513, 3, 96
    x = seeded_normal(21, (rows, parts * w))
    outs = [torch.empty(rows, w, device="cuda") for _ in range(parts)]
    pa_capi.split_last_dim(_cu(x), outs, rows, w)
    ref = oracle.split_last_dim(x, parts)
    for p in range(parts):
        np.testing.assert_array_equal(_np(outs[p]), ref[p])
    g0 = seeded_normal(22, (rows, parts * w))
    gin = _cu(g0)
    pa_capi.concat_last_dim_grad(outs, gin, rows, w)
    np.testing.assert_allclose(_np(gin), oracle.concat_last_dim_grad(ref, g0), rtol=1e-6)


@pytest.mark.gpu
@pytest.mark.parametrize("M,IN,OUT,n", [
    (8192, 512, 1536, 3),   # pre-LN block in-projection: Q, K, V written directly
    (8192, 512, 512, 1),    # out-projection with bias
    (100, 70, 48, 3),       # ragged: partial tiles, 16-column blocks
    (300, 64, 96, 2),
])
def test_linear_fwd_matches_oracle(M, IN, OUT, n):
    import oracle
    import pa_capi
    x = seeded_normal(M + 31, (M, IN))
    w = seeded_normal(IN + 32, (IN, OUT))
    bias = seeded_normal(OUT + 33, (OUT,))
    outs = [torch.full((M, OUT // n), float("nan"), device="cuda") for _ in range(n)]
    pa_capi.linear_fwd(_cu(x), _cu(w), _cu(bias), outs, M, IN, OUT)
    assert pa_capi.device_status() == 0
    ref = oracle.bias_add(oracle.matmul(x, w), bias)
    for c in range(n):
        assert rel_err(_np(outs[c]), ref[:, c * (OUT // n):(c + 1) * (OUT // n)]) < GEMM_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("M,IN,OUT,n", [(8192, 512, 1536, 3), (100, 70, 48, 3), (256, 192, 320, 1)])
def test_linear_bwd_accumulates_like_oracle(M, IN, OUT, n):
    import oracle
    import pa_capi
    x = seeded_normal(M + 41, (M, IN))
    w = seeded_normal(IN + 42, (IN, OUT))
    parts = [seeded_normal(M + 43 + c, (M, OUT // n)) for c in range(n)]
    dy = np.concatenate(parts, axis=1)
    dx0, dw0, db0 = seeded_normal(1, (M, IN)), seeded_normal(2, (IN, OUT)), seeded_normal(3, (OUT,))
    dx, dw, db = _cu(dx0), _cu(dw0), _cu(db0)
    pa_capi.linear_bwd(_cu(x), _cu(w), [_cu(p) for p in parts], dx, dw, db, M, IN, OUT)
    assert pa_capi.device_status() == 0
    assert rel_err(_np(dx), oracle.matmul_grad_x(dy, w, dx0)) < GEMM_TOL
    assert rel_err(_np(dw), oracle.matmul_grad_w(x, dy, dw0)) < GEMM_TOL
    assert rel_err(_np(db), oracle.bias_grad(dy, db0)) < 1e-5  # fp32 column sums over M rows
    # skipped outputs are left alone
    dw2 = _cu(dw0)
    pa_capi.linear_bwd(_cu(x), _cu(w), [_cu(p) for p in parts], None, dw2, None, M, IN, OUT)
    assert rel_err(_np(dw2), oracle.matmul_grad_w(x, dy, dw0)) < GEMM_TOL


# ---------------------------------------------------------------- bf16 math mode
BF16_MATH_TOL = 1e-5


def _rb(x):
    """x rounded to bf16 (round to nearest even), back as float32."""
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).float().numpy()


@pytest.fixture
def bf16_math():
    import pa_capi
    pa_capi.set_f32_math("bf16")
    assert pa_capi.get_f32_math() == "bf16"
    yield
    pa_capi.set_f32_math("split3")


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(256, 192, 320), (100, 70, 50), (8192, 1536, 512)])
def test_matmul_bf16_math_matches_rounded_oracle(M, N, K, bf16_math):
    import oracle
    import pa_capi
    a, b = seeded_normal(M, (M, K)), seeded_normal(N, (K, N))
    c = torch.empty(M, N, device="cuda")
    pa_capi.matmul(_cu(a), _cu(b), c, M, N, K)
    assert rel_err(_np(c), oracle.matmul(_rb(a), _rb(b))) < BF16_MATH_TOL
    dy, w = seeded_normal(K + 1, (M, K)), seeded_normal(K + 2, (N, K))
    dx0 = seeded_normal(3, (M, N))
    dx = _cu(dx0)
    pa_capi.matmul_grad_x(_cu(dy), _cu(w), dx, M, N, K)
    assert rel_err(_np(dx), oracle.matmul_grad_x(_rb(dy), _rb(w), dx0)) < BF16_MATH_TOL
    x = seeded_normal(K + 3, (M, N))
    dw0 = seeded_normal(4, (N, K))
    dw = _cu(dw0)
    pa_capi.matmul_grad_w(_cu(x), _cu(dy), dw, M, N, K)
    assert rel_err(_np(dw), oracle.matmul_grad_w(_rb(x), _rb(dy), dw0)) < BF16_MATH_TOL


@pytest.mark.gpu
def test_linear_bf16_math_matches_rounded_oracle(bf16_math):
    """Fused projection (three column blocks, bias) forward and backward in
    the bf16 math mode; the bias and its gradient stay fp32."""
    import oracle
    import pa_capi
    M, IN, OUT, n = 4096, 256, 768, 3
    x, w, bias = seeded_normal(1, (M, IN)), seeded_normal(2, (IN, OUT)), seeded_normal(3, (OUT,))
    outs = [torch.empty(M, OUT // n, device="cuda") for _ in range(n)]
    ws = torch.empty(pa_capi.linear_workspace_size(M, IN, OUT), dtype=torch.uint8, device="cuda")
    pa_capi.linear_fwd(_cu(x), _cu(w), _cu(bias), outs, M, IN, OUT, ws)
    ref = oracle.matmul(_rb(x), _rb(w)) + bias
    got = np.concatenate([_np(o) for o in outs], axis=1)
    assert rel_err(got, ref) < BF16_MATH_TOL
    dys = [seeded_normal(10 + i, (M, OUT // n)) for i in range(n)]
    dy = np.concatenate(dys, axis=1)
    dx0, dw0, db0 = seeded_normal(4, (M, IN)), seeded_normal(5, (IN, OUT)), seeded_normal(6, (OUT,))
    dx, dw, db = _cu(dx0), _cu(dw0), _cu(db0)
    pa_capi.linear_bwd(_cu(x), _cu(w), [_cu(d) for d in dys], dx, dw, db, M, IN, OUT, ws)
    assert rel_err(_np(dx), oracle.matmul_grad_x(_rb(dy), _rb(w), dx0)) < BF16_MATH_TOL
    assert rel_err(_np(dw), oracle.matmul_grad_w(_rb(x), _rb(dy), dw0)) < BF16_MATH_TOL
    assert rel_err(_np(db), oracle.bias_grad(dy, db0)) < 1e-6


@pytest.mark.gpu
@pytest.mark.parametrize("math_mode", ["split3", "bf16"])
def test_linear_relu_matches_oracle(math_mode):
    """Y = max(0, X W + b) with the clamp in the GEMM epilogue; backward masks
    dY by Y > 0 in the operand gather and in the bias column sums."""
    import oracle
    import pa_capi
    M, IN, OUT = 2048, 256, 1024
    x, w, bias = seeded_normal(31, (M, IN)), seeded_normal(32, (IN, OUT), 0.1), seeded_normal(33, (OUT,))
    dy = seeded_normal(34, (M, OUT))
    rb = _rb if math_mode == "bf16" else (lambda a: a)
    tol = BF16_MATH_TOL if math_mode == "bf16" else GEMM_TOL
    pa_capi.set_f32_math(math_mode)
    try:
        y = torch.full((M, OUT), float("nan"), device="cuda")
        ws = torch.empty(pa_capi.linear_workspace_size(M, IN, OUT), dtype=torch.uint8, device="cuda")
        pa_capi.linear_relu_fwd(_cu(x), _cu(w), _cu(bias), y, M, IN, OUT, ws)
        z = oracle.matmul(rb(x), rb(w)) + bias
        yn = _np(y)
        assert rel_err(yn, np.maximum(z, 0.0)) < tol
        assert (yn >= 0).all() and 0.2 < (yn > 0).mean() < 0.8
        dx0, dw0, db0 = seeded_normal(35, (M, IN)), seeded_normal(36, (IN, OUT)), seeded_normal(37, (OUT,))
        dx, dw, db = _cu(dx0), _cu(dw0), _cu(db0)
        pa_capi.linear_relu_bwd(_cu(x), _cu(w), y, _cu(dy), dx, dw, db, M, IN, OUT, ws)
        dz = np.where(yn > 0, dy, 0.0)
        assert rel_err(_np(dx), oracle.matmul_grad_x(rb(dz), rb(w), dx0)) < tol
        assert rel_err(_np(dw), oracle.matmul_grad_w(rb(x), rb(dz), dw0)) < tol
        assert rel_err(_np(db), oracle.bias_grad(dz, db0)) < 1e-6
    finally:
        pa_capi.set_f32_math("split3")


@pytest.mark.gpu
@pytest.mark.parametrize("math_mode", ["split3", "bf16"])
@pytest.mark.parametrize("M,IN,OUT,n,relu", [(16384, 128, 3072, 3, False), (16384, 128, 4096, 1, True),
                                             (3000, 64, 200, 1, False), (40, 64, 96, 3, False)])
def test_linear_bwd_bias_grad_same_bits_as_column_sum_kernel(M, IN, OUT, n, relu, math_mode):
    """The projection backward sums the bias gradient in the same pass that
    gathers dY into bf16 planes; its chunked column sums are the two-stage
    pa_bias_grad_ws kernel's, so db matches that kernel bit for bit (masked
    by the ReLU output when there is one), and dX matches the oracle."""
    import oracle
    import pa_capi
    x, w = seeded_normal(51, (M, IN)), seeded_normal(52, (IN, OUT), 0.1)
    parts = [seeded_normal(60 + c, (M, OUT // n)) for c in range(n)]
    y = np.maximum(seeded_normal(59, (M, OUT)), 0.0) if relu else None
    db0 = seeded_normal(53, (OUT,))
    pa_capi.set_f32_math(math_mode)
    try:
        db, dx = _cu(db0), torch.zeros(M, IN, device="cuda")
        if relu:
            pa_capi.linear_relu_bwd(_cu(x), _cu(w), _cu(y), _cu(parts[0]), dx, None, db, M, IN, OUT)
        else:
            pa_capi.linear_bwd(_cu(x), _cu(w), [_cu(p) for p in parts], dx, None, db, M, IN, OUT)
        assert pa_capi.device_status() == 0
        ref = _cu(db0)
        W = OUT // n
        ws = torch.empty(pa_capi.bias_grad_workspace_size(M, W), dtype=torch.uint8, device="cuda")
        for c in range(n):
            d = np.where(y > 0, parts[c], 0.0).astype(np.float32) if relu else parts[c]
            pa_capi.bias_grad(_cu(d), ref[c * W:(c + 1) * W], M, W, workspace=ws)
        assert torch.equal(db, ref)
        dz = np.concatenate([np.where(y > 0, p, 0.0) if relu else p for p in parts], axis=1)
        rb = _rb if math_mode == "bf16" else (lambda a: a)
        tol = BF16_MATH_TOL if math_mode == "bf16" else GEMM_TOL
        assert rel_err(_np(dx), oracle.matmul_grad_x(rb(dz), rb(w), np.zeros((M, IN)))) < tol
    finally:
        pa_capi.set_f32_math("split3")


@pytest.mark.gpu
def test_adam_multi_tensor_matches_single_tensor_updates():
    """pa_adam_step_multi over 100 tensors (three launches of up to 48; sizes
    ragged, empty, one element and several chunks) equals pa_adam_step per
    tensor."""
    import ctypes
    import pa_capi
    lib = pa_capi.load()
    rng = np.random.default_rng(40)
    sizes = [int(s) for s in rng.integers(1, 20000, size=96)] + [0, 1, 3, 70001]
    def make(seed):
        g = np.random.default_rng(seed)
        return [torch.from_numpy(g.standard_normal(max(n, 1)).astype(np.float32)).cuda() for n in sizes]
    w1, g1, m1, v1 = make(1), make(2), make(3), [t.abs() for t in make(4)]
    w2, m2, v2 = [t.clone() for t in w1], [t.clone() for t in m1], [t.clone() for t in v1]
    args = (1e-3, 0.9, 0.999, 1e-8, 0.19, 0.002)
    for i, n in enumerate(sizes):
        assert lib.pa_adam_step(w1[i].data_ptr(), g1[i].data_ptr(), m1[i].data_ptr(), v1[i].data_ptr(),
                                n, *args, None) == 0
    arr = lambda ts: (ctypes.c_void_p * len(ts))(*[t.data_ptr() for t in ts])
    szs = (ctypes.c_size_t * len(sizes))(*sizes)
    assert lib.pa_adam_step_multi(arr(w2), arr(g1), arr(m2), arr(v2), szs, len(sizes), *args, None) == 0
    assert pa_capi.device_status() == 0
    for a, b in zip(w1 + m1 + v1, w2 + m2 + v2):
        np.testing.assert_allclose(_np(b), _np(a), rtol=2e-6, atol=1e-7)


@pytest.mark.gpu
@pytest.mark.parametrize("fwd_mode,bwd_mode", [("split3", "split3"), ("bf16", "bf16"),
                                               ("split3", "bf16"), ("bf16", "split3")])
def test_linear_kept_planes_match_plain_calls(fwd_mode, bwd_mode):
    """pa_linear_fwd_keep / pa_linear_bwd_kept (X's operand planes kept from the
    forward) give the plain calls' results, also when the math mode changed in
    between (split3 planes serve bf16; bf16 planes make a split3 backward
    convert X again); ReLU form included."""
    import pa_capi
    M, IN, OUT = 1024, 256, 384
    x, w, bias = seeded_normal(51, (M, IN)), seeded_normal(52, (IN, OUT), 0.1), seeded_normal(53, (OUT,))
    dy = seeded_normal(54, (M, OUT))
    ws = torch.empty(pa_capi.linear_workspace_size(M, IN, OUT), dtype=torch.uint8, device="cuda")
    try:
        for relu in (False, True):
            pa_capi.set_f32_math(fwd_mode)
            kept = torch.empty(pa_capi.linear_kept_size(M, IN), dtype=torch.uint8, device="cuda")
            y_keep, y_ref = (torch.empty(M, OUT, device="cuda") for _ in range(2))
            pa_capi.linear_fwd_keep(_cu(x), _cu(w), _cu(bias), [y_keep], M, IN, OUT, kept, relu=relu,
                                    workspace=ws)
            if relu:
                pa_capi.linear_relu_fwd(_cu(x), _cu(w), _cu(bias), y_ref, M, IN, OUT, ws)
            else:
                pa_capi.linear_fwd(_cu(x), _cu(w), _cu(bias), [y_ref], M, IN, OUT, ws)
            np.testing.assert_array_equal(_np(y_keep), _np(y_ref))
            pa_capi.set_f32_math(bwd_mode)
            g1 = [torch.zeros(M, IN, device="cuda"), torch.zeros(IN, OUT, device="cuda"),
                  torch.zeros(OUT, device="cuda")]
            g2 = [torch.zeros_like(t) for t in g1]
            pa_capi.linear_bwd_kept(_cu(x), _cu(w), kept, fwd_mode, y_keep if relu else None, [_cu(dy)],
                                    *g1, M, IN, OUT, workspace=ws)
            if relu:
                pa_capi.linear_relu_bwd(_cu(x), _cu(w), y_ref, _cu(dy), *g2, M, IN, OUT, ws)
            else:
                pa_capi.linear_bwd(_cu(x), _cu(w), [_cu(dy)], *g2, M, IN, OUT, ws)
            for a, b in zip(g1, g2):
                assert rel_err(_np(a), _np(b)) < 1e-6
    finally:
        pa_capi.set_f32_math("split3")
    assert pa_capi.device_status() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("M,IN,OUT,relu", [(16384, 1024, 4096, True), (1000, 200, 96, False)])
def test_linear_bwd_dx_overwrite(M, IN, OUT, relu):
    """PA_LINEAR_DX_OVERWRITE writes dX = dY W^T over whatever the buffer held
    (NaN here): the values of accumulating into zeros (which may split K into
    slices added in any order, so within fp32 reordering: 1e-5), the other
    gradients untouched by the flag."""
    import pa_capi
    x, w, bias = seeded_normal(71, (M, IN)), seeded_normal(72, (IN, OUT), 0.05), seeded_normal(73, (OUT,))
    dy = seeded_normal(74, (M, OUT))
    ws = torch.empty(pa_capi.linear_workspace_size(M, IN, OUT), dtype=torch.uint8, device="cuda")
    pa_capi.set_f32_math("bf16")
    try:
        kept = torch.empty(pa_capi.linear_kept_size(M, IN), dtype=torch.uint8, device="cuda")
        y = torch.empty(M, OUT, device="cuda")
        pa_capi.linear_fwd_keep(_cu(x), _cu(w), _cu(bias), [y], M, IN, OUT, kept, relu=relu, workspace=ws)
        grads = []
        for overwrite in (False, True):
            dx = torch.full((M, IN), float("nan"), device="cuda") if overwrite else torch.zeros(M, IN, device="cuda")
            dw, db = torch.zeros(IN, OUT, device="cuda"), torch.zeros(OUT, device="cuda")
            pa_capi.linear_bwd_kept(_cu(x), _cu(w), kept, "bf16", y if relu else None, [_cu(dy)], dx, dw, db,
                                    M, IN, OUT, workspace=ws, dx_overwrite=overwrite)
            grads.append((dx, dw, db))
        assert pa_capi.device_status() == 0
        assert not torch.isnan(grads[1][0]).any()
        for a, b in zip(*grads):
            assert rel_err(_np(b), _np(a)) < 1e-5
        assert torch.equal(grads[0][2], grads[1][2])  # bias gradient: fixed-order sums
    finally:
        pa_capi.set_f32_math("split3")


@pytest.mark.gpu
@pytest.mark.parametrize("math_mode", ["bf16", "split3"])
@pytest.mark.parametrize("M,IN,HID,OUT", [(4096, 256, 1024, 256), (300, 64, 200, 72)])
def test_linear_output_planes_feed_the_next_projection(math_mode, M, IN, HID, OUT):
    """pa_linear_fwd_planes writes the hidden layer's bf16 planes from its GEMM
    epilogue: byte for byte the planes the next projection would make from the
    stored output, so that projection, taking them as kept (PA_LINEAR_KEPT_VALID),
    gives the same output bits as converting them itself."""
    import pa_capi
    x, w1, b1 = seeded_normal(81, (M, IN)), seeded_normal(82, (IN, HID), 0.1), seeded_normal(83, (HID,))
    w2, b2 = seeded_normal(84, (HID, OUT), 0.05), seeded_normal(85, (OUT,))
    pa_capi.set_f32_math(math_mode)
    try:
        kept1 = torch.empty(pa_capi.linear_kept_size(M, IN), dtype=torch.uint8, device="cuda")
        yp = torch.zeros(pa_capi.linear_kept_size(M, HID), dtype=torch.uint8, device="cuda")
        h = torch.empty(M, HID, device="cuda")
        pa_capi.linear_fwd_planes(_cu(x), _cu(w1), _cu(b1), [h], M, IN, HID, kept1, math_mode,
                                  y_planes=yp, relu=True)
        h_ref = torch.empty_like(h)
        pa_capi.linear_relu_fwd(_cu(x), _cu(w1), _cu(b1), h_ref, M, IN, HID)
        assert torch.equal(h, h_ref)
        # the planes the next projection makes from h itself
        kept2 = torch.zeros_like(yp)
        y_conv = torch.empty(M, OUT, device="cuda")
        pa_capi.linear_fwd_keep(h, _cu(w2), _cu(b2), [y_conv], M, HID, OUT, kept2)
        assert torch.equal(yp, kept2)
        y_taken = torch.empty_like(y_conv)
        pa_capi.linear_fwd_planes(h, _cu(w2), _cu(b2), [y_taken], M, HID, OUT, yp, math_mode,
                                  kept_valid=True)
        assert torch.equal(y_taken, y_conv)
        assert pa_capi.device_status() == 0
    finally:
        pa_capi.set_f32_math("split3")


@pytest.mark.gpu
@pytest.mark.parametrize("math_mode", ["bf16", "split3"])
@pytest.mark.parametrize("residual", [False, True])
@pytest.mark.parametrize("M,N,OUT", [(4096, 1024, 512), (300, 100, 72), (5, 12, 8)])
def test_layer_norm_output_planes_feed_the_next_projection(math_mode, residual, M, N, OUT):
    """pa_layer_norm_fwd_planes writes y, mean and rstd bit for bit as the plain
    (add +) LayerNorm forward, and y's bf16 planes byte for byte as the next
    projection would make them from y (zero padding of the row pitch included);
    that projection, taking them as kept (PA_LINEAR_KEPT_VALID), gives the same
    output bits as converting y itself."""
    import pa_capi
    x, r = seeded_normal(M + 91, (M, N)), seeded_normal(M + 92, (M, N))
    gamma = 1.0 + 0.1 * seeded_normal(N + 93, (N,))
    beta = 0.1 * seeded_normal(N + 94, (N,))
    w, b = seeded_normal(95, (N, OUT), 0.05), seeded_normal(96, (OUT,))
    pa_capi.set_f32_math(math_mode)
    try:
        xs, rs_, g, bt = _cu(x), _cu(r), _cu(gamma), _cu(beta)
        y, mean, rstd = (torch.empty(M, N, device="cuda"), torch.empty(M, device="cuda"),
                         torch.empty(M, device="cuda"))
        s = torch.empty(M, N, device="cuda") if residual else None
        yp = torch.full((pa_capi.linear_kept_size(M, N),), 0x5A, dtype=torch.uint8, device="cuda")
        pa_capi.layer_norm_fwd_planes(xs, g, bt, y, mean, rstd, yp, r=rs_ if residual else None,
                                      out_sum=s)
        y2, m2, r2 = torch.empty_like(y), torch.empty_like(mean), torch.empty_like(rstd)
        if residual:
            s2 = torch.empty_like(y)
            pa_capi.add_layer_norm_fwd(xs, rs_, s2, g, bt, y2, m2, r2)
            assert torch.equal(s, s2)
        else:
            pa_capi.layer_norm_fwd(xs, g, bt, y2, m2, r2)
        assert torch.equal(y, y2) and torch.equal(mean, m2) and torch.equal(rstd, r2)
        kept = torch.full_like(yp, 0x5A)
        out_conv = torch.empty(M, OUT, device="cuda")
        pa_capi.linear_fwd_keep(y, _cu(w), _cu(b), [out_conv], M, N, OUT, kept)
        assert torch.equal(yp, kept)
        out_taken = torch.empty_like(out_conv)
        pa_capi.linear_fwd_planes(y, _cu(w), _cu(b), [out_taken], M, N, OUT, yp, math_mode,
                                  kept_valid=True)
        assert torch.equal(out_taken, out_conv)
        assert pa_capi.device_status() == 0
    finally:
        pa_capi.set_f32_math("split3")


@pytest.mark.gpu
def test_layer_norm_planes_reject_bad_arguments():
    """Too small a plane buffer, a misaligned one, or a residual without its sum
    are refused before any launch."""
    import pa_capi
    M, N = 64, 128
    x = torch.randn(M, N, device="cuda")
    g, b = torch.ones(N, device="cuda"), torch.zeros(N, device="cuda")
    y, mean, rstd = torch.empty_like(x), torch.empty(M, device="cuda"), torch.empty(M, device="cuda")
    n = pa_capi.linear_kept_size(M, N)
    buf = torch.empty(n + 512, dtype=torch.uint8, device="cuda")
    with pytest.raises(pa_capi.PaError):
        pa_capi.layer_norm_fwd_planes(x, g, b, y, mean, rstd, buf[:n - 256])
    with pytest.raises(pa_capi.PaError):
        pa_capi.layer_norm_fwd_planes(x, g, b, y, mean, rstd, buf[16:16 + n])
    with pytest.raises(pa_capi.PaError):
        pa_capi.layer_norm_fwd_planes(x, g, b, y, mean, rstd, buf[:n], r=x)
    pa_capi.layer_norm_fwd_planes(x, g, b, y, mean, rstd, buf[:n])
    assert pa_capi.device_status() == 0
