"""Parity of the attention block's non-attention kernels (through the C ABI)
with the float64 oracle: the matmul forward and both gradients, LayerNorm
forward and backward, bias add / bias grad / grad accumulate / residual add,
and the last-dimension split and its adjoint.

Tolerances (fp32 path): GEMMs 1e-4 norm-wise (bf16 hi/lo split products),
LayerNorm 1e-5 (y, dgamma, dbeta) and 1e-4 (dX), elementwise 1e-6."""
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
