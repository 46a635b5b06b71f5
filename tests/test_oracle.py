"""The float64 oracle against independent float64 references (torch autograd on
CPU, numpy) on small seeded cases. Runs without a GPU."""
import numpy as np
import pytest

from conftest import rel_err, seeded_normal

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module")
def oracle():
    import oracle as o
    o.lib()
    return o


def _torch_attn(q, k, v, dO, scale):
    tq, tk, tv = (torch.tensor(x, dtype=torch.float64, requires_grad=True) for x in (q, k, v))
    # [B, L, H, D] -> [B, H, L, D]
    s = torch.einsum("bihd,bjhd->bhij", tq, tk) * scale
    lse = torch.logsumexp(s, dim=-1)
    p = torch.softmax(s, dim=-1)
    o = torch.einsum("bhij,bjhd->bihd", p, tv)
    o.backward(torch.tensor(dO, dtype=torch.float64))
    B, L, H, D = q.shape
    return (o.detach().numpy(), lse.detach().numpy().reshape(B * H, L), tq.grad.numpy(),
            tk.grad.numpy(), tv.grad.numpy())


@pytest.mark.parametrize("B,L,H,D", [(1, 128, 1, 32), (2, 37, 3, 16), (1, 64, 2, 64)])
def test_attention_oracle_matches_torch_float64(oracle, B, L, H, D):
    shape = (B, L, H, D)
    q, k, v, g = (seeded_normal(s, shape).astype(np.float64) for s in (1, 2, 3, 4))
    scale = 1.0 / np.sqrt(D)
    to, tl, tdq, tdk, tdv = _torch_attn(q, k, v, g, scale)
    o, lse = oracle.attn_fwd(q, k, v)
    dq, dk, dv, delta = oracle.attn_bwd(q, k, v, o, g, lse)
    for a, b in ((o, to), (lse, tl), (dq, tdq), (dk, tdk), (dv, tdv)):
        assert rel_err(a, b) < 1e-12
    np.testing.assert_allclose(delta, np.einsum("blhd,blhd->blh", g, o), rtol=1e-12, atol=1e-12)


def test_layer_norm_oracle_matches_torch_float64(oracle):
    M, N = 33, 64
    x = seeded_normal(7, (M, N)).astype(np.float64)
    gamma = 1.0 + 0.1 * seeded_normal(8, (N,)).astype(np.float64)
    beta = 0.1 * seeded_normal(9, (N,)).astype(np.float64)
    dy = seeded_normal(10, (M, N)).astype(np.float64)
    tx = torch.tensor(x, requires_grad=True)
    tg = torch.tensor(gamma, requires_grad=True)
    tb = torch.tensor(beta, requires_grad=True)
    ty = torch.nn.functional.layer_norm(tx, (N,), tg, tb, eps=1e-5)
    ty.backward(torch.tensor(dy))
    y, mean, rstd = oracle.layer_norm_fwd(x, gamma, beta, 1e-5)
    dx, dg, db = oracle.layer_norm_bwd(dy, x, mean, rstd, gamma)
    assert rel_err(y, ty.detach().numpy()) < 1e-12
    assert rel_err(dx, tx.grad.numpy()) < 1e-10
    assert rel_err(dg, tg.grad.numpy()) < 1e-12
    assert rel_err(db, tb.grad.numpy()) < 1e-12


def test_matmul_oracles_match_numpy(oracle):
    M, N, K = 17, 23, 31
    a = seeded_normal(11, (M, K)).astype(np.float64)
    b = seeded_normal(12, (K, N)).astype(np.float64)
    np.testing.assert_allclose(oracle.matmul(a, b), a @ b, rtol=1e-12, atol=1e-12)
    dy = seeded_normal(13, (M, K)).astype(np.float64)
    w = seeded_normal(14, (N, K)).astype(np.float64)
    dx0 = seeded_normal(15, (M, N)).astype(np.float64)
    np.testing.assert_allclose(oracle.matmul_grad_x(dy, w, dx0), dx0 + dy @ w.T, rtol=1e-12,
                               atol=1e-12)
    x = seeded_normal(16, (M, N)).astype(np.float64)
    dw0 = seeded_normal(17, (N, K)).astype(np.float64)
    np.testing.assert_allclose(oracle.matmul_grad_w(x, dy, dw0), dw0 + x.T @ dy, rtol=1e-12,
                               atol=1e-12)


def test_elementwise_oracles(oracle):
    M, N = 9, 12
    a = seeded_normal(18, (M, N)).astype(np.float64)
    bias = seeded_normal(19, (N,)).astype(np.float64)
    np.testing.assert_allclose(oracle.bias_add(a, bias), a + bias[None, :])
    np.testing.assert_allclose(oracle.bias_grad(a, bias), bias + a.sum(0), rtol=1e-12)
    x = seeded_normal(20, (M, 3 * 4)).astype(np.float64)
    parts = oracle.split_last_dim(x, 3)
    for p in range(3):
        np.testing.assert_array_equal(parts[p], x[:, p * 4:(p + 1) * 4])
    np.testing.assert_array_equal(oracle.concat_last_dim_grad(parts), x)


def test_cpu_baseline_matches_oracle(oracle):
    """The fp32 multithreaded CPU implementation agrees with the float64 oracle."""
    B, L, H, D = 1, 200, 2, 64
    q, k, v, g = (seeded_normal(s, (B, L, H, D), 0.5) for s in (31, 32, 33, 34))
    o, lse, dq, dk, dv, nt = oracle.cpu_attn_fwd_bwd(q, k, v, g, nthreads=2)
    assert nt == 2
    ro, rl = oracle.attn_fwd(q, k, v)
    rdq, rdk, rdv, _ = oracle.attn_bwd(q, k, v, ro, g, rl)
    assert rel_err(o, ro) < 1e-5
    assert rel_err(lse, rl) < 1e-6
    for a, b in ((dq, rdq), (dk, rdk), (dv, rdv)):
        assert rel_err(a, b) < 1e-4


def test_sampled_row_oracle_equals_full_oracle(oracle):
    """oracle.attn_sampled (LSE of every row; O, dQ of sampled queries; dK, dV of
    sampled keys) computes the same numbers as the full float64 forward and
    backward, at a ragged length."""
    B, L, H, D = 1, 300, 2, 64
    q, k, v, g = (seeded_normal(s, (B, L, H, D), 0.5).astype(np.float64) for s in (41, 42, 43, 44))
    o, lse = oracle.attn_fwd(q, k, v)
    dq, dk, dv, _ = oracle.attn_bwd(q, k, v, o, g, lse)
    h = 1
    sl = lambda a: np.ascontiguousarray(a[0, :, h, :])
    qr, kr = [0, 5, 127, 128, 299], [1, 2, 150, 298, 299]
    rl, ro, rdq, rdk, rdv = oracle.attn_sampled(sl(q), sl(k), sl(v), sl(g), qr, kr)
    np.testing.assert_allclose(rl, lse[h], rtol=0, atol=1e-12)
    np.testing.assert_allclose(ro, sl(o)[qr], rtol=1e-12, atol=1e-13)
    np.testing.assert_allclose(rdq, sl(dq)[qr], rtol=1e-10, atol=1e-13)
    np.testing.assert_allclose(rdk, sl(dk)[kr], rtol=1e-10, atol=1e-13)
    np.testing.assert_allclose(rdv, sl(dv)[kr], rtol=1e-10, atol=1e-13)
    with pytest.raises(ValueError):
        oracle.attn_sampled(sl(q), sl(k), sl(v), sl(g), [L], [])
