"""Parity of the sm_100a flash-attention kernels (through the C ABI) with the
float64 oracle on the same seeded, bf16-rounded inputs.

Tolerance (bf16 path): norm-wise relative error <= 2e-2 on O, dQ, dK, dV;
LSE within 2e-3 absolute."""
import numpy as np
import pytest

from conftest import rel_err, seeded_normal

BF16_TOL = 2e-2
LSE_TOL = 2e-3

torch = pytest.importorskip("torch")


def _bf16(x):
    """Round a float32 numpy array to bf16; returns (torch bf16 on cuda, float64 numpy)."""
    t = torch.from_numpy(x).to(torch.bfloat16)
    return t.cuda(), t.float().numpy().astype(np.float64)


def _run(B, L, H, D, seed, scale_in=0.5, accumulate=False):
    import pa_capi
    shape = (B, L, H, D)
    q, qn = _bf16(seeded_normal(seed, shape, scale_in))
    k, kn = _bf16(seeded_normal(seed + 1000, shape, scale_in))
    v, vn = _bf16(seeded_normal(seed + 2000, shape, scale_in))
    g, gn = _bf16(seeded_normal(seed + 3000, shape, scale_in))
    o = torch.empty_like(q)
    lse = torch.empty(B * H, L, dtype=torch.float32, device="cuda")
    pa_capi.attn_fwd(q, k, v, o, lse)
    d = pa_capi.attn_desc(q)
    ws = torch.empty(pa_capi.attn_bwd_workspace_size(d), dtype=torch.uint8, device="cuda")
    if accumulate:
        dq = torch.ones_like(q)
        dk = torch.ones_like(q)
        dv = torch.ones_like(q)
    else:
        dq, dk, dv = (torch.full_like(q, float("nan")) for _ in range(3))
    pa_capi.attn_bwd(q, k, v, o, g, lse, dq, dk, dv, ws, accumulate=accumulate)
    assert pa_capi.device_status() == 0
    torch.cuda.synchronize()
    f = lambda t: t.float().cpu().numpy().astype(np.float64)
    return (qn, kn, vn, gn), (f(o), lse.cpu().numpy().astype(np.float64), f(dq), f(dk), f(dv))


def _check(inputs, outs, heads=None, accumulate=False):
    import oracle
    qn, kn, vn, gn = inputs
    o, lse, dq, dk, dv = outs
    B, L, H, D = qn.shape
    sel = heads or [(b, h) for b in range(B) for h in range(H)]
    for (b, h) in sel:
        sl = (slice(b, b + 1), slice(None), slice(h, h + 1), slice(None))
        ro, rl = oracle.attn_fwd(qn[sl], kn[sl], vn[sl])
        # the oracle's dO path uses the kernel-independent exact O
        rdq, rdk, rdv, _ = oracle.attn_bwd(qn[sl], kn[sl], vn[sl], ro, gn[sl], rl)
        off = 1.0 if accumulate else 0.0
        errs = {
            "o": rel_err(o[sl], ro),
            "dq": rel_err(dq[sl] - off, rdq),
            "dk": rel_err(dk[sl] - off, rdk),
            "dv": rel_err(dv[sl] - off, rdv),
        }
        lse_err = float(np.max(np.abs(lse[b * H + h] - rl[0])))
        print(f"(b={b},h={h}) L={L} D={D} rel errs {errs} lse max abs {lse_err:.2e}")
        for name, e in errs.items():
            assert e <= BF16_TOL, (name, e)
        assert lse_err <= LSE_TOL


@pytest.mark.gpu
@pytest.mark.parametrize("B,L,H,D", [
    (1, 128, 1, 64),     # one query tile pair / one KV tile
    (2, 512, 2, 64),
    (1, 256, 3, 128),
    (1, 200, 2, 64),     # ragged: partial query and key tiles
    (1, 333, 1, 128),    # ragged, d = 128
    (1, 1024, 2, 64),    # several KV tiles, exercises the stage ring
    (1, 64, 2, 64),      # shorter than one tile
    (2, 300, 3, 64),     # odd number of key tiles: the last cluster's second CTA has no keys
])
def test_attention_bf16_matches_oracle(B, L, H, D):
    inputs, outs = _run(B, L, H, D, seed=B * 131 + L * 7 + H * 3 + D)
    _check(inputs, outs)


@pytest.mark.gpu
def test_attention_bf16_accumulate_adds_into_grads():
    """accumulate=1 adds into dq/dk/dv: a second call onto the first call's
    result doubles it (grads of the same magnitude, so bf16 keeps them)."""
    import pa_capi
    B, L, H, D = 1, 256, 2, 64
    q, k, v, g = (_bf16(seeded_normal(s, (B, L, H, D), 0.5))[0] for s in (11, 12, 13, 14))
    o = torch.empty_like(q)
    lse = torch.empty(B * H, L, device="cuda")
    pa_capi.attn_fwd(q, k, v, o, lse)
    ws = torch.empty(pa_capi.attn_bwd_workspace_size(pa_capi.attn_desc(q)), dtype=torch.uint8,
                     device="cuda")
    grads = [torch.empty_like(q) for _ in range(3)]
    pa_capi.attn_bwd(q, k, v, o, g, lse, *grads, ws)
    first = [t.float().cpu().numpy() for t in grads]
    pa_capi.attn_bwd(q, k, v, o, g, lse, *grads, ws, accumulate=True)
    torch.cuda.synchronize()
    for f, t in zip(first, grads):
        assert rel_err(t.float().cpu().numpy(), 2.0 * f) < 5e-3


@pytest.mark.gpu
def test_attention_bf16_headline_shape_slices():
    """B=8, H=16, L=4096, d=64 (the headline shape): six (b, h) slices spread
    over batches and heads against the full float64 oracle, and LSE / O / dQ /
    dK / dV on sampled rows of six more."""
    inputs, outs = _run(8, 4096, 16, 64, seed=3)
    _check(inputs, outs, heads=[(0, 0), (1, 7), (3, 3), (4, 12), (6, 9), (7, 15)])
    _check_sampled(inputs, outs, heads=[(0, 15), (2, 1), (3, 14), (5, 5), (6, 0), (7, 8)],
                   n_rows=128)


@pytest.mark.gpu
@pytest.mark.parametrize("D", [64, 128])
def test_attention_bf16_uneven_work_per_cta(D):
    """B=3, H=13, L=1000 (ragged last tiles): 156 forward units of 256 query
    rows over 148 CTAs and, at d=64, 156 backward items over 74 CTA pairs, so
    some CTAs carry their ring slots and barrier phases into a second or third
    item. Every output element is written (the gradients start as NaN); four
    heads match the float64 oracle; and each checked head, run again alone as
    a one-head problem, gives bit-identical O, LSE, dK and dV (dQ is reduced
    in no fixed order: within one bf16 ulp per element, plus 1e-5 of max |dQ|
    where the reduction cancels)."""
    import pa_capi
    B, L, H = 3, 1000, 13
    inputs, outs = _run(B, L, H, D, seed=17 + D)
    for t in outs:
        assert np.isfinite(t).all()
    heads = [(0, 0), (1, 7), (2, 11), (2, 12)]
    _check(inputs, outs, heads=heads)
    o, lse, dq, dk, dv = outs
    f = lambda t: t.float().cpu().numpy().astype(np.float64)
    for (b, h) in heads:
        sl = (slice(b, b + 1), slice(None), slice(h, h + 1), slice(None))
        q1, k1, v1, g1 = (torch.from_numpy(np.ascontiguousarray(x[sl]).astype(np.float32))
                          .to(torch.bfloat16).cuda() for x in inputs)
        o1 = torch.empty_like(q1)
        lse1 = torch.empty(1, L, dtype=torch.float32, device="cuda")
        pa_capi.attn_fwd(q1, k1, v1, o1, lse1)
        d1 = pa_capi.attn_desc(q1)
        ws1 = torch.empty(pa_capi.attn_bwd_workspace_size(d1), dtype=torch.uint8, device="cuda")
        dq1, dk1, dv1 = (torch.empty_like(q1) for _ in range(3))
        pa_capi.attn_bwd(q1, k1, v1, o1, g1, lse1, dq1, dk1, dv1, ws1)
        assert pa_capi.device_status() == 0
        np.testing.assert_array_equal(f(o1), o[sl])
        np.testing.assert_array_equal(lse1.cpu().numpy().astype(np.float64)[0], lse[b * H + h])
        np.testing.assert_array_equal(f(dk1), dk[sl])
        np.testing.assert_array_equal(f(dv1), dv[sl])
        a, r = f(dq1), dq[sl]
        # one bf16 ulp, plus fp32 reduction-order noise where dQ cancels to near 0
        assert np.all(np.abs(a - r) <= np.maximum(np.abs(a), np.abs(r)) * 2.0 ** -7
                      + 1e-5 * np.max(np.abs(r)))


@pytest.mark.gpu
def test_attention_bf16_d128_two_heads_oracle():
    """d = 128 at L = 2048 (all heads) against the oracle."""
    inputs, outs = _run(1, 2048, 2, 128, seed=4)
    _check(inputs, outs)


def _sampled_rows(L, n, seed):
    """n distinct rows of [0, L): both ends (tile edges), the rest spread at random."""
    rng = np.random.default_rng(seed)
    ends = [0, 1, 127, 128, L // 2, L - 129, L - 128, L - 2, L - 1]
    rest = rng.choice(np.setdiff1d(np.arange(L), ends), size=n - len(ends), replace=False)
    return np.sort(np.concatenate([ends, rest])).astype(np.int32)


def _check_sampled(inputs, outs, heads, n_rows=256):
    """Oracle parity at lengths where the full float64 backward is too slow:
    for each (b, h), LSE of every query row, and O / dQ on n_rows sampled query
    rows, dK / dV on n_rows sampled key rows (oracle.attn_sampled)."""
    import oracle
    qn, kn, vn, gn = inputs
    o, lse, dq, dk, dv = outs
    B, L, H, D = qn.shape
    for (b, h) in heads:
        sl = lambda a: np.ascontiguousarray(a[b, :, h, :])
        qr = _sampled_rows(L, n_rows, 17 * b + h)
        kr = _sampled_rows(L, n_rows, 1000 + 17 * b + h)
        rl, ro, rdq, rdk, rdv = oracle.attn_sampled(sl(qn), sl(kn), sl(vn), sl(gn), qr, kr)
        errs = {"o": rel_err(sl(o)[qr], ro), "dq": rel_err(sl(dq)[qr], rdq),
                "dk": rel_err(sl(dk)[kr], rdk), "dv": rel_err(sl(dv)[kr], rdv)}
        lse_err = float(np.max(np.abs(lse[b * H + h] - rl)))
        print(f"(b={b},h={h}) L={L} D={D} sampled rel errs {errs} lse (all rows) max abs {lse_err:.2e}")
        for name, e in errs.items():
            assert e <= BF16_TOL, (b, h, name, e)
        assert lse_err <= LSE_TOL, (b, h, lse_err)


@pytest.mark.gpu
def test_attention_bf16_long_sequence_d128_oracle():
    """B=2, H=16, L=16384, d=128 (the long-sequence shape): 128 query tiles per
    key tile, LSE / Delta over 16 384 rows. Against the float64 oracle on two
    (b, h) slices: LSE of every row, O and dQ on 256 sampled query rows, dK and
    dV on 256 sampled key rows. Then identities of the math over every head:
      sum_j dV_j = sum_i dO_i   (rows of P sum to 1)
      sum_j dK_j = 0            (rows of dS sum to 0)
      O rows lie in the range of V's columns (convex combinations)."""
    inputs, outs = _run(2, 16384, 16, 128, seed=4)
    _check_sampled(inputs, outs, heads=[(0, 0), (1, 15)])
    (qn, kn, vn, gn), (o, lse, dq, dk, dv) = inputs, outs
    assert rel_err(dv.sum(axis=1), gn.sum(axis=1)) < 2e-2
    assert np.abs(dk.sum(axis=1)).max() <= 2e-2 * np.abs(dk).sum(axis=1).max()
    assert np.all(o <= vn.max(axis=1, keepdims=True) + 1e-2)
    assert np.all(o >= vn.min(axis=1, keepdims=True) - 1e-2)
    assert np.all(np.isfinite(dq)) and np.all(np.isfinite(lse))


@pytest.mark.gpu
def test_attention_bf16_long_sequence_d64_properties():
    """B=1, H=4, L=16384, d=64: 128 query tiles per key tile, so the per-cluster
    query-tile order wraps around. Sampled-row oracle parity on two heads, and
    the exact identities of the d=128 test over every head."""
    inputs, outs = _run(1, 16384, 4, 64, seed=6)
    _check_sampled(inputs, outs, heads=[(0, 0), (0, 3)])
    (qn, kn, vn, gn), (o, lse, dq, dk, dv) = inputs, outs
    assert rel_err(dv.sum(axis=1), gn.sum(axis=1)) < 2e-2
    assert np.abs(dk.sum(axis=1)).max() <= 2e-2 * np.abs(dk).sum(axis=1).max()
    assert np.all(o <= vn.max(axis=1, keepdims=True) + 1e-2)
    assert np.all(o >= vn.min(axis=1, keepdims=True) - 1e-2)
    assert np.all(np.isfinite(dq)) and np.all(np.isfinite(lse))


@pytest.mark.gpu
def test_attention_deterministic_forward():
    _, a = _run(1, 512, 2, 64, seed=5)
    _, b = _run(1, 512, 2, 64, seed=5)
    np.testing.assert_array_equal(a[0], b[0])
    np.testing.assert_array_equal(a[1], b[1])
    # dK / dV are accumulated in TMEM in a fixed order: bitwise equal as well
    np.testing.assert_array_equal(a[3], b[3])
    np.testing.assert_array_equal(a[4], b[4])


@pytest.mark.gpu
def test_attention_delta_matches_oracle():
    import oracle
    import pa_capi
    B, L, H, D = 2, 300, 3, 64
    o, on = _bf16(seeded_normal(21, (B, L, H, D)))
    g, gn = _bf16(seeded_normal(22, (B, L, H, D)))
    delta = torch.zeros(B, L, H, dtype=torch.float32, device="cuda")
    pa_capi.attn_delta(g, o, delta)
    torch.cuda.synchronize()
    ref = np.einsum("blhd,blhd->blh", gn, on)
    assert rel_err(delta.cpu().numpy(), ref) < 1e-5


@pytest.mark.gpu
def test_attention_rejects_bad_arguments():
    import pa_capi
    q = torch.zeros(1, 128, 1, 96, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(pa_capi.PaError) as e:
        pa_capi.attn_fwd(q, q, q, q, torch.zeros(128, device="cuda"))
    assert e.value.status == 4  # PA_ERR_UNSUPPORTED
    q = torch.zeros(1, 128, 1, 64, dtype=torch.bfloat16, device="cuda")
    d = pa_capi.attn_desc(q)
    small = torch.empty(16, dtype=torch.uint8, device="cuda")
    with pytest.raises(pa_capi.PaError) as e:
        pa_capi.attn_bwd(q, q, q, q, q, torch.zeros(128, device="cuda"), q, q, q, small)
    assert e.value.status == 7  # PA_ERR_WORKSPACE


# ---------------------------------------------------------------- fp32 path
F32_TOL = 1e-3  # norm-wise relative error on O, dQ, dK, dV (fp32 path)


def _run_f32(q, k, v, g, accumulate=False):
    import pa_capi
    B, L, H, D = q.shape
    tq, tk, tv, tg = (torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()
                      for x in (q, k, v, g))
    o = torch.empty_like(tq)
    lse = torch.empty(B * H, L, device="cuda")
    pa_capi.attn_fwd(tq, tk, tv, o, lse)
    d = pa_capi.attn_desc(tq)
    ws = torch.empty(pa_capi.attn_bwd_workspace_size(d), dtype=torch.uint8, device="cuda")
    dq, dk, dv = (torch.full_like(tq, float("nan")) for _ in range(3))
    pa_capi.attn_bwd(tq, tk, tv, o, tg, lse, dq, dk, dv, ws)
    assert pa_capi.device_status() == 0
    torch.cuda.synchronize()
    f = lambda t: t.cpu().numpy().astype(np.float64)
    return f(o), f(lse), f(dq), f(dk), f(dv)


@pytest.mark.gpu
@pytest.mark.parametrize("B,L,H,D,heads", [
    (1, 128, 1, 32, None),     # single-head C1 shape
    (2, 256, 2, 64, None),
    (1, 200, 3, 32, None),     # ragged tiles, d = 32 (padded planes)
    (8, 1024, 8, 64, [(0, 0), (3, 5), (7, 7)]),  # the pre-LN block's attention shape
])
def test_attention_f32_matches_oracle(B, L, H, D, heads):
    import oracle
    shape = (B, L, H, D)
    q, k, v, g = (seeded_normal(s, shape) for s in (B + L, B + L + 1, B + L + 2, B + L + 3))
    o, lse, dq, dk, dv = _run_f32(q, k, v, g)
    for (b, h) in heads or [(b, h) for b in range(B) for h in range(H)]:
        sl = (slice(b, b + 1), slice(None), slice(h, h + 1), slice(None))
        ro, rl = oracle.attn_fwd(q[sl], k[sl], v[sl])
        rdq, rdk, rdv, _ = oracle.attn_bwd(q[sl], k[sl], v[sl], ro, g[sl], rl)
        errs = {"o": rel_err(o[sl], ro), "dq": rel_err(dq[sl], rdq), "dk": rel_err(dk[sl], rdk),
                "dv": rel_err(dv[sl], rdv)}
        print(f"f32 (b={b},h={h}) L={L} D={D} rel errs {errs}")
        for name, e in errs.items():
            assert e <= F32_TOL, (name, e)
        assert np.max(np.abs(lse[b * H + h] - rl[0])) < 1e-4


@pytest.mark.gpu
def test_attention_f32_matches_reference_golden_c1():
    """fp32 path on the exact inputs of the golden fixture produced by the
    reference's own kernels (B=1, H=1, L=128, d=32): O, LSE, dK, dV."""
    import os
    z = np.load(os.path.join(os.path.dirname(__file__), "golden", "ref_c1_attention.npz"))
    o, lse, dq, dk, dv = _run_f32(z["q"], z["k"], z["v"], z["dO"])
    assert rel_err(o, z["o"]) < F32_TOL
    assert np.max(np.abs(lse - z["lse"])) < 1e-4
    assert rel_err(dk, z["dk"]) < F32_TOL
    assert rel_err(dv, z["dv"]) < F32_TOL


# ---------------------------------------------------------------- fp32 tensors, bf16 math
@pytest.fixture
def bf16_math():
    import pa_capi
    pa_capi.set_f32_math("bf16")
    yield
    pa_capi.set_f32_math("split3")


@pytest.mark.gpu
@pytest.mark.parametrize("B,L,H,D", [(2, 256, 2, 64), (1, 300, 3, 64)])
def test_attention_f32_tensors_bf16_math(B, L, H, D, bf16_math):
    """fp32 q, k, v, dO computed in the bf16 math mode (the bf16 d=64 kernels
    on bf16 roundings, fp32 O / dQ / dK / dV): the bf16 path's accuracy
    against the oracle on the rounded inputs, and accumulate adds into the
    fp32 gradients."""
    import pa_capi
    shape = (B, L, H, D)
    raw = [seeded_normal(s, shape, 0.5) for s in (B + L + 7, B + L + 8, B + L + 9, B + L + 10)]
    rounded = [torch.from_numpy(x).to(torch.bfloat16).float().numpy().astype(np.float64) for x in raw]
    tq, tk, tv, tg = (torch.from_numpy(x).cuda() for x in raw)
    o = torch.empty_like(tq)
    lse = torch.empty(B * H, L, device="cuda")
    pa_capi.attn_fwd(tq, tk, tv, o, lse)
    d = pa_capi.attn_desc(tq)
    ws = torch.empty(pa_capi.attn_bwd_workspace_size(d), dtype=torch.uint8, device="cuda")
    dq, dk, dv = (torch.ones_like(tq) for _ in range(3))
    pa_capi.attn_bwd(tq, tk, tv, o, tg, lse, dq, dk, dv, ws, accumulate=True)
    assert pa_capi.device_status() == 0
    f = lambda t: t.cpu().numpy().astype(np.float64)
    _check(tuple(rounded), (f(o), f(lse), f(dq), f(dk), f(dv)), accumulate=True)


@pytest.mark.gpu
@pytest.mark.parametrize("fwd_mode,bwd_mode", [("bf16", "bf16"), ("split3", "split3"),
                                               ("split3", "bf16"), ("bf16", "split3")])
def test_attention_f32_backward_with_kept_planes(fwd_mode, bwd_mode):
    """pa_attn_bwd_kept reuses the q, k, v planes the fp32 forward left in its
    workspace: the same results as pa_attn_bwd (dK, dV bit for bit; dQ within
    the fp32 reduction order of its accumulator), also when the math mode
    changed in between (split3 planes serve bf16; bf16 planes make a split3
    backward convert q, k, v again)."""
    import pa_capi
    B, L, H, D = 2, 384, 3, 64
    shape = (B, L, H, D)
    tq, tk, tv, tg = (torch.from_numpy(seeded_normal(40 + i, shape, 0.5)).cuda() for i in range(4))
    d = pa_capi.attn_desc(tq)
    o, lse = torch.empty_like(tq), torch.empty(B * H, L, device="cuda")
    try:
        pa_capi.set_f32_math(fwd_mode)
        fws = torch.empty(pa_capi.attn_fwd_workspace_size(d), dtype=torch.uint8, device="cuda")
        pa_capi.attn_fwd(tq, tk, tv, o, lse, workspace=fws)
        pa_capi.set_f32_math(bwd_mode)
        ws = torch.empty(pa_capi.attn_bwd_workspace_size(d), dtype=torch.uint8, device="cuda")
        got = [torch.full_like(tq, float("nan")) for _ in range(3)]
        pa_capi.attn_bwd_kept(tq, tk, tv, o, tg, lse, *got, fws, fwd_mode, ws)
        want = [torch.full_like(tq, float("nan")) for _ in range(3)]
        pa_capi.attn_bwd(tq, tk, tv, o, tg, lse, *want, ws)
        assert pa_capi.device_status() == 0
    finally:
        pa_capi.set_f32_math("split3")
    assert torch.equal(got[1], want[1]) and torch.equal(got[2], want[2])
    assert rel_err(got[0].cpu().numpy(), want[0].cpu().numpy()) < 1e-6
