"""Failure detection of the kernels' bounded waits, and first calls from
several host threads at once.

Every mbarrier wait in the attention and GEMM kernels gives up after a time
limit, records PA_ERR_TIMEOUT in a per-device status word and lets its role
leave its loop, so a lost arrival cannot hang the GPU. pa_wait_selftest runs
that same bounded wait in a one-thread kernel whose barrier nothing completes
(a flag that nothing sets), with a short limit: the wait runs out, the status
word reports it, the kernels launched while it is set skip their work, and
after pa_device_status clears it the next call computes normally. No GPU
fault, trap or hang is involved: the kernel returns on its own.

The C ABI may be called from one host thread per GPU; its per-device caches
(shared-memory attributes, SM counts, status-word and scratch addresses) are
set up on first use. The threaded test drives several threads into their
first calls at the same moment, in a fresh process, and checks every result
against the same calls made afterwards from one thread."""
import os
import subprocess
import sys
import textwrap
import time

import numpy as np
import pytest

from conftest import PKG, REPO, rel_err, seeded_normal

torch = pytest.importorskip("torch")


def test_selftest_rejects_bad_limits_without_a_gpu():
    import pa_capi
    lib = pa_capi.load()
    assert lib.pa_wait_selftest(0, 0, None) == 1              # PA_ERR_SHAPE
    assert lib.pa_wait_selftest(6_000_000_000, 0, None) == 1  # above the 5 s cap


def _small_attention():
    shape = (1, 256, 2, 64)
    q, k, v = (torch.from_numpy(seeded_normal(s, shape, 0.5)).to(torch.bfloat16).cuda()
               for s in (301, 302, 303))
    return q, k, v


@pytest.mark.gpu
def test_wait_that_completes_records_nothing():
    import pa_capi
    assert pa_capi.device_status() == 0
    pa_capi.wait_selftest(1_000_000_000, arrive=True)
    assert pa_capi.device_status() == 0


@pytest.mark.gpu
def test_wait_that_runs_out_reports_timeout_and_the_next_call_succeeds():
    import oracle
    import pa_capi
    assert pa_capi.device_status() == 0
    limit_ns = 200_000_000  # 0.2 s
    t0 = time.perf_counter()
    pa_capi.wait_selftest(limit_ns, arrive=False)
    assert pa_capi.device_status(clear=False) == 6  # PA_ERR_TIMEOUT, left set
    assert time.perf_counter() - t0 >= 0.9 * limit_ns * 1e-9  # the wait ran its limit

    # while the word is set, kernels skip their work (outputs stay untouched)
    q, k, v = _small_attention()
    o = torch.full_like(q, float("nan"))
    lse = torch.full((2, 256), float("nan"), device="cuda")
    pa_capi.attn_fwd(q, k, v, o, lse)
    assert pa_capi.device_status(clear=False) == 6
    assert torch.isnan(o).all() and torch.isnan(lse).all()

    # reading with clear resets it; the context is still usable
    assert pa_capi.device_status(clear=True) == 6
    assert pa_capi.device_status() == 0
    pa_capi.attn_fwd(q, k, v, o, lse)
    assert pa_capi.device_status() == 0
    f = lambda t: t.float().cpu().numpy().astype(np.float64)
    ro, rl = oracle.attn_fwd(f(q), f(k), f(v))
    assert rel_err(f(o), ro) < 2e-2
    assert np.max(np.abs(lse.cpu().numpy() - rl)) < 2e-3


_THREADED = textwrap.dedent(r"""
    import sys, threading
    sys.path.insert(0, {pkg!r})
    import numpy as np
    import torch
    import pa_capi

    n_dev = torch.cuda.device_count()
    n_thr = max(2, min(n_dev, 4))
    devs = [i % n_dev for i in range(n_thr)]

    def inputs(t):
        torch.cuda.set_device(devs[t])
        g = torch.Generator(device="cpu").manual_seed(100 + t)
        L = 256 + 128 * t  # a different shape per thread
        qkvg = [(torch.randn(1, L, 2, 64, generator=g) * 0.5).to(torch.bfloat16).cuda()
                for _ in range(4)]
        x = torch.randn(512, 256, generator=g).cuda()
        w = (torch.randn(256, 384, generator=g) * 0.05).cuda()
        return qkvg, x, w

    def run(t, data):
        torch.cuda.set_device(devs[t])
        s = torch.cuda.Stream()
        with torch.cuda.stream(s):
            (q, k, v, g), x, w = data
            o = torch.empty_like(q)
            lse = torch.empty(2, q.shape[1], device="cuda")
            d = pa_capi.attn_desc(q)
            ws = torch.empty(pa_capi.attn_bwd_workspace_size(d), dtype=torch.uint8, device="cuda")
            dq, dk, dv = (torch.empty_like(q) for _ in range(3))
            y = torch.empty(512, 384, device="cuda")
            gamma = torch.ones(256, device="cuda")
            beta = torch.zeros(256, device="cuda")
            ln = torch.empty_like(x)
            mu = torch.empty(512, device="cuda")
            rs = torch.empty(512, device="cuda")
            barrier.wait()  # every thread makes its first calls at the same moment
            pa_capi.attn_fwd(q, k, v, o, lse, d)
            pa_capi.attn_bwd(q, k, v, o, g, lse, dq, dk, dv, ws, desc=d)
            pa_capi.matmul(x, w, y, 512, 384, 256)
            pa_capi.layer_norm_fwd(x, gamma, beta, ln, mu, rs)
            assert pa_capi.device_status() == 0
        return [t_.float().cpu() for t_ in (o, lse, dk, dv, y, ln)]

    data = [inputs(t) for t in range(n_thr)]
    barrier = threading.Barrier(n_thr)
    results = [None] * n_thr
    errors = []

    def body(t):
        try:
            results[t] = run(t, data[t])
        except Exception as e:  # reported below
            errors.append(repr(e))

    threads = [threading.Thread(target=body, args=(t,)) for t in range(n_thr)]
    for th in threads: th.start()
    for th in threads: th.join()
    assert not errors, errors
    barrier = threading.Barrier(1)
    for t in range(n_thr):  # the same calls again, one thread: identical results
        again = run(t, data[t])
        for a, b in zip(results[t], again):
            assert torch.equal(a, b), t
    print("threads", n_thr, "devices", sorted(set(devs)))
""")


@pytest.mark.gpu
def test_first_calls_from_several_host_threads_at_once():
    code = _THREADED.format(pkg=PKG)
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=600,
                       cwd=REPO, env=dict(os.environ))
    assert r.returncode == 0, r.stdout + r.stderr
    assert "threads" in r.stdout
