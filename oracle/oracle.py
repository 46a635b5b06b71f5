"""ctypes front end of the test oracle (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and the CPU-baseline leg of bench.py use
this module, as the checker or the timed CPU baseline. Product code never
imports it.

  float64 restatement     liboracle.so   (pa_oracle.c)
  fp32 multithreaded CPU  libcpuattn.so  (cpu_attention.cpp)
  reference kernels       _ref/libpa_ref.so (the reference's own CUDA code,
                          built from its sources by `make -C oracle ref`)
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
_dp = ctypes.POINTER(ctypes.c_double)
_fp = ctypes.POINTER(ctypes.c_float)
_i = ctypes.c_int


def _load(name):
    path = os.path.join(HERE, name)
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} not built (run `make -C oracle`)")
    return ctypes.CDLL(path)


_lib = None
_cpu = None
_ref = None


def lib():
    global _lib
    if _lib is None:
        _lib = _load("liboracle.so")
        for n in ("oracle_attn_fwd",):
            getattr(_lib, n).argtypes = [_dp] * 5 + [_i] * 4 + [ctypes.c_double]
        _lib.oracle_attn_bwd.argtypes = [_dp] * 10 + [_i] * 4 + [ctypes.c_double]
        _lib.oracle_attn_delta.argtypes = [_dp] * 3 + [_i] * 4
        _ip = ctypes.POINTER(ctypes.c_int)
        _lib.oracle_attn_sampled.argtypes = ([_dp] * 4 + [_i, _i, ctypes.c_double, _ip, _i, _ip, _i]
                                             + [_dp] * 5)
        _lib.oracle_layer_norm_fwd.argtypes = [_dp] * 6 + [_i] * 2 + [ctypes.c_double]
        _lib.oracle_layer_norm_bwd.argtypes = [_dp] * 8 + [_i] * 2
        for n in ("oracle_matmul", "oracle_matmul_grad_x", "oracle_matmul_grad_w"):
            getattr(_lib, n).argtypes = [_dp] * 3 + [_i] * 3
        _lib.oracle_bias_add.argtypes = [_dp] * 3 + [_i] * 2
        _lib.oracle_bias_grad.argtypes = [_dp] * 2 + [_i] * 2
        _lib.oracle_split_last_dim.argtypes = [_dp] * 2 + [_i] * 3
        _lib.oracle_concat_last_dim_grad.argtypes = [_dp] * 2 + [_i] * 3
        _lib.oracle_num_threads.restype = _i
    return _lib


def _d(a):
    """Contiguous float64 copy and its pointer."""
    a = np.ascontiguousarray(a, dtype=np.float64)
    return a, a.ctypes.data_as(_dp)


def _null():
    return ctypes.cast(None, _dp)


# ------------------------------------------------------------------ attention
def attn_fwd(q, k, v, scale=None):
    """q, k, v: [B, L, H, D]. Returns (o [B, L, H, D], lse [B*H, L]) in float64."""
    B, L, H, D = q.shape
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    q, qp = _d(q)
    k, kp = _d(k)
    v, vp = _d(v)
    o = np.zeros((B, L, H, D))
    lse = np.zeros((B * H, L))
    lib().oracle_attn_fwd(qp, kp, vp, o.ctypes.data_as(_dp), lse.ctypes.data_as(_dp), B, L, H, D,
                          float(scale))
    return o, lse


def attn_bwd(q, k, v, o, dO, lse, scale=None):
    """Returns (dq, dk, dv, delta[B, L, H]) in float64."""
    B, L, H, D = q.shape
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    arrs = [_d(x) for x in (q, k, v, o, dO, lse)]
    dq, dk, dv = (np.zeros((B, L, H, D)) for _ in range(3))
    delta = np.zeros((B, L, H))
    lib().oracle_attn_bwd(*[p for _, p in arrs], dq.ctypes.data_as(_dp), dk.ctypes.data_as(_dp),
                          dv.ctypes.data_as(_dp), delta.ctypes.data_as(_dp), B, L, H, D,
                          float(scale))
    return dq, dk, dv, delta


def attn_sampled(q, k, v, dO, qrows, krows, scale=None):
    """One (batch, head) slice, q/k/v/dO as [L, D]: LSE of every query row,
    and O, dQ of the query rows `qrows`, dK, dV of the key rows `krows`, in
    float64. Returns (lse[L], o[nq, D], dq[nq, D], dk[nk, D], dv[nk, D])."""
    L, D = q.shape
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    arrs = [_d(x) for x in (q, k, v, dO)]
    qr = np.ascontiguousarray(qrows, dtype=np.int32)
    kr = np.ascontiguousarray(krows, dtype=np.int32)
    if qr.size and (qr.min() < 0 or qr.max() >= L) or kr.size and (kr.min() < 0 or kr.max() >= L):
        raise ValueError("sampled row out of range")
    ip = ctypes.POINTER(ctypes.c_int)
    lse = np.zeros(L)
    o, dq = np.zeros((qr.size, D)), np.zeros((qr.size, D))
    dk, dv = np.zeros((kr.size, D)), np.zeros((kr.size, D))
    lib().oracle_attn_sampled(*[p for _, p in arrs], L, D, float(scale), qr.ctypes.data_as(ip),
                              int(qr.size), kr.ctypes.data_as(ip), int(kr.size),
                              *[a.ctypes.data_as(_dp) for a in (lse, o, dq, dk, dv)])
    return lse, o, dq, dk, dv


# ------------------------------------------------------------------ layer norm
def layer_norm_fwd(x, gamma, beta, eps=1e-5):
    M, N = x.shape
    x, xp = _d(x)
    g, gp = _d(gamma)
    b, bp = _d(beta)
    y = np.zeros((M, N))
    mean = np.zeros(M)
    rstd = np.zeros(M)
    lib().oracle_layer_norm_fwd(xp, gp, bp, y.ctypes.data_as(_dp), mean.ctypes.data_as(_dp),
                                rstd.ctypes.data_as(_dp), M, N, float(eps))
    return y, mean, rstd


def layer_norm_bwd(dy, x, mean, rstd, gamma):
    """Returns (dx, dgamma, dbeta); dgamma/dbeta start from zero."""
    M, N = x.shape
    arrs = [_d(a) for a in (dy, x, mean, rstd, gamma)]
    dx = np.zeros((M, N))
    dg = np.zeros(N)
    db = np.zeros(N)
    lib().oracle_layer_norm_bwd(*[p for _, p in arrs], dx.ctypes.data_as(_dp),
                                dg.ctypes.data_as(_dp), db.ctypes.data_as(_dp), M, N)
    return dx, dg, db


# ------------------------------------------------------------------ matmul
def matmul(a, b):
    M, K = a.shape
    N = b.shape[1]
    a, ap = _d(a)
    b, bp = _d(b)
    c = np.zeros((M, N))
    lib().oracle_matmul(ap, bp, c.ctypes.data_as(_dp), M, N, K)
    return c


def matmul_grad_x(dy, w, dx0=None):
    """dX[M,N] = dX0 + dY[M,K] W[N,K]^T."""
    M, K = dy.shape
    N = w.shape[0]
    dy, dyp = _d(dy)
    w, wp = _d(w)
    dx = np.zeros((M, N)) if dx0 is None else np.array(dx0, dtype=np.float64, copy=True)
    lib().oracle_matmul_grad_x(dyp, wp, dx.ctypes.data_as(_dp), M, N, K)
    return dx


def matmul_grad_w(x, dy, dw0=None):
    """dW[N,K] = dW0 + X[M,N]^T dY[M,K]."""
    M, N = x.shape
    K = dy.shape[1]
    x, xp = _d(x)
    dy, dyp = _d(dy)
    dw = np.zeros((N, K)) if dw0 is None else np.array(dw0, dtype=np.float64, copy=True)
    lib().oracle_matmul_grad_w(xp, dyp, dw.ctypes.data_as(_dp), M, N, K)
    return dw


def bias_add(a, bias):
    M, N = a.shape
    a, ap = _d(a)
    b, bp = _d(bias)
    out = np.zeros((M, N))
    lib().oracle_bias_add(ap, bp, out.ctypes.data_as(_dp), M, N)
    return out


def bias_grad(dy, db0=None):
    M, N = dy.shape
    dy, dyp = _d(dy)
    db = np.zeros(N) if db0 is None else np.array(db0, dtype=np.float64, copy=True)
    lib().oracle_bias_grad(dyp, db.ctypes.data_as(_dp), M, N)
    return db


def split_last_dim(x, parts):
    rows, n = x.shape
    w = n // parts
    x, xp = _d(x)
    out = np.zeros((parts, rows, w))
    lib().oracle_split_last_dim(xp, out.ctypes.data_as(_dp), rows, parts, w)
    return out


def concat_last_dim_grad(parts_grad, grad_in0=None):
    parts, rows, w = parts_grad.shape
    pg, pgp = _d(parts_grad)
    gi = (np.zeros((rows, parts * w)) if grad_in0 is None
          else np.array(grad_in0, dtype=np.float64, copy=True))
    lib().oracle_concat_last_dim_grad(pgp, gi.ctypes.data_as(_dp), rows, parts, w)
    return gi


# ------------------------------------------------------------------ CPU baseline
_AVX512 = ("avx512f", "avx512bw", "avx512dq", "avx512vl")


def cpu_isa():
    """'avx512' when every host core reports AVX-512 F/BW/DQ/VL (and that
    build exists), else 'avx2'."""
    try:
        with open("/proc/cpuinfo") as f:
            flags = [ln.split(":", 1)[1].split() for ln in f if ln.startswith("flags")]
    except OSError:
        flags = []
    ok = flags and all(all(x in fl for x in _AVX512) for fl in flags)
    return "avx512" if ok and os.path.exists(os.path.join(HERE, "libcpuattn_avx512.so")) else "avx2"


def cpu():
    global _cpu
    if _cpu is None:
        _cpu = _load("libcpuattn_avx512.so" if cpu_isa() == "avx512" else "libcpuattn.so")
        _cpu.cpu_attn_fwd_bwd.argtypes = [_fp] * 9 + [_i] * 4 + [ctypes.c_float] + [_i] * 3
        _cpu.cpu_attn_fwd_bwd.restype = _i
        _cpu.cpu_hardware_threads.restype = _i
    return _cpu


def cpu_attn_fwd_bwd(q, k, v, dO, scale=None, nthreads=0, units=None, outs=None):
    """fp32 CPU forward+backward over (batch, head) units [u0, u1).

    Returns (o, lse, dq, dk, dv, threads_used); only the selected units' rows
    are written."""
    B, L, H, D = q.shape
    scale = 1.0 / np.sqrt(D) if scale is None else scale
    f = [np.ascontiguousarray(x, dtype=np.float32) for x in (q, k, v, dO)]
    if outs is None:
        outs = (np.zeros((B, L, H, D), np.float32), np.zeros((B * H, L), np.float32),
                np.zeros((B, L, H, D), np.float32), np.zeros((B, L, H, D), np.float32),
                np.zeros((B, L, H, D), np.float32))
    u0, u1 = (0, B * H) if units is None else units
    ptr = lambda a: a.ctypes.data_as(_fp)
    nt = cpu().cpu_attn_fwd_bwd(*[ptr(a) for a in f], *[ptr(a) for a in outs], B, L, H, D,
                                float(scale), int(nthreads), int(u0), int(u1))
    return (*outs, nt)


# ------------------------------------------------------------------ reference kernels
def ref_available():
    return os.path.exists(os.path.join(HERE, "_ref", "libpa_ref.so"))


def ref():
    global _ref
    if _ref is None:
        _ref = _load(os.path.join("_ref", "libpa_ref.so"))
        _ref.ref_flash_fwd.argtypes = [_fp] * 5 + [_i] * 4
        _ref.ref_flash_bwd.argtypes = [_fp] * 9 + [_i] * 4
        _ref.ref_flash_bwd_relaunch_d64.argtypes = [_fp] * 8 + [_i] * 3
        _ref.ref_layer_norm_fwd.argtypes = [_fp] * 6 + [_i] * 2 + [ctypes.c_float]
        _ref.ref_layer_norm_bwd.argtypes = [_fp] * 8 + [_i] * 2
        for n in ("ref_matmul", "ref_matmul_grad_x", "ref_matmul_grad_w"):
            getattr(_ref, n).argtypes = [_fp] * 3 + [_i] * 3
        if hasattr(_ref, "ref_time_flash"):
            _ref.ref_time_flash.argtypes = [_fp] * 4 + [_i] * 5 + [_fp] * 2
    return _ref


def _f(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(_fp)


def _chk(rc, what):
    if rc != 0:
        raise RuntimeError(f"reference {what} failed with code {rc}")


def ref_flash_fwd(q, k, v):
    B, L, H, D = q.shape
    (q, qp), (k, kp), (v, vp) = _f(q), _f(k), _f(v)
    o = np.zeros((B, L, H, D), np.float32)
    lse = np.zeros((B * H, L), np.float32)
    _chk(ref().ref_flash_fwd(qp, kp, vp, o.ctypes.data_as(_fp), lse.ctypes.data_as(_fp), B, L, H,
                             D), "flash forward")
    return o, lse


def ref_flash_bwd(q, k, v, o, dO, lse):
    """Shipped backward (D = 32 only). Returns (dq_stub, dk, dv)."""
    B, L, H, D = q.shape
    arrs = [_f(a) for a in (q, k, v, o, dO, lse)]
    dq, dk, dv = (np.zeros((B, L, H, D), np.float32) for _ in range(3))
    _chk(ref().ref_flash_bwd(*[p for _, p in arrs], dq.ctypes.data_as(_fp), dk.ctypes.data_as(_fp),
                             dv.ctypes.data_as(_fp), B, L, H, D), "flash backward")
    return dq, dk, dv


def ref_flash_bwd_relaunch_d64(q, k, v, o, dO, lse):
    B, L, H, D = q.shape
    arrs = [_f(a) for a in (q, k, v, o, dO, lse)]
    dk, dv = (np.zeros((B, L, H, D), np.float32) for _ in range(2))
    _chk(ref().ref_flash_bwd_relaunch_d64(*[p for _, p in arrs], dk.ctypes.data_as(_fp),
                                          dv.ctypes.data_as(_fp), B, L, H), "flash backward d64")
    return dk, dv


def ref_layer_norm_fwd(x, gamma, beta, eps=1e-5):
    M, N = x.shape
    (x, xp), (g, gp), (b, bp) = _f(x), _f(gamma), _f(beta)
    y = np.zeros((M, N), np.float32)
    mean = np.zeros(M, np.float32)
    rstd = np.zeros(M, np.float32)
    _chk(ref().ref_layer_norm_fwd(xp, gp, bp, y.ctypes.data_as(_fp), mean.ctypes.data_as(_fp),
                                  rstd.ctypes.data_as(_fp), M, N, float(eps)), "layer norm fwd")
    return y, mean, rstd


def ref_layer_norm_bwd(dy, x, mean, rstd, gamma):
    M, N = x.shape
    arrs = [_f(a) for a in (dy, x, mean, rstd, gamma)]
    dx = np.zeros((M, N), np.float32)
    dg = np.zeros(N, np.float32)
    db = np.zeros(N, np.float32)
    _chk(ref().ref_layer_norm_bwd(*[p for _, p in arrs], dx.ctypes.data_as(_fp),
                                  dg.ctypes.data_as(_fp), db.ctypes.data_as(_fp), M, N),
         "layer norm bwd")
    return dx, dg, db


def ref_matmul(a, b):
    M, K = a.shape
    N = b.shape[1]
    (a, ap), (b, bp) = _f(a), _f(b)
    c = np.zeros((M, N), np.float32)
    _chk(ref().ref_matmul(ap, bp, c.ctypes.data_as(_fp), M, N, K), "matmul")
    return c


def ref_matmul_grad_x(dy, w, dx0):
    M, K = dy.shape
    N = w.shape[0]
    (dy, dyp), (w, wp) = _f(dy), _f(w)
    dx = np.array(dx0, dtype=np.float32, copy=True)
    _chk(ref().ref_matmul_grad_x(dyp, wp, dx.ctypes.data_as(_fp), M, N, K), "matmul grad X")
    return dx


def ref_matmul_grad_w(x, dy, dw0):
    M, N = x.shape
    K = dy.shape[1]
    (x, xp), (dy, dyp) = _f(x), _f(dy)
    dw = np.array(dw0, dtype=np.float32, copy=True)
    _chk(ref().ref_matmul_grad_w(xp, dyp, dw.ctypes.data_as(_fp), M, N, K), "matmul grad W")
    return dw


def ref_time_flash(q, k, v, dO, reps):
    """Milliseconds per call of the reference's flash forward and backward on
    the GPU (inputs [B, L, H, D] fp32; D = 32 shipped backward, D = 64 the
    in-bounds relaunch). Returns (fwd_ms, bwd_ms)."""
    B, L, H, D = q.shape
    arrs = [_f(a) for a in (q, k, v, dO)]
    fwd = ctypes.c_float(0.0)
    bwd = ctypes.c_float(0.0)
    _chk(ref().ref_time_flash(*[p for _, p in arrs], B, L, H, D, int(reps),
                              ctypes.byref(fwd), ctypes.byref(bwd)), "flash timing")
    return float(fwd.value), float(bwd.value)
