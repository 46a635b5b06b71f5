"""ctypes binding of libpa_kernels.so (the C ABI in include/pa_kernels.h).

This is the Python face of the drop-in boundary: the functions take torch CUDA
tensors (or raw device pointers), call the extern "C" entry points on the
current CUDA stream and raise on any non-zero status. There is no fallback: a
missing library or a missing GPU raises immediately.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libpa_kernels.so")

PA_F32, PA_BF16 = 0, 1

STATUS = {
    0: "PA_OK", 1: "PA_ERR_SHAPE", 2: "PA_ERR_DTYPE", 3: "PA_ERR_ALIGN",
    4: "PA_ERR_UNSUPPORTED", 5: "PA_ERR_LAUNCH", 6: "PA_ERR_TIMEOUT",
    7: "PA_ERR_WORKSPACE", 8: "PA_ERR_NULL", 9: "PA_ERR_DEVICE",
}

# Every symbol include/pa_kernels.h declares.
EXPORTS = [
    "pa_abi_version", "pa_status_string", "pa_device_status", "pa_wait_selftest", "pa_set_f32_math",
    "pa_get_f32_math",
    "pa_attn_fwd_workspace_size", "pa_attn_fwd", "pa_attn_bwd_workspace_size", "pa_attn_bwd", "pa_attn_bwd_kept", "pa_attn_bwd_noalloc",
    "pa_attn_delta",
    "pa_layer_norm_fwd", "pa_add_layer_norm_fwd", "pa_layer_norm_fwd_planes", "pa_layer_norm_bwd_workspace_size", "pa_layer_norm_bwd",
    "pa_layer_norm_bwd_accumulate", "pa_add_layer_norm_bwd",
    "pa_matmul_workspace_size", "pa_matmul", "pa_matmul_grad_x", "pa_matmul_grad_w",
    "pa_linear_workspace_size", "pa_linear_fwd", "pa_linear_bwd", "pa_linear_relu_fwd",
    "pa_linear_relu_bwd", "pa_linear_kept_size", "pa_linear_fwd_keep", "pa_linear_fwd_planes", "pa_linear_bwd_kept",
    "pa_bias_add", "pa_add", "pa_grad_accumulate", "pa_bias_grad", "pa_bias_grad_workspace_size", "pa_bias_grad_ws",
    "pa_split_last_dim", "pa_concat_last_dim_grad",
    "pa_relu_fwd", "pa_relu_bwd", "pa_mse_fwd", "pa_mse_fwd_workspace_size", "pa_mse_fwd_ws", "pa_mse_bwd", "pa_adam_step", "pa_adam_step_multi",
    "pa_fill_normal", "pa_fill",
]


class PaError(RuntimeError):
    def __init__(self, fn, status):
        self.status = status
        super().__init__(f"{fn} failed: {STATUS.get(status, status)}")


class AttnDesc(ctypes.Structure):
    _fields_ = [("batch", ctypes.c_int32), ("seq_len", ctypes.c_int32),
                ("num_heads", ctypes.c_int32), ("head_dim", ctypes.c_int32),
                ("dtype", ctypes.c_int32), ("softmax_scale", ctypes.c_float)]


_vp = ctypes.c_void_p
_sz = ctypes.c_size_t
_u32 = ctypes.c_uint32
_int = ctypes.c_int
_flt = ctypes.c_float

_SIGS = {
    "pa_abi_version": (_int, []),
    "pa_set_f32_math": (_int, [_int]),
    "pa_get_f32_math": (_int, []),
    "pa_status_string": (ctypes.c_char_p, [_int]),
    "pa_device_status": (_int, [_vp, _int]),
    "pa_wait_selftest": (_int, [ctypes.c_uint64, _int, _vp]),
    "pa_attn_fwd_workspace_size": (_sz, [ctypes.POINTER(AttnDesc)]),
    "pa_attn_fwd": (_int, [ctypes.POINTER(AttnDesc), _vp, _vp, _vp, _vp, _vp, _vp, _sz, _vp]),
    "pa_attn_bwd_workspace_size": (_sz, [ctypes.POINTER(AttnDesc)]),
    "pa_attn_bwd": (_int, [ctypes.POINTER(AttnDesc)] + [_vp] * 9 + [_int, _vp, _sz, _vp]),
    "pa_attn_bwd_kept": (_int, [ctypes.POINTER(AttnDesc)] + [_vp] * 9 + [_int, _vp, _sz, _int, _vp, _sz, _vp]),
    "pa_attn_bwd_noalloc": (_int, [ctypes.POINTER(AttnDesc)] + [_vp] * 9 + [_int, _vp]),
    "pa_attn_delta": (_int, [ctypes.POINTER(AttnDesc), _vp, _vp, _vp, _vp]),
    "pa_layer_norm_fwd": (_int, [_vp] * 6 + [_u32, _u32, _flt, _vp]),
    "pa_add_layer_norm_fwd": (_int, [_vp] * 8 + [_u32, _u32, _flt, _vp]),
    "pa_layer_norm_fwd_planes": (_int, [_vp] * 8 + [_u32, _u32, _flt, _vp, _sz, _vp]),
    "pa_layer_norm_bwd_workspace_size": (_sz, [_u32, _u32]),
    "pa_layer_norm_bwd": (_int, [_vp] * 8 + [_u32, _u32, _vp, _sz, _vp]),
    "pa_layer_norm_bwd_accumulate": (_int, [_vp] * 8 + [_u32, _u32, _vp, _sz, _vp]),
    "pa_add_layer_norm_bwd": (_int, [_vp] * 10 + [_u32, _u32, _int, _vp, _sz, _vp]),
    "pa_matmul_workspace_size": (_sz, [_int] * 3),
    "pa_matmul": (_int, [_vp] * 3 + [_int] * 3 + [_vp, _sz, _vp]),
    "pa_matmul_grad_x": (_int, [_vp] * 3 + [_int] * 3 + [_vp, _sz, _vp]),
    "pa_matmul_grad_w": (_int, [_vp] * 3 + [_int] * 3 + [_vp, _sz, _vp]),
    "pa_linear_workspace_size": (_sz, [_int] * 3),
    "pa_linear_relu_fwd": (_int, [_vp] * 4 + [_int] * 3 + [_vp, _sz, _vp]),
    "pa_linear_relu_bwd": (_int, [_vp] * 7 + [_int] * 3 + [_vp, _sz, _vp]),
    "pa_linear_kept_size": (_sz, [_int, _int]),
    "pa_linear_fwd_keep": (_int, [_vp, _vp, _vp, ctypes.POINTER(_vp)] + [_int] * 5 + [_vp, _sz, _vp, _sz, _vp]),
    "pa_linear_fwd_planes": (_int, [_vp, _vp, _vp, ctypes.POINTER(_vp)] + [_int] * 5 + [_vp, _sz, _int, _int, _vp, _sz, _vp, _sz, _vp]),
    "pa_linear_bwd_kept": (_int, [_vp, _vp, _vp, _sz, _int, _vp, ctypes.POINTER(_vp), _int, _vp, _vp, _vp]
                           + [_int] * 4 + [_vp, _sz, _vp]),
    "pa_linear_fwd": (_int, [_vp, _vp, _vp, ctypes.POINTER(_vp), _int, _int, _int, _int, _vp, _sz, _vp]),
    "pa_linear_bwd": (_int, [_vp, _vp, ctypes.POINTER(_vp), _int, _vp, _vp, _vp, _int, _int, _int,
                             _vp, _sz, _vp]),
    "pa_bias_add": (_int, [_vp] * 3 + [_int] * 2 + [_vp]),
    "pa_add": (_int, [_vp] * 3 + [_sz, _vp]),
    "pa_grad_accumulate": (_int, [_vp] * 2 + [_sz, _vp]),
    "pa_bias_grad": (_int, [_vp] * 2 + [_int] * 2 + [_vp]),
    "pa_bias_grad_workspace_size": (_sz, [_int, _int]),
    "pa_bias_grad_ws": (_int, [_vp, _vp, _int, _int, _vp, _sz, _vp]),
    "pa_split_last_dim": (_int, [_vp, ctypes.POINTER(_vp), _u32, _u32, _u32, _vp]),
    "pa_concat_last_dim_grad": (_int, [ctypes.POINTER(_vp), _vp, _u32, _u32, _u32, _vp]),
    "pa_relu_fwd": (_int, [_vp, _vp, _sz, _vp]),
    "pa_relu_bwd": (_int, [_vp, _vp, _vp, _sz, _vp]),
    "pa_mse_fwd": (_int, [_vp, _vp, _vp, _sz, _vp]),
    "pa_mse_fwd_workspace_size": (_sz, [_sz]),
    "pa_mse_fwd_ws": (_int, [_vp, _vp, _vp, _sz, _vp, _sz, _vp]),
    "pa_mse_bwd": (_int, [_vp, _vp, _vp, _vp, _sz, _vp]),
    "pa_adam_step": (_int, [_vp, _vp, _vp, _vp, _sz] + [_flt] * 6 + [_vp]),
    "pa_adam_step_multi": (_int, [_vp] * 5 + [_int] + [_flt] * 6 + [_vp]),
    "pa_fill_normal": (_int, [_vp, _sz, _flt, ctypes.c_uint64, _vp]),
    "pa_fill": (_int, [_vp, _sz, _flt, _vp]),
}

_lib = None


def load(path=LIB_PATH):
    """Load the library and bind every declared symbol (no GPU needed)."""
    global _lib
    if _lib is None:
        if not os.path.exists(path):
            raise FileNotFoundError(f"{path} is not built; run pure-attention_b200/build.py")
        lib = ctypes.CDLL(path)
        for name, (res, args) in _SIGS.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def _ptr(t):
    if t is None:
        return None
    if isinstance(t, int):
        return t
    return t.data_ptr()


def _stream():
    import torch
    return torch.cuda.current_stream().cuda_stream


F32_MATH = {"split3": 0, "bf16": 1}


def set_f32_math(mode):
    """Arithmetic of the fp32 entry points for this thread: "split3" (default,
    fp32-level accuracy) or "bf16" (one bf16 product, fp32 accumulation)."""
    _check("pa_set_f32_math", load().pa_set_f32_math(F32_MATH[mode]))


def get_f32_math():
    return {v: k for k, v in F32_MATH.items()}[load().pa_get_f32_math()]


def _check(fn, st):
    if st != 0:
        raise PaError(fn, st)


def _dtype_code(t):
    import torch
    if t.dtype == torch.bfloat16:
        return PA_BF16
    if t.dtype == torch.float32:
        return PA_F32
    raise TypeError(f"unsupported dtype {t.dtype}")


def attn_desc(q, num_heads=None, scale=0.0):
    """Descriptor for q of shape [B, L, H, D] (or [B, L, E] with num_heads)."""
    if q.dim() == 4:
        B, L, H, D = q.shape
    else:
        B, L, E = q.shape
        H = num_heads
        D = E // H
    return AttnDesc(B, L, H, D, _dtype_code(q), float(scale))


def attn_fwd_workspace_size(desc):
    return load().pa_attn_fwd_workspace_size(ctypes.byref(desc))


def attn_fwd(q, k, v, o, lse, desc=None, stream=None, workspace=None):
    """Forward. bf16 needs no workspace; for fp32 one is allocated here with
    torch unless `workspace` is given."""
    d = desc or attn_desc(q)
    if workspace is None:
        need = attn_fwd_workspace_size(d)
        if need:
            import torch
            workspace = torch.empty(need, dtype=torch.uint8, device=q.device)
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    st = load().pa_attn_fwd(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(lse),
                            _ptr(workspace), ws_bytes, _stream() if stream is None else stream)
    _check("pa_attn_fwd", st)


def attn_bwd_workspace_size(desc):
    return load().pa_attn_bwd_workspace_size(ctypes.byref(desc))


def attn_bwd(q, k, v, o, dO, lse, dq, dk, dv, workspace, accumulate=False, desc=None,
             stream=None):
    d = desc or attn_desc(q)
    ws_bytes = workspace.numel() * workspace.element_size()
    st = load().pa_attn_bwd(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dO),
                            _ptr(lse), _ptr(dq), _ptr(dk), _ptr(dv), int(bool(accumulate)),
                            _ptr(workspace), ws_bytes, _stream() if stream is None else stream)
    _check("pa_attn_bwd", st)


def attn_bwd_kept(q, k, v, o, dO, lse, dq, dk, dv, fwd_workspace, fwd_mode, workspace,
                  accumulate=False, desc=None, stream=None):
    """attn_bwd reusing the q, k, v planes an fp32 attn_fwd left in its workspace
    (made under f32 math mode fwd_mode, 'split3' or 'bf16')."""
    d = desc or attn_desc(q)
    st = load().pa_attn_bwd_kept(
        ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(o), _ptr(dO), _ptr(lse), _ptr(dq),
        _ptr(dk), _ptr(dv), int(bool(accumulate)), _ptr(fwd_workspace),
        fwd_workspace.numel() * fwd_workspace.element_size(), F32_MATH[fwd_mode], _ptr(workspace),
        workspace.numel() * workspace.element_size(), _stream() if stream is None else stream)
    _check("pa_attn_bwd_kept", st)


# Scratch limit of pa_attn_bwd_noalloc (PA_ATTN_BWD_NOALLOC_MAX_WORKSPACE).
NOALLOC_MAX_WORKSPACE = 32 << 20


def attn_bwd_noalloc(q, k, v, o, dO, lse, dq, dk, dv, accumulate=False, desc=None, stream=None):
    """Backward using the library's built-in scratch instead of a caller
    workspace (for callers that cannot allocate device memory)."""
    d = desc or attn_desc(q)
    st = load().pa_attn_bwd_noalloc(ctypes.byref(d), _ptr(q), _ptr(k), _ptr(v), _ptr(o),
                                    _ptr(dO), _ptr(lse), _ptr(dq), _ptr(dk), _ptr(dv),
                                    int(bool(accumulate)), _stream() if stream is None else stream)
    _check("pa_attn_bwd_noalloc", st)


def attn_delta(dO, o, delta, desc=None, stream=None):
    d = desc or attn_desc(o)
    st = load().pa_attn_delta(ctypes.byref(d), _ptr(dO), _ptr(o), _ptr(delta),
                              _stream() if stream is None else stream)
    _check("pa_attn_delta", st)


def device_status(clear=True, stream=None):
    """Synchronise and return the device status word (0 = no kernel timed out)."""
    return load().pa_device_status(_stream() if stream is None else stream, int(clear))


def wait_selftest(limit_ns, arrive, stream=None):
    """Enqueue the failure-detection self-test: one bounded mbarrier wait of
    limit_ns that completes (arrive=True) or runs out (arrive=False)."""
    _check("pa_wait_selftest", load().pa_wait_selftest(int(limit_ns), int(bool(arrive)),
                                                        _stream() if stream is None else stream))


def layer_norm_fwd(x, gamma, beta, y, mean, rstd, eps=1e-5, stream=None):
    M = x.numel() // x.shape[-1]
    N = x.shape[-1]
    st = load().pa_layer_norm_fwd(_ptr(x), _ptr(gamma), _ptr(beta), _ptr(y), _ptr(mean),
                                  _ptr(rstd), M, N, float(eps),
                                  _stream() if stream is None else stream)
    _check("pa_layer_norm_fwd", st)


def add_layer_norm_fwd(x, r, out_sum, gamma, beta, y, mean, rstd, eps=1e-5, stream=None):
    """out_sum = x + r, y = LayerNorm(out_sum) in one pass."""
    M = x.numel() // x.shape[-1]
    N = x.shape[-1]
    st = load().pa_add_layer_norm_fwd(_ptr(x), _ptr(r), _ptr(out_sum), _ptr(gamma), _ptr(beta),
                                      _ptr(y), _ptr(mean), _ptr(rstd), M, N, float(eps),
                                      _stream() if stream is None else stream)
    _check("pa_add_layer_norm_fwd", st)


def layer_norm_fwd_planes(x, gamma, beta, y, mean, rstd, y_planes, r=None, out_sum=None, eps=1e-5,
                          stream=None):
    """layer_norm_fwd (r None) or add_layer_norm_fwd that also writes y's bf16
    operand planes into y_planes (uint8, >= linear_kept_size(M, N) bytes) under
    the current f32 math mode."""
    M = x.numel() // x.shape[-1]
    N = x.shape[-1]
    st = load().pa_layer_norm_fwd_planes(_ptr(x), _ptr(r) if r is not None else None,
                                         _ptr(out_sum) if out_sum is not None else None, _ptr(gamma),
                                         _ptr(beta), _ptr(y), _ptr(mean), _ptr(rstd), M, N, float(eps),
                                         _ptr(y_planes), y_planes.numel() * y_planes.element_size(),
                                         _stream() if stream is None else stream)
    _check("pa_layer_norm_fwd_planes", st)


def layer_norm_bwd_workspace_size(M, N):
    return load().pa_layer_norm_bwd_workspace_size(M, N)


def layer_norm_bwd(dy, x, mean, rstd, gamma, dx, dgamma, dbeta, workspace, stream=None,
                   accumulate=False):
    """dx is overwritten, or accumulated into with accumulate=True."""
    M = x.numel() // x.shape[-1]
    N = x.shape[-1]
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    name = "pa_layer_norm_bwd_accumulate" if accumulate else "pa_layer_norm_bwd"
    st = getattr(load(), name)(_ptr(dy), _ptr(x), _ptr(mean), _ptr(rstd), _ptr(gamma),
                               _ptr(dx), _ptr(dgamma), _ptr(dbeta), M, N, _ptr(workspace),
                               ws_bytes, _stream() if stream is None else stream)
    _check(name, st)


def add_layer_norm_bwd(dy, dsum, s, mean, rstd, gamma, dx, dr, dgamma, dbeta, workspace,
                       acc_dx=False, acc_dr=False, stream=None):
    """Backward of sum = x + r, y = LayerNorm(sum): with G = LN_bwd(dy) + dsum
    (dsum may be None), dx and dr get G (added to their contents with acc_dx /
    acc_dr); dgamma, dbeta accumulate. Any output may be None."""
    M = s.numel() // s.shape[-1]
    N = s.shape[-1]
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    opt = lambda t: _ptr(t) if t is not None else None
    flags = (1 if acc_dx else 0) | (2 if acc_dr else 0)
    _check("pa_add_layer_norm_bwd", load().pa_add_layer_norm_bwd(
        _ptr(dy), opt(dsum), _ptr(s), _ptr(mean), _ptr(rstd), _ptr(gamma), opt(dx), opt(dr),
        opt(dgamma), opt(dbeta), M, N, flags, opt(workspace), ws_bytes,
        _stream() if stream is None else stream))


def matmul_workspace_size(M, N, K):
    return load().pa_matmul_workspace_size(M, N, K)


def _gemm_ws(M, N, K, workspace, device):
    if workspace is None:
        import torch
        workspace = torch.empty(matmul_workspace_size(M, N, K), dtype=torch.uint8, device=device)
    return workspace, workspace.numel() * workspace.element_size()


def matmul(a, b, c, M, N, K, workspace=None, stream=None):
    """c[M,N] = a[M,K] b[K,N] (fp32)."""
    ws, nb = _gemm_ws(M, N, K, workspace, a.device)
    _check("pa_matmul", load().pa_matmul(_ptr(a), _ptr(b), _ptr(c), M, N, K, _ptr(ws), nb,
                                         _stream() if stream is None else stream))


def matmul_grad_x(dy, w, dx, M, N, K, workspace=None, stream=None):
    """dx[M,N] += dy[M,K] w[N,K]^T."""
    ws, nb = _gemm_ws(M, N, K, workspace, dy.device)
    _check("pa_matmul_grad_x", load().pa_matmul_grad_x(_ptr(dy), _ptr(w), _ptr(dx), M, N, K,
                                                       _ptr(ws), nb,
                                                       _stream() if stream is None else stream))


def matmul_grad_w(x, dy, dw, M, N, K, workspace=None, stream=None):
    """dw[N,K] += x[M,N]^T dy[M,K]."""
    ws, nb = _gemm_ws(M, N, K, workspace, x.device)
    _check("pa_matmul_grad_w", load().pa_matmul_grad_w(_ptr(x), _ptr(dy), _ptr(dw), M, N, K,
                                                       _ptr(ws), nb,
                                                       _stream() if stream is None else stream))


def bias_add(a, bias, out, M, N, stream=None):
    _check("pa_bias_add", load().pa_bias_add(_ptr(a), _ptr(bias), _ptr(out), M, N,
                                             _stream() if stream is None else stream))


def add(a, b, out, n, stream=None):
    _check("pa_add", load().pa_add(_ptr(a), _ptr(b), _ptr(out), n,
                                   _stream() if stream is None else stream))


def grad_accumulate(src, dst, n, stream=None):
    _check("pa_grad_accumulate", load().pa_grad_accumulate(_ptr(src), _ptr(dst), n,
                                                           _stream() if stream is None else stream))


def bias_grad(dy, db, M, N, stream=None, workspace=None):
    """db += column sums of dy; with a workspace (bias_grad_workspace_size bytes) over the whole GPU."""
    st = _stream() if stream is None else stream
    if workspace is None:
        _check("pa_bias_grad", load().pa_bias_grad(_ptr(dy), _ptr(db), M, N, st))
    else:
        _check("pa_bias_grad_ws", load().pa_bias_grad_ws(
            _ptr(dy), _ptr(db), M, N, _ptr(workspace), workspace.numel() * workspace.element_size(), st))


def bias_grad_workspace_size(M, N):
    return load().pa_bias_grad_workspace_size(M, N)


def linear_workspace_size(M, in_features, out_features):
    return load().pa_linear_workspace_size(M, in_features, out_features)


def _linear_ws(M, i, o, workspace, device):
    if workspace is None:
        import torch
        workspace = torch.empty(linear_workspace_size(M, i, o), dtype=torch.uint8, device=device)
    return workspace, workspace.numel() * workspace.element_size()


def linear_fwd(x, w, bias, outs, M, in_features, out_features, workspace=None, stream=None):
    """outs[c] = (x[M,in] w[in,out] + bias)[:, c*out/n : (c+1)*out/n] (bias may be None)."""
    ws, nb = _linear_ws(M, in_features, out_features, workspace, x.device)
    arr = (_vp * len(outs))(*[_ptr(o) for o in outs])
    _check("pa_linear_fwd", load().pa_linear_fwd(_ptr(x), _ptr(w), _ptr(bias) if bias is not None else None,
                                                 arr, len(outs), M, in_features, out_features,
                                                 _ptr(ws), nb, _stream() if stream is None else stream))


def linear_bwd(x, w, dy_parts, dx, dw, dbias, M, in_features, out_features, workspace=None,
               stream=None):
    """dx += dY w^T, dw += x^T dY, dbias += colsum(dY), dY = concat(dy_parts); any output may be None."""
    ws, nb = _linear_ws(M, in_features, out_features, workspace, x.device)
    arr = (_vp * len(dy_parts))(*[_ptr(t) for t in dy_parts])
    opt = lambda t: _ptr(t) if t is not None else None
    _check("pa_linear_bwd", load().pa_linear_bwd(_ptr(x), _ptr(w), arr, len(dy_parts), opt(dx), opt(dw),
                                                 opt(dbias), M, in_features, out_features, _ptr(ws),
                                                 nb, _stream() if stream is None else stream))


def linear_relu_fwd(x, w, bias, y, M, in_features, out_features, workspace=None, stream=None):
    """y = max(0, x w + bias) (bias may be None)."""
    ws, nb = _linear_ws(M, in_features, out_features, workspace, x.device)
    _check("pa_linear_relu_fwd", load().pa_linear_relu_fwd(
        _ptr(x), _ptr(w), _ptr(bias) if bias is not None else None, _ptr(y), M, in_features,
        out_features, _ptr(ws), nb, _stream() if stream is None else stream))


def linear_relu_bwd(x, w, y, dy, dx, dw, dbias, M, in_features, out_features, workspace=None,
                    stream=None):
    """With dZ = dy * (y > 0): dx += dZ w^T, dw += x^T dZ, dbias += colsum(dZ)."""
    ws, nb = _linear_ws(M, in_features, out_features, workspace, x.device)
    opt = lambda t: _ptr(t) if t is not None else None
    _check("pa_linear_relu_bwd", load().pa_linear_relu_bwd(
        _ptr(x), _ptr(w), _ptr(y), _ptr(dy), opt(dx), opt(dw), opt(dbias), M, in_features,
        out_features, _ptr(ws), nb, _stream() if stream is None else stream))


def linear_kept_size(M, in_features):
    return load().pa_linear_kept_size(M, in_features)


def linear_fwd_keep(x, w, bias, outs, M, in_features, out_features, kept, relu=False,
                    workspace=None, stream=None):
    """linear_fwd / linear_relu_fwd that also leaves x's operand planes in `kept`."""
    ws, nb = _linear_ws(M, in_features, out_features, workspace, x.device)
    arr = (_vp * len(outs))(*[_ptr(o) for o in outs])
    _check("pa_linear_fwd_keep", load().pa_linear_fwd_keep(
        _ptr(x), _ptr(w), _ptr(bias) if bias is not None else None, arr, len(outs), int(relu), M,
        in_features, out_features, _ptr(kept), kept.numel() * kept.element_size(), _ptr(ws), nb,
        _stream() if stream is None else stream))


def linear_fwd_planes(x, w, bias, outs, M, in_features, out_features, kept, kept_mode="bf16",
                      kept_valid=False, y_planes=None, relu=False, workspace=None, stream=None):
    """linear_fwd_keep with X's planes already in `kept` (kept_valid, made under
    kept_mode) and, optionally, Y's planes written to y_planes."""
    ws, nb = _linear_ws(M, in_features, out_features, workspace, x.device)
    arr = (_vp * len(outs))(*[_ptr(o) for o in outs])
    yb = 0 if y_planes is None else y_planes.numel() * y_planes.element_size()
    _check("pa_linear_fwd_planes", load().pa_linear_fwd_planes(
        _ptr(x), _ptr(w), _ptr(bias) if bias is not None else None, arr, len(outs), int(relu), M,
        in_features, out_features, _ptr(kept), kept.numel() * kept.element_size(),
        F32_MATH[kept_mode], 1 if kept_valid else 0, _ptr(y_planes), yb, _ptr(ws), nb,
        _stream() if stream is None else stream))


def linear_bwd_kept(x, w, kept, kept_mode, y, dy_parts, dx, dw, dbias, M, in_features, out_features,
                    workspace=None, stream=None, dx_overwrite=False):
    """linear_bwd (y None) / linear_relu_bwd (y = ReLU output) using the kept planes of x;
    dx_overwrite: dx = dY w^T instead of dx += dY w^T."""
    ws, nb = _linear_ws(M, in_features, out_features, workspace, x.device)
    arr = (_vp * len(dy_parts))(*[_ptr(t) for t in dy_parts])
    opt = lambda t: _ptr(t) if t is not None else None
    _check("pa_linear_bwd_kept", load().pa_linear_bwd_kept(
        _ptr(x), _ptr(w), _ptr(kept), kept.numel() * kept.element_size(), F32_MATH[kept_mode],
        opt(y), arr, len(dy_parts), opt(dx), opt(dw), opt(dbias), M, in_features, out_features,
        1 if dx_overwrite else 0, _ptr(ws), nb, _stream() if stream is None else stream))


def split_last_dim(inp, outs, rows, width, stream=None):
    arr = (_vp * len(outs))(*[_ptr(o) for o in outs])
    _check("pa_split_last_dim", load().pa_split_last_dim(_ptr(inp), arr, len(outs), rows, width,
                                                         _stream() if stream is None else stream))


def concat_last_dim_grad(part_grads, grad_in, rows, width, stream=None):
    arr = (_vp * len(part_grads))(*[_ptr(o) for o in part_grads])
    _check("pa_concat_last_dim_grad",
           load().pa_concat_last_dim_grad(arr, _ptr(grad_in), len(part_grads), rows, width,
                                          _stream() if stream is None else stream))
