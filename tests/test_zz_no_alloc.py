"""pa_attn_bwd_noalloc: the backward for callers that cannot allocate device
memory (frameworks that own all GPU memory and hand a plugin only its op's
tensors, or runtimes that forbid allocations once a model is loaded). It uses
scratch built into the library instead of a caller workspace.

Checked through the C ABI against pa_attn_bwd with a caller workspace, on two
calls in a row with different inputs (the built-in scratch keeps the first
call's contents, which must not leak into the second). Both entry points run
the same kernels on the same inputs, so:
  - dK and dV, accumulated in a fixed order, must match bit for bit;
  - dQ is summed into an fp32 accumulator by several CTAs in no fixed order,
    so it may differ by that reduction order only: for bf16 outputs at most
    one bf16 unit in the last place (plus 1e-5 of the largest |dQ| where
    cancellation leaves a tiny value), for fp32 outputs 1e-5 of the largest
    |dQ|.
A stale-scratch leak would show as a difference far above these bounds.
This file is collected last so that a failure here stops a run only after all
other tests have run; it also passes alone in a fresh process."""
import ctypes

import numpy as np
import pytest

from conftest import seeded_normal

torch = pytest.importorskip("torch")

BF16_ULP = 2.0 ** -7   # spacing of bf16 values relative to their magnitude (upper bound)
ABS_SLACK = 1e-5       # of max |dQ|, for values left tiny by cancellation


def test_noalloc_rejects_shapes_beyond_its_scratch():
    import pa_capi
    lib = pa_capi.load()
    d = pa_capi.AttnDesc(8, 4096, 16, 64, pa_capi.PA_BF16, 0.0)  # needs ~155 MB of scratch
    assert lib.pa_attn_bwd_workspace_size(ctypes.byref(d)) > pa_capi.NOALLOC_MAX_WORKSPACE
    assert lib.pa_attn_bwd_noalloc(ctypes.byref(d), *([16] * 9), 0, None) == 7  # PA_ERR_WORKSPACE
    assert lib.pa_attn_bwd_noalloc(None, *([16] * 9), 0, None) == 8            # PA_ERR_NULL
    # the fp32 path keeps operand planes in the scratch too: its limit is lower
    f = pa_capi.AttnDesc(1, 4096, 16, 64, pa_capi.PA_F32, 0.0)
    assert lib.pa_attn_bwd_workspace_size(ctypes.byref(f)) > pa_capi.NOALLOC_MAX_WORKSPACE
    assert lib.pa_attn_bwd_noalloc(ctypes.byref(f), *([16] * 9), 0, None) == 7


def _inputs(shape, seed, dtype):
    ts = []
    for s in range(4):
        t = torch.from_numpy(seeded_normal(seed + s, shape, 0.5))
        ts.append((t.to(torch.bfloat16) if dtype == "bf16" else t).cuda())
    return ts


def _compare(got, ref, dtype, call):
    for name, a, r in zip(("dq", "dk", "dv"), got, ref):
        a = a.float().cpu().numpy().astype(np.float64)
        r = r.float().cpu().numpy().astype(np.float64)
        assert np.all(np.isfinite(a)), (call, name)
        if name != "dq":
            np.testing.assert_array_equal(a, r, err_msg=f"call {call}: {name} not bit-identical")
            continue
        diff = np.abs(a - r)
        big = np.abs(r).max()
        if dtype == "bf16":
            bound = BF16_ULP * np.maximum(np.abs(a), np.abs(r)) + ABS_SLACK * big
        else:
            bound = np.full_like(diff, ABS_SLACK * big)
        worst = float((diff - bound).max())
        assert worst <= 0.0, (call, name, float(diff.max()), big)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,B,L,H,D", [
    ("bf16", 1, 512, 4, 64),   # the head-dim-64 kernel: extension tiles in the scratch
    ("bf16", 1, 300, 2, 128),  # head dim 128, ragged tiles
    ("f32", 1, 256, 2, 64),    # fp32: eight operand planes in the scratch
    ("f32", 1, 128, 1, 32),    # fp32 at head dim 32 (planes padded to 64)
])
def test_noalloc_backward_matches_workspace_backward_twice(dtype, B, L, H, D):
    import pa_capi
    shape = (B, L, H, D)
    for call, seed in enumerate((91, 191)):  # different inputs on each call
        q, k, v, g = _inputs(shape, seed + D, dtype)
        o = torch.empty_like(q)
        lse = torch.empty(B * H, L, device="cuda")
        desc = pa_capi.attn_desc(q)
        pa_capi.attn_fwd(q, k, v, o, lse, desc)
        ws = torch.empty(pa_capi.attn_bwd_workspace_size(desc), dtype=torch.uint8, device="cuda")
        ref = [torch.empty_like(q) for _ in range(3)]
        pa_capi.attn_bwd(q, k, v, o, g, lse, *ref, ws, desc=desc)
        got = [torch.full_like(q, float("nan")) for _ in range(3)]
        pa_capi.attn_bwd_noalloc(q, k, v, o, g, lse, *got, desc=desc)
        assert pa_capi.device_status() == 0
        _compare(got, ref, dtype, call)
