"""pa_attn_bwd_noalloc: the backward for callers that cannot allocate device
memory (frameworks that own all GPU memory and hand a plugin only its op's
tensors, or runtimes that forbid allocations once a model is loaded). It uses
scratch built into the library instead of a caller workspace.

Checked through the C ABI against pa_attn_bwd with a caller workspace, on two
calls in a row (the built-in scratch keeps the first call's contents, which
must not leak into the second), within the bf16 tolerance of the other tests.
This file is collected last so that a failure here stops a run only after all
other tests have run; it also passes alone in a fresh process."""
import ctypes

import pytest

from conftest import rel_err, seeded_normal

BF16_TOL = 2e-2

torch = pytest.importorskip("torch")


def test_noalloc_rejects_shapes_beyond_its_scratch():
    import pa_capi
    lib = pa_capi.load()
    d = pa_capi.AttnDesc(8, 4096, 16, 64, pa_capi.PA_BF16, 0.0)  # needs ~170 MB of scratch
    assert lib.pa_attn_bwd_workspace_size(ctypes.byref(d)) > pa_capi.NOALLOC_MAX_WORKSPACE
    assert lib.pa_attn_bwd_noalloc(ctypes.byref(d), *([16] * 9), 0, None) == 7  # PA_ERR_WORKSPACE
    assert lib.pa_attn_bwd_noalloc(None, *([16] * 9), 0, None) == 8            # PA_ERR_NULL


@pytest.mark.gpu
def test_noalloc_backward_matches_workspace_backward_twice():
    import pa_capi
    B, L, H, D = 1, 512, 4, 64
    q, k, v, g = (torch.from_numpy(seeded_normal(s, (B, L, H, D), 0.5)).to(torch.bfloat16).cuda()
                  for s in (91, 92, 93, 94))
    o = torch.empty_like(q)
    lse = torch.empty(B * H, L, device="cuda")
    pa_capi.attn_fwd(q, k, v, o, lse)
    desc = pa_capi.attn_desc(q)
    ws = torch.empty(pa_capi.attn_bwd_workspace_size(desc), dtype=torch.uint8, device="cuda")
    ref = [torch.empty_like(q) for _ in range(3)]
    pa_capi.attn_bwd(q, k, v, o, g, lse, *ref, ws)
    ref = [t.float().cpu().numpy() for t in ref]
    for call in range(2):
        got = [torch.full_like(q, float("nan")) for _ in range(3)]
        pa_capi.attn_bwd_noalloc(q, k, v, o, g, lse, *got)
        assert pa_capi.device_status() == 0
        for name, a, r in zip(("dq", "dk", "dv"), got, ref):
            err = rel_err(a.float().cpu().numpy(), r)
            assert err <= BF16_TOL, (call, name, err)
