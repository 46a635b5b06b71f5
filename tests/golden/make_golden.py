"""Generate golden fixtures from the reference's OWN CUDA kernels.

Runs on a machine with a GPU and oracle/_ref/libpa_ref.so built (the reference
sources compiled by `make -C oracle ref`). Writes
tests/golden/ref_c1_attention.npz and tests/golden/ref_layernorm_matmul.npz
(or into the directory given as argv[1]); the CPU test test_golden.py checks
the float64 oracle against them, which pins the oracle to the reference.

  python tests/golden/make_golden.py [out_dir]
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(REPO, "oracle"))
sys.path.insert(0, os.path.join(REPO, "tests"))

import oracle  # noqa: E402
from conftest import seeded_normal  # noqa: E402


def main(out_dir):
    os.makedirs(out_dir, exist_ok=True)
    # Single-head attention, fp32: B=1, H=1, L=128, d=32, Q/K/V/dO ~ N(0,1), seeds 1..4.
    B, L, H, D = 1, 128, 1, 32
    q, k, v, g = (seeded_normal(s, (B, L, H, D)) for s in (1, 2, 3, 4))
    o, lse = oracle.ref_flash_fwd(q, k, v)
    dq_stub, dk, dv = oracle.ref_flash_bwd(q, k, v, o, g, lse)
    # d = 64 through the relaunch of the reference's own backward kernel
    q6, k6, v6, g6 = (seeded_normal(s, (1, 128, 2, 64)) for s in (5, 6, 7, 8))
    o6, l6 = oracle.ref_flash_fwd(q6, k6, v6)
    dk6, dv6 = oracle.ref_flash_bwd_relaunch_d64(q6, k6, v6, o6, g6, l6)
    np.savez_compressed(os.path.join(out_dir, "ref_c1_attention.npz"),
                        q=q, k=k, v=v, dO=g, o=o, lse=lse, dk=dk, dv=dv,
                        q64=q6, k64=k6, v64=v6, dO64=g6, o64=o6, lse64=l6, dk64=dk6, dv64=dv6)
    # LayerNorm and matmul gradients at a small 2-D size.
    M, N = 64, 128
    x = seeded_normal(50, (M, N))
    gamma = 1.0 + 0.1 * seeded_normal(51, (N,))
    beta = 0.1 * seeded_normal(52, (N,))
    dy = seeded_normal(53, (M, N))
    y, mean, rstd = oracle.ref_layer_norm_fwd(x, gamma, beta)
    dx, dgam, dbet = oracle.ref_layer_norm_bwd(dy, x, mean, rstd, gamma)
    Mm, Nm, Km = 48, 40, 56
    a = seeded_normal(60, (Mm, Km))
    b = seeded_normal(61, (Km, Nm))
    c = oracle.ref_matmul(a, b)
    dym = seeded_normal(62, (Mm, Km))
    w = seeded_normal(63, (Nm, Km))
    dx0 = np.zeros((Mm, Nm), np.float32)
    gx = oracle.ref_matmul_grad_x(dym, w, dx0)
    xm = seeded_normal(65, (Mm, Nm))
    dw0 = np.zeros((Nm, Km), np.float32)
    gw = oracle.ref_matmul_grad_w(xm, dym, dw0)
    np.savez_compressed(os.path.join(out_dir, "ref_layernorm_matmul.npz"),
                        x=x, gamma=gamma, beta=beta, dy=dy, y=y, mean=mean, rstd=rstd, dx=dx,
                        dgamma=dgam, dbeta=dbet, a=a, b=b, c=c, dym=dym, w=w, gx=gx, xm=xm, gw=gw)
    print("wrote golden fixtures to", out_dir)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else HERE)
