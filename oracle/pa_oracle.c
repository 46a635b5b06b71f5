/*
 * Float64 CPU restatement of Pure-Attention's attention-block hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the oracle: tests, the smoke check
 * and the CPU-baseline leg of the benchmark call it to CHECK the CUDA library.
 * No product code path links, loads or calls it.
 *
 * Every function restates the math of one reference kernel (cited by
 * file:line within the Pure-Attention source tree) in double precision, with
 * the defects of the reference left out and named where they matter:
 *   - attention forward: O is divided by l exactly (the reference adds 1e-6 to l);
 *   - attention backward: dQ = dS K is computed (the reference's dQ is a stub);
 *   - layer-norm backward: block sums are exact (the reference's have a race).
 *
 * Layouts follow the reference boundary:
 *   q, k, v, o, dO, dq, dk, dv : [B, L, H, D] (heads interleaved along E = H*D)
 *   lse                        : [B*H, L]
 *   delta                      : [B, L, H]
 *   matrices                   : row-major
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define IDX4(b, l, h, d, L, H, D) ((((size_t)(b) * (L) + (l)) * (H) + (h)) * (D) + (d))

/* Forward, flash_attn_forward_kernel.cu:105-185: S = (q.k) * scale (scale applied
 * after the dot product, :118-124), out-of-range keys masked (:126), row max m,
 * l = sum exp(S - m), O = sum exp(S - m) V / l (:150-178), LSE = m + log(l)
 * (:181-184). The online rescaling of the reference is algebraically the same
 * as this two-pass form. */
void oracle_attn_fwd(const double* q, const double* k, const double* v, double* o, double* lse,
                     int B, int L, int H, int D, double scale) {
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h) {
      double* s = (double*)malloc(sizeof(double) * (size_t)L);
      for (int i = 0; i < L; ++i) {
        const double* qi = q + IDX4(b, i, h, 0, L, H, D);
        double m = -INFINITY;
        for (int j = 0; j < L; ++j) {
          const double* kj = k + IDX4(b, j, h, 0, L, H, D);
          double acc = 0.0;
          for (int x = 0; x < D; ++x) acc += qi[x] * kj[x];
          s[j] = acc * scale;
          if (s[j] > m) m = s[j];
        }
        double l = 0.0;
        for (int j = 0; j < L; ++j) {
          s[j] = exp(s[j] - m);
          l += s[j];
        }
        double* oi = o + IDX4(b, i, h, 0, L, H, D);
        for (int x = 0; x < D; ++x) oi[x] = 0.0;
        for (int j = 0; j < L; ++j) {
          const double* vj = v + IDX4(b, j, h, 0, L, H, D);
          const double p = s[j] / l;
          for (int x = 0; x < D; ++x) oi[x] += p * vj[x];
        }
        lse[((size_t)b * H + h) * L + i] = m + log(l);
      }
      free(s);
    }
}

/* Delta = rowsum(dO * O), flash_attn_backward_kernel.cu:25-41, stored [B, L, H]. */
void oracle_attn_delta(const double* dO, const double* o, double* delta, int B, int L, int H,
                       int D) {
  for (size_t r = 0; r < (size_t)B * L * H; ++r) {
    double acc = 0.0;
    for (int x = 0; x < D; ++x) acc += dO[r * D + x] * o[r * D + x];
    delta[r] = acc;
  }
}

/* Backward, flash_attn_backward_kernel.cu:153-197 and doc/flash_backward.md (section 5):
 *   P  = exp(S*scale - LSE)            (:172, recomputed from the saved LSE)
 *   dP = dO V^T                        (:174-178)
 *   dS = P (dP - Delta) * scale        (:180)
 *   dV = P^T dO, dK = dS^T Q           (:193-197)
 *   dQ = dS K                          (the intended math of :182-191)
 * Outputs are overwritten. delta_out (may be NULL) receives Delta as [B, L, H]. */
void oracle_attn_bwd(const double* q, const double* k, const double* v, const double* o,
                     const double* dO, const double* lse, double* dq, double* dk, double* dv,
                     double* delta_out, int B, int L, int H, int D, double scale) {
  const size_t n = (size_t)B * L * H;
  double* delta = (double*)malloc(sizeof(double) * n);
  oracle_attn_delta(dO, o, delta, B, L, H, D);
  if (delta_out) memcpy(delta_out, delta, sizeof(double) * n);
  memset(dq, 0, sizeof(double) * n * D);
  memset(dk, 0, sizeof(double) * n * D);
  memset(dv, 0, sizeof(double) * n * D);
#pragma omp parallel for collapse(2) schedule(dynamic, 1)
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < H; ++h) {
      double* p = (double*)malloc(sizeof(double) * (size_t)L);
      double* ds = (double*)malloc(sizeof(double) * (size_t)L);
      for (int i = 0; i < L; ++i) {
        const double* qi = q + IDX4(b, i, h, 0, L, H, D);
        const double* doi = dO + IDX4(b, i, h, 0, L, H, D);
        const double lse_i = lse[((size_t)b * H + h) * L + i];
        const double di = delta[((size_t)b * L + i) * H + h];
        for (int j = 0; j < L; ++j) {
          const double* kj = k + IDX4(b, j, h, 0, L, H, D);
          const double* vj = v + IDX4(b, j, h, 0, L, H, D);
          double sacc = 0.0, dpacc = 0.0;
          for (int x = 0; x < D; ++x) {
            sacc += qi[x] * kj[x];
            dpacc += doi[x] * vj[x];
          }
          p[j] = exp(sacc * scale - lse_i);
          ds[j] = p[j] * (dpacc - di) * scale;
        }
        double* dqi = dq + IDX4(b, i, h, 0, L, H, D);
        for (int j = 0; j < L; ++j) {
          const double* kj = k + IDX4(b, j, h, 0, L, H, D);
          double* dkj = dk + IDX4(b, j, h, 0, L, H, D);
          double* dvj = dv + IDX4(b, j, h, 0, L, H, D);
          for (int x = 0; x < D; ++x) {
            dqi[x] += ds[j] * kj[x];
            dkj[x] += ds[j] * qi[x];
            dvj[x] += p[j] * doi[x];
          }
        }
      }
      free(p);
      free(ds);
    }
  free(delta);
}

/* One (batch, head) slice at sequence lengths too long for the full backward
 * above: the same math, evaluated for sampled rows only. Inputs are the
 * slice's rows, q, k, v, dO as [L, D] (row-major, contiguous).
 *   - every query row: the two-pass forward of oracle_attn_fwd
 *     (flash_attn_forward_kernel.cu:105-185), giving lse_all[L], the row's O
 *     and Delta_i = dO_i . O_i (flash_attn_backward_kernel.cu:25-41);
 *   - sampled queries qrows[0..nq): O_i (o_rows) and
 *     dQ_i = sum_j dS_ij K_j with dS_ij = P_ij (dP_ij - Delta_i) * scale,
 *     P_ij = exp(S_ij*scale - LSE_i), dP_ij = dO_i . V_j (doc/flash_backward.md
 *     section 5; flash_attn_backward_kernel.cu:153-197);
 *   - sampled keys krows[0..nk): dV_j = sum_i P_ij dO_i and dK_j = sum_i dS_ij Q_i
 *     (:193-197), which need column j of P and dS over every query.
 * Outputs are [nq, D] / [nk, D] float64, overwritten. */
void oracle_attn_sampled(const double* q, const double* k, const double* v, const double* dO,
                         int L, int D, double scale, const int* qrows, int nq, const int* krows,
                         int nk, double* lse_all, double* o_rows, double* dq_rows, double* dk_rows,
                         double* dv_rows) {
  double* delta = (double*)malloc(sizeof(double) * (size_t)L);
  int* qpos = (int*)malloc(sizeof(int) * (size_t)L); /* query row -> sample index, or -1 */
  for (int i = 0; i < L; ++i) qpos[i] = -1;
  for (int t = 0; t < nq; ++t) qpos[qrows[t]] = t;
#pragma omp parallel
  {
    double* s = (double*)malloc(sizeof(double) * (size_t)L);
    double* oi = (double*)malloc(sizeof(double) * (size_t)D);
#pragma omp for schedule(dynamic, 16)
    for (int i = 0; i < L; ++i) {
      const double* qi = q + (size_t)i * D;
      double m = -INFINITY;
      for (int j = 0; j < L; ++j) {
        const double* kj = k + (size_t)j * D;
        double acc = 0.0;
        for (int x = 0; x < D; ++x) acc += qi[x] * kj[x];
        s[j] = acc * scale;
        if (s[j] > m) m = s[j];
      }
      double l = 0.0;
      for (int j = 0; j < L; ++j) {
        s[j] = exp(s[j] - m);
        l += s[j];
      }
      for (int x = 0; x < D; ++x) oi[x] = 0.0;
      for (int j = 0; j < L; ++j) {
        const double* vj = v + (size_t)j * D;
        const double pj = s[j] / l;
        for (int x = 0; x < D; ++x) oi[x] += pj * vj[x];
      }
      lse_all[i] = m + log(l);
      const double* doi = dO + (size_t)i * D;
      double d = 0.0;
      for (int x = 0; x < D; ++x) d += doi[x] * oi[x];
      delta[i] = d;
      if (qpos[i] >= 0) memcpy(o_rows + (size_t)qpos[i] * D, oi, sizeof(double) * (size_t)D);
    }
    free(s);
    free(oi);
  }
  /* dQ of the sampled queries */
#pragma omp parallel for schedule(dynamic, 1)
  for (int t = 0; t < nq; ++t) {
    const int i = qrows[t];
    const double* qi = q + (size_t)i * D;
    const double* doi = dO + (size_t)i * D;
    double* dqi = dq_rows + (size_t)t * D;
    for (int x = 0; x < D; ++x) dqi[x] = 0.0;
    for (int j = 0; j < L; ++j) {
      const double* kj = k + (size_t)j * D;
      const double* vj = v + (size_t)j * D;
      double sacc = 0.0, dpacc = 0.0;
      for (int x = 0; x < D; ++x) {
        sacc += qi[x] * kj[x];
        dpacc += doi[x] * vj[x];
      }
      const double p = exp(sacc * scale - lse_all[i]);
      const double ds = p * (dpacc - delta[i]) * scale;
      for (int x = 0; x < D; ++x) dqi[x] += ds * kj[x];
    }
  }
  /* dK, dV of the sampled keys */
#pragma omp parallel for schedule(dynamic, 1)
  for (int t = 0; t < nk; ++t) {
    const int j = krows[t];
    const double* kj = k + (size_t)j * D;
    const double* vj = v + (size_t)j * D;
    double* dkj = dk_rows + (size_t)t * D;
    double* dvj = dv_rows + (size_t)t * D;
    for (int x = 0; x < D; ++x) dkj[x] = dvj[x] = 0.0;
    for (int i = 0; i < L; ++i) {
      const double* qi = q + (size_t)i * D;
      const double* doi = dO + (size_t)i * D;
      double sacc = 0.0, dpacc = 0.0;
      for (int x = 0; x < D; ++x) {
        sacc += qi[x] * kj[x];
        dpacc += doi[x] * vj[x];
      }
      const double p = exp(sacc * scale - lse_all[i]);
      const double ds = p * (dpacc - delta[i]) * scale;
      for (int x = 0; x < D; ++x) {
        dvj[x] += p * doi[x];
        dkj[x] += ds * qi[x];
      }
    }
  }
  free(delta);
  free(qpos);
}

/* LayerNorm forward, layer_norm_forward_kernel.cu:40-82: mean, biased variance
 * var = E[x^2] - mean^2 (:63-64), rstd = 1/sqrt(var + eps) (:65),
 * y = gamma * (x - mean) * rstd + beta (:79-82). */
void oracle_layer_norm_fwd(const double* x, const double* gamma, const double* beta, double* y,
                           double* mean, double* rstd, int M, int N, double eps) {
  for (int r = 0; r < M; ++r) {
    const double* xr = x + (size_t)r * N;
    double s = 0.0, s2 = 0.0;
    for (int c = 0; c < N; ++c) {
      s += xr[c];
      s2 += xr[c] * xr[c];
    }
    const double mu = s / N;
    const double var = s2 / N - mu * mu;
    const double rs = 1.0 / sqrt(var + eps);
    mean[r] = mu;
    rstd[r] = rs;
    for (int c = 0; c < N; ++c) y[(size_t)r * N + c] = gamma[c] * (xr[c] - mu) * rs + beta[c];
  }
}

/* LayerNorm backward, layer_norm_backward.cu:17-66 (dgamma += sum dY*xhat,
 * dbeta += sum dY; accumulated) and :97-157 (dX overwritten):
 * dX = rstd/N * (N*dY*gamma - sum(dY*gamma) - xhat*sum(dY*gamma*xhat)).
 * Any of dx, dgamma, dbeta may be NULL (skipped, as in the launcher). */
void oracle_layer_norm_bwd(const double* dy, const double* x, const double* mean,
                           const double* rstd, const double* gamma, double* dx, double* dgamma,
                           double* dbeta, int M, int N) {
  for (int r = 0; r < M; ++r) {
    const double* xr = x + (size_t)r * N;
    const double* dyr = dy + (size_t)r * N;
    const double mu = mean[r], rs = rstd[r];
    double s1 = 0.0, s2 = 0.0;
    for (int c = 0; c < N; ++c) {
      const double xh = (xr[c] - mu) * rs;
      const double t = dyr[c] * gamma[c];
      s1 += t;
      s2 += t * xh;
      if (dgamma) dgamma[c] += dyr[c] * xh;
      if (dbeta) dbeta[c] += dyr[c];
    }
    if (dx)
      for (int c = 0; c < N; ++c) {
        const double xh = (xr[c] - mu) * rs;
        dx[(size_t)r * N + c] = ((double)N * dyr[c] * gamma[c] - s1 - xh * s2) * rs / N;
      }
  }
}

/* C[M,N] = A[M,K] B[K,N], matmul_kernel.cu:4-50. */
void oracle_matmul(const double* A, const double* Bm, double* C, int M, int N, int K) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < M; ++i) {
    double* ci = C + (size_t)i * N;
    for (int j = 0; j < N; ++j) ci[j] = 0.0;
    for (int kk = 0; kk < K; ++kk) {
      const double a = A[(size_t)i * K + kk];
      const double* bk = Bm + (size_t)kk * N;
      for (int j = 0; j < N; ++j) ci[j] += a * bk[j];
    }
  }
}

/* dX[M,N] += dY[M,K] W[N,K]^T, matmul_backward_X_kernel.cu:5-54 (accumulates, :102). */
void oracle_matmul_grad_x(const double* dY, const double* W, double* dX, int M, int N, int K) {
#pragma omp parallel for schedule(static)
  for (int i = 0; i < M; ++i)
    for (int j = 0; j < N; ++j) {
      double acc = 0.0;
      for (int kk = 0; kk < K; ++kk) acc += dY[(size_t)i * K + kk] * W[(size_t)j * K + kk];
      dX[(size_t)i * N + j] += acc;
    }
}

/* dW[N,K] += X[M,N]^T dY[M,K], matmul_backward_W_kernel.cu:5-55 (accumulates, :157). */
void oracle_matmul_grad_w(const double* X, const double* dY, double* dW, int M, int N, int K) {
#pragma omp parallel for schedule(static)
  for (int j = 0; j < N; ++j) {
    double* dwj = dW + (size_t)j * K;
    for (int i = 0; i < M; ++i) {
      const double xij = X[(size_t)i * N + j];
      const double* dyi = dY + (size_t)i * K;
      for (int kk = 0; kk < K; ++kk) dwj[kk] += xij * dyi[kk];
    }
  }
}

/* out[M,N] = A[M,N] + bias[N], matadd_kernel.cu:4-12. */
void oracle_bias_add(const double* A, const double* bias, double* out, int M, int N) {
  for (int i = 0; i < M; ++i)
    for (int j = 0; j < N; ++j) out[(size_t)i * N + j] = A[(size_t)i * N + j] + bias[j];
}

/* db[N] += sum_i dY[i, :], sum_rows_grad_kernel.cu:4-13. */
void oracle_bias_grad(const double* dY, double* db, int M, int N) {
  for (int j = 0; j < N; ++j) {
    double acc = 0.0;
    for (int i = 0; i < M; ++i) acc += dY[(size_t)i * N + j];
    db[j] += acc;
  }
}

/* Last-dimension split of [rows, parts*w] into parts x [rows, w], split_forward_kernel.cu:4-21. */
void oracle_split_last_dim(const double* in, double* out, int rows, int parts, int w) {
  for (int p = 0; p < parts; ++p)
    for (int r = 0; r < rows; ++r)
      for (int c = 0; c < w; ++c)
        out[((size_t)p * rows + r) * w + c] = in[(size_t)r * parts * w + (size_t)p * w + c];
}

/* Adjoint of the split: grad_in[r, p*w + c] += grad_parts[p][r][c], split_backward_kernel.cu:4-22. */
void oracle_concat_last_dim_grad(const double* parts_grad, double* grad_in, int rows, int parts,
                                 int w) {
  for (int p = 0; p < parts; ++p)
    for (int r = 0; r < rows; ++r)
      for (int c = 0; c < w; ++c)
        grad_in[(size_t)r * parts * w + (size_t)p * w + c] +=
            parts_grad[((size_t)p * rows + r) * w + c];
}

/* Number of OpenMP threads the oracle uses (1 without OpenMP). */
int oracle_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
