// Multithreaded fp32 CPU flash-attention forward + backward.
//
// TEST / BASELINE INFRASTRUCTURE ONLY: this is the CPU implementation timed
// beside the CUDA library (the benchmark's cpu_baseline leg and its
// `--impl reference` arm). No product code path links or calls it.
//
// Algorithm: the reference's flash-attention math (forward
// flash_attn_forward_kernel.cu:80-185, backward flash_attn_backward_kernel.cu:
// 124-201 and doc/flash_backward.md section 5), restated for CPU cores:
// one (batch, head) unit per task, 64-row query x 64-key tiles, online
// softmax in the forward, P recomputed from the saved LSE in the backward,
// dK/dV accumulated per key tile and dQ per unit (so no atomics are needed).
// Inner loops run along the contiguous dimension so the compiler vectorises
// them; fp32 accumulation throughout.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

namespace {

constexpr int BR = 64;  // query rows per tile
constexpr int BC = 64;  // keys per tile

struct Problem {
  const float *q, *k, *v, *dO;
  float *o, *lse, *dq, *dk, *dv;
  int B, L, H, D;
  float scale;
};

inline size_t idx(const Problem& p, int b, int l, int h) {
  return ((static_cast<size_t>(b) * p.L + l) * p.H + h) * p.D;
}

// Forward of one (b, h) unit. o/lse are written; rows are independent.
void unit_forward(const Problem& p, int b, int h, std::vector<float>& kt, std::vector<float>& vb,
                  std::vector<float>& s) {
  const int L = p.L, D = p.D;
  std::vector<float> acc(static_cast<size_t>(BR) * D), m(BR), l(BR);
  for (int i0 = 0; i0 < L; i0 += BR) {
    const int br = std::min(BR, L - i0);
    std::fill(acc.begin(), acc.end(), 0.f);
    std::fill(m.begin(), m.end(), -INFINITY);
    std::fill(l.begin(), l.end(), 0.f);
    for (int j0 = 0; j0 < L; j0 += BC) {
      const int bc = std::min(BC, L - j0);
      for (int j = 0; j < bc; ++j) {
        const float* kj = p.k + idx(p, b, j0 + j, h);
        const float* vj = p.v + idx(p, b, j0 + j, h);
        for (int x = 0; x < D; ++x) kt[static_cast<size_t>(x) * BC + j] = kj[x];
        std::memcpy(&vb[static_cast<size_t>(j) * D], vj, sizeof(float) * D);
      }
      for (int i = 0; i < br; ++i) {
        const float* qi = p.q + idx(p, b, i0 + i, h);
        float* si = &s[static_cast<size_t>(i) * BC];
        for (int j = 0; j < bc; ++j) si[j] = 0.f;
        for (int x = 0; x < D; ++x) {
          const float qx = qi[x];
          const float* kx = &kt[static_cast<size_t>(x) * BC];
          for (int j = 0; j < bc; ++j) si[j] += qx * kx[j];
        }
        float mx = m[i];
        for (int j = 0; j < bc; ++j) {
          si[j] *= p.scale;
          mx = std::max(mx, si[j]);
        }
        const float corr = std::exp(m[i] - mx);
        float rs = 0.f;
        for (int j = 0; j < bc; ++j) {
          si[j] = std::exp(si[j] - mx);
          rs += si[j];
        }
        l[i] = l[i] * corr + rs;
        m[i] = mx;
        float* ai = &acc[static_cast<size_t>(i) * D];
        for (int x = 0; x < D; ++x) ai[x] *= corr;
        for (int j = 0; j < bc; ++j) {
          const float pj = si[j];
          const float* vj = &vb[static_cast<size_t>(j) * D];
          for (int x = 0; x < D; ++x) ai[x] += pj * vj[x];
        }
      }
    }
    for (int i = 0; i < br; ++i) {
      float* oi = p.o + idx(p, b, i0 + i, h);
      const float inv = 1.f / l[i];
      for (int x = 0; x < D; ++x) oi[x] = acc[static_cast<size_t>(i) * D + x] * inv;
      p.lse[(static_cast<size_t>(b) * p.H + h) * L + i0 + i] = m[i] + std::log(l[i]);
    }
  }
}

// Backward of one (b, h) unit; needs o and lse from the forward.
void unit_backward(const Problem& p, int b, int h, std::vector<float>& kt, std::vector<float>& vt,
                   std::vector<float>& s, std::vector<float>& dp) {
  const int L = p.L, D = p.D;
  std::vector<float> delta(L), dqacc(static_cast<size_t>(L) * D, 0.f);
  std::vector<float> dkb(static_cast<size_t>(BC) * D), dvb(static_cast<size_t>(BC) * D);
  for (int i = 0; i < L; ++i) {
    const float* oi = p.o + idx(p, b, i, h);
    const float* gi = p.dO + idx(p, b, i, h);
    float a = 0.f;
    for (int x = 0; x < D; ++x) a += oi[x] * gi[x];
    delta[i] = a;
  }
  const float* lse = p.lse + (static_cast<size_t>(b) * p.H + h) * L;
  for (int j0 = 0; j0 < L; j0 += BC) {
    const int bc = std::min(BC, L - j0);
    for (int j = 0; j < bc; ++j) {
      const float* kj = p.k + idx(p, b, j0 + j, h);
      const float* vj = p.v + idx(p, b, j0 + j, h);
      for (int x = 0; x < D; ++x) {
        kt[static_cast<size_t>(x) * BC + j] = kj[x];
        vt[static_cast<size_t>(x) * BC + j] = vj[x];
      }
    }
    std::fill(dkb.begin(), dkb.end(), 0.f);
    std::fill(dvb.begin(), dvb.end(), 0.f);
    for (int i = 0; i < L; ++i) {
      const float* qi = p.q + idx(p, b, i, h);
      const float* gi = p.dO + idx(p, b, i, h);
      float* si = &s[0];
      float* dpi = &dp[0];
      for (int j = 0; j < bc; ++j) si[j] = dpi[j] = 0.f;
      for (int x = 0; x < D; ++x) {
        const float qx = qi[x], gx = gi[x];
        const float* kx = &kt[static_cast<size_t>(x) * BC];
        const float* vx = &vt[static_cast<size_t>(x) * BC];
        for (int j = 0; j < bc; ++j) {
          si[j] += qx * kx[j];
          dpi[j] += gx * vx[j];
        }
      }
      const float li = lse[i], di = delta[i];
      for (int j = 0; j < bc; ++j) {
        const float pj = std::exp(si[j] * p.scale - li);
        si[j] = pj;                                // P
        dpi[j] = pj * (dpi[j] - di) * p.scale;     // dS
      }
      float* dqi = &dqacc[static_cast<size_t>(i) * D];
      for (int j = 0; j < bc; ++j) {
        const float pj = si[j], dsj = dpi[j];
        float* dvj = &dvb[static_cast<size_t>(j) * D];
        float* dkj = &dkb[static_cast<size_t>(j) * D];
        const float* kj = p.k + idx(p, b, j0 + j, h);
        for (int x = 0; x < D; ++x) {
          dvj[x] += pj * gi[x];
          dkj[x] += dsj * qi[x];
          dqi[x] += dsj * kj[x];
        }
      }
    }
    for (int j = 0; j < bc; ++j) {
      std::memcpy(p.dk + idx(p, b, j0 + j, h), &dkb[static_cast<size_t>(j) * D], sizeof(float) * D);
      std::memcpy(p.dv + idx(p, b, j0 + j, h), &dvb[static_cast<size_t>(j) * D], sizeof(float) * D);
    }
  }
  for (int i = 0; i < L; ++i)
    std::memcpy(p.dq + idx(p, b, i, h), &dqacc[static_cast<size_t>(i) * D], sizeof(float) * D);
}

}  // namespace

extern "C" {

// Forward (+ backward when dO != nullptr) over units [unit_begin, unit_end) of
// the B*H (batch, head) units, on `nthreads` threads (<= 0: all hardware threads).
// Returns the number of threads used.
int cpu_attn_fwd_bwd(const float* q, const float* k, const float* v, const float* dO, float* o,
                     float* lse, float* dq, float* dk, float* dv, int B, int L, int H, int D,
                     float scale, int nthreads, int unit_begin, int unit_end) {
  Problem p{q, k, v, dO, o, lse, dq, dk, dv, B, L, H, D, scale};
  if (nthreads <= 0) nthreads = static_cast<int>(std::max(1u, std::thread::hardware_concurrency()));
  unit_begin = std::max(0, unit_begin);
  unit_end = std::min(unit_end, B * H);
  std::atomic<int> next(unit_begin);
  auto worker = [&]() {
    std::vector<float> kt(static_cast<size_t>(D) * BC), vt(static_cast<size_t>(D) * BC),
        vb(static_cast<size_t>(BC) * D), s(static_cast<size_t>(BR) * BC), dp(BC);
    for (int u = next.fetch_add(1); u < unit_end; u = next.fetch_add(1)) {
      const int b = u / H, h = u % H;
      unit_forward(p, b, h, kt, vb, s);
      if (dO) unit_backward(p, b, h, kt, vt, s, dp);
    }
  };
  const int nt = std::min(nthreads, std::max(1, unit_end - unit_begin));
  std::vector<std::thread> pool;
  for (int t = 1; t < nt; ++t) pool.emplace_back(worker);
  worker();
  for (auto& t : pool) t.join();
  return nt;
}

int cpu_hardware_threads(void) {
  return static_cast<int>(std::thread::hardware_concurrency());
}

}  // extern "C"
