// Flash-attention forward for sm_100a: bf16 Q/K/V, fp32 accumulation in TMEM.
//
// Computes, per (batch, head) and query row, the reference's forward
// (flash_attn_forward_kernel.cu:80-185): S = Q K^T * scale, online softmax,
// O = softmax(S) V and LSE = rowmax + log(rowsum) (natural log). Unlike the
// reference, O is divided by the row sum exactly (no +1e-6).
//
// Persistent: one CTA per SM walks work items (batch*head, block of two
// 128-row query tiles = 256 rows), item = blockIdx.x + k * gridDim.x; the K/V
// ring, the barrier phases and (where shared memory allows) a double-buffered
// Q carry across items, so the next item's first S MMAs and loads overlap the
// current item's last tiles and its O write-back.
//   warp 0      : TMA producer (Q per item, K/V ring of STAGES stages)
//   warp 1      : TMEM allocator + tcgen05.mma issuer (single elected lane)
//   warps 4-7   : softmax of query tile 0   (thread = one query row)
//   warps 8-11  : softmax of query tile 1
// The two softmax warpgroups ping-pong so the tensor core computes one tile's
// S or P*V while the other tile's softmax runs.
//
// TMEM columns (d = 64): S0 [0,128) S1 [128,256) O0 [256,320) O1 [320,384)
// P0 [384,448) P1 [448,512). P has its own columns, so a softmax warpgroup
// releases S (s_free) as soon as it has loaded it into registers and the next
// tile's S = Q K^T runs while it computes the exponentials.
// (d = 128: O takes 128 columns each, so P (bf16 pairs) is written over the
// first 64 columns of its own S tile; the next S MMA is then issued after the
// P*V MMA that reads P - tcgen05.mma ops of one thread execute in order.)
//
// fp32 path (SPLIT): Q, K, V arrive as bf16 hi/lo planes (fp32_split.cu) and
// every product is taken as hi*hi + hi*lo + lo*hi, three chained MMAs into the
// same TMEM accumulator; P is split the same way and stored as hi (columns
// [0,64)) and lo ([64,128)) over its S tile. Head dims 32 and 64 run as 64
// (zero-padded planes); O is written in fp32 with the true head dim.
//
// The row max is kept in the log2 domain and only raised when a new tile's max
// exceeds it by more than 8 (a factor 256): O and the row sum are rescaled
// then, and otherwise P entries may reach 2^8, which fp32/bf16 hold exactly.
#include <type_traits>
#include "host_launchers.h"

namespace pa {

template <int D, bool SPLIT>
struct FwdCfg {
  static constexpr int NP = SPLIT ? 2 : 1;      // operand planes (hi, lo)
  static constexpr int BM = 128;                 // query rows per tile
  static constexpr int BN = 128;                 // keys per KV tile
  static constexpr int KCH = D / 64;             // 128-byte column chunks per row
  static constexpr int STAGES = (D == 64 && !SPLIT) ? 3 : 2;
  static constexpr int CHUNK = 128 * 128;        // bytes of one 128-row x 128-byte box
  static constexpr int Q_BYTES = BM * D * 2;
  static constexpr int KV_BYTES = BN * D * 2;
  static constexpr int KV_RING = NP * STAGES * 2 * KV_BYTES;
  static constexpr int Q_ITEM = NP * 2 * Q_BYTES;  // both query tiles of an item
  // Q buffers: two where they fit next to the K/V ring (the next item's Q then
  // loads while the current item still runs), else one.
  static constexpr int QBUF = (2 * Q_ITEM + KV_RING + 1024 <= 227 * 1024) ? 2 : 1;
  static constexpr int SMEM = QBUF * Q_ITEM + KV_RING + 1024;
  static constexpr int THREADS = 384;
  static constexpr bool SEP_P = (D == 64 && !SPLIT);  // P in its own TMEM columns
  static constexpr uint32_t T_S = 0, T_O = 256;
  static constexpr uint32_t T_P = SEP_P ? 384 : 0;
};

// OutT: __nv_bfloat16 (bf16 path) or float (SPLIT). d_out: head dim of O.
// n_qb: 256-row query blocks per (batch, head); n_items = n_qb * B * H.
template <int D, bool SPLIT, typename OutT>
__global__ void __launch_bounds__(384, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                    const __grid_constant__ CUtensorMap mapV, const __grid_constant__ CUtensorMap mapQl,
                    const __grid_constant__ CUtensorMap mapKl, const __grid_constant__ CUtensorMap mapVl,
                    OutT* __restrict__ O, float* __restrict__ lse, int L, int H, int d_out,
                    float scale_log2, int n_qb, int n_items, uint32_t* status) {
  using C = FwdCfg<D, SPLIT>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bars[24];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  if (cta_aborted(status, &abort_flag)) return;

  uint8_t* smem = align1024(smem_raw);
  // plane p of query tile t of Q buffer u at sQ + u * Q_ITEM + (t * NP + p) * Q_BYTES;
  // K/V plane p of stage s at sK / sV + (s * NP + p) * KV_BYTES
  uint8_t* sQ = smem;
  uint8_t* sK = smem + C::QBUF * C::Q_ITEM;
  uint8_t* sV = sK + C::NP * C::STAGES * C::KV_BYTES;

  auto q_full = [&](int u) { return smem_u32(&bars[0 + u]); };
  auto q_empty = [&](int u) { return smem_u32(&bars[2 + u]); };
  auto kv_full = [&](int s) { return smem_u32(&bars[4 + s]); };
  auto kv_empty = [&](int s) { return smem_u32(&bars[7 + s]); };
  auto s_full = [&](int t) { return smem_u32(&bars[10 + t]); };
  auto p_full = [&](int t) { return smem_u32(&bars[12 + t]); };
  auto o_done = [&](int t) { return smem_u32(&bars[14 + t]); };
  auto s_free = [&](int t) { return smem_u32(&bars[16 + t]); };
  auto pv_done = [&](int t) { return smem_u32(&bars[18 + t]); };

  const int warp = warp_id();
  const int n_kv = (L + C::BN - 1) / C::BN;
  // Items in launch order: consecutive items share (batch, head), so the CTAs
  // running at one time read the K/V of a few heads, which stay in L2.
  const int item0 = static_cast<int>(blockIdx.x), n_cta = static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int u = 0; u < C::QBUF; ++u) {
      mbar_init(q_full(u), 1);
      mbar_init(q_empty(u), 1);
    }
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(kv_full(s), 1);
      mbar_init(kv_empty(s), 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(s_full(t), 1);
      mbar_init(p_full(t), 128);
      mbar_init(o_done(t), 1);
      mbar_init(s_free(t), 128);
      mbar_init(pv_done(t), 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  // it: items done by this CTA; g: KV tiles done over all its items (ring slot
  // and barrier phase); j: KV tile within the item.
  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {
      tma_prefetch_desc(&mapQ);
      tma_prefetch_desc(&mapK);
      tma_prefetch_desc(&mapV);
      bool ok = true;
      for (int item = item0, it = 0; ok && item < n_items; item += n_cta, ++it) {
        const int bh = item / n_qb;
        const int b = bh / H, h = bh % H;
        const int q0 = (item % n_qb) * 256;
        const int u = it % C::QBUF, k = it / C::QBUF;
        if (k > 0 && !(ok = mbar_wait(q_empty(u), (k - 1) & 1, status))) break;
        mbar_arrive_expect_tx(q_full(u), C::Q_ITEM);
        for (int t = 0; t < 2; ++t)
          for (int p = 0; p < C::NP; ++p)
            for (int c = 0; c < C::KCH; ++c)
              tma_load_4d(smem_u32(sQ + u * C::Q_ITEM + (t * C::NP + p) * C::Q_BYTES + c * C::CHUNK),
                          p ? &mapQl : &mapQ, q_full(u), c * 64, h, q0 + t * C::BM, b);
        for (int j = 0; j < n_kv; ++j) {
          const int g = it * n_kv + j;
          const int s = g % C::STAGES;
          if (g >= C::STAGES && !(ok = mbar_wait(kv_empty(s), ((g / C::STAGES) - 1) & 1, status))) break;
          mbar_arrive_expect_tx(kv_full(s), C::NP * 2 * C::KV_BYTES);
          for (int p = 0; p < C::NP; ++p)
            for (int c = 0; c < C::KCH; ++c) {
              tma_load_4d(smem_u32(sK + (s * C::NP + p) * C::KV_BYTES + c * C::CHUNK),
                          p ? &mapKl : &mapK, kv_full(s), c * 64, h, j * C::BN, b);
              tma_load_4d(smem_u32(sV + (s * C::NP + p) * C::KV_BYTES + c * C::CHUNK),
                          p ? &mapVl : &mapV, kv_full(s), c * 64, h, j * C::BN, b);
            }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idS = make_idesc(128, 128, 1, false, false);
      constexpr uint32_t idO = make_idesc(128, D, 1, false, true);
      // Descriptor bases; per-K-step offsets are added to the 16-byte address field.
      const uint64_t dQ0 = make_sdesc(smem_u32(sQ), 16, 1024);
      const uint64_t dK0 = make_sdesc(smem_u32(sK), 16, 1024);
      const uint64_t dV0 = make_sdesc(smem_u32(sV), C::CHUNK, 1024);
      // SPLIT: product terms (A plane, B plane) = (hi,hi), (hi,lo), (lo,hi)
      constexpr int NTERM = SPLIT ? 3 : 1;
      auto issue_S = [&](int t, int u, int g) {
#pragma unroll
        for (int term = 0; term < NTERM; ++term) {
          const int pa = term == 2 ? 1 : 0, pb = term == 1 ? 1 : 0;
          const uint64_t qd = dQ0 + ((u * C::Q_ITEM + (t * C::NP + pa) * C::Q_BYTES) >> 4);
          const uint64_t kd = dK0 + ((((g % C::STAGES) * C::NP + pb) * C::KV_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t off = ((k / 4) * C::CHUNK + (k % 4) * 32) >> 4;
            umma_f16_ss(tmem + C::T_S + t * 128, qd + off, kd + off, idS, (term > 0 || k > 0) ? 1u : 0u);
          }
        }
      };
      // P*V of KV tile g (j-th of the item: j == 0 starts O from zero)
      auto issue_PV = [&](int t, int g, int j) {
        const uint32_t tp = C::SEP_P ? (tmem + C::T_P + t * 64) : (tmem + C::T_S + t * 128);
#pragma unroll
        for (int term = 0; term < NTERM; ++term) {
          const int pa = term == 2 ? 1 : 0, pb = term == 1 ? 1 : 0;
          const uint64_t vd = dV0 + ((((g % C::STAGES) * C::NP + pb) * C::KV_BYTES) >> 4);
#pragma unroll
          for (int k = 0; k < C::BN / 16; ++k)
            umma_f16_ts(tmem + C::T_O + t * D, tp + pa * 64 + k * 8, vd + ((k * 2048) >> 4), idO,
                        (j > 0 || term > 0 || k > 0) ? 1u : 0u);
        }
      };
      bool ok = true;
      for (int item = item0, it = 0; ok && item < n_items; item += n_cta, ++it) {
        const int u = it % C::QBUF, g0 = it * n_kv;
        ok = mbar_wait(q_full(u), (it / C::QBUF) & 1, status) &&
             mbar_wait(kv_full(g0 % C::STAGES), (g0 / C::STAGES) & 1, status);
        if (!ok) break;
        // S of the item's first KV tile. Separate P: S's columns are free once
        // the softmax has loaded the previous tile's S. P over S: the previous
        // tile's P*V, which reads them, was issued before (in order).
        for (int t = 0; t < 2; ++t) {
          if (C::SEP_P && g0 > 0 && !(ok = mbar_wait(s_free(t), (g0 - 1) & 1, status))) break;
          tc_fence_after();
          issue_S(t, u, g0);
          umma_commit(s_full(t));
        }
        if (!ok) break;
        if (n_kv == 1) umma_commit(q_empty(u));
        for (int j = 0; ok && j < n_kv; ++j) {
          const int g = g0 + j;
          const bool more = j + 1 < n_kv;
          if (more && !(ok = mbar_wait(kv_full((g + 1) % C::STAGES), ((g + 1) / C::STAGES) & 1, status)))
            break;
          // P*V of tile j starts O from zero at j == 0: p_full of this item's
          // first tile is arrived only after the softmax has read the previous
          // item's O (its write-back comes first), so O is free then.
          for (int t = 0; t < 2; ++t) {
            if (C::SEP_P) {
              // next S first (its columns were released by s_free), then P*V
              if (more) {
                if (!(ok = mbar_wait(s_free(t), g & 1, status))) break;
                tc_fence_after();
                issue_S(t, u, g + 1);
                umma_commit(s_full(t));
              }
              if (!(ok = mbar_wait(p_full(t), g & 1, status))) break;
              tc_fence_after();
              issue_PV(t, g, j);
              umma_commit(pv_done(t));
            } else {
              // P lives in S's columns: P*V first, then the next S overwrites them
              if (!(ok = mbar_wait(p_full(t), g & 1, status))) break;
              tc_fence_after();
              issue_PV(t, g, j);
              umma_commit(pv_done(t));
              if (more) {
                issue_S(t, u, g + 1);
                umma_commit(s_full(t));
              }
            }
            if (t == 1) umma_commit(kv_empty(g % C::STAGES));
            if (!more) umma_commit(o_done(t));
          }
          if (j + 2 == n_kv) umma_commit(q_empty(u));  // the item's last S MMAs are issued
        }
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ softmax
    const int t = (warp - 4) / 4;                 // query tile of this warpgroup
    const int r = threadIdx.x - 128 * (t + 1);    // row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + C::T_S + t * 128 + lane_base;
    const uint32_t tO = tmem + C::T_O + t * D + lane_base;
    const uint32_t tP = C::SEP_P ? (tmem + C::T_P + t * 64 + lane_base) : tS;
    bool ok = true;
    for (int item = item0, it = 0; ok && item < n_items; item += n_cta, ++it) {
    const int bh = item / n_qb;
    const int b = bh / H, h = bh % H;
    const int row = (item % n_qb) * 256 + t * C::BM + r;
    float m = -INFINITY;  // running max of S * scale * log2(e)
    float l = 0.f;        // running row sum (relative to m)
    for (int j = 0; j < n_kv; ++j) {
      const int g = it * n_kv + j;
      if (!(ok = mbar_wait_warp(s_full(t), g & 1, status))) break;
      tc_fence_after();
      float s[128];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(tS + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&s[c * 32]));
      tmem_ld_wait();
      if (C::SEP_P) {
        tc_fence_before();
        mbar_arrive(s_free(t));  // S may now be overwritten by the next tile's MMA
      }
      const int kv_left = L - j * C::BN;
      if (kv_left < C::BN) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= kv_left) s[i] = -INFINITY;
      }
      // row max over eight independent chains of three-input max (a single
      // chain would be 127 dependent steps)
      float mk[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mk[k] = fmaxf(s[k], s[8 + k]);
#pragma unroll
      for (int i = 16; i < 128; i += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) mk[k] = max3f(mk[k], s[i + k], s[i + 8 + k]);
      const float mx = max3f(max3f(mk[0], mk[1], mk[2]), max3f(mk[3], mk[4], mk[5]), fmaxf(mk[6], mk[7]));
      const float m_new = fmaxf(m, mx * scale_log2);
      const bool need = m_new > m + 8.f;
      const bool warp_need = __any_sync(0xffffffffu, need);
      const float alpha = need ? ex2(m - m_new) : 1.f;
      if (need) {
        l *= alpha;
        m = m_new;
      }
      // P of the previous tile and O are read / accumulated by its P*V MMA:
      // wait for it before overwriting P or rescaling O (normally long done).
      if (C::SEP_P && g > 0) {
        if (!(ok = mbar_wait_warp(pv_done(t), (g - 1) & 1, status))) break;
        tc_fence_after();
      }
      // P = exp2(S * scale * log2(e) - m), packed to bf16 pairs, 16 columns at a time.
      const float neg_m = -m;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        uint32_t pk[8], pl[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float p0 = ex2(fmaf(s[c * 16 + 2 * i], scale_log2, neg_m));
          const float p1 = ex2(fmaf(s[c * 16 + 2 * i + 1], scale_log2, neg_m));
          sum += p0 + p1;
          pk[i] = pack_bf16x2(p0, p1);
          if (SPLIT)
            pl[i] = pack_bf16x2(p0 - __uint_as_float(pk[i] << 16),
                                p1 - __uint_as_float(pk[i] & 0xffff0000u));
        }
        PA_TMEM_ST_X8(tP + c * 8, pk);
        if (SPLIT) PA_TMEM_ST_X8(tP + 64 + c * 8, pl);
      }
      l += sum;
      if (warp_need && j > 0) {
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tO + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(tO + c * 32, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full(t));
    }
    // O write-back. The TMEM loads complete (wait::ld) before this warpgroup's
    // next p_full arrive, which the next item's first P*V waits for.
    if (!ok || !(ok = mbar_wait_warp(o_done(t), it & 1, status))) break;
    tc_fence_after();
    const float inv_l = 1.f / l;
    OutT* orow = O + ((static_cast<size_t>(b) * L + row) * H + h) * d_out;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      uint32_t o[32];
      tmem_ld32(tO + c * 32, o);
      tmem_ld_wait();
      if constexpr (std::is_same<OutT, float>::value) {
        if (row < L && c * 32 < d_out) {
          float4* dst = reinterpret_cast<float4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            dst[i] = make_float4(__uint_as_float(o[4 * i]) * inv_l, __uint_as_float(o[4 * i + 1]) * inv_l,
                                 __uint_as_float(o[4 * i + 2]) * inv_l, __uint_as_float(o[4 * i + 3]) * inv_l);
        }
      } else {
        uint32_t pkd[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pkd[i] = pack_bf16x2(__uint_as_float(o[2 * i]) * inv_l, __uint_as_float(o[2 * i + 1]) * inv_l);
        if (row < L) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(pkd[4 * i], pkd[4 * i + 1], pkd[4 * i + 2], pkd[4 * i + 3]);
        }
      }
    }
    if (row < L) lse[static_cast<size_t>(bh) * L + row] = (m + __log2f(l)) * kLn2;
    }  // item
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool SPLIT, typename OutT>
static int launch_fwd(const AttnShape& shp, const CUtensorMap* m, void* o, float* lse, int d_out,
                      uint32_t* status, cudaStream_t stream) {
  using C = FwdCfg<D, SPLIT>;
  static std::atomic<uint64_t> attr{0};
  if (!ensure_smem_attr(attn_fwd_kernel<D, SPLIT, OutT>, C::SMEM, attr)) return PA_ERR_LAUNCH;
  // persistent: as many CTAs as fit on the device at once, at most one per item
  const int dev = current_device();
  if (dev < 0) return PA_ERR_DEVICE;
  static std::atomic<int> resident[kMaxDevices];
  const int res = cached_per_device(resident, dev, [] {
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, attn_fwd_kernel<D, SPLIT, OutT>, C::THREADS,
                                                      C::SMEM) != cudaSuccess ||
        per_sm <= 0) {
      cudaGetLastError();  // clear a failed query; one CTA per SM
      per_sm = 1;
    }
    return device_sm_count() * per_sm;
  });
  const int n_qb = (shp.L + 255) / 256;
  const long long items = static_cast<long long>(n_qb) * shp.B * shp.H;
  if (items > 0x7fffffffLL) return PA_ERR_SHAPE;
  const int n_items = static_cast<int>(items);
  const int grid = n_items < res ? n_items : res;
  attn_fwd_kernel<D, SPLIT, OutT><<<grid, C::THREADS, C::SMEM, stream>>>(
      m[0], m[1], m[2], m[3], m[4], m[5], static_cast<OutT*>(o), lse, shp.L, shp.H, d_out,
      shp.scale * kLog2e, n_qb, n_items, status);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

// Host launcher. q/k/v/o are [B, L, H, D] bf16, lse is [B*H, L] fp32.
int launch_attn_fwd_bf16(const AttnShape& sh, const void* q, const void* k, const void* v, void* o,
                         float* lse, uint32_t* status, cudaStream_t stream) {
  CUtensorMap m[6];
  if (!make_qkv_map(&m[0], q, sh, 128) || !make_qkv_map(&m[1], k, sh, 128) ||
      !make_qkv_map(&m[2], v, sh, 128))
    return PA_ERR_ALIGN;
  m[3] = m[0];
  m[4] = m[1];
  m[5] = m[2];
  if (sh.D == 64) return launch_fwd<64, false, __nv_bfloat16>(sh, m, o, lse, 64, status, stream);
  if (sh.D == 128) return launch_fwd<128, false, __nv_bfloat16>(sh, m, o, lse, 128, status, stream);
  return PA_ERR_UNSUPPORTED;
}

// Padded head dim of the fp32 path's bf16 planes.
int f32_plane_dim(int D) { return D <= 64 ? 64 : -1; }

size_t attn_fwd_workspace_bytes_f32(const AttnShape& sh) {
  const int Dp = f32_plane_dim(sh.D);
  if (Dp < 0) return 0;
  const size_t plane = static_cast<size_t>(sh.B) * sh.L * sh.H * Dp * 2;
  const size_t up = (plane + 255) & ~static_cast<size_t>(255);
  return 6 * up;
}

// fp32 q/k/v/o [B, L, H, D], D in {32, 64}: split into bf16 hi/lo planes in
// the workspace, then the SPLIT kernel.
int launch_attn_fwd_f32(const AttnShape& sh, const void* q, const void* k, const void* v, void* o,
                        float* lse, void* ws, uint32_t* status, cudaStream_t stream) {
  const int Dp = f32_plane_dim(sh.D);
  if (Dp < 0) return PA_ERR_UNSUPPORTED;
  const size_t rows = static_cast<size_t>(sh.B) * sh.L * sh.H;
  const size_t plane = rows * Dp * 2;
  const size_t up = (plane + 255) & ~static_cast<size_t>(255);
  uint8_t* w = static_cast<uint8_t*>(ws);
  const float* src[3] = {static_cast<const float*>(q), static_cast<const float*>(k),
                         static_cast<const float*>(v)};
  const bool bf16_math = sh.D == 64 && f32_math() == PA_F32_MATH_BF16;
  for (int i = 0; i < 3; ++i) {
    const int st = launch_split_planes(src[i], w + (2 * i) * up,
                                       bf16_math ? nullptr : w + (2 * i + 1) * up, rows, sh.D, Dp,
                                       stream);
    if (st != PA_OK) return st;
  }
  AttnShape ps = sh;
  ps.D = Dp;
  CUtensorMap m[6];
  if (sh.D == 64 && f32_math() == PA_F32_MATH_BF16) {
    // bf16 math: the hi planes alone (bf16 roundings of q, k, v), bf16 kernel, fp32 O
    for (int i = 0; i < 3; ++i) {
      if (!make_qkv_map(&m[i], w + (2 * i) * up, ps, 128)) return PA_ERR_ALIGN;
      m[3 + i] = m[i];
    }
    return launch_fwd<64, false, float>(ps, m, o, lse, 64, status, stream);
  }
  // m[0..2] = hi planes of q, k, v; m[3..5] = lo planes
  for (int i = 0; i < 3; ++i)
    if (!make_qkv_map(&m[i], w + (2 * i) * up, ps, 128) ||
        !make_qkv_map(&m[3 + i], w + (2 * i + 1) * up, ps, 128))
      return PA_ERR_ALIGN;
  return launch_fwd<64, true, float>(ps, m, o, lse, sh.D, status, stream);
}

}  // namespace pa
