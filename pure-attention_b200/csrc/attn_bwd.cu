// Flash-attention backward for sm_100a: bf16 inputs, fp32 accumulation.
//
// Restates the reference's backward (flash_attn_backward_kernel.cu:25-41 for
// Delta, :153-197 for the per-tile math, doc/flash_backward.md section 5):
//   P  = exp(S * scale - LSE)        recomputed from the saved row LSE
//   dP = dO V^T,  Delta = rowsum(dO * O)
//   dS = P * (dP - Delta) * scale
//   dV = P^T dO,  dK = dS^T Q,  dQ = dS K
// with the reference's dQ stub (:182-191) replaced by the real product.
//
// Three kernels:
//   attn_bwd_prep_kernel : Delta and LSE*log2(e) per query row, laid out
//                          [B*H, Lp] (Lp = L rounded up to 128, padded rows
//                          get LSE = +inf so their P is exactly 0).
//   attn_bwd_kernel      : one CTA per (batch, head, 128-key tile), looping
//                          over 128-query tiles:
//       warp 0      TMA producer (K, V once; Q, dO, LSE, Delta per query tile)
//       warp 1      TMEM allocator + tcgen05.mma issuer
//       warps 4-11  P / dS elementwise, thread = one key row and one half of
//                   the 128 queries (two warpgroups); dK/dV epilogue
//       warps 12-15 dQ readout: TMEM -> swizzled shared tile -> TMA tensor
//                   reduce-add into an fp32 dQ accumulator in the workspace
//     MMAs per query tile (M = 128, K-major unless noted):
//       S^T  = K Q^T            (SS)        -> TMEM S
//       dP^T = V dO^T           (SS)        -> TMEM dP
//       dV  += P^T dO           (TS, dO MN-major)
//       dK  += dS^T Q           (TS, Q MN-major)
//       dQ   = dS K             (SS, dS and K MN-major; dS staged in shared)
//     P^T and dS^T (bf16) are written over the S and dP columns their
//     warpgroup has already read. dS is kept without the softmax scale; the
//     scale is applied once in the dK epilogue and in the dQ convert.
//   attn_dq_convert_kernel : fp32 dQ accumulator -> dq in the boundary layout.
//
// fp32 path (SPLIT): Q, K, V, dO arrive as bf16 hi/lo planes (fp32_split.cu,
// head dim padded to 64) and every product is hi*hi + hi*lo + lo*hi, three
// chained MMAs; P and dS are split the same way. In TMEM the hi and lo halves
// of each 16-query K-step sit in adjacent 8-column groups (16k, 16k + 8).
#include <type_traits>
#include "host_launchers.h"

namespace pa {

template <int D, bool SPLIT>
struct BwdCfg {
  static constexpr int NP = SPLIT ? 2 : 1;  // operand planes (hi, lo)
  static constexpr int KCH = D / 64;
  static constexpr int STAGES = (D == 64 && !SPLIT) ? 2 : 1;
  static constexpr int DQB = 1;                      // dQ staging buffers
  // d = 64: dS tile double-buffered and the next tile's S/dP MMAs issued before
  // this tile's dQ MMA (dQ has its own TMEM columns). d = 128: dQ reuses S's
  // TMEM columns, so dQ is issued before the next S.
  static constexpr bool EARLY_S = (D == 64 && !SPLIT);
  static constexpr int DSB = EARLY_S ? 2 : 1;
  static constexpr int CHUNK = 128 * 128;
  static constexpr int KV_BYTES = 128 * D * 2;
  static constexpr int QT_BYTES = 128 * D * 2;
  static constexpr int STAGE_BYTES = NP * 2 * QT_BYTES + 1024;  // Q, dO planes, LSE2[128], Delta[128]
  static constexpr int DS_BYTES = 128 * 128 * 2;
  static constexpr int DQ_BYTES = 128 * D * 4;
  static constexpr int SMEM =
      NP * 2 * KV_BYTES + STAGES * STAGE_BYTES + DSB * NP * DS_BYTES + DQB * DQ_BYTES + 1024;
  static constexpr uint32_t T_S = 0, T_DP = 128, T_DV = 256, T_DK = 256 + D;
  static constexpr uint32_t T_DQ = (D == 64) ? 384 : 0;  // D=128: dQ reuses S's columns
};

// ---------------------------------------------------------------- prep
// v ~= hi + mid + lo in bf16 (about 24 significant bits); packed (hi, mid), (lo, 0).
__device__ __forceinline__ uint2 split3_bf16(float v) {
  const __nv_bfloat16 hi = __float2bfloat16_rn(v);
  const float r1 = v - __bfloat162float(hi);
  const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
  const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
  return make_uint2(static_cast<uint32_t>(__bfloat16_as_ushort(hi)) |
                        (static_cast<uint32_t>(__bfloat16_as_ushort(mid)) << 16),
                    static_cast<uint32_t>(__bfloat16_as_ushort(lo)));
}

// Extension tile of the head-dim-64 backward: per (b*H + h, 128-query tile)
// 4 KB = 128 query rows x 16 bf16 columns in the K-major no-swizzle
// core-matrix layout (row r, column k at byte (r/8)*256 + (k/8)*128 +
// (r%8)*16 + 2*(k%8)). Columns 0-2 hold -LSE/scale split in three bf16
// parts, columns 8-10 -Delta likewise; the rest are zero. Against a tile of
// ones in columns 0-2 (resp. 8-10) they add -LSE/scale to S (resp. -Delta to
// dP) inside the S and dP MMAs. Padded query rows get -1e30 so their P is
// exactly 0.
constexpr int kExtTileBytes = 4096;
__device__ __forceinline__ void write_ext_rows(uint8_t* ext, size_t bh, int Lp, int l, float q_val,
                                               float do_val, bool pad) {
  uint8_t* t = ext + (bh * (Lp / 128) + l / 128) * kExtTileBytes;
  const int r = l % 128;
  const int off = (r / 8) * 256 + (r % 8) * 16;
  const uint2 q = pad ? make_uint2(static_cast<uint32_t>(__bfloat16_as_ushort(__float2bfloat16_rn(-1e30f))), 0u)
                      : split3_bf16(q_val);
  const uint2 d = split3_bf16(do_val);
  *reinterpret_cast<uint4*>(t + off) = make_uint4(q.x, q.y, 0u, 0u);
  *reinterpret_cast<uint4*>(t + off + 128) = make_uint4(d.x, d.y, 0u, 0u);
}

// One thread per (batch*head, query row); a block holds the 128 rows of one
// query tile, so the extension tile, LSE and Delta of a block are contiguous
// and every warp writes them as whole 128-byte lines. Each thread reads its
// rows of dO and O (D values each) with up to 16 independent 16-byte loads in
// flight. With dq_zero the block also clears its tile of the fp32 dQ
// accumulator (128 rows x dq_width floats), which the main kernel reduces into.
template <int D, typename InT>
__global__ void __launch_bounds__(128)
    attn_bwd_prep_kernel(const InT* __restrict__ dO, const InT* __restrict__ O,
                         const float* __restrict__ lse, float* __restrict__ lse2_t,
                         float* __restrict__ delta_t, float* __restrict__ delta_ref,
                         uint8_t* __restrict__ ext, float* __restrict__ dq_zero, int dq_width,
                         float inv_scale, int L, int Lp, int H) {
  constexpr int NV = D * static_cast<int>(sizeof(InT)) / 16;  // 16-byte vectors per row
  constexpr int CH = NV < 8 ? NV : 8;                           // vectors loaded per batch
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int l = blockIdx.x * 128 + static_cast<int>(threadIdx.x);
  const bool real = l < L;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  if (real) {
    const size_t off = ((static_cast<size_t>(b) * L + l) * H + h) * D;
    const uint4* a4 = reinterpret_cast<const uint4*>(dO + off);
    const uint4* c4 = reinterpret_cast<const uint4*>(O + off);
#pragma unroll
    for (int v0 = 0; v0 < NV; v0 += CH) {
      uint4 va[CH], vc[CH];
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        va[i] = a4[v0 + i];
        vc[i] = c4[v0 + i];
      }
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        if constexpr (sizeof(InT) == 2) {
          const __nv_bfloat162* x2 = reinterpret_cast<const __nv_bfloat162*>(&va[i]);
          const __nv_bfloat162* y2 = reinterpret_cast<const __nv_bfloat162*>(&vc[i]);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 fx = __bfloat1622float2(x2[e]);
            const float2 fy = __bfloat1622float2(y2[e]);
            acc[e] = fmaf(fx.x, fy.x, fmaf(fx.y, fy.y, acc[e]));
          }
        } else {
          const float* x = reinterpret_cast<const float*>(&va[i]);
          const float* y = reinterpret_cast<const float*>(&vc[i]);
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[e] = fmaf(x[e], y[e], acc[e]);
        }
      }
    }
  }
  const float delta = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  const size_t row = static_cast<size_t>(bh) * Lp + l;  // rows [B*H, Lp]
  if (l < Lp) {
    if (lse2_t) lse2_t[row] = real ? lse[static_cast<size_t>(bh) * L + l] * kLog2e : INFINITY;
    if (delta_t) delta_t[row] = real ? delta : 0.f;
    if (ext)
      write_ext_rows(ext, bh, Lp, l, real ? -lse[static_cast<size_t>(bh) * L + l] * inv_scale : 0.f,
                     real ? -delta : 0.f, !real);
  }
  if (delta_ref && real) delta_ref[(static_cast<size_t>(b) * L + l) * H + h] = delta;
  if (dq_zero) {
    float4* z = reinterpret_cast<float4*>(dq_zero + (static_cast<size_t>(bh) * Lp +
                                                     static_cast<size_t>(blockIdx.x) * 128) * dq_width);
    const int n4 = 128 * dq_width / 4;
    const float4 zero = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int i = static_cast<int>(threadIdx.x); i < n4; i += 128) z[i] = zero;
  }
}

// ---------------------------------------------------------------- main
// TMEM column of the k-th 16-query K-step of P^T / dS^T: each elementwise
// warpgroup packs its 64 queries (32 columns of bf16 pairs) at the start of
// the 64 fp32 columns it read, so queries [0,64) sit in columns [0,32) and
// queries [64,128) in columns [64,96) of the S (or dP) tile.
__device__ __forceinline__ uint32_t packed_col(int k) { return (k < 4) ? k * 8 : 64 + (k - 4) * 8; }
// SPLIT: hi and lo halves of K-step k in columns 16k and 16k + 8.
template <bool SPLIT>
__device__ __forceinline__ uint32_t step_col(int k, int plane) {
  return SPLIT ? static_cast<uint32_t>(16 * k + 8 * plane) : packed_col(k);
}

// OutT: __nv_bfloat16 (bf16 path) or float (SPLIT); d_out = head dim of dk/dv.
template <int D, bool SPLIT, typename OutT>
__global__ void __launch_bounds__(512, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                    const __grid_constant__ CUtensorMap mapV, const __grid_constant__ CUtensorMap mapdO,
                    const __grid_constant__ CUtensorMap mapQl, const __grid_constant__ CUtensorMap mapKl,
                    const __grid_constant__ CUtensorMap mapVl, const __grid_constant__ CUtensorMap mapdOl,
                    const __grid_constant__ CUtensorMap mapDQ, OutT* __restrict__ dk,
                    OutT* __restrict__ dv, const float* __restrict__ lse2_t,
                    const float* __restrict__ delta_t, int L, int Lp, int H, int d_out, float scale,
                    float scale_log2, int accumulate, uint32_t* status) {
  using C = BwdCfg<D, SPLIT>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bars[16];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  if (cta_aborted(status, &abort_flag)) return;

  uint8_t* smem = align1024(smem_raw);
  // K / V: NP planes each. Stage s: Q planes, dO planes, LSE2, Delta.
  // dS: DSB buffers of NP planes. Plane p of K at sK + p * KV_BYTES, etc.
  uint8_t* sK = smem;
  uint8_t* sV = sK + C::NP * C::KV_BYTES;
  uint8_t* sStage = sV + C::NP * C::KV_BYTES;
  uint8_t* sdS = sStage + C::STAGES * C::STAGE_BYTES;
  uint8_t* sDQ = sdS + C::DSB * C::NP * C::DS_BYTES;

  const uint32_t kv_full = smem_u32(&bars[0]);
  auto q_full = [&](int s) { return smem_u32(&bars[1 + s]); };
  auto q_empty = [&](int s) { return smem_u32(&bars[3 + s]); };
  const uint32_t sd_full = smem_u32(&bars[5]);
  const uint32_t p_full = smem_u32(&bars[6]);
  const uint32_t dq_full = smem_u32(&bars[7]);
  const uint32_t dq_empty = smem_u32(&bars[8]);
  const uint32_t kv_done = smem_u32(&bars[9]);

  const int warp = warp_id();
  const int bh = blockIdx.y;
  const int b = bh / H, h = bh % H;
  const int k0 = blockIdx.x * 128;
  const int n_q = Lp / 128;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(q_full(s), 1);
      mbar_init(q_empty(s), 1);
    }
    mbar_init(sd_full, 1);
    mbar_init(p_full, 256);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 128);
    mbar_init(kv_done, 1);
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

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&mapQ);
      tma_prefetch_desc(&mapdO);
      mbar_arrive_expect_tx(kv_full, C::NP * 2 * C::KV_BYTES);
      for (int p = 0; p < C::NP; ++p)
        for (int c = 0; c < C::KCH; ++c) {
          tma_load_4d(smem_u32(sK + p * C::KV_BYTES + c * C::CHUNK), p ? &mapKl : &mapK, kv_full,
                      c * 64, h, k0, b);
          tma_load_4d(smem_u32(sV + p * C::KV_BYTES + c * C::CHUNK), p ? &mapVl : &mapV, kv_full,
                      c * 64, h, k0, b);
        }
      for (int j = 0; j < n_q; ++j) {
        const int s = j % C::STAGES;
        if (j >= C::STAGES && !mbar_wait(q_empty(s), ((j / C::STAGES) - 1) & 1, status)) break;
        uint8_t* st = sStage + s * C::STAGE_BYTES;
        mbar_arrive_expect_tx(q_full(s), C::NP * 2 * C::QT_BYTES + 1024);
        for (int p = 0; p < C::NP; ++p)
          for (int c = 0; c < C::KCH; ++c) {
            tma_load_4d(smem_u32(st + p * C::QT_BYTES + c * C::CHUNK), p ? &mapQl : &mapQ,
                        q_full(s), c * 64, h, j * 128, b);
            tma_load_4d(smem_u32(st + (C::NP + p) * C::QT_BYTES + c * C::CHUNK),
                        p ? &mapdOl : &mapdO, q_full(s), c * 64, h, j * 128, b);
          }
        const size_t voff = static_cast<size_t>(bh) * Lp + j * 128;
        bulk_load(smem_u32(st + 2 * C::NP * C::QT_BYTES), lse2_t + voff, 512, q_full(s));
        bulk_load(smem_u32(st + 2 * C::NP * C::QT_BYTES + 512), delta_t + voff, 512, q_full(s));
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idSP = make_idesc(128, 128, 1, false, false);
      constexpr uint32_t idKV = make_idesc(128, D, 1, false, true);
      constexpr uint32_t idQ = make_idesc(128, D, 1, true, true);
      // Descriptor bases; offsets are added to the 16-byte address field.
      const uint64_t dK_K = make_sdesc(smem_u32(sK), 16, 1024);              // K, K-major
      const uint64_t dV_K = make_sdesc(smem_u32(sV), 16, 1024);              // V, K-major
      const uint64_t dK_MN = make_sdesc(smem_u32(sK), C::CHUNK, 1024);       // K, MN-major
      const uint64_t dSt_K = make_sdesc(smem_u32(sStage), 16, 1024);         // Q / dO, K-major
      const uint64_t dSt_MN = make_sdesc(smem_u32(sStage), C::CHUNK, 1024);  // Q / dO, MN-major
      const uint64_t dDS_MN = make_sdesc(smem_u32(sdS), C::CHUNK, 1024);     // dS, MN-major
      // SPLIT: product terms (A plane, B plane) = (hi,hi), (hi,lo), (lo,hi)
      constexpr int NTERM = SPLIT ? 3 : 1;
      constexpr uint32_t KVP = C::KV_BYTES >> 4, QTP = C::QT_BYTES >> 4, DSP = C::DS_BYTES >> 4;
      auto issue_SdP = [&](int j) {
        const uint32_t so = ((j % C::STAGES) * C::STAGE_BYTES) >> 4;
#pragma unroll
        for (int term = 0; term < NTERM; ++term) {
          const uint32_t pa = term == 2, pb = term == 1;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t off = ((k / 4) * C::CHUNK + (k % 4) * 32) >> 4;
            umma_f16_ss(tmem + C::T_S, dK_K + pa * KVP + off, dSt_K + so + pb * QTP + off, idSP,
                        (term > 0 || k > 0) ? 1u : 0u);
          }
        }
#pragma unroll
        for (int term = 0; term < NTERM; ++term) {
          const uint32_t pa = term == 2, pb = term == 1;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t off = ((k / 4) * C::CHUNK + (k % 4) * 32) >> 4;
            umma_f16_ss(tmem + C::T_DP, dV_K + pa * KVP + off,
                        dSt_K + so + (C::NP + pb) * QTP + off, idSP, (term > 0 || k > 0) ? 1u : 0u);
          }
        }
      };
      auto issue_dVdK = [&](int j) {
        const uint32_t so = ((j % C::STAGES) * C::STAGE_BYTES) >> 4;
#pragma unroll
        for (int term = 0; term < NTERM; ++term) {
          const int pa = term == 2, pb = term == 1;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            umma_f16_ts(tmem + C::T_DV, tmem + C::T_S + step_col<SPLIT>(k, pa),
                        dSt_MN + so + (C::NP + pb) * QTP + ((k * 2048) >> 4), idKV,
                        (j > 0 || term > 0 || k > 0) ? 1u : 0u);
        }
#pragma unroll
        for (int term = 0; term < NTERM; ++term) {
          const int pa = term == 2, pb = term == 1;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            umma_f16_ts(tmem + C::T_DK, tmem + C::T_DP + step_col<SPLIT>(k, pa),
                        dSt_MN + so + pb * QTP + ((k * 2048) >> 4), idKV,
                        (j > 0 || term > 0 || k > 0) ? 1u : 0u);
        }
      };
      auto issue_dQ = [&](int j) {
        const uint32_t bo = ((j % C::DSB) * C::NP * C::DS_BYTES) >> 4;
#pragma unroll
        for (int term = 0; term < NTERM; ++term) {
          const uint32_t pa = term == 2, pb = term == 1;
#pragma unroll
          for (int k = 0; k < 8; ++k)
            umma_f16_ss(tmem + C::T_DQ, dDS_MN + bo + pa * DSP + ((k * 2048) >> 4),
                        dK_MN + pb * KVP + ((k * 2048) >> 4), idQ, (term > 0 || k > 0) ? 1u : 0u);
        }
      };
      bool ok = mbar_wait(kv_full, 0, status) && mbar_wait(q_full(0), 0, status);
      if (ok) {
        tc_fence_after();
        issue_SdP(0);
        umma_commit(sd_full);
      }
      for (int j = 0; ok && j < n_q; ++j) {
        const int s = j % C::STAGES;
        const bool more = j + 1 < n_q;
        if (!(ok = mbar_wait(p_full, j & 1, status))) break;
        tc_fence_after();
        issue_dVdK(j);
        umma_commit(q_empty(s));
        if (C::EARLY_S) {
          if (more) {
            if (!(ok = mbar_wait(q_full((j + 1) % C::STAGES), ((j + 1) / C::STAGES) & 1, status)))
              break;
            tc_fence_after();
            issue_SdP(j + 1);
            umma_commit(sd_full);
          }
          if (j > 0) {
            if (!(ok = mbar_wait(dq_empty, (j - 1) & 1, status))) break;
            tc_fence_after();
          }
          issue_dQ(j);
          umma_commit(dq_full);
        } else {
          // dQ overwrites S's columns: after dV, before the next S.
          if (j > 0) {
            if (!(ok = mbar_wait(dq_empty, (j - 1) & 1, status))) break;
            tc_fence_after();
          }
          issue_dQ(j);
          umma_commit(dq_full);
          if (more) {
            if (!(ok = mbar_wait(q_full((j + 1) % C::STAGES), ((j + 1) / C::STAGES) & 1, status)))
              break;
            if (!(ok = mbar_wait(dq_empty, j & 1, status))) break;
            tc_fence_after();
            issue_SdP(j + 1);
            umma_commit(sd_full);
          }
        }
      }
      if (ok) umma_commit(kv_done);
    }
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------ P / dS
    // Two warpgroups: grp 0 handles queries [0,64) of each tile, grp 1 [64,128).
    const int grp = (warp - 4) >> 2;
    const int kr = ((warp & 3) << 5) + static_cast<int>(lane_id());  // key row == TMEM lane
    const int key = k0 + kr;
    const bool valid = key < L;
    const bool full_tile = k0 + 128 <= L;  // CTA-uniform: no key masking needed
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + C::T_S + lane_base + grp * 64;
    const uint32_t tdP = tmem + C::T_DP + lane_base + grp * 64;
    bool ok = true;
    for (int j = 0; j < n_q; ++j) {
      const int s = j % C::STAGES;
      if (!(ok = mbar_wait_warp(sd_full, j & 1, status))) break;
      if (!(ok = mbar_wait_warp(q_full(s), (j / C::STAGES) & 1, status))) break;
      tc_fence_after();
      // MN-major dS tile (hi plane; lo plane DS_BYTES further)
      uint8_t* dsrow = sdS + (j % C::DSB) * C::NP * C::DS_BYTES + grp * C::CHUNK;
      const float* lse2s = reinterpret_cast<const float*>(sStage + s * C::STAGE_BYTES +
                                                          2 * C::NP * C::QT_BYTES) + grp * 64;
      const float* dels = lse2s + 128;
      uint32_t sv[2][16], dpv[2][16];
      tmem_ld16(tS, sv[0]);
      tmem_ld16(tdP, dpv[0]);
      tmem_ld_wait();
#pragma unroll
      for (int sc = 0; sc < 4; ++sc) {
        const int cur = sc & 1;
        if (sc < 3) {
          tmem_ld16(tS + (sc + 1) * 16, sv[cur ^ 1]);
          tmem_ld16(tdP + (sc + 1) * 16, dpv[cur ^ 1]);
        }
        float ls[16], de[16];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          *reinterpret_cast<float4*>(&ls[4 * u]) =
              *reinterpret_cast<const float4*>(lse2s + sc * 16 + 4 * u);
          *reinterpret_cast<float4*>(&de[4 * u]) =
              *reinterpret_cast<const float4*>(dels + sc * 16 + 4 * u);
        }
        uint32_t pk[8], dk2[8], pl[8], dl2[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          float p[2], d2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int el = 2 * i + e;
            p[e] = ex2(fmaf(__uint_as_float(sv[cur][el]), scale_log2, -ls[el]));
            d2[e] = p[e] * (__uint_as_float(dpv[cur][el]) - de[el]);
          }
          pk[i] = pack_bf16x2(p[0], p[1]);
          dk2[i] = pack_bf16x2(d2[0], d2[1]);
          if (SPLIT) {
            pl[i] = pack_bf16x2(p[0] - __uint_as_float(pk[i] << 16),
                                p[1] - __uint_as_float(pk[i] & 0xffff0000u));
            dl2[i] = pack_bf16x2(d2[0] - __uint_as_float(dk2[i] << 16),
                                 d2[1] - __uint_as_float(dk2[i] & 0xffff0000u));
          }
        }
        if (!full_tile && !valid) {
#pragma unroll
          for (int i = 0; i < 8; ++i) pk[i] = dk2[i] = pl[i] = dl2[i] = 0u;
        }
        if (SPLIT) {
          PA_TMEM_ST_X8(tS + sc * 16, pk);
          PA_TMEM_ST_X8(tS + sc * 16 + 8, pl);
          PA_TMEM_ST_X8(tdP + sc * 16, dk2);
          PA_TMEM_ST_X8(tdP + sc * 16 + 8, dl2);
        } else {
          PA_TMEM_ST_X8(tS + sc * 8, pk);
          PA_TMEM_ST_X8(tdP + sc * 8, dk2);
        }
        // queries grp*64 + sc*16 .. +16 -> 32 bytes of this key's row in the dS tile
        *reinterpret_cast<uint4*>(dsrow + sw128_offset(kr, (2 * sc) * 16)) =
            make_uint4(dk2[0], dk2[1], dk2[2], dk2[3]);
        *reinterpret_cast<uint4*>(dsrow + sw128_offset(kr, (2 * sc + 1) * 16)) =
            make_uint4(dk2[4], dk2[5], dk2[6], dk2[7]);
        if (SPLIT) {
          *reinterpret_cast<uint4*>(dsrow + C::DS_BYTES + sw128_offset(kr, (2 * sc) * 16)) =
              make_uint4(dl2[0], dl2[1], dl2[2], dl2[3]);
          *reinterpret_cast<uint4*>(dsrow + C::DS_BYTES + sw128_offset(kr, (2 * sc + 1) * 16)) =
              make_uint4(dl2[4], dl2[5], dl2[6], dl2[7]);
        }
        if (sc < 3) tmem_ld_wait();
      }
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full);
    }
    // dK (x scale) and dV epilogue: group 0 writes dV, group 1 writes dK.
    if (ok && mbar_wait_warp(kv_done, 0, status)) {
      tc_fence_after();
      const size_t roff = ((static_cast<size_t>(b) * L + key) * H + h) * d_out;
      OutT* dst = (grp == 0 ? dv : dk) + roff;
      const uint32_t tsrc = tmem + (grp == 0 ? C::T_DV : C::T_DK) + lane_base;
      const float mul = grp == 0 ? 1.f : scale;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(tsrc + c * 32, o);
        tmem_ld_wait();
        if constexpr (SPLIT) {
          if (valid && c * 32 < d_out) {
            float4* d4 = reinterpret_cast<float4*>(dst + c * 32);
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              float4 f = make_float4(__uint_as_float(o[4 * u]) * mul, __uint_as_float(o[4 * u + 1]) * mul,
                                     __uint_as_float(o[4 * u + 2]) * mul,
                                     __uint_as_float(o[4 * u + 3]) * mul);
              if (accumulate) {
                const float4 pv = d4[u];
                f.x += pv.x; f.y += pv.y; f.z += pv.z; f.w += pv.w;
              }
              d4[u] = f;
            }
          }
        } else if (valid) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(o[8 * u + e]) * mul;
            if (accumulate) {
              const uint4 prev = d4[u];
              const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&prev);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const float2 pf = __bfloat1622float2(p2[e]);
                f[2 * e] += pf.x;
                f[2 * e + 1] += pf.y;
              }
            }
            d4[u] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                               pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
          }
        }
      }
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------ dQ readout
    const int qr = threadIdx.x - 384;  // query row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tdQ = tmem + C::T_DQ + lane_base;
    // The loop never exits early: the named barriers below need all 128
    // threads every iteration, so a failed wait only skips the work.
    bool ok = true;
    for (int j = 0; j < n_q; ++j) {
      const int buf = j % C::DQB;
      if (j >= C::DQB) {
        if (qr == 0) bulk_wait_read<C::DQB - 1>();
        named_bar_sync(1, 128);
      }
      ok = ok && mbar_wait_warp(dq_full, j & 1, status);
      if (ok) {
        tc_fence_after();
        // Staging tile = D/32 boxes of 128 rows x 32 fp32 (128 B), 128B-swizzled
        // like the TMA map over dq_acc, so stores are conflict-free.
        uint8_t* sdq = sDQ + buf * C::DQ_BYTES;
#pragma unroll 1
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(tdQ + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(sdq + c * C::CHUNK + sw128_offset(qr, u * 16)) =
                make_uint4(o[4 * u], o[4 * u + 1], o[4 * u + 2], o[4 * u + 3]);
        }
        tc_fence_before();
        mbar_arrive(dq_empty);
        fence_proxy_async_smem();
      }
      named_bar_sync(1, 128);
      if (qr == 0 && !aborted(status)) {
        for (int c = 0; c < D / 32; ++c)
          tma_reduce_add_2d(&mapDQ, smem_u32(sDQ + buf * C::DQ_BYTES + c * C::CHUNK), c * 32,
                            bh * Lp + j * 128);
        tma_store_commit();
      }
    }
    if (qr == 0) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- head dim 64 (bf16)
// Schedule for d = 64 that keeps the tensor pipe fed from one TMEM budget:
//   S [0,128) | dP [128,256) | P^T packed bf16 [256,320) | dV [320,384) | dK [384,448) | dQ [448,512)
// -LSE/scale and -Delta enter the S and dP MMAs as one extra K-step
// (an extension tile written by the prep kernel, against tiles of ones), so
// S' = S - LSE/scale and dP' = dP - Delta come out of the tensor core and the
// elementwise step needs no per-query loads: P = exp2(S' * scale * log2 e),
// dS = P * dP'. (The extra K-step is 6% more tensor-pipe work, but loading
// LSE and Delta per query from shared memory in the elementwise step measured
// 23% slower: the MMAs' shared-memory operand reads are what this kernel is
// sensitive to.)
// Persistent: one two-CTA cluster per SM pair walks (batch*head, pair of key
// tiles) work items; rings, barrier phases and the dS buffers continue across
// items, and the dV/dK write-back of one item overlaps the next item's MMAs.
// Each tile's elementwise work runs in two phases:
//   P phase:  load S (s_free: the next S may start) -> P in registers ->
//             P^T to its own TMEM columns (pt_full: dV may start)
//   dS phase: load dP -> dS = P * dP' -> dS^T packed over the dP columns just
//             read (the A operand of the TS dK MMA) and dS to a double-buffered
//             shared tile (the A operand of dQ) (p_full)
// and the MMA issuer interleaves the tiles on the tensor pipe, per tile j:
//   s_free(j) -> S(j+1);  pt_full(j) -> dV(j);
//   p_full(j) -> dK(j), then dP(j+1) over dS^T(j), then dQ(j). Q and the extension tile are triple-buffered because
// Q(j) is released only by dK(j); dO is double-buffered (released by dV(j)).
// The dQ readout frees dQ's TMEM right after its tcgen05.ld (16x256b shape:
// four neighbouring lanes hold a whole 32-byte sector of a dQ row). The two
// CTAs of a cluster (neighbouring key tiles, same query order) then swap
// halves of their dQ tiles through distributed shared memory: each sends the
// 32 columns its partner owns into the partner's 16 KB receive buffer, adds
// the partner's contribution to its own 32 columns, and reduces only those
// into the fp32 accumulator (8-byte vector reductions straight from
// registers). Global reduction traffic is halved; the L2 reduction rate,
// not the tensor pipe, bounds this kernel without it.
struct Bwd64Cfg {
  static constexpr int EWG = 4;                        // elementwise warpgroups
  static constexpr int QPG = 32;                       // queries per warpgroup
  static constexpr int NEW = 128 * EWG;                // elementwise threads
  static constexpr int EW_WARP = 2;                    // warps 0, 1: producer, MMA issuer
  static constexpr int READOUT_WARP = EW_WARP + 4 * EWG;
  static constexpr int THREADS = 32 * (READOUT_WARP + 4);  // + 4 dQ readout warps
  static constexpr int QSTAGES = 3;                    // Q + extension buffers
  static constexpr int OSTAGES = 2;                    // dO buffers
  static constexpr int CHUNK = 128 * 128;              // one SW128 tile: 128 rows x 128 B
  static constexpr int KV_BYTES = 128 * 64 * 2;
  static constexpr int QT_BYTES = 128 * 64 * 2;
  static constexpr int EXT_BYTES = kExtTileBytes;      // 128 rows x 16 bf16
  static constexpr int QSTAGE_BYTES = QT_BYTES + EXT_BYTES;
  static constexpr int DS_BYTES = 2 * CHUNK;           // queries [0,64) and [64,128)
  static constexpr int RX_BYTES = 128 * 32 * 4;        // partner's half of a dQ tile
  static constexpr int ONES_BYTES = 1024;  // two 256-byte tiles of ones, padded to 1 KB
  static constexpr int SMEM = 2 * KV_BYTES + ONES_BYTES + QSTAGES * QSTAGE_BYTES +
                              OSTAGES * QT_BYTES + 2 * DS_BYTES + RX_BYTES + 1024;
  static constexpr uint32_t T_S = 0, T_DP = 128, T_PT = 256, T_DV = 320, T_DK = 384, T_DQ = 448;
};

// dQ half exchange of the readout. A 16x256b load of 16 rows gives thread t
// r[4i + 2a + q] = (row t/4 + 8a, column 8i + 2(t%4) + q). CTA rank OWN
// reduces column blocks i in [4 OWN, 4 OWN + 4): dq_split sends the other
// four blocks to the partner's receive buffer (slots v0 .. v0+3; slot v of
// thread t at byte v * 2048 + t * 16) with st.async, which completes bytes of
// the partner's rx_full barrier, and keeps its own four in `own`.
template <int OWN>
__device__ __forceinline__ void dq_split(const uint32_t (&r)[32], uint32_t (&own)[16],
                                         uint32_t peer_slot, uint32_t peer_bar, int v0) {
  constexpr int OTHER = 1 - OWN;
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const int i = 4 * OTHER + v;
    st_async_v4(peer_slot + (v0 + v) * 2048, make_uint4(r[4 * i], r[4 * i + 1], r[4 * i + 2], r[4 * i + 3]),
                peer_bar);
#pragma unroll
    for (int e = 0; e < 4; ++e) own[4 * v + e] = r[4 * (4 * OWN + v) + e];
  }
}
__device__ __forceinline__ void dq_add_slots(uint32_t (&own)[16], const uint8_t* rx_slot, int v0) {
#pragma unroll
  for (int v = 0; v < 4; ++v) {
    const uint4 p = *reinterpret_cast<const uint4*>(rx_slot + (v0 + v) * 2048);
    own[4 * v] = __float_as_uint(__uint_as_float(own[4 * v]) + __uint_as_float(p.x));
    own[4 * v + 1] = __float_as_uint(__uint_as_float(own[4 * v + 1]) + __uint_as_float(p.y));
    own[4 * v + 2] = __float_as_uint(__uint_as_float(own[4 * v + 2]) + __uint_as_float(p.z));
    own[4 * v + 3] = __float_as_uint(__uint_as_float(own[4 * v + 3]) + __uint_as_float(p.w));
  }
}
// row = accumulator element (row t/4 of a 16-row group, column 8 * 4 OWN + 2(t%4))
__device__ __forceinline__ void dq_reduce_own(const uint32_t (&own)[16], float* row) {
#pragma unroll
  for (int v = 0; v < 4; ++v)
#pragma unroll
    for (int a = 0; a < 2; ++a)
      red_add_v2_f32(row + (8 * a) * 64 + 8 * v, __uint_as_float(own[4 * v + 2 * a]),
                     __uint_as_float(own[4 * v + 2 * a + 1]));
}

// OutT: dK / dV storage, __nv_bfloat16 (bf16 tensors) or float (fp32 tensors
// computed in the bf16 math mode).
template <typename OutT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Bwd64Cfg::THREADS, 1)
    attn_bwd_d64_kernel(const __grid_constant__ CUtensorMap mapQ, const __grid_constant__ CUtensorMap mapK,
                        const __grid_constant__ CUtensorMap mapV,
                        const __grid_constant__ CUtensorMap mapdO, float* __restrict__ dq_acc,
                        OutT* __restrict__ dk, OutT* __restrict__ dv,
                        const uint8_t* __restrict__ ext, int L, int Lp, int H, float scale,
                        float scale_log2, int accumulate, int n_pairs, int n_items,
                        uint32_t* status) {
  using C = Bwd64Cfg;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bars[24];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  // No early return: both CTAs of the cluster must reach the cluster barriers.
  const bool skip = cta_aborted(status, &abort_flag);

  uint8_t* smem = align1024(smem_raw);
  uint8_t* sK = smem;
  uint8_t* sV = sK + C::KV_BYTES;
  // tiles of ones in the extension layout: columns 0-2 (picks -LSE/scale) and
  // columns 8-10 (picks -Delta). Every 8-row group of the 128-row operand is
  // the same, so each tile is one group (256 B) read with a zero group stride.
  uint8_t* sOnesS = sV + C::KV_BYTES;
  uint8_t* sOnesP = sOnesS + 256;
  uint8_t* sQ = sOnesS + C::ONES_BYTES;  // stage s: Q tile, then its extension tile
  uint8_t* sO = sQ + C::QSTAGES * C::QSTAGE_BYTES;
  uint8_t* sdS = sO + C::OSTAGES * C::QT_BYTES;
  uint8_t* sRX = sdS + 2 * C::DS_BYTES;  // partner's half of the current dQ tile
  if (threadIdx.x < 16) {
    const int r = threadIdx.x >> 1, half = threadIdx.x & 1;
    const uint4 one3 = make_uint4(0x3f803f80u, 0x00003f80u, 0u, 0u);
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    const int off = r * 16 + half * 128;
    *reinterpret_cast<uint4*>(sOnesS + off) = half ? zero : one3;
    *reinterpret_cast<uint4*>(sOnesP + off) = half ? one3 : zero;
    fence_proxy_async_smem();
  }

  const uint32_t kv_full = smem_u32(&bars[0]);
  auto q_full = [&](int s) { return smem_u32(&bars[1 + s]); };
  auto q_empty = [&](int s) { return smem_u32(&bars[4 + s]); };
  auto o_full = [&](int s) { return smem_u32(&bars[18 + s]); };
  auto o_empty = [&](int s) { return smem_u32(&bars[20 + s]); };
  const uint32_t s_full = smem_u32(&bars[7]);    // S' of the tile is in TMEM
  const uint32_t s_free = smem_u32(&bars[8]);    // elementwise warps have read S'
  const uint32_t pt_full = smem_u32(&bars[9]);   // P^T is in TMEM
  const uint32_t pt_free = smem_u32(&bars[10]);  // the dV MMA has read P^T
  const uint32_t dp_full = smem_u32(&bars[11]);  // dP' of the tile is in TMEM
  // dS of tile j is in shared memory. Two barriers, by tile parity: the
  // elementwise warps can finish tile j+1 before the issuer has polled tile j.
  auto p_full = [&](int j) { return smem_u32(&bars[(j & 1) ? 17 : 13]); };
  const uint32_t dq_full = smem_u32(&bars[14]);
  const uint32_t dq_empty = smem_u32(&bars[15]);
  const uint32_t kv_done = smem_u32(&bars[16]);
  const uint32_t rx_full = smem_u32(&bars[22]);  // partner's dQ half is in sRX (16 KB of st.async)
  const uint32_t tx_free = smem_u32(&bars[23]);  // partner has read what this CTA sent
  const uint32_t acc_free = smem_u32(&bars[12]);  // the epilogue has read an item's dV and dK

  const int warp = warp_id();
  const int n_q = Lp / 128;
  // Persistent clusters: cluster cl takes work items cl, cl + n_cl, ...; an item
  // is (batch*head, pair of adjacent key tiles), this CTA's tile of the pair
  // being its rank. Every role walks the same items; barrier phases and ring
  // slots count query tiles over all of them (g = items done * n_q + j).
  const int cl = static_cast<int>(blockIdx.x >> 1), n_cl = static_cast<int>(gridDim.x >> 1);
  const int rank_x = static_cast<int>(blockIdx.x & 1);
  struct Item {
    int bh, b, h, k0, q_first;
  };
  auto item_of = [&](int item) {
    Item w;
    w.bh = item / n_pairs;
    const int pair = item % n_pairs;
    w.b = w.bh / H;
    w.h = w.bh % H;
    w.k0 = (2 * pair + rank_x) * 128;
    // Query tiles are visited from tile `pair` onwards (mod n_q): the clusters
    // of one (batch, head) then reduce into different dQ rows at any moment
    // instead of all into the same tile. Same order in both CTAs of a cluster.
    w.q_first = pair % n_q;
    return w;
  };
  auto jq = [&](const Item& w, int j) { const int t = j + w.q_first; return t < n_q ? t : t - n_q; };

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    for (int s = 0; s < C::QSTAGES; ++s) {
      mbar_init(q_full(s), 1);
      mbar_init(q_empty(s), 1);
    }
    for (int s = 0; s < C::OSTAGES; ++s) {
      mbar_init(o_full(s), 1);
      mbar_init(o_empty(s), 1);
    }
    mbar_init(s_full, 1);
    mbar_init(s_free, C::NEW);
    mbar_init(pt_full, C::NEW);
    mbar_init(pt_free, 1);
    mbar_init(dp_full, 1);
    mbar_init(p_full(0), C::NEW);
    mbar_init(p_full(1), C::NEW);
    mbar_init(dq_full, 1);
    mbar_init(dq_empty, 128);
    mbar_init(kv_done, 1);
    mbar_init(acc_free, C::NEW);
    mbar_init(rx_full, 1);
    mbar_init(tx_free, 128);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  cluster_sync();  // the partner's barriers are initialised before any remote arrive
  const uint32_t tmem = tmem_slot;

  if (skip) {
  } else if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (elect_one()) {
      tma_prefetch_desc(&mapQ);
      tma_prefetch_desc(&mapdO);
      bool ok = true;
      for (int item = cl, it = 0; ok && item < n_items; item += n_cl, ++it) {
        const Item w = item_of(item);
        // buffers free up in the order dK(g-3) < dV(g-2) < dK(g-2) < ..., so the
        // loads below are requested in the order they can be granted
        for (int j = 0; j < n_q; ++j) {
          const int g = it * n_q + j;
          const int s = g % C::QSTAGES, t = g % C::OSTAGES;
          if (g >= C::QSTAGES && !(ok = mbar_wait(q_empty(s), ((g / C::QSTAGES) - 1) & 1, status)))
            break;
          uint8_t* sq = sQ + s * C::QSTAGE_BYTES;
          mbar_arrive_expect_tx(q_full(s), C::QT_BYTES + C::EXT_BYTES);
          tma_load_4d(smem_u32(sq), &mapQ, q_full(s), 0, w.h, jq(w, j) * 128, w.b);
          bulk_load(smem_u32(sq + C::QT_BYTES),
                    ext + (static_cast<size_t>(w.bh) * n_q + jq(w, j)) * C::EXT_BYTES,
                    C::EXT_BYTES, q_full(s));
          if (g >= C::OSTAGES && !(ok = mbar_wait(o_empty(t), ((g / C::OSTAGES) - 1) & 1, status)))
            break;
          mbar_arrive_expect_tx(o_full(t), C::QT_BYTES);
          tma_load_4d(smem_u32(sO + t * C::QT_BYTES), &mapdO, o_full(t), 0, w.h, jq(w, j) * 128,
                      w.b);
          if (j == 0) {
            // K and V of this item, once every MMA of the previous item is done with them
            if (it > 0 && !(ok = mbar_wait(kv_done, (it - 1) & 1, status))) break;
            mbar_arrive_expect_tx(kv_full, 2 * C::KV_BYTES);
            tma_load_4d(smem_u32(sK), &mapK, kv_full, 0, w.h, w.k0, w.b);
            tma_load_4d(smem_u32(sV), &mapV, kv_full, 0, w.h, w.k0, w.b);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {
      constexpr uint32_t idSP = make_idesc(128, 128, 1, false, false);
      constexpr uint32_t idKV = make_idesc(128, 64, 1, false, true);  // A K-major, B MN-major
      constexpr uint32_t idQ = make_idesc(128, 64, 1, true, true);    // A and B MN-major
      const uint64_t dK_K = make_sdesc(smem_u32(sK), 16, 1024);
      const uint64_t dV_K = make_sdesc(smem_u32(sV), 16, 1024);
      const uint64_t dK_MN = make_sdesc(smem_u32(sK), C::CHUNK, 1024);
      const uint64_t dQ_K = make_sdesc(smem_u32(sQ), 16, 1024);
      const uint64_t dQ_MN = make_sdesc(smem_u32(sQ), C::CHUNK, 1024);
      const uint64_t dO_K = make_sdesc(smem_u32(sO), 16, 1024);
      const uint64_t dO_MN = make_sdesc(smem_u32(sO), C::CHUNK, 1024);
      const uint64_t dDS_MN = make_sdesc(smem_u32(sdS), C::CHUNK, 1024);  // dS, MN-major
      // extension tiles: K-major, no swizzle; K-halves 128 B apart, 8-row groups 256 B apart
      const uint64_t dOnesS = make_sdesc(smem_u32(sOnesS), 128, 0, 0);
      const uint64_t dOnesP = make_sdesc(smem_u32(sOnesP), 128, 0, 0);
      const uint64_t dExt = make_sdesc(smem_u32(sQ + C::QT_BYTES), 128, 256, 0);
      // g: query tile counted over all items (ring slots, dS buffer); j: within the item
      auto q_off = [&](int g) { return static_cast<uint32_t>(((g % C::QSTAGES) * C::QSTAGE_BYTES) >> 4); };
      auto o_off = [&](int g) { return static_cast<uint32_t>(((g % C::OSTAGES) * C::QT_BYTES) >> 4); };
      auto issue_S = [&](int g) {  // S'^T = K Q^T - LSE/scale
        const uint32_t so = q_off(g);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16_ss(tmem + C::T_S, dK_K + ((k * 32) >> 4), dQ_K + so + ((k * 32) >> 4), idSP,
                      k > 0 ? 1u : 0u);
        umma_f16_ss(tmem + C::T_S, dOnesS, dExt + so, idSP, 1u);
      };
      auto issue_dP = [&](int g) {  // dP'^T = V dO^T - Delta
        const uint32_t so = o_off(g);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16_ss(tmem + C::T_DP, dV_K + ((k * 32) >> 4), dO_K + so + ((k * 32) >> 4), idSP,
                      k > 0 ? 1u : 0u);
        umma_f16_ss(tmem + C::T_DP, dOnesP, dExt + q_off(g), idSP, 1u);
      };
      auto issue_dV = [&](int g, int j) {  // dV += P^T dO  (P^T from TMEM)
        const uint32_t so = o_off(g);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_f16_ts(tmem + C::T_DV, tmem + C::T_PT + 8 * k, dO_MN + so + ((k * 2048) >> 4), idKV,
                      (j > 0 || k > 0) ? 1u : 0u);
      };
      auto issue_dK = [&](int g, int j) {  // dK += dS^T Q  (dS^T packed over the dP columns)
        const uint32_t so = q_off(g);
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_f16_ts(tmem + C::T_DK, tmem + C::T_DP + 32 * (k / 2) + 8 * (k % 2),
                      dQ_MN + so + ((k * 2048) >> 4), idKV, (j > 0 || k > 0) ? 1u : 0u);
      };
      auto issue_dQ = [&](int g) {  // dQ = dS K
        const uint32_t bo = ((g & 1) * C::DS_BYTES) >> 4;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          umma_f16_ss(tmem + C::T_DQ, dDS_MN + bo + ((k * 2048) >> 4), dK_MN + ((k * 2048) >> 4), idQ,
                      k > 0 ? 1u : 0u);
      };
      bool ok = true;
      for (int item = cl, it = 0; ok && item < n_items; item += n_cl, ++it) {
        const int gb = it * n_q;
        ok = mbar_wait(kv_full, it & 1, status) &&
             mbar_wait(q_full(gb % C::QSTAGES), (gb / C::QSTAGES) & 1, status) &&
             mbar_wait(o_full(gb % C::OSTAGES), (gb / C::OSTAGES) & 1, status);
        if (!ok) break;
        tc_fence_after();
        issue_S(gb);
        umma_commit(s_full);
        issue_dP(gb);
        umma_commit(dp_full);
        for (int j = 0; ok && j < n_q; ++j) {
          const int g = gb + j;
          const bool more = j + 1 < n_q;
          if (!(ok = mbar_wait(s_free, g & 1, status))) break;
          if (more) {
            if (!(ok = mbar_wait(q_full((g + 1) % C::QSTAGES), ((g + 1) / C::QSTAGES) & 1, status)))
              break;
            tc_fence_after();
            issue_S(g + 1);
            umma_commit(s_full);
          }
          if (!(ok = mbar_wait(pt_full, g & 1, status))) break;
          // dV and dK restart from zero: the previous item's epilogue must have read them
          if (j == 0 && it > 0 && !(ok = mbar_wait(acc_free, (it - 1) & 1, status))) break;
          tc_fence_after();
          issue_dV(g, j);
          umma_commit(pt_free);
          umma_commit(o_empty(g % C::OSTAGES));
          if (!(ok = mbar_wait(p_full(g), (g >> 1) & 1, status))) break;
          tc_fence_after();
          issue_dK(g, j);  // reads dS^T(g) from the dP columns before dP(g+1) overwrites them
          umma_commit(q_empty(g % C::QSTAGES));
          if (more) {
            if (!(ok = mbar_wait(o_full((g + 1) % C::OSTAGES), ((g + 1) / C::OSTAGES) & 1, status)))
              break;
            tc_fence_after();
            issue_dP(g + 1);
            umma_commit(dp_full);
          }
          if (g > 0) {
            if (!(ok = mbar_wait(dq_empty, (g - 1) & 1, status))) break;
            tc_fence_after();
          }
          issue_dQ(g);
          umma_commit(dq_full);
        }
        if (ok) umma_commit(kv_done);  // K, V free; dV, dK final
      }
    }
  } else if (warp >= C::EW_WARP && warp < C::READOUT_WARP) {
    // ------------------------------------------------------------ P / dS
    // Warpgroup grp (four consecutive warps, one per TMEM lane quarter warp & 3):
    // queries [32 grp, 32 grp + 32) of each tile; thread = key row.
    const int grp = (warp - C::EW_WARP) >> 2;
    const int kr = ((warp & 3) << 5) + static_cast<int>(lane_id());  // key row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tS = tmem + C::T_S + lane_base + grp * C::QPG;
    const uint32_t tdP = tmem + C::T_DP + lane_base + grp * C::QPG;
    const uint32_t tPT = tmem + C::T_PT + lane_base + grp * C::QPG / 2;
    // this group's 32 queries: 64 bytes of a key row in dS chunk grp / 2, from byte 64 (grp % 2)
    const int dsb0 = 64 * (grp & 1);
    bool ok = true;
    for (int item = cl, it = 0; ok && item < n_items; item += n_cl, ++it) {
    const Item w = item_of(item);
    const int key = w.k0 + kr;
    const bool valid = key < L;
    const bool full_tile = w.k0 + 128 <= L;  // CTA-uniform: no key masking needed
    for (int j = 0; j < n_q; ++j) {
      const int g = it * n_q + j;
      // P phase
      if (!(ok = mbar_wait_warp(s_full, g & 1, status))) break;
      tc_fence_after();
      uint32_t va[16], vb[16];
      tmem_ld16x2_sync(tS, tS + 16, va, vb);
      tc_fence_before();
      mbar_arrive(s_free);
      float p[32];
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        p[e] = ex2(__uint_as_float(va[e]) * scale_log2);
        p[16 + e] = ex2(__uint_as_float(vb[e]) * scale_log2);
      }
      if (!full_tile && !valid) {
#pragma unroll
        for (int e = 0; e < 32; ++e) p[e] = 0.f;
      }
      uint32_t pk0[8], pk1[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        pk0[i] = pack_bf16x2(p[2 * i], p[2 * i + 1]);
        pk1[i] = pack_bf16x2(p[16 + 2 * i], p[16 + 2 * i + 1]);
      }
      if (g > 0) {  // P^T columns are free once the previous tile's dV MMA has read them
        if (!(ok = mbar_wait_warp(pt_free, (g - 1) & 1, status))) break;
        tc_fence_after();
      }
      PA_TMEM_ST_X8(tPT, pk0);
      PA_TMEM_ST_X8(tPT + 8, pk1);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(pt_full);
      // dS phase
      if (!(ok = mbar_wait_warp(dp_full, g & 1, status))) break;
      tc_fence_after();
      tmem_ld16x2_sync(tdP, tdP + 16, va, vb);
      uint32_t ds[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ds[i] = pack_bf16x2(p[2 * i] * __uint_as_float(va[2 * i]),
                            p[2 * i + 1] * __uint_as_float(va[2 * i + 1]));
        ds[8 + i] = pack_bf16x2(p[16 + 2 * i] * __uint_as_float(vb[2 * i]),
                                p[16 + 2 * i + 1] * __uint_as_float(vb[2 * i + 1]));
      }
      // dS^T packed over the first 16 of this group's 32 dP columns (read above)
      PA_TMEM_ST_X8(tdP, ds);
      PA_TMEM_ST_X8(tdP + 8, (ds + 8));
      uint8_t* dsrow = sdS + (g & 1) * C::DS_BYTES + (grp >> 1) * C::CHUNK;
#pragma unroll
      for (int u = 0; u < 4; ++u)
        *reinterpret_cast<uint4*>(dsrow + sw128_offset(kr, dsb0 + 16 * u)) =
            make_uint4(ds[4 * u], ds[4 * u + 1], ds[4 * u + 2], ds[4 * u + 3]);
      tmem_st_wait();
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(p_full(g));
    }
    // dV and dK (x scale) epilogue: groups 0, 1 write dV columns [0,32), [32,64);
    // groups 2, 3 the same columns of dK.
    if (!ok || !(ok = mbar_wait_warp(kv_done, it & 1, status))) break;
    {
      tc_fence_after();
      const bool is_dv = grp < 2;
      const int c = grp & 1;
      const int b = w.b, h = w.h;
      uint32_t o[32];
      tmem_ld32_sync(tmem + (is_dv ? C::T_DV : C::T_DK) + lane_base + c * 32, o);
      tc_fence_before();
      mbar_arrive(acc_free);  // the next item's first dV / dK MMAs may overwrite them
      if (valid && std::is_same<OutT, float>::value) {
        const float mul = is_dv ? 1.f : scale;
        float4* d4 = reinterpret_cast<float4*>((is_dv ? dv : dk) +
                                               ((static_cast<size_t>(b) * L + key) * H + h) * 64 +
                                               c * 32);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          float4 f = make_float4(__uint_as_float(o[4 * u]) * mul, __uint_as_float(o[4 * u + 1]) * mul,
                                 __uint_as_float(o[4 * u + 2]) * mul,
                                 __uint_as_float(o[4 * u + 3]) * mul);
          if (accumulate) {
            const float4 prev = d4[u];
            f.x += prev.x; f.y += prev.y; f.z += prev.z; f.w += prev.w;
          }
          d4[u] = f;
        }
      } else if (valid) {
        const float mul = is_dv ? 1.f : scale;
        OutT* dst =
            (is_dv ? dv : dk) + ((static_cast<size_t>(b) * L + key) * H + h) * 64 + c * 32;
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float f[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = __uint_as_float(o[8 * u + e]) * mul;
          if (accumulate) {
            const uint4 prev = d4[u];
            const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&prev);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 pf = __bfloat1622float2(p2[e]);
              f[2 * e] += pf.x;
              f[2 * e + 1] += pf.y;
            }
          }
          d4[u] = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                             pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
        }
      }
    }
    }  // item
  } else if (warp >= C::READOUT_WARP) {
    // ------------------------------------------------------------ dQ readout
    const int lane = static_cast<int>(lane_id());
    const int tid = threadIdx.x - 32 * C::READOUT_WARP;
    const int wl = (warp & 3) * 32;  // this warp's TMEM lanes (query rows) wl .. wl+31
    const uint32_t tdQ = tmem + C::T_DQ + (static_cast<uint32_t>(wl) << 16);
    const uint32_t rank = cluster_ctarank(), peer = rank ^ 1u;
    const uint32_t peer_slot = mapa_shared(smem_u32(sRX), peer) + tid * 16;
    const uint8_t* rx_slot = sRX + tid * 16;
    const uint32_t rx_full_peer = mapa_shared(rx_full, peer);
    const uint32_t tx_free_peer = mapa_shared(tx_free, peer);
    bool ok = true;
    for (int item = cl, it = 0; ok && item < n_items; item += n_cl, ++it) {
    const Item w = item_of(item);
    for (int j = 0; j < n_q; ++j) {
      const int g = it * n_q + j;
      if (!(ok = mbar_wait_warp(dq_full, g & 1, status))) break;
      // the partner has read what this CTA sent for the previous tile
      if (g > 0 && !(ok = mbar_wait_cluster_warp(tx_free, (g - 1) & 1, status))) break;
      if (tid == 0) mbar_arrive_expect_tx(rx_full, C::RX_BYTES);  // this tile's incoming bytes
      tc_fence_after();
      uint32_t own0[16], own1[16];
      {
        uint32_t r[32];
        tmem_ld_16x256b_x8_sync(tdQ, r);  // rows wl .. wl+15
        if (rank == 0) dq_split<0>(r, own0, peer_slot, rx_full_peer, 0);
        else dq_split<1>(r, own0, peer_slot, rx_full_peer, 0);
      }
      {
        uint32_t r[32];
        tmem_ld_16x256b_x8_sync(tdQ + (16u << 16), r);  // rows wl+16 .. wl+31
        tc_fence_before();
        mbar_arrive(dq_empty);  // dQ's TMEM columns are free for the next tile
        if (rank == 0) dq_split<0>(r, own1, peer_slot, rx_full_peer, 4);
        else dq_split<1>(r, own1, peer_slot, rx_full_peer, 4);
      }
      // add the partner's contribution to this CTA's columns, then reduce them
      if (!(ok = mbar_wait_cluster_warp(rx_full, g & 1, status))) break;
      dq_add_slots(own0, rx_slot, 0);
      dq_add_slots(own1, rx_slot, 4);
      // The partner may now overwrite sRX. The fence orders this thread's reads
      // of sRX before the arrive (a bare relaxed arrive may be issued before
      // those loads return); restricted to shared::cta accesses, it does not
      // wait for the reductions still in flight, as a full release would.
      fence_release_shared_cta_cluster();
      mbar_arrive_cluster_relaxed(tx_free_peer);
      float* row = dq_acc + (static_cast<size_t>(w.bh) * Lp + jq(w, j) * 128 + wl + (lane >> 2)) * 64 +
                   32 * rank + 2 * (lane & 3);
      dq_reduce_own(own0, row);
      dq_reduce_own(own1, row + 16 * 64);
    }
    }  // item
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no remote access into this CTA's shared memory after this point
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- dQ convert
// dq[b, l, h, :] (=|+=) scale * dq_acc[b*H + h, l, :]; 8 values per thread.
// D = row width of dq_acc; d_out (<= D, multiple of 8) = head dim of dq.
template <int D, typename OutT>
__global__ void __launch_bounds__(256)
    attn_dq_convert_kernel(const float* __restrict__ dq_acc, OutT* __restrict__ dq, int B, int L,
                           int Lp, int H, int d_out, float scale, int accumulate) {
  const size_t gt = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int G = d_out / 8;
  const size_t total = static_cast<size_t>(B) * L * H * G;
  if (gt >= total) return;
  const int g = static_cast<int>(gt % G);
  const size_t rowi = gt / G;  // (b, l, h)
  const int h = static_cast<int>(rowi % H);
  const int l = static_cast<int>((rowi / H) % L);
  const int b = static_cast<int>(rowi / (static_cast<size_t>(H) * L));
  const float* src = dq_acc + ((static_cast<size_t>(b) * H + h) * Lp + l) * D + g * 8;
  const float4 a = *reinterpret_cast<const float4*>(src);
  const float4 c = *reinterpret_cast<const float4*>(src + 4);
  float f[8] = {a.x * scale, a.y * scale, a.z * scale, a.w * scale,
                c.x * scale, c.y * scale, c.z * scale, c.w * scale};
  OutT* dst = dq + rowi * d_out + g * 8;
  if constexpr (sizeof(OutT) == 2) {
    uint4* d4 = reinterpret_cast<uint4*>(dst);
    if (accumulate) {
      const uint4 prev = *d4;
      const __nv_bfloat162* p2 = reinterpret_cast<const __nv_bfloat162*>(&prev);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 pf = __bfloat1622float2(p2[e]);
        f[2 * e] += pf.x;
        f[2 * e + 1] += pf.y;
      }
    }
    *d4 = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                     pack_bf16x2(f[6], f[7]));
  } else {
    float4* d4 = reinterpret_cast<float4*>(dst);
    if (accumulate) {
      const float4 p0 = d4[0], p1 = d4[1];
      f[0] += p0.x; f[1] += p0.y; f[2] += p0.z; f[3] += p0.w;
      f[4] += p1.x; f[5] += p1.y; f[6] += p1.z; f[7] += p1.w;
    }
    d4[0] = make_float4(f[0], f[1], f[2], f[3]);
    d4[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

// ---------------------------------------------------------------- host
namespace {
size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

// LSE2 [B*H, Lp], Delta [B*H, Lp], fp32 dQ accumulator [B*H*Lp, Dacc], and
// with `ext` the extension tiles [B*H, Lp/128, 8 KB] of the head-dim-64 kernel.
size_t stats_bytes(const AttnShape& sh, int Dacc, bool ext = false) {
  const size_t Lp = static_cast<size_t>((sh.L + 127) / 128) * 128;
  const size_t bh = static_cast<size_t>(sh.B) * sh.H;
  return up256(bh * Lp * 4) * 2 + up256(bh * Lp * Dacc * 4) +
         (ext ? bh * (Lp / 128) * kExtTileBytes : 0);
}

// Delta (and LSE2, extension tiles, the zeroed dQ accumulator) prep over rows
// of `Dreal` values of type InT: one block per (batch*head, 128-row tile).
// Lp: row pitch of the [B*H, Lp] outputs (a multiple of 128 for the backward;
// L for Delta alone, where only rows < L are written).
template <int Dreal, typename InT>
int launch_prep(const AttnShape& sh, const void* dO, const void* o, const float* lse, float* lse2,
                float* delta_t, float* delta_ref, uint8_t* ext, float* dq_zero, int dq_width, int Lp,
                cudaStream_t stream) {
  const dim3 grid(static_cast<unsigned>((Lp + 127) / 128), static_cast<unsigned>(sh.B * sh.H));
  attn_bwd_prep_kernel<Dreal, InT><<<grid, 128, 0, stream>>>(
      static_cast<const InT*>(dO), static_cast<const InT*>(o), lse, lse2, delta_t, delta_ref, ext,
      dq_zero, dq_width, 1.f / sh.scale, sh.L, Lp, sh.H);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

template <typename InT>
int prep_any(int Dreal, const AttnShape& sh, const void* dO, const void* o, const float* lse,
             float* lse2, float* delta_t, float* delta_ref, int Lp, cudaStream_t stream,
             uint8_t* ext = nullptr, float* dq_zero = nullptr, int dq_width = 0) {
  switch (Dreal) {
    case 32:
      return launch_prep<32, InT>(sh, dO, o, lse, lse2, delta_t, delta_ref, ext, dq_zero, dq_width,
                                  Lp, stream);
    case 64:
      return launch_prep<64, InT>(sh, dO, o, lse, lse2, delta_t, delta_ref, ext, dq_zero, dq_width,
                                  Lp, stream);
    case 128:
      return launch_prep<128, InT>(sh, dO, o, lse, lse2, delta_t, delta_ref, ext, dq_zero, dq_width,
                                   Lp, stream);
    default: return PA_ERR_UNSUPPORTED;
  }
}

// Runs prep + main + dQ convert. m[0..3] = hi (or only) maps of q, k, v, dO;
// m[4..7] = lo maps (SPLIT). sh.D = d_out (true head dim); D = MMA head dim.
template <int D, bool SPLIT, typename T>
int run_bwd(const AttnShape& sh, const CUtensorMap* m, const void* o, const void* dO,
            const float* lse, void* dq, void* dk, void* dv, int accumulate, uint8_t* stats,
            uint32_t* status, cudaStream_t stream) {
  using C = BwdCfg<D, SPLIT>;
  const int Lp = (sh.L + 127) / 128 * 128;
  const size_t bh = static_cast<size_t>(sh.B) * sh.H;
  float* lse2 = reinterpret_cast<float*>(stats);
  float* delta_t = reinterpret_cast<float*>(stats + up256(bh * Lp * 4));
  float* dq_acc = reinterpret_cast<float*>(stats + 2 * up256(bh * Lp * 4));
  // dQ accumulator [B*H*Lp, D] fp32, reduced into by 128-row x 32-column boxes.
  CUtensorMap mdq;
  const uint64_t dims[2] = {static_cast<uint64_t>(D), bh * Lp};
  const uint64_t strides[1] = {static_cast<uint64_t>(D) * 4};
  const uint32_t box[2] = {32, 128};
  if (!make_tmap(&mdq, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, dq_acc, dims, strides, box,
                 CU_TENSOR_MAP_SWIZZLE_128B))
    return PA_ERR_ALIGN;
  // the prep kernel also zeroes the dQ accumulator [B*H*Lp, D]
  constexpr bool kD64 = D == 64 && !SPLIT;
  uint8_t* ext = kD64 ? stats + 2 * up256(bh * Lp * 4) + up256(bh * Lp * D * 4) : nullptr;
  int st = kD64 ? prep_any<T>(sh.D, sh, dO, o, lse, nullptr, nullptr, nullptr, Lp, stream, ext,
                              dq_acc, D)
                : prep_any<T>(sh.D, sh, dO, o, lse, lse2, delta_t, nullptr, Lp, stream, nullptr,
                              dq_acc, D);
  if (st != PA_OK) return st;

  dim3 grid((sh.L + 127) / 128, static_cast<unsigned>(bh));
  if constexpr (D == 64 && !SPLIT) {
    using C64 = Bwd64Cfg;
    static std::atomic<uint64_t> attr64{0};
    if (!ensure_smem_attr(attn_bwd_d64_kernel<T>, C64::SMEM, attr64)) return PA_ERR_LAUNCH;
    // Persistent clusters of two CTAs, as many as fit on the device at once;
    // work items are (batch*head, pair of adjacent key tiles; a tile past L
    // has no keys).
    const int n_pairs = (static_cast<int>(grid.x) + 1) / 2;
    const int n_items = n_pairs * static_cast<int>(bh);
    const int dev = current_device();
    if (dev < 0) return PA_ERR_DEVICE;
    static std::atomic<int> max_clusters[kMaxDevices];
    const int mc = cached_per_device(max_clusters, dev, [] {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(2 * 4096, 1, 1);
      cfg.blockDim = dim3(C64::THREADS, 1, 1);
      cfg.dynamicSmemBytes = C64::SMEM;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, attn_bwd_d64_kernel<T>, &cfg) != cudaSuccess || n <= 0) {
        cudaGetLastError();  // clear a failed query; fall back to one cluster per two SMs
        n = device_sm_count() / 2;
      }
      return n;
    });
    const int n_cl = n_items < mc ? n_items : mc;
    attn_bwd_d64_kernel<T><<<dim3(2 * n_cl, 1, 1), C64::THREADS, C64::SMEM, stream>>>(
        m[0], m[1], m[2], m[3], dq_acc, static_cast<T*>(dk), static_cast<T*>(dv), ext, sh.L, Lp,
        sh.H, sh.scale, sh.scale * kLog2e, accumulate, n_pairs, n_items, status);
  } else {
    static std::atomic<uint64_t> attr{0};
    if (!ensure_smem_attr(attn_bwd_kernel<D, SPLIT, T>, C::SMEM, attr)) return PA_ERR_LAUNCH;
    attn_bwd_kernel<D, SPLIT, T><<<grid, 512, C::SMEM, stream>>>(
        m[0], m[1], m[2], m[3], m[4], m[5], m[6], m[7], mdq, static_cast<T*>(dk),
        static_cast<T*>(dv), lse2, delta_t, sh.L, Lp, sh.H, sh.D, sh.scale, sh.scale * kLog2e,
        accumulate, status);
  }
  if (cudaGetLastError() != cudaSuccess) return PA_ERR_LAUNCH;

  const size_t threads = static_cast<size_t>(sh.B) * sh.L * sh.H * (sh.D / 8);
  attn_dq_convert_kernel<D, T><<<static_cast<unsigned>((threads + 255) / 256), 256, 0, stream>>>(
      dq_acc, static_cast<T*>(dq), sh.B, sh.L, Lp, sh.H, sh.D, sh.scale, accumulate);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}
}  // namespace

size_t attn_bwd_workspace_bytes(const AttnShape& sh) { return stats_bytes(sh, sh.D, sh.D == 64); }

int launch_attn_delta_bf16(const AttnShape& sh, const void* dO, const void* o, float* delta,
                           cudaStream_t stream) {
  if (sh.D != 64 && sh.D != 128) return PA_ERR_UNSUPPORTED;
  return prep_any<__nv_bfloat16>(sh.D, sh, dO, o, nullptr, nullptr, nullptr, delta, sh.L, stream);
}

int launch_attn_bwd_bf16(const AttnShape& sh, const void* q, const void* k, const void* v,
                         const void* o, const void* dO, const float* lse, void* dq, void* dk,
                         void* dv, int accumulate, void* ws, uint32_t* status, cudaStream_t stream) {
  CUtensorMap m[8];
  if (!make_qkv_map(&m[0], q, sh, 128) || !make_qkv_map(&m[1], k, sh, 128) ||
      !make_qkv_map(&m[2], v, sh, 128) || !make_qkv_map(&m[3], dO, sh, 128))
    return PA_ERR_ALIGN;
  for (int i = 0; i < 4; ++i) m[4 + i] = m[i];
  uint8_t* w = static_cast<uint8_t*>(ws);
  if (sh.D == 64)
    return run_bwd<64, false, __nv_bfloat16>(sh, m, o, dO, lse, dq, dk, dv, accumulate, w, status,
                                              stream);
  if (sh.D == 128)
    return run_bwd<128, false, __nv_bfloat16>(sh, m, o, dO, lse, dq, dk, dv, accumulate, w, status,
                                               stream);
  return PA_ERR_UNSUPPORTED;
}

// fp32 path: bf16 hi/lo planes of q, k, v, dO (head dim padded to 64), then
// the statistics block.
// (The bf16 math mode uses the hi planes only, plus the key-extension tiles
// of the d64 kernel; the size covers both modes.)
size_t attn_bwd_workspace_bytes_f32(const AttnShape& sh) {
  const int Dp = f32_plane_dim(sh.D);
  if (Dp < 0) return 0;
  const size_t plane = up256(static_cast<size_t>(sh.B) * sh.L * sh.H * Dp * 2);
  return 8 * plane + stats_bytes(sh, Dp, sh.D == 64);
}

// kept: the forward's workspace (launch_attn_fwd_f32), which holds the planes
// of q, k, v in the same layout as planes 0-5 here (hi of operand i at 2i, lo
// at 2i + 1); then only dO is converted. kept_lo: it holds the lo planes too.
int launch_attn_bwd_f32(const AttnShape& sh, const void* q, const void* k, const void* v,
                        const void* o, const void* dO, const float* lse, void* dq, void* dk,
                        void* dv, int accumulate, void* ws, uint32_t* status, cudaStream_t stream,
                        const void* kept, bool kept_lo) {
  const int Dp = f32_plane_dim(sh.D);
  if (Dp != 64) return PA_ERR_UNSUPPORTED;
  const size_t rows = static_cast<size_t>(sh.B) * sh.L * sh.H;
  const size_t plane = up256(rows * Dp * 2);
  uint8_t* w = static_cast<uint8_t*>(ws);
  const float* src[4] = {static_cast<const float*>(q), static_cast<const float*>(k),
                         static_cast<const float*>(v), static_cast<const float*>(dO)};
  AttnShape ps = sh;
  ps.D = Dp;
  CUtensorMap m[8];
  const bool bf16_math = sh.D == 64 && f32_math() == PA_F32_MATH_BF16;
  // planes of operand i: from the forward's kept workspace (q, k, v) or converted here
  uint8_t* kp = const_cast<uint8_t*>(static_cast<const uint8_t*>(kept));
  const bool use_kept = kp && (bf16_math || kept_lo);
  auto planes_of = [&](int i) { return (use_kept && i < 3 ? kp : w) + (2 * i) * plane; };
  if (bf16_math) {
    // one bf16 plane per operand, the bf16 d64 kernel with fp32 dK / dV
    for (int i = 0; i < 4; ++i) {
      uint8_t* hi = planes_of(i);
      if (!(use_kept && i < 3)) {
        const int st = launch_split_planes(src[i], hi, nullptr, rows, sh.D, Dp, stream);
        if (st != PA_OK) return st;
      }
      if (!make_qkv_map(&m[i], hi, ps, 128)) return PA_ERR_ALIGN;
      m[4 + i] = m[i];
    }
    return run_bwd<64, false, float>(sh, m, o, dO, lse, dq, dk, dv, accumulate, w + 8 * plane,
                                     status, stream);
  }
  for (int i = 0; i < 4; ++i) {
    uint8_t* hi = planes_of(i);
    uint8_t* lo = hi + plane;
    if (!(use_kept && i < 3)) {
      const int st = launch_split_planes(src[i], hi, lo, rows, sh.D, Dp, stream);
      if (st != PA_OK) return st;
    }
    if (!make_qkv_map(&m[i], hi, ps, 128) || !make_qkv_map(&m[4 + i], lo, ps, 128))
      return PA_ERR_ALIGN;
  }
  return run_bwd<64, true, float>(sh, m, o, dO, lse, dq, dk, dv, accumulate, w + 8 * plane, status,
                                  stream);
}

int launch_attn_delta_f32(const AttnShape& sh, const void* dO, const void* o, float* delta,
                          cudaStream_t stream) {
  if (sh.D != 32 && sh.D != 64) return PA_ERR_UNSUPPORTED;
  return prep_any<float>(sh.D, sh, dO, o, nullptr, nullptr, nullptr, delta, sh.L, stream);
}

}  // namespace pa
