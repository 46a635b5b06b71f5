// tcgen05 GEMM for the projection forward and the matmul gradients (fp32 in/out).
//
// Restates the reference's three tiled fp32 GEMMs:
//   mode 0  C[M,N]   = A[M,K] B[K,N]      matmul_kernel.cu:4-50
//   mode 1  dX[M,N] += dY[M,K] W[N,K]^T   matmul_backward_X_kernel.cu:5-54
//   mode 2  dW[N,K] += X[M,N]^T dY[M,K]   matmul_backward_W_kernel.cu:5-55
// on the bf16 tensor cores at fp32-level accuracy: each fp32 operand is split
// into bf16 hi/lo planes in the caller's workspace (fp32_split.cu) and every
// product is hi*hi + hi*lo + lo*hi, three MMAs into one fp32 TMEM accumulator
// (in the bf16 math mode, pa_set_f32_math, only the hi planes and one MMA).
//
// The transposes of the gradients cost nothing: a row-major operand whose
// reduction index is the row index is simply fed as an MN-major tcgen05
// operand, so each mode reads its inputs in place.
//
// The projection layer built on it (launch_linear_fwd / _bwd) fuses what the
// reference does in separate passes around each projection
// (Functional.cpp:12-52 matmul, matadd_kernel.cu bias add, split_forward_kernel.cu
// and its adjoint, sum_rows_grad_kernel.cu): the forward epilogue adds the
// bias and writes the output as up to three column blocks (Q, K, V of the
// attention in-projection) to separate tensors; the backward gathers the
// column-block gradients straight into one pair of bf16 planes, shared by
// the dX and dW GEMMs. A projection followed by a ReLU (the feed-forward's
// first layer) clamps in the same epilogue, and its backward masks the
// incoming gradient by the saved output while gathering it (no ReLU passes,
// no pre-activation tensor).
//
// Persistent clusters of two CTAs (one MMA unit, tcgen05 cta_group::2) walk
// 256 x 256 output tiles (work units: tiles, or tiles x K slices for
// accumulating GEMMs that would fill the GPU badly); K in blocks of 64
// through a TMA ring of bf16 planes; the fp32 accumulator is double-buffered
// in TMEM so the epilogue of one unit overlaps the MMAs of the next; the
// epilogue stages 128 x 32 chunks in shared memory for TMA stores or TMA
// add-reductions. In each CTA:
//   warp 0     TMA producer (its own 128 rows of A, 128 columns of B)
//   warp 1     TMEM allocator; in the even CTA also the MMA issuer
//   warps 4-7  epilogue: TMEM -> registers (+ bias, ReLU) -> shared -> TMA
#include <cuda_bf16.h>
#include "host_launchers.h"

namespace pa {

namespace {

constexpr int GB = 128;          // output tile rows (the tile is GB x PB_N)
constexpr int GK = 64;           // K block (one 128-byte swizzle row of bf16)

// Output tiles are 256 x 256 (a CTA pair) walked by persistent pairs; K in
// blocks of 64. The fp32 accumulator is double-buffered in TMEM (2 x 256
// columns per CTA): the epilogue warps drain unit i while the MMAs accumulate
// unit i + 1. Epilogue with tma_out: each 128 x 32 chunk is staged in shared
// memory (128-byte swizzled, two buffers) and written by one TMA store - or,
// when accumulating, one TMA add-reduction - per chunk, so the stores are
// whole 128-byte row segments instead of one row per thread. Without tma_out
// (unaligned outputs, column blocks not multiples of 32) each thread stores
// its own row. The bias of the tile's 256 columns is staged in shared memory
// once per tile.
constexpr int PB_N = 256;              // output tile columns
constexpr int PB_A = GB * GK * 2;      // 16 KB: one A plane of one stage (128 rows)
constexpr int PB_STG = 128 * 32 * 4;   // one 128-row x 32-column fp32 output chunk (16 KB)

// ---------------------------------------------------------------- paired GEMM
// Two CTAs of a cluster act as one MMA unit (tcgen05 cta_group::2) on a
// 256 x 256 output tile: per K block each CTA loads its 128 rows of A and its
// 128 of the tile's 256 columns of B, and the even CTA's MMAs (M=256 N=256
// K=16) read both CTAs' shared memory and leave each CTA's 128 output rows in
// its own TMEM. Per SM that is 32 KB of operands per K block for the MMA work
// the one-CTA 128 x 256 tile needs 48 KB for, so the same shared memory holds
// a ring half again as deep in time (6 stages in bf16 math, 3 of hi/lo planes
// in split3) and the L2 reads per FLOP drop by a third. Both CTAs' TMA loads
// count towards the even CTA's full barrier (cta_group::2 loads: no
// multicast, each CTA fetches its own tiles); one commit, multicast to both
// CTAs, frees a stage in both, and another hands an accumulator to both
// epilogues, which report back to the even CTA (4 warps each).
constexpr int PP_BH = 128 * GK * 2;  // 16 KB: this CTA's 128 columns of one B plane
template <int NT>
struct PairCfg {
  static constexpr int NP = NT == 3 ? 2 : 1;
  static constexpr int STAGE = NP * (PB_A + PP_BH);
  static constexpr int STAGES = NT == 3 ? 3 : 6;
  static constexpr int SMEM = STAGES * STAGE + 2 * PB_STG + 1024;
};

template <bool A_MN, bool B_MN, int NT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(256, 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap mA, const __grid_constant__ CUtensorMap mAl,
                     const __grid_constant__ CUtensorMap mB, const __grid_constant__ CUtensorMap mBl,
                     const __grid_constant__ CUtensorMap mC0, const __grid_constant__ CUtensorMap mC1,
                     const __grid_constant__ CUtensorMap mC2, int tma_out, int ksplit,
                     float* __restrict__ C, int ldc, int Mout, int Nout, int Kred, int accumulate,
                     const float* __restrict__ bias, float* __restrict__ C1, float* __restrict__ C2,
                     int nsplit, int relu, int n_fast, __nv_bfloat16* __restrict__ yp_hi,
                     __nv_bfloat16* __restrict__ yp_lo, int yp_ld, uint32_t* status) {
  using P = PairCfg<NT>;
  constexpr int ST = P::STAGES, STG = P::STAGE, NP = P::NP;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bars[2 * ST + 4];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ __align__(16) float bias_s[PB_N];  // the current tile's bias (0 past Nout)
  // No early return: both CTAs must take part in the paired TMEM allocation
  // and the cluster barriers. A status word set by an earlier failure skips
  // the work loops (a pair that disagrees on it ends in bounded waits).
  const bool skip = cta_aborted(status, &abort_flag);
  uint8_t* smem = align1024(smem_raw);
  const uint32_t rank = cluster_ctarank();
  const bool even = rank == 0;
  auto full = [&](int s) { return smem_u32(&bars[s]); };
  auto empty = [&](int s) { return smem_u32(&bars[ST + s]); };
  auto acc_full = [&](int b) { return smem_u32(&bars[2 * ST + b]); };
  auto acc_empty = [&](int b) { return smem_u32(&bars[2 * ST + 2 + b]); };  // the even CTA's
  const int warp = warp_id();
  const int tiles_m = (Mout + 2 * GB - 1) / (2 * GB);
  const int tiles_n = (Nout + PB_N - 1) / PB_N;
  const int units = tiles_m * tiles_n * ksplit;
  // Tile order: consecutive units (which run at the same time) share the
  // operand indexed by the slow index, so with n_fast the A rows of a tile
  // come from DRAM once and serve its column tiles from L2 (A the larger
  // operand); else the B columns do.
  auto tile_m = [&](int tile) { return n_fast ? tile / tiles_n : tile % tiles_m; };
  auto tile_n = [&](int tile) { return n_fast ? tile % tiles_n : tile / tiles_m; };
  const int nk_all = (Kred + GK - 1) / GK;
  const int cl = static_cast<int>(blockIdx.x) / 2, ncl = static_cast<int>(gridDim.x) / 2;
  auto kslice = [&](int u, int& kb0, int& kb1) {
    const int sl = u % ksplit;
    kb0 = static_cast<int>((static_cast<long long>(nk_all) * sl) / ksplit);
    kb1 = static_cast<int>((static_cast<long long>(nk_all) * (sl + 1)) / ksplit);
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < ST; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 8);  // lane 0 of the four epilogue warps of both CTAs
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(&tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem = tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (!skip && elect_one()) {
      int g = 0;  // k-blocks loaded so far: ring slot and phase
      bool ok = true;
      for (int u = cl; ok && u < units; u += ncl) {
        const int tile = u / ksplit;
        const int m0 = tile_m(tile) * 2 * GB + static_cast<int>(rank) * GB;
        const int n0 = tile_n(tile) * PB_N + static_cast<int>(rank) * 128;
        int kb0, kb1;
        kslice(u, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = g % ST;
          // both CTAs' MMAs on this slot are done (the commit reaches both)
          if (g >= ST && !(ok = mbar_wait(empty(s), ((g / ST) - 1) & 1, status))) break;
          if (even) mbar_arrive_expect_tx(full(s), 2 * STG);
          const uint32_t bar = mapa_shared(full(s), 0);
          const uint32_t st0 = smem_u32(smem + s * STG);
#pragma unroll
          for (int pl = 0; pl < NP; ++pl) {
            const uint32_t da = st0 + pl * PB_A, db = st0 + NP * PB_A + pl * PP_BH;
            const CUtensorMap* ma = pl ? &mAl : &mA;
            const CUtensorMap* mb = pl ? &mBl : &mB;
            if (A_MN) {  // two 64-wide M groups of 64 K rows
              tma_load_2d_pair(da, ma, bar, m0, kb * GK);
              tma_load_2d_pair(da + PB_A / 2, ma, bar, m0 + 64, kb * GK);
            } else {
              tma_load_2d_pair(da, ma, bar, kb * GK, m0);
            }
            if (B_MN) {  // two 64-wide N groups of 64 K rows
              tma_load_2d_pair(db, mb, bar, n0, kb * GK);
              tma_load_2d_pair(db + PP_BH / 2, mb, bar, n0 + 64, kb * GK);
            } else {
              tma_load_2d_pair(db, mb, bar, kb * GK, n0);
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (even && !skip && elect_one()) {
      constexpr uint32_t idesc = make_idesc(2 * GB, PB_N, 1, A_MN, B_MN);
      const uint32_t s0 = smem_u32(smem);
      int g = 0, it = 0;
      bool ok = true;
      for (int u = cl; ok && u < units; u += ncl, ++it) {
        const int b = it & 1;
        int kb0, kb1;
        kslice(u, kb0, kb1);
        // both epilogues have drained this accumulator buffer (unit it - 2)
        if (it >= 2 && !(ok = mbar_wait_cluster(acc_empty(b), ((it >> 1) - 1) & 1, status))) break;
        tc_fence_after();
        const uint32_t d = tmem + b * PB_N;
        for (int kb = kb0; kb < kb1; ++kb, ++g) {
          const int s = g % ST;
          if (!(ok = mbar_wait_cluster(full(s), (g / ST) & 1, status))) break;
          tc_fence_after();
#pragma unroll
          for (int term = 0; term < NT; ++term) {
            // planes (A, B) of each term: (hi, hi), (hi, lo), (lo, hi)
            const uint32_t sa = s0 + s * STG + (term == 2 ? PB_A : 0);
            const uint32_t sb = s0 + s * STG + NP * PB_A + (term == 1 ? PP_BH : 0);
#pragma unroll
            for (int ks = 0; ks < GK / 16; ++ks) {
              const uint64_t da = A_MN ? make_sdesc(sa + ks * 2048, PB_A / 2, 1024)
                                       : make_sdesc(sa + ks * 32, 16, 1024);
              const uint64_t db = B_MN ? make_sdesc(sb + ks * 2048, PP_BH / 2, 1024)
                                       : make_sdesc(sb + ks * 32, 16, 1024);
              umma_f16_ss_pair(d, da, db, idesc, (kb > kb0 || term > 0 || ks > 0) ? 1u : 0u);
            }
          }
          umma_commit_pair(empty(s));
        }
        if (ok) umma_commit_pair(acc_full(b));
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int r = threadIdx.x - 128;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const bool leader = threadIdx.x == 128;
    uint8_t* stg = smem + ST * STG;
    int q = 0;  // staged chunks so far (buffer q & 1)
    int it = 0;
    for (int u = cl; !skip && u < units; u += ncl, ++it) {
      const int tile = u / ksplit;
      const int b = it & 1;
      bool ok = mbar_wait_cluster_warp(acc_full(b), (it >> 1) & 1, status);
      ok = named_bar_and(1, 128, ok);  // the four warps leave together
      if (!ok) break;
      tc_fence_after();
      const int row0 = tile_m(tile) * 2 * GB + static_cast<int>(rank) * GB;
      const int row = row0 + r, n0 = tile_n(tile) * PB_N;
      if (bias) {
        // every thread is past the previous tile's reads of bias_s (the barrier
        // above), so it can be refilled; the barrier below publishes it
#pragma unroll
        for (int h = 0; h < PB_N / 128; ++h) {
          const int col = n0 + r + 128 * h;
          bias_s[r + 128 * h] = col < Nout ? bias[col] : 0.f;
        }
        named_bar_sync(1, 128);
      }
      // Output column `col` goes to C[row * ldc + col], or with nsplit > 0 to
      // part p = col / nsplit (C, C1, C2) at [row * nsplit + col - p * nsplit].
      auto dst_of = [&](int col) -> float* {
        if (nsplit <= 0) return C + static_cast<size_t>(row) * ldc + col;
        const int p = col / nsplit;
        float* base = p == 0 ? C : (p == 1 ? C1 : C2);
        return base + static_cast<size_t>(row) * nsplit + (col - p * nsplit);
      };
#pragma unroll 1
      for (int c = 0; c < PB_N / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + b * PB_N + c * 32 + lane_base, v);
        tmem_ld_wait();
        if (c == PB_N / 32 - 1) {  // the buffer is free for tile it + 2 (in both CTAs)
          tc_fence_before();
          __syncwarp();
          if (lane_id() == 0) mbar_arrive_cluster(mapa_shared(acc_empty(b), 0));
        }
        const int col0 = n0 + c * 32;
        // this row's 32 values of the chunk, with the bias and the ReLU
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          float4 f = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                 __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
          if (bias) {
            const float4 bb = reinterpret_cast<const float4*>(bias_s)[c * 8 + e];
            f.x += bb.x; f.y += bb.y; f.z += bb.z; f.w += bb.w;
          }
          if (relu) {
            f.x = fmaxf(f.x, 0.f); f.y = fmaxf(f.y, 0.f);
            f.z = fmaxf(f.z, 0.f); f.w = fmaxf(f.w, 0.f);
          }
          v[4 * e] = __float_as_uint(f.x); v[4 * e + 1] = __float_as_uint(f.y);
          v[4 * e + 2] = __float_as_uint(f.z); v[4 * e + 3] = __float_as_uint(f.w);
        }
        // the output's bf16 operand planes (hi = bf16(y), lo = bf16(y - hi)), for a
        // projection that reads this output next: 64 contiguous bytes per row
        if (yp_hi && row < Mout && col0 < Nout) {
          __nv_bfloat16* ph = yp_hi + static_cast<size_t>(row) * yp_ld + col0;
          __nv_bfloat16* pl = yp_lo ? yp_lo + static_cast<size_t>(row) * yp_ld + col0 : nullptr;
          if (col0 + 32 <= Nout) {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              uint32_t h[4], l[4];
#pragma unroll
              for (int k = 0; k < 4; ++k) {
                const float a = __uint_as_float(v[8 * e + 2 * k]);
                const float b2 = __uint_as_float(v[8 * e + 2 * k + 1]);
                h[k] = pack_bf16x2(a, b2);
                l[k] = pack_bf16x2(a - __uint_as_float(h[k] << 16),
                                   b2 - __uint_as_float(h[k] & 0xffff0000u));
              }
              reinterpret_cast<uint4*>(ph)[e] = make_uint4(h[0], h[1], h[2], h[3]);
              if (pl) reinterpret_cast<uint4*>(pl)[e] = make_uint4(l[0], l[1], l[2], l[3]);
            }
          } else {
#pragma unroll
            for (int e = 0; e < 32; ++e) {  // constant indices: v stays in registers
              if (col0 + e < Nout) {
                const float a = __uint_as_float(v[e]);
                const __nv_bfloat16 h = __float2bfloat16_rn(a);
                ph[e] = h;
                if (pl) pl[e] = __float2bfloat16_rn(a - __bfloat162float(h));
              }
            }
          }
        }
        if (tma_out) {
          // uniform over the epilogue warps (an odd CTA past the last row stores nothing)
          if (col0 >= Nout || row0 >= Mout) continue;
          const int buf = q++ & 1;
          if (leader) bulk_wait_read<1>();  // the store of two chunks ago has read this buffer
          named_bar_sync(1, 128);
          uint8_t* srow = stg + buf * PB_STG;
#pragma unroll
          for (int e = 0; e < 8; ++e)
            *reinterpret_cast<uint4*>(srow + sw128_offset(r, 16 * e)) =
                make_uint4(v[4 * e], v[4 * e + 1], v[4 * e + 2], v[4 * e + 3]);
          fence_proxy_async_smem();
          named_bar_sync(1, 128);
          if (leader) {
            const int p = nsplit > 0 ? col0 / nsplit : 0;
            const CUtensorMap* map = p == 0 ? &mC0 : (p == 1 ? &mC1 : &mC2);
            const int x = col0 - p * (nsplit > 0 ? nsplit : 0);
            if (accumulate)
              tma_reduce_add_2d(map, smem_u32(srow), x, row0);
            else
              tma_store_2d(map, smem_u32(srow), x, row0);
            tma_store_commit();
          }
          continue;
        }
        if (row >= Mout || col0 >= Nout) continue;
        float* dst = dst_of(col0);
        const bool one_part = nsplit <= 0 || (col0 % nsplit) + 32 <= nsplit;
        const int ld = nsplit > 0 ? nsplit : ldc;
        const bool vec = (col0 + 32 <= Nout) && one_part && ((ld & 3) == 0) &&
                         ((reinterpret_cast<uintptr_t>(dst) & 15u) == 0);
        if (vec) {
          float4* d4 = reinterpret_cast<float4*>(dst);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            float4 f = make_float4(__uint_as_float(v[4 * e]), __uint_as_float(v[4 * e + 1]),
                                   __uint_as_float(v[4 * e + 2]), __uint_as_float(v[4 * e + 3]));
            if (accumulate) {
              const float4 p = d4[e];
              f.x += p.x; f.y += p.y; f.z += p.z; f.w += p.w;
            }
            d4[e] = f;
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int col = col0 + e;
            if (col < Nout) {
              float* de = dst_of(col);
              *de = __uint_as_float(v[e]) + (accumulate ? *de : 0.f);
            }
          }
        }
      }
    }
    if (leader) bulk_wait_all();  // staged chunks fully written before the CTA ends
  }
  tc_fence_before();
  cluster_sync();  // the other CTA no longer reaches into this one's barriers or TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }
int round8(int x) { return (x + 7) & ~7; }

// Bytes of the hi + lo planes of a [rows, cols] fp32 operand (rows padded to 8 columns).
size_t planes_bytes(int rows, int cols) {
  return 2 * up256(static_cast<size_t>(rows) * round8(cols) * 2);
}

// 2-D TMA map over a bf16 plane of `rows` x `cols` (row pitch round8(cols)).
// K-major operand: box {64 cols, 128 rows}; MN-major operand: box {64, 64}.
bool plane_map(CUtensorMap* m, const void* base, int rows, int cols, bool mn,
               uint32_t kmajor_rows = 128) {
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(round8(cols)) * 2};
  const uint32_t box[2] = {64, mn ? 64u : kmajor_rows};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

struct Epilogue {
  const float* bias = nullptr;
  float* c1 = nullptr;
  float* c2 = nullptr;
  int nsplit = 0;
  int relu = 0;  // max(0, .) after the bias (forward projections only)
  // the output's bf16 planes as well (lo: split3 only; row pitch round8(Nout)),
  // for a single-output forward projection
  void* y_hi = nullptr;
  void* y_lo = nullptr;
};

// fp32 [rows, cols] output with row pitch ld, as 128-row x 32-column TMA boxes.
bool out_map(CUtensorMap* m, const float* base, int rows, int cols, int ld) {
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(ld) * 4};
  const uint32_t box[2] = {32, 128};
  return make_tmap(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box,
                   CU_TENSOR_MAP_SWIZZLE_128B);
}

// The paired kernel: the same work units over 256-row tiles, one CTA pair per
// two SMs (as many pairs as the device holds at once).
template <bool A_MN, bool B_MN, int NT>
int run_gemm_pair(const CUtensorMap* m, float* C, int ldc, int Mout, int Nout, int Kred,
                  int accumulate, const Epilogue& ep, uint32_t* status, cudaStream_t s) {
  const CUtensorMap& mA = m[0];
  static std::atomic<uint64_t> attr{0};
  if (!ensure_smem_attr(gemm_pair_kernel<A_MN, B_MN, NT>, PairCfg<NT>::SMEM, attr))
    return PA_ERR_LAUNCH;
  CUtensorMap mc[3];
  const bool al = [&] {
    auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
    if (ep.nsplit > 0) {
      const int parts = Nout / ep.nsplit;
      if (ep.nsplit % 32 != 0 || Nout % ep.nsplit != 0 || parts > 3) return false;
      float* outs[3] = {C, ep.c1, ep.c2};
      for (int p = 0; p < parts; ++p)
        if (!outs[p] || !a16(outs[p]) || !out_map(&mc[p], outs[p], Mout, ep.nsplit, ep.nsplit))
          return false;
      for (int p = parts; p < 3; ++p) mc[p] = mc[0];
      return true;
    }
    if (ldc % 4 != 0 || !a16(C) || !out_map(&mc[0], C, Mout, Nout, ldc)) return false;
    mc[1] = mc[2] = mc[0];
    return true;
  }();
  if (!al) mc[0] = mc[1] = mc[2] = mA;  // unused
  const int dev = current_device();
  if (dev < 0) return PA_ERR_DEVICE;
  static std::atomic<int> max_pairs[kMaxDevices];
  const int pairs = cached_per_device(max_pairs, dev, [] {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 1024, 1, 1);
    cfg.blockDim = dim3(256, 1, 1);
    cfg.dynamicSmemBytes = PairCfg<NT>::SMEM;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_pair_kernel<A_MN, B_MN, NT>, &cfg) != cudaSuccess ||
        n <= 0) {
      cudaGetLastError();  // clear a failed query; fall back to one pair per two SMs
      n = device_sm_count() / 2;
    }
    return n;
  });
  const int tiles = ((Mout + 2 * GB - 1) / (2 * GB)) * ((Nout + PB_N - 1) / PB_N);
  // Accumulating GEMMs through the TMA path may split K so that the work units
  // fill whole waves of pairs: the slices add into C in any order, so their
  // results can differ in the last bits from run to run.
  int ksplit = 1;
  if (accumulate && al && !ep.bias && !ep.relu) {
    const int nk = (Kred + GK - 1) / GK;
    double best = 0.0;
    for (int sp = 1; sp <= 16 && nk / sp >= 4; ++sp) {
      const int units = tiles * sp, waves = (units + pairs - 1) / pairs;
      const double eff = static_cast<double>(units) / (static_cast<double>(waves) * pairs);
      if (eff > best + 0.02) {
        best = eff;
        ksplit = sp;
      }
    }
  }
  const int units = tiles * ksplit;
  const int grid = 2 * (units < pairs ? units : pairs);
  // walk N fastest when A (Mout x Kred) is the larger operand: it then streams once
  const int n_fast = Mout > Nout ? 1 : 0;
  gemm_pair_kernel<A_MN, B_MN, NT><<<grid, 256, PairCfg<NT>::SMEM, s>>>(
      m[0], m[1], m[2], m[3], mc[0], mc[1], mc[2], al ? 1 : 0, ksplit, C, ldc, Mout, Nout, Kred,
      accumulate, ep.bias, ep.c1, ep.c2, ep.nsplit, ep.relu, n_fast,
      static_cast<__nv_bfloat16*>(ep.y_hi), static_cast<__nv_bfloat16*>(ep.y_lo), round8(Nout),
      status);
  return cudaGetLastError() == cudaSuccess ? PA_OK : PA_ERR_LAUNCH;
}

// bf16 hi/lo planes of one [rows, cols] operand in the workspace (row pitch round8(cols)).
struct Planes {
  uint8_t* hi;
  uint8_t* lo;
  int rows, cols;
};
size_t plane_size(int rows, int cols) { return up256(static_cast<size_t>(rows) * round8(cols) * 2); }
Planes carve(uint8_t*& w, int rows, int cols) {
  const size_t b = plane_size(rows, cols);
  Planes p{w, w + b, rows, cols};
  w += 2 * b;
  return p;
}
// hi and lo planes, or the hi plane alone in the bf16 math mode
int split_into(const float* x, const Planes& p, cudaStream_t s) {
  return launch_split_planes(x, p.hi, f32_math() == PA_F32_MATH_BF16 ? nullptr : p.lo,
                             static_cast<size_t>(p.rows), p.cols, round8(p.cols), s);
}

// GEMM of `mode` (see launch_gemm_f32) on operands already split into planes.
// Modes 1 and 2 add into C unless accumulate is 0, when they overwrite it.
int gemm_planes(int mode, const Planes& a, const Planes& b, float* C, int M, int N, int K,
                const Epilogue& ep, uint32_t* status, cudaStream_t s, int accumulate = 1) {
  const bool a_mn = (mode == 2), b_mn = (mode != 1);
  // paired 256 x 256 kernel: maps A hi, A lo, B hi, B lo (K-major boxes of 128 rows:
  // each CTA loads its 128 rows of A and its 128 columns of B)
  {
    const bool one = f32_math() == PA_F32_MATH_BF16;
    CUtensorMap m[4];
    if (!plane_map(&m[0], a.hi, a.rows, a.cols, a_mn, 128) ||
        !plane_map(&m[2], b.hi, b.rows, b.cols, b_mn, 128))
      return PA_ERR_ALIGN;
    if (one) {
      m[1] = m[0];
      m[3] = m[2];
    } else if (!plane_map(&m[1], a.lo, a.rows, a.cols, a_mn, 128) ||
               !plane_map(&m[3], b.lo, b.rows, b.cols, b_mn, 128)) {
      return PA_ERR_ALIGN;
    }
    const int acc = accumulate ? 1 : 0;
    if (one) {
      if (mode == 0) return run_gemm_pair<false, true, 1>(m, C, N, M, N, K, 0, ep, status, s);
      if (mode == 1) return run_gemm_pair<false, false, 1>(m, C, N, M, N, K, acc, ep, status, s);
      return run_gemm_pair<true, true, 1>(m, C, K, N, K, M, acc, ep, status, s);
    }
    if (mode == 0) return run_gemm_pair<false, true, 3>(m, C, N, M, N, K, 0, ep, status, s);
    if (mode == 1) return run_gemm_pair<false, false, 3>(m, C, N, M, N, K, acc, ep, status, s);
    return run_gemm_pair<true, true, 3>(m, C, K, N, K, M, acc, ep, status, s);
  }
}

}  // namespace

size_t gemm_workspace_bytes(int M, int N, int K) {
  const size_t m0 = planes_bytes(M, K) + planes_bytes(K, N);   // A [M,K], B [K,N]
  const size_t m1 = planes_bytes(M, K) + planes_bytes(N, K);   // dY [M,K], W [N,K]
  const size_t m2 = planes_bytes(M, N) + planes_bytes(M, K);   // X [M,N], dY [M,K]
  size_t mx = m0 > m1 ? m0 : m1;
  return mx > m2 ? mx : m2;
}

int launch_gemm_f32(int mode, const float* A, const float* B, float* C, int M, int N, int K,
                    void* ws, uint32_t* status, cudaStream_t s) {
  // (rows, cols) of the two stored operands, per mode
  int ar, ac, br, bc;
  if (mode == 0) { ar = M; ac = K; br = K; bc = N; }
  else if (mode == 1) { ar = M; ac = K; br = N; bc = K; }
  else { ar = M; ac = N; br = M; bc = K; }
  uint8_t* w = static_cast<uint8_t*>(ws);
  const Planes a = carve(w, ar, ac), b = carve(w, br, bc);
  int st = split_into(A, a, s);
  if (st != PA_OK) return st;
  st = split_into(B, b, s);
  if (st != PA_OK) return st;
  return gemm_planes(mode, a, b, C, M, N, K, Epilogue{}, status, s);
}

// Projection Y[M, OUT] = X[M, IN] W[IN, OUT] (+ bias), as column blocks.
// Bias-gradient partials of the widest column block (1, 2 or 3 blocks).
size_t bias_partials_bytes(int M, int OUT) {
  size_t b = 0;
  for (int n = 1; n <= 3; ++n)
    if (OUT % n == 0) {
      const size_t x = up256(bias_grad_workspace_bytes(static_cast<uint32_t>(M),
                                                       static_cast<uint32_t>(OUT / n)));
      b = x > b ? x : b;
    }
  return b;
}

size_t linear_workspace_bytes(int M, int IN, int OUT) {
  const size_t fwd = planes_bytes(M, IN) + planes_bytes(IN, OUT);
  const size_t bwd = planes_bytes(M, OUT) + planes_bytes(IN, OUT) + planes_bytes(M, IN) +
                     bias_partials_bytes(M, OUT);
  return fwd > bwd ? fwd : bwd;
}

// Kept planes of X: the hi plane and, under split3 math, the lo plane, in the
// layout of the GEMM operands, written by a forward for its backward.
size_t linear_kept_bytes(int M, int IN, int mode) {
  return static_cast<size_t>(mode == PA_F32_MATH_BF16 ? 1 : 2) * plane_size(M, IN);
}

int launch_linear_fwd(const float* x, const float* wt, const float* bias, float* const* outs,
                      int n_outs, int M, int IN, int OUT, int relu, void* ws, uint32_t* status,
                      cudaStream_t s, void* kept, int kept_valid, void* y_planes) {
  uint8_t* w = static_cast<uint8_t*>(ws);
  uint8_t* kp = static_cast<uint8_t*>(kept);
  const Planes a = kept ? Planes{kp, kp + plane_size(M, IN), M, IN} : carve(w, M, IN);
  const Planes b = carve(w, IN, OUT);
  int st = kept && kept_valid ? PA_OK : split_into(x, a, s);  // valid: X's planes are there
  if (st != PA_OK) return st;
  st = split_into(wt, b, s);
  if (st != PA_OK) return st;
  Epilogue ep;
  ep.bias = bias;
  ep.relu = relu;
  if (n_outs > 1) {
    ep.nsplit = OUT / n_outs;
    ep.c1 = outs[1];
    ep.c2 = n_outs > 2 ? outs[2] : nullptr;
  }
  if (y_planes) {  // Y's planes in the kept layout of a projection that reads Y next
    uint8_t* yp = static_cast<uint8_t*>(y_planes);
    ep.y_hi = yp;
    ep.y_lo = f32_math() == PA_F32_MATH_BF16 ? nullptr : yp + plane_size(M, OUT);
  }
  return gemm_planes(0, a, b, outs[0], M, OUT, IN, ep, status, s);
}

int launch_linear_bwd(const float* x, const float* wt, const float* const* dy_parts, int n_parts,
                      const float* relu_out, float* dx, float* dw, float* dbias, int M, int IN,
                      int OUT, void* ws, uint32_t* status, cudaStream_t s, const void* kept,
                      int dx_accumulate) {
  uint8_t* w = static_cast<uint8_t*>(ws);
  const Planes dy = carve(w, M, OUT), wp = carve(w, IN, OUT);
  Planes xp = carve(w, M, IN);
  if (kept) {  // X's planes from the forward, valid for the current math mode
    uint8_t* kp = const_cast<uint8_t*>(static_cast<const uint8_t*>(kept));
    xp = Planes{kp, kp + plane_size(M, IN), M, IN};
  }
  float* bias_ws = reinterpret_cast<float*>(w);  // bias_partials_bytes(M, OUT)
  // gather the column-block gradients into one pair of planes (row pitch
  // round8(OUT)), with the bias gradient summed in the same pass over dY
  const int part = OUT / n_parts;
  void* dy_lo = f32_math() == PA_F32_MATH_BF16 ? nullptr : dy.lo;
  for (int p = 0; p < n_parts; ++p) {
    const int width = p + 1 < n_parts ? part : round8(OUT) - p * part;  // last block takes the pad
    // relu_out: single-part projections only
    const int st =
        dbias ? launch_split_planes_colsum(dy_parts[p], relu_out, dy.hi, dy_lo,
                                           static_cast<uint32_t>(M), part, width,
                                           static_cast<size_t>(round8(OUT)), p * part,
                                           dbias + p * part, bias_ws, s)
              : launch_split_planes_masked(dy_parts[p], relu_out, dy.hi, dy_lo,
                                           static_cast<size_t>(M), part, width,
                                           static_cast<size_t>(round8(OUT)), p * part, s);
    if (st != PA_OK) return st;
  }
  if (dx) {
    int st = split_into(wt, wp, s);
    if (st != PA_OK) return st;
    st = gemm_planes(1, dy, wp, dx, M, IN, OUT, Epilogue{}, status, s, dx_accumulate);
    if (st != PA_OK) return st;
  }
  if (dw) {
    int st = kept ? PA_OK : split_into(x, xp, s);
    if (st != PA_OK) return st;
    st = gemm_planes(2, xp, dy, dw, M, IN, OUT, Epilogue{}, status, s);
    if (st != PA_OK) return st;
  }
  return PA_OK;
}

}  // namespace pa
