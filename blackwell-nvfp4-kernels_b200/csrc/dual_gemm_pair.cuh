// NVFP4 dual GEMM on CTA pairs (cta_group::2), sm_100a: the large-M kernel.
//
//   C = silu(A . B1ᵀ) * (A . B2ᵀ)   (fp32 accumulate in TMEM, fp16 out)
//
// A pair of CTAs (a cluster of 2 on neighbouring SMs) owns a 256 x 128 tile
// of C.  CTA r holds A rows [256*mp + 128*r, +128) and one B tile: CTA 0 the
// 128 rows of B1, CTA 1 the 128 rows of B2 for the tile's columns.  One
// tcgen05.mma.cta_group::2 with M = 256, N = 256 then computes, in each CTA's
// TMEM, its 128 rows x [gate (N rows 0..127 from CTA 0's B1) | up (N rows
// 128..255 from CTA 1's B2)], so the accumulator layout and the epilogue are
// those of the single-CTA kernel while every SM loads only
// A 16 KB + B 16 KB + scales 6 KB per 256-deep K step (54 KB single-CTA).
//
// Protocol (all waits bounded):
// * both producers wait on their own stage-free barrier and load into their
//   own shared memory, counting bytes on the LEADER's stage-full barrier
//   (TMA with .cta_group::2, no multicast); only the leader's producer posts
//   the expected byte count (both CTAs' bytes);
// * the leader's MMA warp copies every CTA's scale atoms into that CTA's TMEM
//   (tcgen05.cp.cta_group::2), issues the pair MMAs, and commits to the
//   stage-free and accumulator-full barriers of both CTAs (commit multicast);
// * each CTA's epilogue drains its own TMEM; the accumulator is handed back
//   by arrivals of both CTAs' epilogue warps on the leader's barrier;
// * cluster barriers after initialisation and before teardown keep every
//   remote arrive and shared-memory read inside both CTAs' lifetimes.
#pragma once
#include <cuda.h>
#include "kernel_common.cuh"

namespace nvfp4 {

struct DualPairParams {
  CUtensorMap tmap_a;     // bytes [L][M][K/2], box {128 B, 128 rows, 1}
  CUtensorMap tmap_b1;    // bytes [L][N][K/2], box {128 B, 128 rows, 1}
  CUtensorMap tmap_b2;
  CUtensorMap tmap_sfa;   // u64 [L*ceil(M/128)][K/64][64], box {64, 4, 1}: 4 atoms
  CUtensorMap tmap_sfb1;  // u64 [L*ceil(N/128)][K/64][64]
  CUtensorMap tmap_sfb2;
  __half* c;              // [L][M][N]
  int m, n, k, l;
  int mp_blocks, n_blocks, k_blocks, tiles;  // tiles = L * mp_blocks * n_blocks
  int sfa_blocks, sfb_blocks;                // ceil(M/128), ceil(N/128)
  int group_m;                               // raster: pair M-blocks per group
  unsigned* status;
  long long wait_limit;
};

template <int kStages>
struct DualPairCfg {
  static constexpr int kBN = 128;                   // output columns per pair tile
  static constexpr int kEpiWarps = 8;
  static constexpr int kABytes = kBM * kBK / 2;     // 16 KB: this CTA's 128 A rows
  static constexpr int kBBytes = kBN * kBK / 2;     // 16 KB: B1 (CTA 0) or B2 (CTA 1)
  static constexpr int kStageBytes = kABytes + kBBytes + 3 * kSfStageBytes;
  static constexpr int kPairTxBytes = 2 * kStageBytes;
  static constexpr int kThreads = 32 * (kEpiWarps + 2);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;
  static constexpr int kTmemCols = 512;
  static constexpr int kAccCols = 2 * kBN;          // gate | up
  static constexpr int kSfCol = kAccCols;
  static constexpr int kSfBufCols = 48;             // SFA 4x4 + [SFB1|SFB2] 4x8
  static constexpr int kColsPerWarp = kBN / (kEpiWarps / 4);
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(kSfCol + 2 * kSfBufCols <= kTmemCols, "TMEM budget");
  static_assert(kSfCol % 4 == 0 && kSfBufCols % 4 == 0, "tcgen05.cp needs 4-column alignment");
};

struct PairTile { int l, mp, nb; };

__device__ __forceinline__ PairTile pair_tile_coord(const DualPairParams& p, int t) {
  const int per_l = p.mp_blocks * p.n_blocks;
  PairTile tc;
  tc.l = t / per_l;
  const int local = t - tc.l * per_l;
  const int span = p.group_m * p.n_blocks;
  const int g = local / span;
  const int first = g * p.group_m;
  const int gsz = min(p.mp_blocks - first, p.group_m);
  const int r = local - g * span;
  tc.mp = first + r % gsz;
  tc.nb = r / gsz;
  return tc;
}

template <int kStages>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(DualPairCfg<kStages>::kThreads, 1)
dual_gemm_pair_kernel(const __grid_constant__ DualPairParams p) {
  using Cfg = DualPairCfg<kStages>;
  constexpr int kProd = Cfg::kEpiWarps, kMma = Cfg::kEpiWarps + 1;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full[kStages], bar_empty[kStages];
  __shared__ uint64_t bar_acc_full, bar_acc_empty, bar_drain;
  __shared__ uint32_t s_tmem_base;
  __shared__ volatile int s_abort;

  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();
  const uint32_t rank = cluster_ctarank();   // 0 = leader
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, num_pairs = gridDim.x >> 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bar_full[s]), 1);
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    mbar_init(smem_u32(&bar_acc_full), 1);
    mbar_init(smem_u32(&bar_acc_empty), 2 * Cfg::kEpiWarps);   // both CTAs' epilogue warps
    mbar_init(smem_u32(&bar_drain), 1);
    s_abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == kProd && lane == 0) {
    tma_prefetch_desc(&p.tmap_a);
    tma_prefetch_desc(rank == 0 ? &p.tmap_b1 : &p.tmap_b2);
    tma_prefetch_desc(&p.tmap_sfa);
    tma_prefetch_desc(&p.tmap_sfb1);
    tma_prefetch_desc(&p.tmap_sfb2);
  }
  if (warp == kMma) tmem_alloc_pair<Cfg::kTmemCols>(smem_u32(&s_tmem_base));
  tc_fence_before();
  __syncthreads();
  cluster_sync();   // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem = s_tmem_base;
  const AbortCtl ctl{&s_abort, p.status, p.wait_limit};

  if (warp == kProd) {
    // ------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      const uint64_t pol = policy_evict_normal();
      const CUtensorMap* tmap_b = rank == 0 ? &p.tmap_b1 : &p.tmap_b2;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_phase[kStages];
      bool issued[kStages];
      for (int s = 0; s < kStages; ++s) issued[s] = false, last_phase[s] = 0;
      bool ok = true;
      for (int t = pair; t < p.tiles && ok; t += num_pairs) {
        const PairTile tc = pair_tile_coord(p, t);
        const int m0 = tc.mp * 2 * kBM + (int)rank * kBM;   // this CTA's A rows
        const int n0 = tc.nb * Cfg::kBN;
        const int sfa_row = tc.l * p.sfa_blocks + m0 / 128;
        const int sfb_row = tc.l * p.sfb_blocks + n0 / 128;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ctl.wait(smem_u32(&bar_empty[stage]), phase ^ 1u, kDevTimeoutStageFree)) {
            ok = false;
            break;
          }
          const uint32_t full = mapa_shared(smem_u32(&bar_full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(smem_u32(&bar_full[stage]), Cfg::kPairTxBytes);
          const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sb = sa + Cfg::kABytes;
          const uint32_t ssf = sb + Cfg::kBBytes;
          tma_load_3d_pair(sa, &p.tmap_a, full, kb * 128, m0, tc.l, pol);
          tma_load_3d_pair(sb, tmap_b, full, kb * 128, n0, tc.l, pol);
          tma_load_3d_pair(ssf, &p.tmap_sfa, full, 0, kb * 4, sfa_row, pol);
          tma_load_3d_pair(ssf + kSfStageBytes, &p.tmap_sfb1, full, 0, kb * 4, sfb_row, pol);
          tma_load_3d_pair(ssf + 2 * kSfStageBytes, &p.tmap_sfb2, full, 0, kb * 4, sfb_row, pol);
          issued[stage] = true;
          last_phase[stage] = phase;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
      }
      if (!ok && leader) {  // the leader's full barriers count both CTAs' bytes
        for (int s = 0; s < kStages; ++s)
          if (issued[s]) ctl.drain(smem_u32(&bar_full[s]), last_phase[s]);
      }
    }
  } else if (warp == kMma) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && lane == 0) {
      constexpr uint32_t idesc = (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) |
                                 ((uint32_t)(256 >> 4) << 24);   // M=256, N=256, e2m1 x e2m1, e4m3 scales
      constexpr uint16_t kBoth = 0x3;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      uint32_t sf_buf = 0;
      bool ok = true, any = false;
      for (int t = pair; t < p.tiles && ok; t += num_pairs) {
        if (!ctl.wait(smem_u32(&bar_acc_empty), acc_phase ^ 1u, kDevTimeoutAccFree)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ctl.wait(smem_u32(&bar_full[stage]), phase, kDevTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sb = sa + Cfg::kABytes;
          const uint32_t ssf = sb + Cfg::kBBytes;
          const uint32_t sf_a = tmem + Cfg::kSfCol + sf_buf * Cfg::kSfBufCols;
          const uint32_t sf_b = sf_a + 16;
          #pragma unroll
          for (int j = 0; j < kBK / kKStep; ++j) {
            tc_cp_sf_atom_pair(sf_a + 4 * j, sf_atom_desc(ssf + j * kSfAtom));
            tc_cp_sf_atom_pair(sf_b + 8 * j, sf_atom_desc(ssf + kSfStageBytes + j * kSfAtom));
            tc_cp_sf_atom_pair(sf_b + 8 * j + 4, sf_atom_desc(ssf + 2 * kSfStageBytes + j * kSfAtom));
          }
          #pragma unroll
          for (int j = 0; j < kBK / kKStep; ++j) {
            tc_mma_nvf4_pair(tmem, kmajor_sw128_desc(sa + 32 * j), kmajor_sw128_desc(sb + 32 * j),
                             idesc, sf_a + 4 * j, sf_b + 8 * j, (kb | j) != 0);
          }
          tc_commit_pair(smem_u32(&bar_empty[stage]), kBoth);   // stage free in both CTAs
          any = true;
          sf_buf ^= 1u;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        tc_commit_pair(smem_u32(&bar_acc_full), kBoth);         // accumulators ready in both
        acc_phase ^= 1u;
      }
      if (!ok && any) {
        tc_commit_pair(smem_u32(&bar_drain), 0x1);
        ctl.drain(smem_u32(&bar_drain), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;
    const int part = warp >> 2;
    constexpr int kCW = Cfg::kColsPerWarp;
    constexpr int kChunks = kCW / 32;
    static_assert(kCW == 64, "one 128-byte fp16 line per lane");
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&bar_acc_empty), 0);
    uint32_t acc_phase = 0;
    for (int t = pair; t < p.tiles; t += num_pairs) {
      const PairTile tc = pair_tile_coord(p, t);
      if (!ctl.wait(smem_u32(&bar_acc_full), acc_phase, kDevTimeoutAccFull)) break;
      tc_fence_after();
      const uint32_t t_gate = tmem + ((uint32_t)(quad * 32) << 16) + part * kCW;
      const uint32_t t_up = t_gate + Cfg::kBN;
      uint32_t g[kChunks][32], u[kChunks][32];
      #pragma unroll
      for (int c = 0; c < kChunks; ++c) {
        tmem_ld_32x32b_x32(t_gate + 32 * c, g[c]);
        tmem_ld_32x32b_x32(t_up + 32 * c, u[c]);
      }
      tmem_ld_wait();
      #pragma unroll
      for (int c = 0; c < kChunks; ++c) tmem_regs_ready(g[c]), tmem_regs_ready(u[c]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_leader);   // TMEM may be overwritten now
      uint32_t w[32];
      #pragma unroll
      for (int c = 0; c < kChunks; ++c)
        #pragma unroll
        for (int e = 0; e < 16; ++e)
          w[16 * c + e] =
              pack_half2(silu_gate(__uint_as_float(g[c][2 * e]), __uint_as_float(u[c][2 * e])),
                         silu_gate(__uint_as_float(g[c][2 * e + 1]), __uint_as_float(u[c][2 * e + 1])));
      const int row0 = tc.mp * 2 * kBM + (int)rank * kBM + quad * 32;
      const int col0 = tc.nb * Cfg::kBN + part * kCW;
      store_lines_coalesced(w, p.c + ((size_t)tc.l * p.m + row0) * (size_t)p.n + col0, p.n,
                            p.m - row0, p.n - col0);
      acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();   // no MMA, copy or remote arrive of either CTA is still in flight
  if (warp == kMma) {
    tc_fence_after();
    tmem_dealloc_pair<Cfg::kTmemCols>(tmem);
  }
}

}  // namespace nvfp4
