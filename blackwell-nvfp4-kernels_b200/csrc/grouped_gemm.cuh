// NVFP4 grouped GEMM, sm_100a: one persistent launch computes
//
//   C_g[l] = A_g[l] . B_g[l]ᵀ   for every group g   (fp32 accumulate, fp16 out)
//
// Same computation as the reference's ref_kernel
// (nvfp4_group_gemm/reference.py:39-74) and its best submission's
// persistent_group_gemm_kernel (nvfp4_group_gemm/submission_v7.py:188-438);
// own design:
//
// * the group table (one TMA descriptor pair + sizes + scale/output pointers
//   per group) travels in the kernel parameter block (__grid_constant__), so
//   a launch needs no host->device copy and no descriptor fencing; kMaxGroups
//   is a template parameter and the host splits larger problems;
// * tiles of all groups form one list (group-major, M-blocks fastest inside a
//   column so a B tile is reused from L2 by all M-blocks of its group); every
//   CTA walks the list round-robin and finds its group by binary search over
//   the tile-start prefix sums;
// * two TMEM accumulator buffers, so the epilogue of one tile overlaps the
//   MMAs of the next; empty groups are compacted out on the host.
#pragma once
#include <cuda.h>
#include "kernel_common.cuh"

namespace nvfp4 {

struct GroupInfo {
  const uint8_t* sfa;   // permuted scale atoms [L][ceil(M/128)][K/64][512]
  const uint8_t* sfb;   // [L][ceil(N/128)][K/64][512]
  __half* c;            // [L][M][N]
  int m, n, k, l;
  int m_blocks, n_blocks, tile_start, pad_;
};

template <int kMaxGroups>
struct GroupedParams {
  CUtensorMap tmap_a[kMaxGroups];  // bytes [L][M][K/2], box {128 B, 128 rows, 1}
  CUtensorMap tmap_b[kMaxGroups];  // bytes [L][N][K/2], box {128 B, BN rows, 1}
  GroupInfo g[kMaxGroups];
  int num_groups, tiles;
  unsigned* status;
  long long wait_limit;
};

template <int kBN, int kStages>
struct GroupedCfg {
  static constexpr int kEpiWarps = 4;
  static constexpr int kAccBufs = 2;
  static constexpr int kABytes = kBM * kBK / 2;
  static constexpr int kBBytes = kBN * kBK / 2;
  static constexpr int kStageBytes = kABytes + kBBytes + 2 * kSfStageBytes;
  static constexpr int kThreads = 32 * (kEpiWarps + 2);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;
  static constexpr int kTmemCols = 512;
  static constexpr int kSfCol = kAccBufs * kBN;
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(kSfCol + 32 <= kTmemCols, "TMEM budget");
  static_assert(kBN == 128 || kBN == 64, "tile N");
};

struct GTile { int g, l, mb, nb; };

template <int kMaxGroups>
__device__ __forceinline__ GTile grouped_tile(const GroupedParams<kMaxGroups>& p, int t) {
  int lo = 0, hi = p.num_groups - 1;  // largest g with tile_start <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.g[mid].tile_start <= t) lo = mid; else hi = mid - 1;
  }
  const GroupInfo& gi = p.g[lo];
  GTile r;
  r.g = lo;
  int local = t - gi.tile_start;
  const int per_l = gi.m_blocks * gi.n_blocks;
  r.l = local / per_l;
  local -= r.l * per_l;
  r.mb = local % gi.m_blocks;
  r.nb = local / gi.m_blocks;
  return r;
}

template <int kBN, int kStages, int kMaxGroups>
__global__ void __launch_bounds__(GroupedCfg<kBN, kStages>::kThreads, 1)
grouped_gemm_kernel(const __grid_constant__ GroupedParams<kMaxGroups> p) {
  using Cfg = GroupedCfg<kBN, kStages>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full[kStages], bar_empty[kStages];
  __shared__ uint64_t bar_acc_full[Cfg::kAccBufs], bar_acc_empty[Cfg::kAccBufs];
  __shared__ uint64_t bar_drain;
  __shared__ uint32_t s_tmem_base;
  __shared__ volatile int s_abort;

  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();
  constexpr int kProd = Cfg::kEpiWarps, kMma = Cfg::kEpiWarps + 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bar_full[s]), 1);
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    for (int b = 0; b < Cfg::kAccBufs; ++b) {
      mbar_init(smem_u32(&bar_acc_full[b]), 1);
      mbar_init(smem_u32(&bar_acc_empty[b]), Cfg::kEpiWarps);
    }
    mbar_init(smem_u32(&bar_drain), 1);
    s_abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == kMma) tmem_alloc<Cfg::kTmemCols>(smem_u32(&s_tmem_base));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem_base;
  const AbortCtl ctl{&s_abort, p.status, p.wait_limit};

  if (warp == kProd) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_phase[kStages];
      bool issued[kStages];
      for (int s = 0; s < kStages; ++s) issued[s] = false, last_phase[s] = 0;
      bool ok = true;
      int prev_g = -1;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        const GTile tc = grouped_tile(p, t);
        const GroupInfo& gi = p.g[tc.g];
        if (tc.g != prev_g) {
          tma_prefetch_desc(&p.tmap_a[tc.g]);
          tma_prefetch_desc(&p.tmap_b[tc.g]);
          prev_g = tc.g;
        }
        const int k_blocks = gi.k / kBK;
        const int rest_k = gi.k / kKStep;
        const size_t sfa_l = (size_t)gi.m_blocks * rest_k * kSfAtom;
        const size_t sfb_l = (size_t)((gi.n + 127) / 128) * rest_k * kSfAtom;
        const int n0 = tc.nb * kBN;
        const uint8_t* sfa_t = gi.sfa + tc.l * sfa_l + (size_t)tc.mb * rest_k * kSfAtom;
        const uint8_t* sfb_t = gi.sfb + tc.l * sfb_l + (size_t)(n0 / 128) * rest_k * kSfAtom;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!ctl.wait(smem_u32(&bar_empty[stage]), phase ^ 1u, kDevTimeoutStageFree)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&bar_full[stage]);
          const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sb = sa + Cfg::kABytes;
          const uint32_t ssf = sb + Cfg::kBBytes;
          mbar_arrive_expect_tx(full, Cfg::kStageBytes);
          tma_load_3d(sa, &p.tmap_a[tc.g], full, kb * 128, tc.mb * kBM, tc.l, pol);
          tma_load_3d(sb, &p.tmap_b[tc.g], full, kb * 128, n0, tc.l, pol);
          const size_t sf_off = (size_t)kb * kSfStageBytes;
          bulk_load(ssf, sfa_t + sf_off, kSfStageBytes, full, pol);
          bulk_load(ssf + kSfStageBytes, sfb_t + sf_off, kSfStageBytes, full, pol);
          issued[stage] = true;
          last_phase[stage] = phase;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
      }
      if (!ok) {
        for (int s = 0; s < kStages; ++s)
          if (issued[s]) ctl.drain(smem_u32(&bar_full[s]), last_phase[s]);
      }
    }
  } else if (warp == kMma) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_mxf4nvf4<kBM, kBN>();
      const uint32_t sf_a = tmem + Cfg::kSfCol;
      const uint32_t sf_b = sf_a + 16;
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, any = false;
      for (int t = blockIdx.x; t < p.tiles && ok; t += gridDim.x) {
        const GTile tc = grouped_tile(p, t);
        const int k_blocks = p.g[tc.g].k / kBK;
        const uint32_t sfb_sub = (kBN == 64) ? (uint32_t)((tc.nb & 1) * 2) : 0u;
        if (!ctl.wait(smem_u32(&bar_acc_empty[acc]), acc_phase ^ 1u, kDevTimeoutAccFree)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * kBN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!ctl.wait(smem_u32(&bar_full[stage]), phase, kDevTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sb = sa + Cfg::kABytes;
          const uint32_t ssf = sb + Cfg::kBBytes;
          #pragma unroll
          for (int j = 0; j < kBK / kKStep; ++j) {
            tc_cp_sf_atom(sf_a + 4 * j, sf_atom_desc(ssf + j * kSfAtom));
            tc_cp_sf_atom(sf_b + 4 * j, sf_atom_desc(ssf + kSfStageBytes + j * kSfAtom));
          }
          #pragma unroll
          for (int j = 0; j < kBK / kKStep; ++j) {
            tc_mma_nvf4(d, kmajor_sw128_desc(sa + 32 * j), kmajor_sw128_desc(sb + 32 * j), idesc,
                        sf_a + 4 * j, sf_b + 4 * j + sfb_sub, (kb | j) != 0);
          }
          tc_commit(smem_u32(&bar_empty[stage]));
          any = true;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        tc_commit(smem_u32(&bar_acc_full[acc]));
        if (++acc == Cfg::kAccBufs) acc = 0, acc_phase ^= 1u;
      }
      if (!ok && any) {
        tc_commit(smem_u32(&bar_drain));
        ctl.drain(smem_u32(&bar_drain), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < p.tiles; t += gridDim.x) {
      const GTile tc = grouped_tile(p, t);
      const GroupInfo& gi = p.g[tc.g];
      if (!ctl.wait(smem_u32(&bar_acc_full[acc]), acc_phase, kDevTimeoutAccFull)) break;
      tc_fence_after();
      const uint32_t t_acc = tmem + ((uint32_t)(quad * 32) << 16) + acc * kBN;
      const int row = tc.mb * kBM + quad * 32 + (int)lane;
      const int col0 = tc.nb * kBN;
      __half* crow = gi.c + ((size_t)tc.l * gi.m + row) * (size_t)gi.n + col0;
      const bool row_ok = row < gi.m;
      #pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(t_acc + 32 * c, v);
        tmem_ld_wait();
        tmem_regs_ready(v);
        #pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int col = col0 + 32 * c + 8 * q;
          if (row_ok && col < gi.n) {
            const int i = 8 * q;
            st_global_v4(crow + 32 * c + 8 * q,
                         pack_half2(__uint_as_float(v[i + 0]), __uint_as_float(v[i + 1])),
                         pack_half2(__uint_as_float(v[i + 2]), __uint_as_float(v[i + 3])),
                         pack_half2(__uint_as_float(v[i + 4]), __uint_as_float(v[i + 5])),
                         pack_half2(__uint_as_float(v[i + 6]), __uint_as_float(v[i + 7])));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[acc]));
      if (++acc == Cfg::kAccBufs) acc = 0, acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMma) {
    tc_fence_after();
    tmem_dealloc<Cfg::kTmemCols>(tmem);
  }
}

}  // namespace nvfp4
