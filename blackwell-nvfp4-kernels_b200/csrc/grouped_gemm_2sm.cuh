// NVFP4 grouped GEMM on CTA pairs (tcgen05.mma.cta_group::2), sm_100a:
//
//   C_g[l] = A_g[l] . B_g[l]ᵀ   for every group g   (fp32 accumulate in TMEM, fp16 out)
//
// Same computation as the reference's ref_kernel
// (nvfp4_group_gemm/reference.py:39-74); own design, the dual GEMM's CTA-pair
// kernel (dual_gemm_2sm.cuh) applied to one GEMM per group:
//
// * one persistent launch over the tiles of all groups.  A CTA pair (cluster
//   of 2) owns a 256 x 256 tile of one group's C: CTA r holds A rows
//   [256*mp + 128*r, +128) and B rows [256*nb + 128*r, +128).  One
//   tcgen05.mma.cta_group::2 with M = 256, N = 256 per 64-deep K step writes
//   each CTA's 128 rows x 256 columns into its TMEM.  Per SM and 256-deep K
//   block: A 16 KB + B 16 KB for 128 x 256 outputs (the single-CTA kernel:
//   16 + 32 KB);
// * scale factors: each CTA loads its 4 SFA atoms and the 4 + 4 atoms of the
//   tile's two 128-row B blocks per K block by TMA onto the leader's stage
//   barrier; the MMA thread copies them into TMEM itself
//   (tcgen05.cp.cta_group::2.32x128b.warpx4) right before the step's MMA;
// * the group table (four tensor maps per group, sizes, output pointer)
//   travels in the kernel parameter block; tiles are listed group-major with
//   pair M-blocks fastest inside a column, and every pair walks the list
//   round-robin, finding its group by binary search over the tile starts;
// * a group's rows are covered in 256-row pair blocks, except that a last
//   block holding at most 128 rows is a "half tile": the pair computes its
//   128 x 256 block of C transposed, Cᵀ = B . Aᵀ, with the tile's B rows as
//   the M = 256 operand (128 per CTA) and the block's A rows as the N = 128
//   operand (64 per CTA), so no CTA works on rows past M (per SM and K
//   block: 8 + 16 KB of operands for 128 x 128 outputs).  Half tiles keep
//   their place in the list, next to the group's other blocks of the same
//   columns, which read the same B rows from L2; rows past M_g in a full
//   tile's second CTA load as TMA zero fill and are not stored.  A loads as
//   64-row boxes (two per full tile), so both tile kinds share one map.  A
//   half tile does half a full tile's MMA work in ~0.95 of its time: with
//   28 KB per stage in flight, the stage round trip paces its K blocks;
// * a call of more than 48 groups is several launches; each later one is
//   "chained" (it waits for the previous launch at its end, not its start);
// * issue threads chosen with elect.sync, descriptors advanced from the
//   stage-0 ones, one accumulator that the eight epilogue warps of each CTA
//   pull into registers and release before the stores, all waits bounded.
#pragma once
#include <cuda.h>
#include "kernel_common.cuh"

namespace nvfp4 {

struct GroupPairInfo {
  __half* c;              // [L][M][N]
  int m, n, k, l;
  int mp_blocks, n_blocks, tile_start;   // 256-row pair blocks, 256-column blocks
  int half;                              // the last pair block holds <= 128 rows
  int sfa_blocks, sfb_blocks;            // ceil(M/128), ceil(N/128)
  int lines32;                           // C rows start 32-byte aligned
};

template <int kMaxGroups>
struct GroupedPairParams {
  CUtensorMap tmap_a[kMaxGroups];    // bytes [L][M][K/2], box {128 B, 64 rows, 1}
  CUtensorMap tmap_b[kMaxGroups];    // bytes [L][N][K/2], box {128 B, 128 rows, 1}
  // scale atoms [L * blocks * K/64][128 x 32-bit], box {128, 4}: the four
  // atoms of one 256-deep K block of one 128-row block
  CUtensorMap tmap_sfa[kMaxGroups];
  CUtensorMap tmap_sfb[kMaxGroups];
  GroupPairInfo g[kMaxGroups];
  int num_groups, tiles;
  // a later launch of the same call (other groups, same inputs' producers):
  // it may start on SMs the previous launch frees, and waits for that launch
  // before it exits instead of before it starts
  int chained;
  unsigned* status;
  long long wait_limit;
};

template <int kStages_>
struct GroupedPairCfg {
  static constexpr int kStages = kStages_;
  static constexpr int kBN = 256;                      // C columns per tile
  static constexpr int kABytes = kBM * kBK / 2;        // 16 KB
  static constexpr int kBBytes = (kBN / 2) * kBK / 2;  // this CTA's 128 B rows: 16 KB
  static constexpr int kSfaBytes = kSfStageBytes;      // 4 atoms of this CTA's A rows
  static constexpr int kSfbBytes = 2 * kSfStageBytes;  // 4 atoms of each of the tile's B blocks
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + kSfbBytes;   // 38 KB
  static constexpr int kPairTxBytes = 2 * kStageBytes;  // both CTAs' copies of a stage
  // half tile, per CTA: 64 A rows, 128 B rows, the atoms of its B block and of the A block
  static constexpr int kHalfABytes = kABytes / 2;
  static constexpr int kHalfPairTxBytes = 2 * (kHalfABytes + kBBytes + 2 * kSfStageBytes);
  static constexpr int kEpiWarps = 8;                   // 2 per TMEM quadrant
  static constexpr int kColsPerWarp = kBN / 2;         // 128
  // warp roles: epilogue [0, 8), tile producer 8, MMA 9, scale producer 10
  static constexpr int kProdWarp = kEpiWarps, kMmaWarp = kEpiWarps + 1, kSfProdWarp = kEpiWarps + 2;
  static constexpr int kThreads = 32 * (kEpiWarps + 3);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;
  static constexpr int kTmemCols = 512;
  static constexpr int kAccCols = kBN;
  static constexpr int kSfCol = kAccCols;
  static constexpr int kSfBufCols = 48;                // per stage: SFA 16, SFB 2 x 16
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(kSfCol + kStages * kSfBufCols <= kTmemCols, "TMEM budget: one scale buffer per stage");
};

struct GPairTile { int g, l, mp, nb; bool half; };

template <int kMaxGroups>
__device__ __forceinline__ GPairTile gpair_tile(const GroupedPairParams<kMaxGroups>& p, int t) {
  int lo = 0, hi = p.num_groups - 1;   // largest g with tile_start <= t
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.g[mid].tile_start <= t) lo = mid; else hi = mid - 1;
  }
  const GroupPairInfo& gi = p.g[lo];
  GPairTile r;
  r.g = lo;
  int local = t - gi.tile_start;
  const int per_l = gi.mp_blocks * gi.n_blocks;
  r.l = local / per_l;
  local -= r.l * per_l;
  r.mp = local % gi.mp_blocks;
  r.nb = local / gi.mp_blocks;
  r.half = gi.half && r.mp == gi.mp_blocks - 1;
  return r;
}

template <int kStages, int kMaxGroups>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(GroupedPairCfg<kStages>::kThreads, 1)
grouped_gemm_2sm_kernel(const __grid_constant__ GroupedPairParams<kMaxGroups> p) {
  using Cfg = GroupedPairCfg<kStages>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full[kStages], bar_empty[kStages];
  __shared__ uint64_t bar_acc_full, bar_acc_empty;
  __shared__ uint64_t bar_drain;
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
      // the leader's expect_tx arrival (+ the copy bytes of both CTAs)
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
  if (warp == Cfg::kMmaWarp) tmem_alloc_pair<Cfg::kTmemCols>(smem_u32(&s_tmem_base));
  tc_fence_before();
  __syncthreads();
  cluster_sync();   // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem = s_tmem_base;
  // the prologue above overlaps the previous kernel; global memory only after
  // it.  A chained launch reads nothing the previous one writes: that launch
  // let it start only after its own wait, so the inputs are complete.
  if (!p.chained) griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();
  const AbortCtl ctl{&s_abort, p.status, p.wait_limit};

  if (warp == Cfg::kProdWarp || warp == Cfg::kSfProdWarp) {
    // ------------------------------------------------------------ TMA producers (both CTAs)
    // warp kProdWarp the operand tiles, warp kSfProdWarp the scale atoms, all
    // onto the leader's stage barrier
    if (elect_one()) {
      const bool tile_role = warp == Cfg::kProdWarp;
      const uint64_t pol = policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      // per stage: ever issued, and the phase of its last issue (abort drain)
      uint32_t issued = 0, last_phase = 0;
      bool ok = true;
      int prev_g = -1;
      for (int t = pair; t < p.tiles && ok; t += num_pairs) {
        const GPairTile tc = gpair_tile(p, t);
        const GroupPairInfo& gi = p.g[tc.g];
        if (tc.g != prev_g) {
          if (tile_role) {
            tma_prefetch_desc(&p.tmap_a[tc.g]);
            tma_prefetch_desc(&p.tmap_b[tc.g]);
          } else {
            tma_prefetch_desc(&p.tmap_sfa[tc.g]);
            tma_prefetch_desc(&p.tmap_sfb[tc.g]);
          }
          prev_g = tc.g;
        }
        const int k_blocks = gi.k / kBK;
        const int rest_k = gi.k / kKStep;   // 64-deep atoms per 128-row block
        const int nb0 = tc.nb * Cfg::kBN + (int)rank * (Cfg::kBN / 2);   // this CTA's B rows
        // full tile: this CTA's 128 A rows, their scale block and the tile's
        // two B blocks.  Half tile: 64 of the block's A rows (the N = 128
        // operand), this CTA's own B block (the M = 256 operand's scales)
        // and the A block.  A B block past N re-reads the last real one
        // (its columns are never stored).
        const int m0 = tc.mp * 2 * kBM + (int)rank * (tc.half ? kBM / 2 : kBM);
        const int ablk = min(tc.mp * 2 + (tc.half ? 0 : (int)rank), gi.sfa_blocks - 1);
        const int blk0 = min(tc.nb * (Cfg::kBN / 128) + (tc.half ? (int)rank : 0), gi.sfb_blocks - 1);
        const int blk1 = min(tc.nb * (Cfg::kBN / 128) + 1, gi.sfb_blocks - 1);
        const int a_atom0 = (tc.l * gi.sfa_blocks + ablk) * rest_k;
        const int b_atom0 = (tc.l * gi.sfb_blocks + blk0) * rest_k;
        const int b_atom1 = (tc.l * gi.sfb_blocks + blk1) * rest_k;
        const uint32_t tx = tc.half ? Cfg::kHalfPairTxBytes : Cfg::kPairTxBytes;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!ctl.wait(smem_u32(&bar_empty[stage]), phase ^ 1u, kDevTimeoutStageFree)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sb = sa + Cfg::kABytes;
          const uint32_t full = mapa_shared(smem_u32(&bar_full[stage]), 0);
          if (tile_role) {
            if (leader) mbar_arrive_expect_tx(smem_u32(&bar_full[stage]), tx);
            tma_load_3d_pair(sa, &p.tmap_a[tc.g], full, kb * 128, m0, tc.l, pol);
            if (!tc.half)
              tma_load_3d_pair(sa + Cfg::kHalfABytes, &p.tmap_a[tc.g], full, kb * 128, m0 + kBM / 2,
                               tc.l, pol);
            tma_load_3d_pair(sb, &p.tmap_b[tc.g], full, kb * 128, nb0, tc.l, pol);
          } else {
            // full tile: [SFA][SFB block 0][SFB block 1]; half tile: [SFB
            // block of this CTA][SFA], 4 atoms each
            const uint32_t ssf = sb + Cfg::kBBytes;
            const int ka = kb * (kBK / kKStep);
            if (tc.half) {
              tma_load_2d_pair(ssf, &p.tmap_sfb[tc.g], full, 0, b_atom0 + ka, pol);
              tma_load_2d_pair(ssf + kSfStageBytes, &p.tmap_sfa[tc.g], full, 0, a_atom0 + ka, pol);
            } else {
              tma_load_2d_pair(ssf, &p.tmap_sfa[tc.g], full, 0, a_atom0 + ka, pol);
              tma_load_2d_pair(ssf + Cfg::kSfaBytes, &p.tmap_sfb[tc.g], full, 0, b_atom0 + ka, pol);
              tma_load_2d_pair(ssf + Cfg::kSfaBytes + kSfStageBytes, &p.tmap_sfb[tc.g], full, 0,
                               b_atom1 + ka, pol);
            }
          }
          issued |= 1u << stage;
          last_phase = (last_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
      }
      if (!ok && leader) {
        // in-flight copies land before the CTA winds down (a peer's copies
        // land on the leader's stage barriers: the leader drains them, and
        // the closing cluster barrier holds the peer)
        for (int s = 0; s < kStages; ++s)
          if ((issued >> s) & 1u) ctl.drain_copies(smem_u32(&bar_full[s]), (last_phase >> s) & 1u);
      }
    }
  } else if (warp == Cfg::kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer (leader only)
    if (leader && elect_one()) {
      // e2m1 x e2m1, e4m3 scales; M = 256 and N = 256 (full tile) or 128 (half tile)
      constexpr uint32_t idesc = (1u << 7) | (1u << 10) | ((uint32_t)(Cfg::kBN >> 3) << 17) |
                                 ((uint32_t)(256 >> 4) << 24);
      constexpr uint32_t idesc_half = (1u << 7) | (1u << 10) | ((uint32_t)(128 >> 3) << 17) |
                                      ((uint32_t)(256 >> 4) << 24);
      constexpr uint16_t kBoth = 0x3;
      const uint64_t a_desc0 = kmajor_sw128_desc(smem_base);   // stage 0's A tile
      const uint64_t sf_desc0 = sf_atom_desc(smem_base + Cfg::kABytes + Cfg::kBBytes);   // its first SFA atom
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true, any = false;
      for (int t = pair; t < p.tiles && ok; t += num_pairs) {
        const GPairTile tc = gpair_tile(p, t);
        const int k_blocks = p.g[tc.g].k / kBK;
        if (!ctl.wait(smem_u32(&bar_acc_empty), acc_phase ^ 1u, kDevTimeoutAccFree)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < k_blocks; ++kb) {
          // both CTAs' tiles and scale atoms landed: one barrier counts it all
          if (!ctl.wait(smem_u32(&bar_full[stage]), phase, kDevTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t so = (uint32_t)stage * Cfg::kStageBytes;
          const uint64_t da = desc_advance(a_desc0, so);
          const uint64_t db = desc_advance(da, Cfg::kABytes);   // this CTA's B rows
          const uint64_t dsf = desc_advance(sf_desc0, so);
          const uint32_t sf_a = tmem + Cfg::kSfCol + stage * Cfg::kSfBufCols;
          const uint32_t sf_b = sf_a + 16;
          if (tc.half) {
            // Cᵀ block: the CTA's B rows are the M operand (its B block's
            // atom into [4j, +4)), the A rows the N operand (the A block's
            // atom into [16 + 8j, +4))
            #pragma unroll
            for (int j = 0; j < kBK / kKStep; ++j) {
              const uint64_t dsa = desc_advance(dsf, j * kSfAtom);
              tc_cp_pair_32x128b_x4(sf_a + 4 * j, dsa);
              tc_cp_pair_32x128b_x4(sf_b + 8 * j, desc_advance(dsa, kSfStageBytes));
              tc_mma_nvf4_pair(tmem, desc_advance(db, 32 * j), desc_advance(da, 32 * j), idesc_half,
                               sf_a + 4 * j, sf_b + 8 * j, (kb | j) != 0);
            }
          } else {
            // per 64-deep step j: its SFA atom into columns [4j, +4), the two B
            // blocks' atoms into [16 + 8j, +8) (B rows 0-127, then 128-255), then the MMA
            #pragma unroll
            for (int j = 0; j < kBK / kKStep; ++j) {
              const uint64_t dsa = desc_advance(dsf, j * kSfAtom);
              tc_cp_pair_32x128b_x4(sf_a + 4 * j, dsa);
              tc_cp_pair_32x128b_x4(sf_b + 8 * j, desc_advance(dsa, Cfg::kSfaBytes));
              tc_cp_pair_32x128b_x4(sf_b + 8 * j + 4, desc_advance(dsa, Cfg::kSfaBytes + kSfStageBytes));
              tc_mma_nvf4_pair(tmem, desc_advance(da, 32 * j), desc_advance(db, 32 * j), idesc,
                               sf_a + 4 * j, sf_b + 8 * j, (kb | j) != 0);
            }
          }
          tc_commit_pair(smem_u32(&bar_empty[stage]), kBoth);   // stage (and scale buffer) free
          any = true;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        tc_commit_pair(smem_u32(&bar_acc_full), kBoth);
        acc_phase ^= 1u;
      }
      if (!ok && any) {
        tc_commit_pair(smem_u32(&bar_drain), 0x1);
        ctl.drain(smem_u32(&bar_drain), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;        // TMEM lane quadrant
    const int part = warp >> 2;       // columns [128*part, +128) of the tile
    constexpr int kCW = Cfg::kColsPerWarp;
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&bar_acc_empty), 0);
    uint32_t acc_phase = 0;
    for (int t = pair; t < p.tiles; t += num_pairs) {
      const GPairTile tc = gpair_tile(p, t);
      const GroupPairInfo& gi = p.g[tc.g];
      if (!ctl.wait(smem_u32(&bar_acc_full), acc_phase, kDevTimeoutAccFull)) break;
      tc_fence_after();
      if (tc.half) {
        // Cᵀ block: TMEM lane = C column nb*256 + 128*rank + lane, TMEM column
        // j = C row 256*mp + j; the warp pulls columns [64*part, +64), hands
        // TMEM back, and stores one C row per register (32 lanes = 64
        // contiguous bytes)
        const uint32_t t_acc = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(64 * part);
        uint32_t v[2][32];
        tmem_ld_32x32b_x32(t_acc, v[0]);
        tmem_ld_32x32b_x32(t_acc + 32, v[1]);
        tmem_ld_wait();
        tmem_regs_ready(v[0]);
        tmem_regs_ready(v[1]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acc_empty_leader);
        acc_phase ^= 1u;
        const int col = tc.nb * Cfg::kBN + (int)rank * (Cfg::kBN / 2) + quad * 32 + (int)lane;
        const int row0 = tc.mp * 2 * kBM + 64 * part;
        if (col < gi.n) {
          __half* c0 = gi.c + ((size_t)tc.l * gi.m + row0) * (size_t)gi.n + col;
          const int rows = min(64, gi.m - row0);
          #pragma unroll
          for (int e = 0; e < 64; ++e)
            if (e < rows) c0[(size_t)e * gi.n] = __float2half_rn(__uint_as_float(v[e >> 5][e & 31]));
        }
        continue;
      }
      const uint32_t t_acc = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(kCW * part);
      // pull the warp's 128 columns into registers, hand TMEM back, pack to
      // fp16 (two 64-column lines per lane), then store whole lines
      uint32_t w[2][32];
      {
        uint32_t v[4][32];
        #pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(t_acc + 32 * c, v[c]);
        tmem_ld_wait();
        #pragma unroll
        for (int c = 0; c < 4; ++c) tmem_regs_ready(v[c]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acc_empty_leader);
        #pragma unroll
        for (int ln = 0; ln < 2; ++ln)
          #pragma unroll
          for (int e = 0; e < 16; ++e) {
            w[ln][e] = pack_half2(__uint_as_float(v[2 * ln][2 * e]), __uint_as_float(v[2 * ln][2 * e + 1]));
            w[ln][16 + e] =
                pack_half2(__uint_as_float(v[2 * ln + 1][2 * e]), __uint_as_float(v[2 * ln + 1][2 * e + 1]));
          }
      }
      acc_phase ^= 1u;
      const int row0 = tc.mp * 2 * kBM + (int)rank * kBM + quad * 32;
      const int col0 = tc.nb * Cfg::kBN + kCW * part;
      __half* cl0 = gi.c + ((size_t)tc.l * gi.m + row0) * (size_t)gi.n + col0;
      #pragma unroll
      for (int ln = 0; ln < 2; ++ln) {
        if (gi.lines32)
          store_lines_coalesced_v8(w[ln], cl0 + 64 * ln, gi.n, gi.m - row0, gi.n - col0 - 64 * ln);
        else
          store_lines_coalesced(w[ln], cl0 + 64 * ln, gi.n, gi.m - row0, gi.n - col0 - 64 * ln);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();   // no MMA, copy or remote arrive of either CTA is still in flight
  if (warp == Cfg::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair<Cfg::kTmemCols>(tmem);
  }
  // a chained launch completes only after the previous one: whatever waits
  // for this kernel then sees every launch of the call done
  if (p.chained && threadIdx.x == 0) griddep_wait();
}

}  // namespace nvfp4
