// NVFP4 dual GEMM on CTA pairs (tcgen05.mma.cta_group::2), sm_100a.
//
//   C = silu(A . B1ᵀ) * (A . B2ᵀ)   (fp32 accumulate in TMEM, fp16 out)
//
// Same computation as the reference's ref_kernel
// (nvfp4_dual_gemm/reference.py:27-77); own design:
//
// * a CTA pair (cluster of 2 on neighbouring SMs) owns a 256 x kBN tile of C
//   (kBN = 128 or 64).  CTA r holds A rows [256*mp + 128*r, +128) and half
//   of the tile's B1 rows and half of its B2 rows (rows [n0 + r*kBN/2,
//   +kBN/2) of each).  Per 64-deep K step two tcgen05.mma.cta_group::2 with
//   M = 256, N = kBN (whose B operand is split half per CTA) write gate and
//   up into each CTA's TMEM: its 128 rows x [gate kBN | up kBN].  The second
//   MMA takes A from the tensor core's collector buffer, where the first left
//   it, so A is read from shared memory once.  Per SM and 256-deep K block:
//   A 16 KB + B kBN/8 KB for 128 x kBN outputs (the single-CTA kernel: 48 KB
//   for 128 x 128);
// * scale factors: each CTA loads its 4 SFA atoms and the 4 SFB1 and 4 SFB2
//   atoms of the tile's 128-row block per K block by TMA, onto the same
//   leader stage barrier as the tiles.  The MMA thread copies them into TMEM
//   itself (tcgen05.cp.cta_group::2.32x128b.warpx4, one instruction per atom
//   and pair: row i of the atom to lane i of every lane quadrant of both
//   CTAs, 4 columns) right before the MMAs that read them; the tensor pipe
//   runs one thread's copies and MMAs in issue order.  A 64-wide tile reads
//   columns (n0 % 128) / 32 + {0, 1} of the B atoms.  Each pipeline stage
//   owns one TMEM scale buffer (48 columns);
// * one accumulator; eight epilogue warps per CTA pull their gate and up
//   columns into registers and release the accumulator (remote arrives on
//   the leader's barrier) before the math and the stores;
// * each CTA issues its copies from two threads in parallel (operand tiles;
//   scale atoms), both counting on the leader's stage barrier (TMA
//   .cta_group::2, no multicast); the leader commits to both CTAs
//   (tcgen05.commit multicast); cross-CTA handshakes use CTA-scope-release
//   remote arrives; cluster barriers bracket setup and teardown.  The
//   issuing threads are chosen with elect.sync and the MMA thread advances
//   precomputed descriptors: both keep its per-instruction cost low, which
//   sets the pace of small tiles.  All waits are bounded.  The second CTA of
//   the last pair block may lie wholly past M: its A rows load as zeros, it
//   stores nothing, and it re-reads the last real A-scale block.
#pragma once
#include <cuda.h>
#include "kernel_common.cuh"

namespace nvfp4 {

struct Dual2smParams {
  CUtensorMap tmap_a;    // bytes [L][M][K/2], box {128 B, 128 rows, 1}
  CUtensorMap tmap_b1;   // bytes [L][N][K/2], box {128 B, kBN/2 rows, 1}
  CUtensorMap tmap_b2;
  // scale atoms as 2-D [atoms][128 x 32-bit] maps, box {128, 4}: the four
  // atoms of one 256-deep K block of one 128-row block
  CUtensorMap tmap_sfa, tmap_sfb1, tmap_sfb2;
  __half* c;             // [L][M][N]
  int m, n, k, l;
  int mp_blocks, n_blocks, k_blocks, tiles;  // 256-row pair blocks, kBN-column blocks
  int sfa_blocks, sfb_blocks;                // ceil(M/128), ceil(N/128)
  int group_m;                               // raster: pair M-blocks per group
  int c_lines32;                             // C rows start 32-byte aligned
  unsigned* status;
  long long wait_limit;
};

template <int kBN_, int kStages>
struct Dual2smCfg {
  static constexpr int kBN = kBN_;                     // C columns per tile: 64 or 128
  static constexpr int kABytes = kBM * kBK / 2;        // 16 KB
  static constexpr int kBHalfBytes = (kBN / 2) * kBK / 2;   // this CTA's B1 (or B2) rows: 4 or 8 KB
  static constexpr int kBBytes = 2 * kBHalfBytes;      // B1 half, then B2 half
  static constexpr int kSfaBytes = kSfStageBytes;      // 4 atoms of this CTA's A rows
  static constexpr int kSfbBytes = kSfStageBytes;      // 4 atoms of the tile's B1 (or B2) block
  static constexpr int kStageBytes = kABytes + kBBytes + kSfaBytes + 2 * kSfbBytes;   // 30 or 38 KB
  static constexpr int kPairTxBytes = 2 * kStageBytes;  // both CTAs' copies of a stage
  static constexpr int kEpiWarps = 8;                   // 2 per TMEM quadrant
  static constexpr int kColsPerWarp = kBN / 2;         // 32 or 64 columns of gate and of up
  // warp roles: epilogue [0, 8), tile producer 8, MMA 9, scale producer 10
  static constexpr int kProdWarp = kEpiWarps, kMmaWarp = kEpiWarps + 1, kSfProdWarp = kEpiWarps + 2;
  static constexpr int kThreads = 32 * (kEpiWarps + 3);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;
  static constexpr int kTmemCols = 512;
  static constexpr int kAccBufs = 1;
  static constexpr int kAccCols = 2 * kBN;             // gate columns, then up columns
  static constexpr int kSfCol = kAccBufs * kAccCols;
  static constexpr int kSfBufCols = 48;                // per stage: SFA, SFB1, SFB2 x 4 atoms x 4 columns
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(kSfCol + kStages * kSfBufCols <= kTmemCols, "TMEM budget: one scale buffer per stage");
  static_assert(kBN == 64 || kBN == 128, "tile width: a tile lies in one 128-row scale block");
};

struct PairTile2 { int l, mp, nb; };

__device__ __forceinline__ PairTile2 pair2_tile_coord(const Dual2smParams& p, int t) {
  const int per_l = p.mp_blocks * p.n_blocks;
  PairTile2 tc;
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

template <int kBN, int kStages>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(Dual2smCfg<kBN, kStages>::kThreads, 1)
dual_gemm_2sm_kernel(const __grid_constant__ Dual2smParams p) {
  using Cfg = Dual2smCfg<kBN, kStages>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full[kStages], bar_empty[kStages];
  __shared__ uint64_t bar_acc_full[Cfg::kAccBufs], bar_acc_empty[Cfg::kAccBufs];
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
    for (int b = 0; b < Cfg::kAccBufs; ++b) {
      mbar_init(smem_u32(&bar_acc_full[b]), 1);
      mbar_init(smem_u32(&bar_acc_empty[b]), 2 * Cfg::kEpiWarps);   // both CTAs' epilogue warps
    }
    mbar_init(smem_u32(&bar_drain), 1);
    s_abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == Cfg::kProdWarp && lane == 0) {
    tma_prefetch_desc(&p.tmap_a);
    tma_prefetch_desc(&p.tmap_b1);
    tma_prefetch_desc(&p.tmap_b2);
    tma_prefetch_desc(&p.tmap_sfa);
    tma_prefetch_desc(&p.tmap_sfb1);
    tma_prefetch_desc(&p.tmap_sfb2);
  }
  if (warp == Cfg::kMmaWarp) tmem_alloc_pair<Cfg::kTmemCols>(smem_u32(&s_tmem_base));
  tc_fence_before();
  __syncthreads();
  cluster_sync();   // the peer's barriers exist before anyone signals them
  tc_fence_after();
  const uint32_t tmem = s_tmem_base;
  // the prologue above overlaps the previous kernel; global memory only after it
  griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();
  const AbortCtl ctl{&s_abort, p.status, p.wait_limit};
  const int rest_k = p.k / kKStep;   // 64-deep atoms per 128-row block

  if (warp == Cfg::kProdWarp || warp == Cfg::kSfProdWarp) {
    // ------------------------------------------------------------ TMA producers (both CTAs)
    // Two threads issue each stage's copies in parallel: warp kProdWarp the
    // operand tiles, warp kSfProdWarp the scale atoms, all onto the leader's
    // stage barrier (every copy instruction and barrier operation costs its
    // issuing thread tens of cycles).  elect.sync rather than lane == 0: the
    // compiler then knows one thread runs the region and keeps its addresses
    // in uniform registers, which the copy instructions take directly.
    if (elect_one()) {
      const bool tile_role = warp == Cfg::kProdWarp;
      const uint64_t pol = policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      // per stage: ever issued, and the phase of its last issue (abort drain)
      uint32_t issued = 0, last_phase = 0;
      bool ok = true;
      for (int t = pair; t < p.tiles && ok; t += num_pairs) {
        const PairTile2 tc = pair2_tile_coord(p, t);
        const int m0 = tc.mp * 2 * kBM + (int)rank * kBM;   // this CTA's A rows
        const int n0 = tc.nb * kBN;
        const int nb0 = n0 + (int)rank * (kBN / 2);         // this CTA's B1 / B2 rows
        // the second CTA of the last pair block may lie wholly past M (odd
        // ceil(M/128)): its A rows load as zeros, it stores nothing, and it
        // re-reads the last real scale block rather than reading past the tensor
        const int ablk = min(m0 / 128, p.sfa_blocks - 1);
        const int a_atom0 = (tc.l * p.sfa_blocks + ablk) * rest_k;
        const int b_atom0 = (tc.l * p.sfb_blocks + n0 / 128) * rest_k;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!ctl.wait(smem_u32(&bar_empty[stage]), phase ^ 1u, kDevTimeoutStageFree)) {
            ok = false;
            break;
          }
          const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sb = sa + Cfg::kABytes;
          const uint32_t full = mapa_shared(smem_u32(&bar_full[stage]), 0);
          if (tile_role) {
            if (leader) mbar_arrive_expect_tx(smem_u32(&bar_full[stage]), Cfg::kPairTxBytes);
            tma_load_3d_pair(sa, &p.tmap_a, full, kb * 128, m0, tc.l, pol);
            tma_load_3d_pair(sb, &p.tmap_b1, full, kb * 128, nb0, tc.l, pol);
            tma_load_3d_pair(sb + Cfg::kBHalfBytes, &p.tmap_b2, full, kb * 128, nb0, tc.l, pol);
          } else {
            // [SFA][SFB1][SFB2], 4 atoms each
            const uint32_t ssf = sb + Cfg::kBBytes;
            const int ka = kb * (kBK / kKStep);
            tma_load_2d_pair(ssf, &p.tmap_sfa, full, 0, a_atom0 + ka, pol);
            tma_load_2d_pair(ssf + Cfg::kSfaBytes, &p.tmap_sfb1, full, 0, b_atom0 + ka, pol);
            tma_load_2d_pair(ssf + Cfg::kSfaBytes + Cfg::kSfbBytes, &p.tmap_sfb2, full, 0, b_atom0 + ka,
                             pol);
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
      // M = 256, N = kBN, e2m1 x e2m1, e4m3 scales
      constexpr uint32_t idesc = (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                                 ((uint32_t)(256 >> 4) << 24);
      constexpr uint16_t kBoth = 0x3;
      const uint64_t a_desc0 = kmajor_sw128_desc(smem_base);   // stage 0's A tile
      const uint64_t sf_desc0 = sf_atom_desc(smem_base + Cfg::kABytes + Cfg::kBBytes);   // its first SFA atom
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, any = false;
      for (int t = pair; t < p.tiles && ok; t += num_pairs) {
        if (!ctl.wait(smem_u32(&bar_acc_empty[acc]), acc_phase ^ 1u, kDevTimeoutAccFree)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_acc = tmem + acc * Cfg::kAccCols;
        // the tile's B rows start at column (n0 % 128) / 32 of their scale atoms
        const uint32_t b_col = (uint32_t)((pair2_tile_coord(p, t).nb * kBN) % 128) / 32u;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          // both CTAs' tiles and scale atoms landed: one barrier counts it all
          if (!ctl.wait(smem_u32(&bar_full[stage]), phase, kDevTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // descriptors of this stage's tiles and atoms: the stage-0 ones advanced
          const uint32_t so = (uint32_t)stage * Cfg::kStageBytes;
          const uint64_t da = desc_advance(a_desc0, so);
          const uint64_t db = desc_advance(da, Cfg::kABytes);   // this CTA's B1 rows, then B2 rows
          const uint64_t dsf = desc_advance(sf_desc0, so);
          const uint32_t sf_a = tmem + Cfg::kSfCol + stage * Cfg::kSfBufCols;
          const uint32_t sf_b1 = sf_a + 16, sf_b2 = sf_a + 32;
          // per 64-deep step j: its SFA, SFB1 and SFB2 atoms into TMEM
          // (columns [4j, +4) of each 16-column part), then gate and up
          #pragma unroll
          for (int j = 0; j < kBK / kKStep; ++j) {
            const uint64_t dsa = desc_advance(dsf, j * kSfAtom);
            tc_cp_pair_32x128b_x4(sf_a + 4 * j, dsa);
            tc_cp_pair_32x128b_x4(sf_b1 + 4 * j, desc_advance(dsa, Cfg::kSfaBytes));
            tc_cp_pair_32x128b_x4(sf_b2 + 4 * j, desc_advance(dsa, Cfg::kSfaBytes + Cfg::kSfbBytes));
            const uint64_t daj = desc_advance(da, 32 * j), db1 = desc_advance(db, 32 * j);
            const uint32_t acc_in = (kb | j) != 0;
            tc_mma_nvf4_pair_ca<CollectorA::kFill>(d_acc, daj, db1, idesc, sf_a + 4 * j,
                                                  sf_b1 + 4 * j + b_col, acc_in);
            tc_mma_nvf4_pair_ca<CollectorA::kLastUse>(d_acc + kBN, daj, desc_advance(db1, Cfg::kBHalfBytes),
                                                     idesc, sf_a + 4 * j, sf_b2 + 4 * j + b_col, acc_in);
          }
          tc_commit_pair(smem_u32(&bar_empty[stage]), kBoth);   // stage (and scale buffer) free
          any = true;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        tc_commit_pair(smem_u32(&bar_acc_full[acc]), kBoth);
        if (++acc == Cfg::kAccBufs) acc = 0, acc_phase ^= 1u;
      }
      if (!ok && any) {
        tc_commit_pair(smem_u32(&bar_drain), 0x1);
        ctl.drain(smem_u32(&bar_drain), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int quad = warp & 3;        // TMEM lane quadrant
    const int part = warp >> 2;       // columns [kColsPerWarp*part, +kColsPerWarp) of gate and up
    constexpr int kCW = Cfg::kColsPerWarp;
    constexpr int kC16 = kCW / 16;
    const uint32_t acc_empty_leader = mapa_shared(smem_u32(&bar_acc_empty[0]), 0);
    uint32_t acc_phase = 0;
    for (int t = pair; t < p.tiles; t += num_pairs) {
      const PairTile2 tc = pair2_tile_coord(p, t);
      if (!ctl.wait(smem_u32(&bar_acc_full[0]), acc_phase, kDevTimeoutAccFull)) break;
      tc_fence_after();
      const uint32_t t_gate = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(kCW * part);
      const uint32_t t_up = t_gate + Cfg::kBN;
      // pull this warp's gate and up columns into registers, hand TMEM back
      uint32_t w[32];
      if constexpr (kCW == 64) {
        uint32_t g[2][32], u[2][32];
        #pragma unroll
        for (int c = 0; c < 2; ++c) {
          tmem_ld_32x32b_x32(t_gate + 32 * c, g[c]);
          tmem_ld_32x32b_x32(t_up + 32 * c, u[c]);
        }
        tmem_ld_wait();
        #pragma unroll
        for (int c = 0; c < 2; ++c) tmem_regs_ready(g[c]), tmem_regs_ready(u[c]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acc_empty_leader);
        #pragma unroll
        for (int c = 0; c < 2; ++c)
          #pragma unroll
          for (int e = 0; e < 16; ++e)
            w[16 * c + e] = pack_half2(silu_gate(__uint_as_float(g[c][2 * e]), __uint_as_float(u[c][2 * e])),
                                       silu_gate(__uint_as_float(g[c][2 * e + 1]),
                                                 __uint_as_float(u[c][2 * e + 1])));
      } else {
        uint32_t g[kC16][16], u[kC16][16];
        #pragma unroll
        for (int c = 0; c < kC16; ++c) {
          tmem_ld_32x32b_x16(t_gate + 16 * c, g[c]);
          tmem_ld_32x32b_x16(t_up + 16 * c, u[c]);
        }
        tmem_ld_wait();
        #pragma unroll
        for (int c = 0; c < kC16; ++c) tmem_regs_ready16(g[c]), tmem_regs_ready16(u[c]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_remote(acc_empty_leader);
        #pragma unroll
        for (int c = 0; c < kC16; ++c)
          #pragma unroll
          for (int e = 0; e < 8; ++e)
            w[8 * c + e] = pack_half2(silu_gate(__uint_as_float(g[c][2 * e]), __uint_as_float(u[c][2 * e])),
                                      silu_gate(__uint_as_float(g[c][2 * e + 1]),
                                                __uint_as_float(u[c][2 * e + 1])));
        #pragma unroll
        for (int e = 8 * kC16; e < 32; ++e) w[e] = 0u;
      }
      acc_phase ^= 1u;
      // kCW columns per row (32 / 48: two / three 32-byte chunks of a line, 64: a line)
      const int row0 = tc.mp * 2 * kBM + (int)rank * kBM + quad * 32;
      const int col0 = tc.nb * Cfg::kBN + kCW * part;
      __half* c_line0 = p.c + ((size_t)tc.l * p.m + row0) * (size_t)p.n + col0;
      const int cols = min(kCW, p.n - col0);
      if (p.c_lines32)
        store_lines_coalesced_v8(w, c_line0, p.n, p.m - row0, cols);
      else
        store_lines_coalesced(w, c_line0, p.n, p.m - row0, cols);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();   // no MMA, copy or remote arrive of either CTA is still in flight
  if (warp == Cfg::kMmaWarp) {
    tc_fence_after();
    tmem_dealloc_pair<Cfg::kTmemCols>(tmem);
  }
}

}  // namespace nvfp4
