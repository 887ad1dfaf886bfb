// NVFP4 dual GEMM with fused SiLU-gate epilogue, sm_100a.
//
//   C[l] = silu(A[l] . B1[l]ᵀ) * (A[l] . B2[l]ᵀ)   (fp32 accumulate, fp16 out)
//
// Same computation as the reference's ref_kernel
// (nvfp4_dual_gemm/reference.py:27-77) and its submissions' custom_kernel
// (e.g. nvfp4_dual_gemm/submission_v4.py:1256-1284); own design:
//
// * persistent grid (one CTA per SM), static round-robin over output tiles in
//   a grouped-M raster so concurrently running CTAs share A rows and B
//   columns in L2;
// * warp roles: warps [0, kEpiWarps) drain TMEM and run the epilogue, warp
//   kEpiWarps issues TMA (A, B1, B2 tiles with 128-byte swizzle, scale atoms
//   with bulk copies), warp kEpiWarps+1 owns TMEM and issues tcgen05.cp +
//   tcgen05.mma;
// * B1 and B2 tiles sit back to back in shared memory, so for 128-wide tiles
//   one tcgen05.mma with N = 256 computes gate and up together from a single
//   read of the A tile (accumulator columns [0,128) = gate, [128,256) = up);
//   64-wide tiles issue two N=64 MMAs;
// * scale factors go shared -> TMEM with tcgen05.cp (one 512-byte atom per
//   64-K step per operand); the scale region is double-buffered across
//   stages, so copying the next stage's scales never has to wait for the
//   MMAs still reading the current ones;
// * kAccBufs accumulator sets (gate + up, kBN columns each) in TMEM; with one
//   set the epilogue loads all of its columns to registers and releases TMEM
//   before doing the math and stores, so the next tile's MMAs start early;
// * split-K for shapes with too few tiles to fill the GPU: each split's
//   partial gate/up sums go to an fp32 workspace slot; the split that draws
//   the last ticket sums the slots in split order and alone applies the SiLU
//   gate (the epilogue is not linear, so the reduction must finish first).
#pragma once
#include <cuda.h>
#include "kernel_common.cuh"

namespace nvfp4 {

struct DualParams {
  CUtensorMap tmap_a;    // bytes [L][M][K/2], box {128 B, 128 rows, 1}
  CUtensorMap tmap_b1;   // bytes [L][N][K/2], box {128 B, BN rows, 1}
  CUtensorMap tmap_b2;
  const uint8_t* sfa;    // permuted scale atoms [L][ceil(M/128)][K/64][512]
  const uint8_t* sfb1;   // [L][ceil(N/128)][K/64][512]
  const uint8_t* sfb2;
  __half* c;             // [L][M][N]
  int m, n, k, l;
  int m_blocks, n_blocks, k_blocks, tiles;
  int group_m;           // raster: M-blocks per group
  // split-K (splits > 1, 128-wide tiles only): work unit u = tile * splits +
  // split covers k-blocks [split*k_blocks/splits, (split+1)*k_blocks/splits)
  int splits;
  float* ws;             // `splits` fp32 partial slots per tile, [256 cols][128 rows] each
  int* ws_ctr;           // one ticket counter per tile; zero between calls
  unsigned* status;
  long long wait_limit;
};

template <int kBN, int kStages, int kEpiWarps, int kAccBufs>
struct DualCfg {
  static constexpr int kABytes = kBM * kBK / 2;
  static constexpr int kBBytes = kBN * kBK / 2;
  static constexpr int kStageBytes = kABytes + 2 * kBBytes + 3 * kSfStageBytes;
  static constexpr int kTxBytes = kStageBytes;
  static constexpr int kThreads = 32 * (kEpiWarps + 2);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;  // + alignment slack
  static constexpr int kTmemCols = 512;
  static constexpr int kAccCols = 2 * kBN;            // gate + up
  static constexpr int kSfCol = kAccBufs * kAccCols;  // TMEM column of the scale regions
  static constexpr int kSfBufCols = 48;               // per buffer: SFA 4x4 + SFB 4x8 columns
  static constexpr int kColsPerWarp = kBN / (kEpiWarps / 4);
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(kSfCol + 2 * kSfBufCols <= kTmemCols, "TMEM budget");
  static_assert(kSfCol % 4 == 0 && kSfBufCols % 4 == 0, "tcgen05.cp needs 4-column alignment");
  static_assert(kEpiWarps % 4 == 0, "epilogue warps cover all four TMEM lane quadrants");
  static_assert(kColsPerWarp % 32 == 0, "epilogue loads 32 columns at a time");
  static_assert(kBN == 64 || kBN == 128, "tile N");
};

struct TileCoord { int l, mb, nb; };

// Grouped-M raster: tiles of `group_m` consecutive M-blocks are walked
// column by column, so ~148 concurrent tiles touch few A and B blocks.
__device__ __forceinline__ TileCoord dual_tile_coord(const DualParams& p, int t) {
  const int per_l = p.m_blocks * p.n_blocks;
  TileCoord tc;
  tc.l = t / per_l;
  const int local = t - tc.l * per_l;
  const int span = p.group_m * p.n_blocks;
  const int g = local / span;
  const int first_mb = g * p.group_m;
  const int gsz = min(p.m_blocks - first_mb, p.group_m);
  const int r = local - g * span;
  tc.mb = first_mb + r % gsz;
  tc.nb = r / gsz;
  return tc;
}

struct KRange { int tile, split, kb0, kb1; };

template <bool kSplitK>
__device__ __forceinline__ KRange dual_unit(const DualParams& p, int u) {
  if constexpr (!kSplitK) return KRange{u, 0, 0, p.k_blocks};   // one unit per tile
  KRange r;
  r.tile = u / p.splits;
  r.split = u - r.tile * p.splits;
  r.kb0 = r.split * p.k_blocks / p.splits;          // splits <= 16: no 32-bit overflow
  r.kb1 = (r.split + 1) * p.k_blocks / p.splits;
  return r;
}

template <int kBN, int kStages, int kEpiWarps, int kAccBufs, bool kSplitK>
__global__ void __launch_bounds__(DualCfg<kBN, kStages, kEpiWarps, kAccBufs>::kThreads, 1)
dual_gemm_kernel(const __grid_constant__ DualParams p) {
  using Cfg = DualCfg<kBN, kStages, kEpiWarps, kAccBufs>;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full[kStages], bar_empty[kStages];
  __shared__ uint64_t bar_acc_full[kAccBufs], bar_acc_empty[kAccBufs];
  __shared__ uint64_t bar_drain;
  __shared__ uint32_t s_tmem_base;
  __shared__ volatile int s_abort;
  __shared__ volatile int s_ticket, s_fail;   // split-K epilogue decisions (uniform after a barrier)

  // 1024-byte aligned stage ring (SWIZZLE_128B atoms are 1024 bytes).
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&bar_full[s]), 1);
      mbar_init(smem_u32(&bar_empty[s]), 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(smem_u32(&bar_acc_full[b]), 1);
      mbar_init(smem_u32(&bar_acc_empty[b]), kEpiWarps);
    }
    mbar_init(smem_u32(&bar_drain), 1);
    s_abort = 0;
    s_fail = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == kEpiWarps) {
    if (lane == 0) {
      tma_prefetch_desc(&p.tmap_a);
      tma_prefetch_desc(&p.tmap_b1);
      tma_prefetch_desc(&p.tmap_b2);
    }
  }
  if (warp == kEpiWarps + 1) tmem_alloc<Cfg::kTmemCols>(smem_u32(&s_tmem_base));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem_base;
  const AbortCtl ctl{&s_abort, p.status, p.wait_limit};

  if (warp == kEpiWarps) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol = policy_evict_normal();
      const int rest_k = p.k_blocks * (kBK / kKStep);  // 64-K atoms per 128 rows
      const size_t sfa_l = (size_t)p.m_blocks * rest_k * kSfAtom;
      const size_t sfb_l = (size_t)((p.n + 127) / 128) * rest_k * kSfAtom;
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_phase[kStages];
      bool issued[kStages];
      for (int s = 0; s < kStages; ++s) issued[s] = false, last_phase[s] = 0;
      bool ok = true;
      const int units = kSplitK ? p.tiles * p.splits : p.tiles;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const KRange kr = dual_unit<kSplitK>(p, u);
        const TileCoord tc = dual_tile_coord(p, kr.tile);
        const int n0 = tc.nb * kBN;
        const uint8_t* sfa_t = p.sfa + tc.l * sfa_l + (size_t)tc.mb * rest_k * kSfAtom;
        const uint8_t* sfb1_t = p.sfb1 + tc.l * sfb_l + (size_t)(n0 / 128) * rest_k * kSfAtom;
        const uint8_t* sfb2_t = p.sfb2 + tc.l * sfb_l + (size_t)(n0 / 128) * rest_k * kSfAtom;
        for (int kb = kr.kb0; kb < kr.kb1; ++kb) {
          if (!ctl.wait(smem_u32(&bar_empty[stage]), phase ^ 1u, kDevTimeoutStageFree)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&bar_full[stage]);
          const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sb1 = sa + Cfg::kABytes;
          const uint32_t sb2 = sb1 + Cfg::kBBytes;
          const uint32_t ssf = sb2 + Cfg::kBBytes;
          mbar_arrive_expect_tx(full, Cfg::kTxBytes);
          tma_load_3d(sa, &p.tmap_a, full, kb * 128, tc.mb * kBM, tc.l, pol);
          tma_load_3d(sb1, &p.tmap_b1, full, kb * 128, n0, tc.l, pol);
          tma_load_3d(sb2, &p.tmap_b2, full, kb * 128, n0, tc.l, pol);
          const size_t sf_off = (size_t)kb * kSfStageBytes;
          bulk_load(ssf, sfa_t + sf_off, kSfStageBytes, full, pol);
          bulk_load(ssf + kSfStageBytes, sfb1_t + sf_off, kSfStageBytes, full, pol);
          bulk_load(ssf + 2 * kSfStageBytes, sfb2_t + sf_off, kSfStageBytes, full, pol);
          issued[stage] = true;
          last_phase[stage] = phase;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
      }
      if (!ok) {  // let in-flight copies land before the CTA winds down
        for (int s = 0; s < kStages; ++s)
          if (issued[s]) ctl.drain(smem_u32(&bar_full[s]), last_phase[s]);
      }
    }
  } else if (warp == kEpiWarps + 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // 128-wide tiles: one M=128, N=256 MMA per 64-K step over [B1 tile ; B2 tile];
      // 64-wide tiles: two N=64 MMAs (gate, up)
      constexpr uint32_t idesc = idesc_mxf4nvf4<kBM, kBN == 128 ? 2 * kBN : kBN>();
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      uint32_t sf_buf = 0;
      bool ok = true, any = false;
      const int units = kSplitK ? p.tiles * p.splits : p.tiles;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        const KRange kr = dual_unit<kSplitK>(p, u);
        const TileCoord tc = dual_tile_coord(p, kr.tile);
        // 64-wide tiles use half of each 128-row scale atom: columns {0,1} or {2,3}
        const uint32_t sub = (kBN == 64) ? (uint32_t)((tc.nb & 1) * 2) : 0u;
        if (!ctl.wait(smem_u32(&bar_acc_empty[acc]), acc_phase ^ 1u, kDevTimeoutAccFree)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_acc = tmem + acc * Cfg::kAccCols;
        for (int kb = kr.kb0; kb < kr.kb1; ++kb) {
          if (!ctl.wait(smem_u32(&bar_full[stage]), phase, kDevTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sb = sa + Cfg::kABytes;             // B1 rows then B2 rows
          const uint32_t ssf = sb + 2 * Cfg::kBBytes;
          const uint32_t sf_a = tmem + Cfg::kSfCol + sf_buf * Cfg::kSfBufCols;
          const uint32_t sf_b = sf_a + 16;
          // scale atoms for k-step j: SFA -> [sf_a+4j, +4), SFB1 | SFB2 -> [sf_b+8j, +8)
          // (tcgen05.cp destinations stay 4-column aligned)
          #pragma unroll
          for (int j = 0; j < kBK / kKStep; ++j) {
            tc_cp_sf_atom(sf_a + 4 * j, sf_atom_desc(ssf + j * kSfAtom));
            tc_cp_sf_atom(sf_b + 8 * j, sf_atom_desc(ssf + kSfStageBytes + j * kSfAtom));
            tc_cp_sf_atom(sf_b + 8 * j + 4, sf_atom_desc(ssf + 2 * kSfStageBytes + j * kSfAtom));
          }
          #pragma unroll
          for (int j = 0; j < kBK / kKStep; ++j) {
            const uint64_t da = kmajor_sw128_desc(sa + 32 * j);
            const uint32_t accum = kSplitK ? ((kb != kr.kb0) || (j != 0)) : ((kb | j) != 0);
            if constexpr (kBN == 128) {
              // one N=256 MMA over [B1 ; B2]: the 8 scale columns are exactly
              // SFB1 rows 0..127 then SFB2 rows 0..127
              tc_mma_nvf4(d_acc, da, kmajor_sw128_desc(sb + 32 * j), idesc, sf_a + 4 * j,
                          sf_b + 8 * j, accum);
            } else {
              // 64-row halves of the atoms sit in columns {0,1} or {2,3}: two N=64 MMAs
              tc_mma_nvf4(d_acc, da, kmajor_sw128_desc(sb + 32 * j), idesc, sf_a + 4 * j,
                          sf_b + 8 * j + sub, accum);
              tc_mma_nvf4(d_acc + kBN, da, kmajor_sw128_desc(sb + Cfg::kBBytes + 32 * j), idesc,
                          sf_a + 4 * j, sf_b + 8 * j + 4 + sub, accum);
            }
          }
          tc_commit(smem_u32(&bar_empty[stage]));  // frees the stage once these MMAs finish
          any = true;
          sf_buf ^= 1u;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        tc_commit(smem_u32(&bar_acc_full[acc]));  // accumulators ready for the epilogue
        if (++acc == kAccBufs) acc = 0, acc_phase ^= 1u;
      }
      if (!ok && any) {  // no MMA may still write TMEM when it is released
        tc_commit(smem_u32(&bar_drain));
        ctl.drain(smem_u32(&bar_drain), 0);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;             // TMEM lane quadrant this warp may access
    const int part = warp >> 2;            // which 64-column slice of the tile
    constexpr int kCW = Cfg::kColsPerWarp;
    static_assert(kCW == 64, "64 columns (one 128-byte fp16 line) per lane");
    constexpr int kEpiThreads = 32 * kEpiWarps;
    const int et = threadIdx.x;                          // epilogue thread index
    const int trow = quad * 32 + (int)lane;              // row within the tile
    int acc = 0;
    uint32_t acc_phase = 0;
    const int units = kSplitK ? p.tiles * p.splits : p.tiles;
    for (int uu = blockIdx.x; uu < units; uu += gridDim.x) {
      const KRange kr = dual_unit<kSplitK>(p, uu);
      const TileCoord tc = dual_tile_coord(p, kr.tile);
      const bool got = ctl.wait(smem_u32(&bar_acc_full[acc]), acc_phase, kDevTimeoutAccFull);
      if constexpr (!kSplitK) {
        if (!got) break;
      } else {
        // split-K: every epilogue thread must reach each named barrier, so
        // failures become a shared decision read after the barrier
        if (!got) s_fail = 1;
        named_bar_sync(1, kEpiThreads);
        if (s_fail) break;
      }
      tc_fence_after();
      const uint32_t t_gate = tmem + ((uint32_t)(quad * 32) << 16) + acc * Cfg::kAccCols + part * kCW;
      const uint32_t t_up = t_gate + kBN;
      // pull gate and up for this lane's row into registers, hand TMEM back
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
      if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[acc]));
      if (++acc == kAccBufs) acc = 0, acc_phase ^= 1u;
      if constexpr (kSplitK) {
        // Every split publishes its partial in its own slot ([col][row]: a
        // warp writes 128 contiguous bytes per column), fences, and draws a
        // ticket; whoever draws the last ticket finds all other partials
        // already visible, sums all slots in split order (deterministic) and
        // alone applies the SiLU gate.
        const size_t slot_elems = (size_t)2 * kBN * kBM;
        float* slots = p.ws + (size_t)kr.tile * p.splits * slot_elems;
        float* own = slots + (size_t)kr.split * slot_elems;
        #pragma unroll
        for (int c = 0; c < 2; ++c)
          #pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int col = part * kCW + 32 * c + i;
            __stcg(own + (size_t)col * kBM + trow, __uint_as_float(g[c][i]));
            __stcg(own + (size_t)(kBN + col) * kBM + trow, __uint_as_float(u[c][i]));
          }
        __threadfence();
        named_bar_sync(1, kEpiThreads);
        if (et == 0) s_ticket = atomicAdd(&p.ws_ctr[kr.tile], 1);
        named_bar_sync(1, kEpiThreads);
        if (s_ticket != p.splits - 1) continue;
        __threadfence();
        if (et == 0) p.ws_ctr[kr.tile] = 0;   // zero again for the next call
        #pragma unroll
        for (int c = 0; c < 2; ++c)
          #pragma unroll
          for (int i = 0; i < 32; ++i) g[c][i] = u[c][i] = 0u;
        for (int sp = 0; sp < p.splits; ++sp) {
          const float* slot = slots + (size_t)sp * slot_elems;
          #pragma unroll
          for (int c = 0; c < 2; ++c)
            #pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = part * kCW + 32 * c + i;
              g[c][i] = __float_as_uint(__uint_as_float(g[c][i]) +
                                        __ldcg(slot + (size_t)col * kBM + trow));
              u[c][i] = __float_as_uint(__uint_as_float(u[c][i]) +
                                        __ldcg(slot + (size_t)(kBN + col) * kBM + trow));
            }
        }
      }
      // each lane writes its own row's 128-byte line (8 x 16 B); measured
      // faster here than a shuffle-transposed full-line store (the extra
      // epilogue instructions slow the MMA and TMA warps more than the
      // partial-line writes cost)
      const int row = tc.mb * kBM + quad * 32 + (int)lane;
      const int col0 = tc.nb * kBN + part * kCW;
      if (row < p.m) {
        __half* crow = p.c + ((size_t)tc.l * p.m + row) * (size_t)p.n + col0;
        #pragma unroll
        for (int c = 0; c < 2; ++c) {
          #pragma unroll
          for (int v = 0; v < 4; ++v) {
            if (col0 + 32 * c + 8 * v < p.n) {
              uint32_t w[4];
              #pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int i = 8 * v + 2 * e;
                w[e] = pack_half2(silu_gate(__uint_as_float(g[c][i]), __uint_as_float(u[c][i])),
                                  silu_gate(__uint_as_float(g[c][i + 1]), __uint_as_float(u[c][i + 1])));
              }
              st_global_v4(crow + 32 * c + 8 * v, w[0], w[1], w[2], w[3]);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kEpiWarps + 1) {
    tc_fence_after();
    tmem_dealloc<Cfg::kTmemCols>(tmem);
  }
}

}  // namespace nvfp4
