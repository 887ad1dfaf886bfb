// NVFP4 dual GEMM with fused SiLU-gate epilogue, sm_100a: the single-CTA
// kernel, which the host picks for few-tile, long-K shapes (its split-K
// forms); the CTA-pair kernel (dual_gemm_2sm.cuh) serves the others.
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
//   with bulk copies), warp kEpiWarps+1 owns TMEM and issues tcgen05.mma,
//   warps [kEpiWarps+2, kEpiWarps+6) stage the scale factors into TMEM;
// * B1 and B2 tiles sit back to back in shared memory, so for 128-wide tiles
//   one tcgen05.mma with N = 256 computes gate and up together from a single
//   read of the A tile (accumulator columns [0,128) = gate, [128,256) = up);
//   64-wide tiles issue two N=64 MMAs;
// * scale factors reach TMEM through four staging warps (one per 32-lane
//   TMEM quadrant) that read each stage's 512-byte atoms from shared memory
//   and write them with tcgen05.st, every quadrant receiving the full atom
//   rows (the image tcgen05.cp.32x128b.warpx4 would produce).  Staged by
//   CUDA cores the scales cost the tensor pipe nothing (the CTA-pair kernel,
//   dual_gemm_2sm.cuh, copies them with tcgen05.cp from its MMA thread
//   instead).  The scale atoms land on their own mbarrier, so staging
//   overlaps the operand-tile transfer.  Each
//   pipeline stage owns one TMEM scale buffer, rewritten only after the MMAs
//   that read it have released the stage;
// * kAccBufs accumulator sets (gate + up, kBN columns each) in TMEM; with one
//   set the epilogue loads all of its columns to registers and releases TMEM
//   before doing the math and stores, so the next tile's MMAs start early;
// * the epilogue transposes each warp's 32 rows x 64 fp16 columns through
//   shuffles so every store instruction writes whole 128-byte lines;
// * split-K for shapes with too few tiles to fill the GPU, in two forms.
//   Cluster split-K (kCluster = 2 or 4): the splits of a tile run as one
//   thread-block cluster; after the main loop every CTA owns 128/kCluster of
//   the tile's output columns, the others write their fp32 gate/up partials
//   for that slice into the owner's (now idle) pipeline shared memory over
//   the cluster (st.shared::cluster), and the owner sums them in split order
//   (deterministic), applies the SiLU gate and stores.  Workspace split-K
//   (kCluster = 0): each split's partials go to an fp32 global workspace
//   slot; the split that draws the last ticket sums the slots in split order
//   and alone applies the gate (the epilogue is not linear, so the reduction
//   must finish first).
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
  int c_lines32;         // C rows start 32-byte aligned (N % 16 == 0, C 32-byte aligned)
  unsigned* status;
  long long wait_limit;
};

template <int kBN, int kStages, int kEpiWarps, int kAccBufs>
struct DualCfg {
  static constexpr int kABytes = kBM * kBK / 2;
  static constexpr int kBBytes = kBN * kBK / 2;
  static constexpr int kStageBytes = kABytes + 2 * kBBytes + 3 * kSfStageBytes;
  static constexpr int kTxBytes = kABytes + 2 * kBBytes;   // operand tiles (scales land apart)
  static constexpr int kSfWarps = 4;                  // one per TMEM lane quadrant
  static constexpr int kThreads = 32 * (kEpiWarps + 2 + kSfWarps);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;  // + alignment slack
  static constexpr int kTmemCols = 512;
  static constexpr int kAccCols = 2 * kBN;            // gate + up
  static constexpr int kSfCol = kAccBufs * kAccCols;  // TMEM column of the scale buffers
  static constexpr int kSfBufCols = 48;               // per stage: SFA 4x4 + [SFB1|SFB2] 4x8 columns
  static constexpr int kColsPerWarp = kBN / (kEpiWarps / 4);
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(kSfCol + kStages * kSfBufCols <= kTmemCols, "TMEM budget: one scale buffer per stage");
  static_assert(kSfCol % 4 == 0 && kSfBufCols % 4 == 0, "scale columns stay 4-aligned");
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

template <int kBN, int kStages, int kEpiWarps, int kAccBufs, bool kSplitK, int kCluster = 0>
__global__ void __launch_bounds__(DualCfg<kBN, kStages, kEpiWarps, kAccBufs>::kThreads, 1)
dual_gemm_kernel(const __grid_constant__ DualParams p) {
  using Cfg = DualCfg<kBN, kStages, kEpiWarps, kAccBufs>;
  static_assert(kCluster == 0 || (kSplitK && kBN == 128 && kEpiWarps == 8 &&
                                  (kCluster == 2 || kCluster == 4)),
                "cluster split-K: 128-wide tiles, 8 epilogue warps, 2 or 4 splits");
  // cluster split-K receive buffer in the owner's stage ring: per sending
  // split, gate and up of the owned 128/kCluster columns, [col][row] fp32
  constexpr int kOwnCols = kCluster ? 128 / kCluster : 128;
  constexpr int kRxSlotFloats = 2 * kOwnCols * kBM;
  static_assert(kCluster == 0 || (kCluster - 1) * kRxSlotFloats * 4 <= kStages * Cfg::kStageBytes,
                "receive buffer fits the stage ring");
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full[kStages], bar_empty[kStages];
  __shared__ uint64_t bar_sf_landed[kStages];
  __shared__ uint64_t bar_acc_full[kAccBufs], bar_acc_empty[kAccBufs];
  __shared__ uint64_t bar_drain;
  __shared__ uint64_t bar_peer_ready, bar_rx_full;   // cluster split-K exchange
  __shared__ uint32_t s_tmem_base;
  __shared__ volatile int s_abort;
  __shared__ volatile int s_ticket, s_fail;   // split-K epilogue decisions (uniform after a barrier)

  // 1024-byte aligned stage ring (SWIZZLE_128B atoms are 1024 bytes).
  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      // the producer's expect_tx arrival + one per staging warp (+ the TMA bytes)
      mbar_init(smem_u32(&bar_full[s]), 1 + Cfg::kSfWarps);
      mbar_init(smem_u32(&bar_empty[s]), 1);
      mbar_init(smem_u32(&bar_sf_landed[s]), 1);
    }
    for (int b = 0; b < kAccBufs; ++b) {
      mbar_init(smem_u32(&bar_acc_full[b]), 1);
      mbar_init(smem_u32(&bar_acc_empty[b]), kEpiWarps);
    }
    mbar_init(smem_u32(&bar_drain), 1);
    if constexpr (kCluster > 0) {
      mbar_init(smem_u32(&bar_peer_ready), kCluster - 1);        // one arrive per other CTA
      // every lane of the 4 warps holding an owned column range arrives once
      // per 32-column chunk it sends, from each of the kCluster-1 other CTAs
      mbar_init(smem_u32(&bar_rx_full), (kCluster - 1) * 4 * 32 * (kOwnCols / 32));
    }
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
  if constexpr (kCluster > 0) cluster_sync();   // peers' barriers exist before any remote arrive
  tc_fence_after();
  const uint32_t tmem = s_tmem_base;
  const AbortCtl ctl{&s_abort, p.status, p.wait_limit};
  // everything above (barriers, TMEM, descriptor prefetch) overlaps the
  // previous kernel in the stream; global memory only after it completed
  griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();

  if (warp == kEpiWarps) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {   // one thread; uniform registers for the issue
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
          const uint32_t landed = smem_u32(&bar_sf_landed[stage]);
          const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sb1 = sa + Cfg::kABytes;
          const uint32_t sb2 = sb1 + Cfg::kBBytes;
          const uint32_t ssf = sb2 + Cfg::kBBytes;
          // scales first, on their own barrier: the staging warps move them
          // into TMEM while the operand tiles are still landing
          mbar_arrive_expect_tx(landed, 3 * kSfStageBytes);
          const size_t sf_off = (size_t)kb * kSfStageBytes;
          bulk_load(ssf, sfa_t + sf_off, kSfStageBytes, landed, pol);
          bulk_load(ssf + kSfStageBytes, sfb1_t + sf_off, kSfStageBytes, landed, pol);
          bulk_load(ssf + 2 * kSfStageBytes, sfb2_t + sf_off, kSfStageBytes, landed, pol);
          mbar_arrive_expect_tx(full, Cfg::kTxBytes);
          tma_load_3d(sa, &p.tmap_a, full, kb * 128, tc.mb * kBM, tc.l, pol);
          tma_load_3d(sb1, &p.tmap_b1, full, kb * 128, n0, tc.l, pol);
          tma_load_3d(sb2, &p.tmap_b2, full, kb * 128, n0, tc.l, pol);
          issued[stage] = true;
          last_phase[stage] = phase;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
      }
      if (!ok) {  // let in-flight copies land before the CTA winds down
        for (int s = 0; s < kStages; ++s)
          if (issued[s]) {
            ctl.drain(smem_u32(&bar_sf_landed[s]), last_phase[s]);
            ctl.drain_copies(smem_u32(&bar_full[s]), last_phase[s]);
          }
      }
    }
  } else if (warp == kEpiWarps + 1) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {   // one thread; uniform registers for the issue
      // 128-wide tiles: one M=128, N=256 MMA per 64-K step over [B1 tile ; B2 tile];
      // 64-wide tiles: two N=64 MMAs (gate, up)
      constexpr uint32_t idesc = idesc_mxf4nvf4<kBM, kBN == 128 ? 2 * kBN : kBN>();
      const uint64_t a_desc0 = kmajor_sw128_desc(smem_base);   // stage 0's A tile
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
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
          // operand tiles landed and the stage's scales staged into TMEM: one
          // barrier counts both (the TMA bytes and one arrival per staging
          // warp), so this thread checks one barrier per K step (each check
          // costs it ~100 cycles, and its loop sets the pace of small tiles)
          if (!ctl.wait(smem_u32(&bar_full[stage]), phase, kDevTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da0 = desc_advance(a_desc0, (uint32_t)stage * Cfg::kStageBytes);
          const uint64_t db0 = desc_advance(da0, Cfg::kABytes);   // B1 rows then B2 rows
          // scales of k-step j: SFA in [sf_a+4j, +4), SFB1 | SFB2 in [sf_b+8j, +8)
          const uint32_t sf_a = tmem + Cfg::kSfCol + stage * Cfg::kSfBufCols;
          const uint32_t sf_b = sf_a + 16;
          #pragma unroll
          for (int j = 0; j < kBK / kKStep; ++j) {
            const uint64_t da = desc_advance(da0, 32 * j), db = desc_advance(db0, 32 * j);
            const uint32_t accum = kSplitK ? ((kb != kr.kb0) || (j != 0)) : ((kb | j) != 0);
            if constexpr (kBN == 128) {
              // one N=256 MMA over [B1 ; B2]: the 8 scale columns are exactly
              // SFB1 rows 0..127 then SFB2 rows 0..127
              tc_mma_nvf4(d_acc, da, db, idesc, sf_a + 4 * j, sf_b + 8 * j, accum);
            } else {
              // 64-row halves of the atoms sit in columns {0,1} or {2,3}: two N=64 MMAs
              tc_mma_nvf4(d_acc, da, db, idesc, sf_a + 4 * j, sf_b + 8 * j + sub, accum);
              tc_mma_nvf4(d_acc + kBN, da, desc_advance(db, Cfg::kBBytes), idesc, sf_a + 4 * j,
                          sf_b + 8 * j + 4 + sub, accum);
            }
          }
          tc_commit(smem_u32(&bar_empty[stage]));  // frees the stage (and its scale buffer)
          any = true;
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
  } else if (warp >= kEpiWarps + 2) {
    // ------------------------------------------------------------ scale staging
    // Warp w writes TMEM lanes [32*(w%4), +32).  Lane i of every quadrant
    // receives row i of each 512-byte atom (16 bytes = 4 columns): SFA atom j
    // at columns [4j, +4), SFB1 / SFB2 atom j at [16+8j, +4) / [20+8j, +4) of
    // the stage's scale buffer.  The MMA reads the scales of tile row r from
    // lane r, column (base + r/32): with every quadrant holding the full atom
    // rows, that is row r's own four scales.
    const uint32_t t_quad = ((uint32_t)(warp & 3) * 32u) << 16;
    int stage = 0;
    uint32_t phase = 0;
    const int units = kSplitK ? p.tiles * p.splits : p.tiles;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const KRange kr = dual_unit<kSplitK>(p, u);
      bool ok = true;
      for (int kb = kr.kb0; kb < kr.kb1; ++kb) {
        // one lane waits (bounded) so the whole warp takes the same branch,
        // then every lane observes the completed phase itself
        bool got = true;
        if (lane == 0) got = ctl.wait(smem_u32(&bar_sf_landed[stage]), phase, kDevTimeoutTmaFull);
        if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) {
          ok = false;
          break;
        }
        mbar_try_wait(smem_u32(&bar_sf_landed[stage]), phase);
        const uint32_t ssf = smem_base + stage * Cfg::kStageBytes + Cfg::kABytes +
                             2 * Cfg::kBBytes + lane * 16u;
        uint32_t ra[16], rb[32];
        #pragma unroll
        for (int j = 0; j < kBK / kKStep; ++j) {
          const uint4 a = lds_v4(ssf + j * kSfAtom);
          const uint4 b1 = lds_v4(ssf + kSfStageBytes + j * kSfAtom);
          const uint4 b2 = lds_v4(ssf + 2 * kSfStageBytes + j * kSfAtom);
          ra[4 * j + 0] = a.x, ra[4 * j + 1] = a.y, ra[4 * j + 2] = a.z, ra[4 * j + 3] = a.w;
          rb[8 * j + 0] = b1.x, rb[8 * j + 1] = b1.y, rb[8 * j + 2] = b1.z, rb[8 * j + 3] = b1.w;
          rb[8 * j + 4] = b2.x, rb[8 * j + 5] = b2.y, rb[8 * j + 6] = b2.z, rb[8 * j + 7] = b2.w;
        }
        const uint32_t t_buf = tmem + t_quad + Cfg::kSfCol + stage * Cfg::kSfBufCols;
        tmem_st_32x32b_x16(t_buf, ra);
        tmem_st_32x32b_x32(t_buf + 16, rb);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bar_full[stage]));
        if (++stage == kStages) stage = 0, phase ^= 1u;
      }
      if (!ok) break;
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
      if constexpr (kCluster > 0) {
        // ---- cluster split-K: one unit per CTA; this CTA is split `rank`
        const uint32_t rank = (uint32_t)kr.split;
        // this CTA's pipeline is drained: its stage ring may now receive
        if (et == 0)
          for (uint32_t o = 0; o < (uint32_t)kCluster; ++o)
            if (o != rank) mbar_arrive_cluster(mapa_shared(smem_u32(&bar_peer_ready), o));
        bool ok = true;
        if (lane == 0) ok = ctl.wait_cluster(smem_u32(&bar_peer_ready), 0, kDevTimeoutPeers);
        ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
        if (!ok) break;
        mbar_try_wait_cluster(smem_u32(&bar_peer_ready), 0);
        // send the 32-column chunks other CTAs own ([gate|up][col][row] in
        // slot (rank < owner ? rank : rank - 1) of the owner's buffer)
        #pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int tcol = part * kCW + 32 * c;          // tile column of the chunk
          const uint32_t owner = (uint32_t)(tcol / kOwnCols);
          if (owner == rank) continue;
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(t_gate + 32 * c, g);
          tmem_ld_32x32b_x32(t_up + 32 * c, u);
          tmem_ld_wait();
          tmem_regs_ready(g), tmem_regs_ready(u);
          const uint32_t slot = rank < owner ? rank : rank - 1;
          const uint32_t rx = mapa_shared(smem_base, owner) +
                              4u * (slot * kRxSlotFloats + (uint32_t)(tcol - owner * kOwnCols) * kBM +
                                    (uint32_t)trow);
          #pragma unroll
          for (int i = 0; i < 32; ++i) {
            st_shared_cluster_f32(rx + 4u * i * kBM, __uint_as_float(g[i]));
            st_shared_cluster_f32(rx + 4u * (kOwnCols + i) * kBM, __uint_as_float(u[i]));
          }
          mbar_arrive_cluster(mapa_shared(smem_u32(&bar_rx_full), owner));   // release: the stores above
        }
        // reduce the chunk(s) this CTA owns: splits in order 0..kCluster-1
        uint32_t w[32];
        int own_c0 = -1, own_n = 0;
        #pragma unroll
        for (int c = 0; c < 2; ++c) {
          const int tcol = part * kCW + 32 * c;
          if ((uint32_t)(tcol / kOwnCols) != rank) continue;
          if (own_c0 < 0) {
            own_c0 = c;
            bool got_rx = true;
            if (lane == 0) got_rx = ctl.wait_cluster(smem_u32(&bar_rx_full), 0, kDevTimeoutPeers);
            if (!__shfl_sync(0xffffffffu, got_rx ? 1 : 0, 0)) { ok = false; break; }
            mbar_try_wait_cluster(smem_u32(&bar_rx_full), 0);
          }
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(t_gate + 32 * c, g);
          tmem_ld_32x32b_x32(t_up + 32 * c, u);
          tmem_ld_wait();
          tmem_regs_ready(g), tmem_regs_ready(u);
          const float* rxl = reinterpret_cast<const float*>(smem_raw + (smem_base - smem_u32(smem_raw))) +
                             (tcol - (int)rank * kOwnCols) * kBM + trow;
          #pragma unroll
          for (int e = 0; e < 16; ++e) {
            float gs[2], us[2];
            #pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int i = 2 * e + h;
              float ga = 0.f, ua = 0.f;
              #pragma unroll
              for (int sp = 0; sp < kCluster; ++sp) {
                if (sp == (int)rank) {
                  ga += __uint_as_float(g[i]);
                  ua += __uint_as_float(u[i]);
                } else {
                  const float* slot = rxl + (sp < (int)rank ? sp : sp - 1) * kRxSlotFloats;
                  ga += slot[i * kBM];
                  ua += slot[(kOwnCols + i) * kBM];
                }
              }
              gs[h] = ga, us[h] = ua;
            }
            // owned chunks: both (2 splits, slot 16c) or one (4 splits, slot 0)
            w[(kOwnCols == 64 ? 16 * c : 0) + e] = pack_half2(silu_gate(gs[0], us[0]), silu_gate(gs[1], us[1]));
          }
          ++own_n;
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[acc]));
        if (++acc == kAccBufs) acc = 0, acc_phase ^= 1u;
        if (!ok) break;
        if (own_n > 0) {
          const int row0 = tc.mb * kBM + quad * 32;
          const int col0 = tc.nb * kBN + part * kCW + 32 * own_c0;
          __half* c_line0 = p.c + ((size_t)tc.l * p.m + row0) * (size_t)p.n + col0;
          const int cols = min(32 * own_n, p.n - col0);
          if (p.c_lines32)
            store_lines_coalesced_v8(w, c_line0, p.n, p.m - row0, cols);
          else
            store_lines_coalesced(w, c_line0, p.n, p.m - row0, cols);
        }
        continue;
      }
      // SiLU gate -> fp16 words w (this lane's row, 64 columns)
      uint32_t w[32];
      if constexpr (!kSplitK) {
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
        #pragma unroll
        for (int c = 0; c < 2; ++c)
          #pragma unroll
          for (int e = 0; e < 16; ++e)
            w[16 * c + e] = pack_half2(silu_gate(__uint_as_float(g[c][2 * e]), __uint_as_float(u[c][2 * e])),
                                       silu_gate(__uint_as_float(g[c][2 * e + 1]),
                                                 __uint_as_float(u[c][2 * e + 1])));
      } else {
        // Every split publishes its partial in its own slot ([col][row]: a
        // warp writes 128 contiguous bytes per column), fences, and draws a
        // ticket; whoever draws the last ticket finds all other partials
        // already visible, sums all slots in split order (deterministic) and
        // alone applies the SiLU gate.  The host's split choice gives each
        // CTA at most one unit, so TMEM is drained one 32-column chunk at a
        // time (fewer live registers; no next tile waits for the accumulator).
        const size_t slot_elems = (size_t)2 * kBN * kBM;
        float* slots = p.ws + (size_t)kr.tile * p.splits * slot_elems;
        float* own = slots + (size_t)kr.split * slot_elems;
        #pragma unroll
        for (int c = 0; c < 2; ++c) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(t_gate + 32 * c, g);
          tmem_ld_32x32b_x32(t_up + 32 * c, u);
          tmem_ld_wait();
          tmem_regs_ready(g), tmem_regs_ready(u);
          #pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int col = part * kCW + 32 * c + i;
            __stcg(own + (size_t)col * kBM + trow, __uint_as_float(g[i]));
            __stcg(own + (size_t)(kBN + col) * kBM + trow, __uint_as_float(u[i]));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[acc]));
        if (++acc == kAccBufs) acc = 0, acc_phase ^= 1u;
        __threadfence();
        named_bar_sync(1, kEpiThreads);
        if (et == 0) s_ticket = atomicAdd(&p.ws_ctr[kr.tile], 1);
        named_bar_sync(1, kEpiThreads);
        if (s_ticket != p.splits - 1) continue;
        __threadfence();
        if (et == 0) p.ws_ctr[kr.tile] = 0;   // zero again for the next call
        #pragma unroll
        for (int c = 0; c < 2; ++c) {
          float g[32], u[32];
          #pragma unroll
          for (int i = 0; i < 32; ++i) g[i] = u[i] = 0.f;
          for (int sp = 0; sp < p.splits; ++sp) {
            const float* slot = slots + (size_t)sp * slot_elems;
            #pragma unroll
            for (int i = 0; i < 32; ++i) {
              const int col = part * kCW + 32 * c + i;
              g[i] += __ldcg(slot + (size_t)col * kBM + trow);
              u[i] += __ldcg(slot + (size_t)(kBN + col) * kBM + trow);
            }
          }
          #pragma unroll
          for (int e = 0; e < 16; ++e)
            w[16 * c + e] = pack_half2(silu_gate(g[2 * e], u[2 * e]), silu_gate(g[2 * e + 1], u[2 * e + 1]));
        }
      }
      // Whole-line stores: the warp transposes its 32 rows x 64 columns so
      // each store instruction writes complete 128-byte lines (32-byte
      // stores where every row start is 32-byte aligned).  Measured on B200:
      // per-lane 16-byte row stores cost ~90 us of the 8192 x 14336 x 4096
      // call, full-line stores ~30.
      const int row0 = tc.mb * kBM + quad * 32;
      const int col0 = tc.nb * kBN + part * kCW;
      __half* c_line0 = p.c + ((size_t)tc.l * p.m + row0) * (size_t)p.n + col0;
      if (p.c_lines32)
        store_lines_coalesced_v8(w, c_line0, p.n, p.m - row0, p.n - col0);
      else
        store_lines_coalesced(w, c_line0, p.n, p.m - row0, p.n - col0);
    }
  }

  tc_fence_before();
  __syncthreads();
  // cluster split-K: no CTA exits while a peer may still write into its
  // shared memory or arrive on its barriers
  if constexpr (kCluster > 0) cluster_sync();
  if (warp == kEpiWarps + 1) {
    tc_fence_after();
    tmem_dealloc<Cfg::kTmemCols>(tmem);
  }
}

}  // namespace nvfp4
