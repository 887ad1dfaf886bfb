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
// * 128x256 tiles (one N=256 MMA per 64-K step, one accumulator buffer whose
//   columns the epilogue pulls into registers before releasing it) or
//   128x128 tiles (two accumulator buffers, so the epilogue of one tile
//   overlaps the MMAs of the next); empty groups are compacted out on the host;
// * scale factors reach TMEM as in the dual kernel: they land on their own
//   mbarrier and four staging warps (one per TMEM lane quadrant) write each
//   stage's atoms with tcgen05.st into that stage's TMEM scale buffer, so
//   the tensor pipe runs MMAs only.
// The host picks this kernel for short-K groups and the MoE path; long-K
// groups go to the CTA-pair kernel (grouped_gemm_2sm.cuh).
#pragma once
#include <cuda.h>
#include "kernel_common.cuh"

namespace nvfp4 {

struct GroupInfo {
  const uint8_t* sfa;   // permuted scale atoms [L][ceil(M/128)][K/64][512]
  const uint8_t* sfb;   // [L][ceil(N/128)][K/64][512]
  __half* c;            // [L][M][N]
  int m, n, k, l;
  int m_blocks, n_blocks, tile_start;
  int lines32;          // C rows start 32-byte aligned (N % 16 == 0, C 32-byte aligned)
};

template <int kMaxGroups>
struct GroupedParams {
  CUtensorMap tmap_a[kMaxGroups];  // bytes [L][M][K/2], box {128 B, 128 rows, 1}
  CUtensorMap tmap_b[kMaxGroups];  // bytes [L][N][K/2], box {128 B, BN rows, 1}
  GroupInfo g[kMaxGroups];
  int num_groups, tiles;
  int chained;   // a later launch of the same call: see the CTA-pair kernel
  unsigned* status;
  long long wait_limit;
};

template <int kBN, int kStages, int kEpiWarps, int kAccBufs>
struct GroupedCfg {
  static constexpr int kABytes = kBM * kBK / 2;
  static constexpr int kBBytes = kBN * kBK / 2;
  static constexpr int kSfbAtoms = kBN / 128;                  // 128-row scale atoms per tile
  static constexpr int kSfbBytes = kSfbAtoms * kSfStageBytes;
  static constexpr int kStageBytes = kABytes + kBBytes + kSfStageBytes + kSfbBytes;
  static constexpr int kSfWarps = 4;                           // one per TMEM lane quadrant
  static constexpr int kThreads = 32 * (kEpiWarps + 2 + kSfWarps);
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;
  static constexpr int kTmemCols = 512;
  static constexpr int kSfCol = kAccBufs * kBN;
  static constexpr int kSfBufCols = 16 + 16 * kSfbAtoms;       // SFA 4x4 + SFB 4x(4*atoms), per stage
  static constexpr int kColsPerWarp = kBN / (kEpiWarps / 4);
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-byte aligned");
  static_assert(kSfCol + kStages * kSfBufCols <= kTmemCols, "TMEM budget: one scale buffer per stage");
  static_assert(kSfCol % 4 == 0 && kSfBufCols % 4 == 0, "scale columns stay 4-aligned");
  static_assert(kBN == 128 || kBN == 256, "tile N");
  static_assert(kEpiWarps % 4 == 0 && kColsPerWarp % 32 == 0, "epilogue split");
};

// MoE mode: the experts' A operands are consecutive row ranges of one packed
// buffer (the MoE dispatch's output) and their sizes live on the device, so
// the launch needs no host round trip.  Expert e0 + i has counts[e0 + i]
// rows from row row_offsets[e0 + i] and its scale atoms from 128-row block
// atom_offsets[e0 + i] of sfa; its output rows are the same rows of c.  The
// tile schedule is built in shared memory from those arrays when the kernel
// starts.  A tile's rows past its expert's count belong to the next expert:
// they are computed and never stored.
template <int kMaxExperts>
struct MoeGemmParams {
  CUtensorMap tmap_a;                // packed rows [rows][K/2], box {128 B, 128 rows, 1}
  CUtensorMap tmap_b[kMaxExperts];   // expert weights [N][K/2], box {128 B, BN rows, 1}
  const uint8_t* sfb[kMaxExperts];   // [ceil(N/128)][K/64][512]
  const uint8_t* sfa;                // dispatch scale atoms
  const int* counts;                 // device arrays of the dispatch, indexed e0 + i
  const int* row_offsets;
  const int* atom_offsets;
  __half* c;                         // [rows][N]
  int e0, experts, n, k, lines32;
  int chained;                       // always 0: one launch per dispatch chunk waits as usual
  unsigned* status;
  long long wait_limit;
};

struct GTile { int g, l, mb, nb; };

// What the kernel roles need of one group.
struct GroupView {
  const CUtensorMap* tmap_a;
  const CUtensorMap* tmap_b;
  int a_row0;                        // first row of the group in tmap_a
  const uint8_t* sfa;
  const uint8_t* sfb;
  __half* c;
  int m, n, k, l, m_blocks, n_blocks, lines32;
};

// Tile schedule: the table mode reads the parameter block, the MoE mode a
// shared-memory copy of the device sizes (filled once per CTA).
template <class P, int kBN> struct Schedule;

template <int kMaxGroups, int kBN>
struct Schedule<GroupedParams<kMaxGroups>, kBN> {
  struct Storage {};
  const GroupedParams<kMaxGroups>& p;
  __device__ Schedule(const GroupedParams<kMaxGroups>& p_, Storage&) : p(p_) {}
  __device__ static constexpr bool needs_fill() { return false; }
  __device__ void fill() {}
  __device__ int tiles() const { return p.tiles; }
  __device__ GTile tile(int t) const {
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
  __device__ GroupView view(int g) const {
    const GroupInfo& gi = p.g[g];
    return GroupView{&p.tmap_a[g], &p.tmap_b[g], 0, gi.sfa, gi.sfb, gi.c, gi.m, gi.n, gi.k, gi.l,
                     gi.m_blocks, gi.n_blocks, gi.lines32};
  }
};

template <int kMaxExperts, int kBN>
struct Schedule<MoeGemmParams<kMaxExperts>, kBN> {
  struct Storage {
    int tile_start[kMaxExperts + 1];
    int rows[kMaxExperts], row0[kMaxExperts], atom0[kMaxExperts];
  };
  const MoeGemmParams<kMaxExperts>& p;
  Storage& s;
  __device__ Schedule(const MoeGemmParams<kMaxExperts>& p_, Storage& s_) : p(p_), s(s_) {}
  __device__ static constexpr bool needs_fill() { return true; }
  // every thread calls this (after the dispatch that wrote the sizes has
  // completed), then __syncthreads()
  __device__ void fill() {
    const int n_blocks = (p.n + kBN - 1) / kBN;
    for (int i = threadIdx.x; i < p.experts; i += blockDim.x) {
      s.rows[i] = p.counts[p.e0 + i];
      s.row0[i] = p.row_offsets[p.e0 + i];
      s.atom0[i] = p.atom_offsets[p.e0 + i];
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      int t = 0;
      for (int i = 0; i < p.experts; ++i) {
        s.tile_start[i] = t;
        t += (s.rows[i] + kBM - 1) / kBM * n_blocks;
      }
      s.tile_start[p.experts] = t;
    }
  }
  __device__ int tiles() const { return s.tile_start[p.experts]; }
  __device__ GTile tile(int t) const {
    int lo = 0, hi = p.experts - 1;     // largest i with tile_start <= t and tiles of its own
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (s.tile_start[mid] <= t) lo = mid; else hi = mid - 1;
    }
    GTile r;
    r.g = lo;
    r.l = 0;
    const int local = t - s.tile_start[lo];
    const int m_blocks = (s.rows[lo] + kBM - 1) / kBM;
    r.mb = local % m_blocks;
    r.nb = local / m_blocks;
    return r;
  }
  __device__ GroupView view(int i) const {
    const int m = s.rows[i];
    return GroupView{&p.tmap_a, &p.tmap_b[i], s.row0[i],
                     p.sfa + (size_t)s.atom0[i] * (p.k / kKStep) * kSfAtom, p.sfb[i],
                     p.c + (size_t)s.row0[i] * p.n, m, p.n, p.k, 1, (m + kBM - 1) / kBM,
                     (p.n + kBN - 1) / kBN, p.lines32};
  }
};

template <int kBN, int kStages, int kEpiWarps, int kAccBufs, class P>
__global__ void __launch_bounds__(GroupedCfg<kBN, kStages, kEpiWarps, kAccBufs>::kThreads, 1)
grouped_gemm_kernel(const __grid_constant__ P p) {
  using Cfg = GroupedCfg<kBN, kStages, kEpiWarps, kAccBufs>;
  using Sched = Schedule<P, kBN>;
  __shared__ typename Sched::Storage s_sched;
  extern __shared__ uint8_t smem_raw[];
  __shared__ uint64_t bar_full[kStages], bar_empty[kStages];
  __shared__ uint64_t bar_sf_landed[kStages];
  __shared__ uint64_t bar_acc_full[kAccBufs], bar_acc_empty[kAccBufs];
  __shared__ uint64_t bar_drain;
  __shared__ uint32_t s_tmem_base;
  __shared__ volatile int s_abort;

  const uint32_t smem_base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5;
  const uint32_t lane = lane_id();
  constexpr int kProd = kEpiWarps, kMma = kEpiWarps + 1;

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
    s_abort = 0;
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == kMma) tmem_alloc<Cfg::kTmemCols>(smem_u32(&s_tmem_base));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem_base;
  // the prologue above overlaps the previous kernel; global memory only after
  // it (a chained launch reads nothing the previous one writes; it waits for
  // it before exiting instead)
  if (!p.chained) griddep_wait();
  if (threadIdx.x == 0) griddep_launch_dependents();
  const AbortCtl ctl{&s_abort, p.status, p.wait_limit};
  Sched sched(p, s_sched);
  if constexpr (Sched::needs_fill()) {
    sched.fill();
    __syncthreads();
  }
  const int total_tiles = sched.tiles();

  if (warp == kProd) {
    // ------------------------------------------------------------ TMA producer
    if (elect_one()) {   // one thread; uniform registers for the issue
      const uint64_t pol = policy_evict_normal();
      int stage = 0;
      uint32_t phase = 0;
      uint32_t last_phase[kStages];
      bool issued[kStages];
      for (int s = 0; s < kStages; ++s) issued[s] = false, last_phase[s] = 0;
      bool ok = true;
      int prev_g = -1;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const GTile tc = sched.tile(t);
        const GroupView gi = sched.view(tc.g);
        if (tc.g != prev_g) {
          tma_prefetch_desc(gi.tmap_a);
          tma_prefetch_desc(gi.tmap_b);
          prev_g = tc.g;
        }
        const int k_blocks = gi.k / kBK;
        const int rest_k = gi.k / kKStep;
        const size_t sfa_l = (size_t)gi.m_blocks * rest_k * kSfAtom;
        const int n_atoms = (gi.n + 127) / 128;
        const size_t sfb_l = (size_t)n_atoms * rest_k * kSfAtom;
        const int n0 = tc.nb * kBN;
        const uint8_t* sfa_t = gi.sfa + tc.l * sfa_l + (size_t)tc.mb * rest_k * kSfAtom;
        const uint8_t* sfb_t = gi.sfb + tc.l * sfb_l + (size_t)(n0 / 128) * rest_k * kSfAtom;
        for (int kb = 0; kb < k_blocks; ++kb) {
          if (!ctl.wait(smem_u32(&bar_empty[stage]), phase ^ 1u, kDevTimeoutStageFree)) {
            ok = false;
            break;
          }
          const uint32_t full = smem_u32(&bar_full[stage]);
          const uint32_t landed = smem_u32(&bar_sf_landed[stage]);
          const uint32_t sa = smem_base + stage * Cfg::kStageBytes;
          const uint32_t sb = sa + Cfg::kABytes;
          const uint32_t ssf = sb + Cfg::kBBytes;
          // scales first, on their own barrier (staged while the tiles land)
          mbar_arrive_expect_tx(landed, kSfStageBytes + Cfg::kSfbBytes);
          const size_t sf_off = (size_t)kb * kSfStageBytes;
          bulk_load(ssf, sfa_t + sf_off, kSfStageBytes, landed, pol);
          #pragma unroll
          for (int a = 0; a < Cfg::kSfbAtoms; ++a) {
            // consecutive 128-row atom blocks; a block past N (rows that are
            // never stored) re-reads the last real block instead
            const int blk = min(n0 / 128 + a, n_atoms - 1) - n0 / 128;
            bulk_load(ssf + (1 + a) * kSfStageBytes,
                      sfb_t + blk * (size_t)rest_k * kSfAtom + sf_off, kSfStageBytes, landed, pol);
          }
          mbar_arrive_expect_tx(full, Cfg::kABytes + Cfg::kBBytes);
          tma_load_3d(sa, gi.tmap_a, full, kb * 128, gi.a_row0 + tc.mb * kBM, tc.l, pol);
          tma_load_3d(sb, gi.tmap_b, full, kb * 128, n0, tc.l, pol);
          issued[stage] = true;
          last_phase[stage] = phase;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
      }
      if (!ok) {
        for (int s = 0; s < kStages; ++s)
          if (issued[s]) {
            ctl.drain(smem_u32(&bar_sf_landed[s]), last_phase[s]);
            ctl.drain_copies(smem_u32(&bar_full[s]), last_phase[s]);
          }
      }
    }
  } else if (warp == kMma) {
    // ------------------------------------------------------------ MMA issuer
    if (elect_one()) {   // one thread; uniform registers for the issue
      constexpr uint32_t idesc = idesc_mxf4nvf4<kBM, kBN>();
      const uint64_t a_desc0 = kmajor_sw128_desc(smem_base);   // stage 0's A tile
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true, any = false;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const GTile tc = sched.tile(t);
        const int k_blocks = sched.view(tc.g).k / kBK;
        if (!ctl.wait(smem_u32(&bar_acc_empty[acc]), acc_phase ^ 1u, kDevTimeoutAccFree)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + acc * kBN;
        for (int kb = 0; kb < k_blocks; ++kb) {
          // operand tiles landed and the stage's scales staged into TMEM: one
          // barrier counts both (the TMA bytes and one arrival per staging
          // warp), so this thread checks one barrier per K step (each check
          // costs it ~100 cycles, and its loop sets the pace of small tiles)
          if (!ctl.wait(smem_u32(&bar_full[stage]), phase, kDevTimeoutTmaFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = desc_advance(a_desc0, (uint32_t)stage * Cfg::kStageBytes);
          const uint64_t db = desc_advance(da, Cfg::kABytes);
          // scales of k-step j: SFA in [sf_a+4j, +4), SFB atom a in [sf_b+4(atoms*j+a), +4)
          const uint32_t sf_a = tmem + Cfg::kSfCol + stage * Cfg::kSfBufCols;
          const uint32_t sf_b = sf_a + 16;
          #pragma unroll
          for (int j = 0; j < kBK / kKStep; ++j) {
            tc_mma_nvf4(d, desc_advance(da, 32 * j), desc_advance(db, 32 * j), idesc,
                        sf_a + 4 * j, sf_b + 4 * Cfg::kSfbAtoms * j, (kb | j) != 0);
          }
          tc_commit(smem_u32(&bar_empty[stage]));   // frees the stage and its scale buffer
          any = true;
          if (++stage == kStages) stage = 0, phase ^= 1u;
        }
        if (!ok) break;
        tc_commit(smem_u32(&bar_acc_full[acc]));
        if (++acc == kAccBufs) acc = 0, acc_phase ^= 1u;
      }
      if (!ok && any) {
        tc_commit(smem_u32(&bar_drain));
        ctl.drain(smem_u32(&bar_drain), 0);
      }
    }
  } else if (warp >= kEpiWarps + 2) {
    // ------------------------------------------------------------ scale staging
    // Warp w writes TMEM lanes [32*(w%4), +32); lane i of every quadrant gets
    // row i of each 512-byte atom (the broadcast image the MMA reads: tile row
    // r's scales at lane r, column base + r/32).
    const uint32_t t_quad = ((uint32_t)(warp & 3) * 32u) << 16;
    constexpr int kSfbRegs = 16 * Cfg::kSfbAtoms;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
      const GTile tc = sched.tile(t);
      const int k_blocks = sched.view(tc.g).k / kBK;
      for (int kb = 0; kb < k_blocks; ++kb) {
        bool got = true;
        if (lane == 0) got = ctl.wait(smem_u32(&bar_sf_landed[stage]), phase, kDevTimeoutTmaFull);
        if (!__shfl_sync(0xffffffffu, got ? 1 : 0, 0)) {
          ok = false;
          break;
        }
        mbar_try_wait(smem_u32(&bar_sf_landed[stage]), phase);   // every lane observes the phase
        const uint32_t ssf = smem_base + stage * Cfg::kStageBytes + Cfg::kABytes + Cfg::kBBytes +
                             lane * 16u;
        uint32_t ra[16], rb[kSfbRegs];
        #pragma unroll
        for (int j = 0; j < kBK / kKStep; ++j) {
          const uint4 v = lds_v4(ssf + j * kSfAtom);
          ra[4 * j + 0] = v.x, ra[4 * j + 1] = v.y, ra[4 * j + 2] = v.z, ra[4 * j + 3] = v.w;
          #pragma unroll
          for (int a = 0; a < Cfg::kSfbAtoms; ++a) {
            const uint4 b = lds_v4(ssf + (1 + a) * kSfStageBytes + j * kSfAtom);
            const int o = 4 * (Cfg::kSfbAtoms * j + a);
            rb[o + 0] = b.x, rb[o + 1] = b.y, rb[o + 2] = b.z, rb[o + 3] = b.w;
          }
        }
        const uint32_t t_buf = tmem + t_quad + Cfg::kSfCol + stage * Cfg::kSfBufCols;
        tmem_st_32x32b_x16(t_buf, ra);
        if constexpr (Cfg::kSfbAtoms == 2) tmem_st_32x32b_x32(t_buf + 16, rb);
        else tmem_st_32x32b_x16(t_buf + 16, rb);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bar_full[stage]));
        if (++stage == kStages) stage = 0, phase ^= 1u;
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quad = warp & 3;        // TMEM lane quadrant this warp may access
    const int part = warp >> 2;       // which column slice of the tile
    constexpr int kCW = Cfg::kColsPerWarp;
    constexpr int kChunks = kCW / 32;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      const GTile tc = sched.tile(t);
      const GroupView gi = sched.view(tc.g);
      if (!ctl.wait(smem_u32(&bar_acc_full[acc]), acc_phase, kDevTimeoutAccFull)) break;
      tc_fence_after();
      const uint32_t t_acc = tmem + ((uint32_t)(quad * 32) << 16) + acc * kBN + part * kCW;
      const int row0 = tc.mb * kBM + quad * 32;
      const int col0 = tc.nb * kBN + part * kCW;
      __half* cl0 = gi.c + ((size_t)tc.l * gi.m + row0) * (size_t)gi.n + col0;
      // fp16 words of one 64-column (128-byte) line per lane -> whole-line stores
      auto pack_line = [&](uint32_t (&w)[32], const uint32_t (&lo)[32], const uint32_t (&hi)[32]) {
        #pragma unroll
        for (int e = 0; e < 16; ++e) {
          w[e] = pack_half2(__uint_as_float(lo[2 * e]), __uint_as_float(lo[2 * e + 1]));
          w[16 + e] = pack_half2(__uint_as_float(hi[2 * e]), __uint_as_float(hi[2 * e + 1]));
        }
      };
      auto store_line = [&](uint32_t (&w)[32], int line) {
        if (gi.lines32)
          store_lines_coalesced_v8(w, cl0 + 64 * line, gi.n, gi.m - row0, gi.n - col0 - 64 * line);
        else
          store_lines_coalesced(w, cl0 + 64 * line, gi.n, gi.m - row0, gi.n - col0 - 64 * line);
      };
      if constexpr (kAccBufs == 1) {
        // pull the whole slice into registers, hand TMEM back, pack to fp16
        // (halving the live registers), then store
        uint32_t w[kChunks / 2][32];
        {
          uint32_t v[kChunks][32];
          #pragma unroll
          for (int c = 0; c < kChunks; ++c) tmem_ld_32x32b_x32(t_acc + 32 * c, v[c]);
          tmem_ld_wait();
          #pragma unroll
          for (int c = 0; c < kChunks; ++c) tmem_regs_ready(v[c]);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[acc]));
          #pragma unroll
          for (int c = 0; c < kChunks; c += 2) pack_line(w[c / 2], v[c], v[c + 1]);
        }
        #pragma unroll
        for (int ln = 0; ln < kChunks / 2; ++ln) store_line(w[ln], ln);
      } else {
        #pragma unroll 1
        for (int c = 0; c < kChunks; c += 2) {
          uint32_t lo[32], hi[32], w[32];
          tmem_ld_32x32b_x32(t_acc + 32 * c, lo);
          tmem_ld_32x32b_x32(t_acc + 32 * c + 32, hi);
          tmem_ld_wait();
          tmem_regs_ready(lo);
          tmem_regs_ready(hi);
          pack_line(w, lo, hi);
          store_line(w, c / 2);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&bar_acc_empty[acc]));
      }
      if (++acc == kAccBufs) acc = 0, acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == kMma) {
    tc_fence_after();
    tmem_dealloc<Cfg::kTmemCols>(tmem);
  }
  if (p.chained && threadIdx.x == 0) griddep_wait();
}

}  // namespace nvfp4
