// MoE dispatch and combine around the grouped GEMM, sm_100a.
//
// Dispatch: T tokens, each with `topk` expert choices ids[t*topk + j] (pair
// index p = t*topk + j; choices outside [0, E) are dropped), become the
// grouped GEMM's per-expert A operands:
//
//   counts[e]        pairs routed to expert e
//   row_offsets[e]   exclusive prefix of counts (row of A_all where expert e starts)
//   atom_offsets[e]  exclusive prefix of ceil(counts/128) (128-row scale blocks)
//   src[row]         the pair that permuted row `row` holds; within an expert
//                    rows follow ascending pair index (a stable sort by expert)
//   dst[p]           the permuted row of pair p, -1 if dropped
//   packed           A_all [R][K/2] e2m1: row r = quantised x[src[r] / topk]
//   sf_perm          expert e's scale atoms [ceil(counts/128)][K/64][512]
//                    from byte atom_offsets[e] * (K/64) * 512 on (padding
//                    rows zero), the layout the GEMMs read
//
// The reference stops at the grouped GEMM (nvfp4_group_gemm/reference.py:
// 39-74 takes per-group A_g as given); producing A_g from routed tokens is
// the caller side of its grouped benchmark.  The quantisation is the same
// device code as nvfp4_quantize.
//
// Kernels (all integer / byte work except the quantiser's arithmetic):
//   1. count:   one warp per chunk of kMoeChunk pairs, a shared-memory
//               histogram per warp -> chunk_counts[chunk][E]
//   2. scan:    one CTA; per expert an exclusive scan over chunks (in place),
//               then exclusive scans over experts -> offsets
//   3. scatter: one warp per chunk walks its pairs in order, 32 at a time;
//               lanes with the same expert find each other with match.any,
//               take consecutive rows after the expert's running count
//               (stable: lower lanes and earlier steps first)
//   4. quantise: one CTA per (128-row block of an expert, up to 4 64-deep K atoms),
//               gathering its rows' tokens; grid sized by the upper bound
//               ceil(pairs/128) + min(E, pairs) blocks, the excess exits
//
// Combine: out[t][n] = sum_j w[t*topk + j] * C_all[dst[t*topk + j]][n]
// (fp32, j ascending, each product and sum rounded separately (no FMA) so
// the result is exactly reproducible on the host; dropped pairs skipped;
// w == nullptr means 1).
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "quantize.cuh"

namespace nvfp4 {

constexpr int kMoeChunk = 1024;          // pairs per warp chunk (32 steps of 32)
constexpr int kMoeMaxExperts = 1024;     // shared-memory histogram / scan bound
constexpr int kMoeWarps = 4;             // chunks per CTA in count / scatter
// K atoms per quantise CTA: the expert lookup, scale tables and row indices
// of a CTA are shared by four atoms, and each row's 128-byte packed line is
// written by one CTA back to back (measured 290 -> 250 us on 32768 x 7168).
constexpr int kMoeAtomsPerCta = 4;

struct MoeParams {
  const float* x;        // [T][K]
  const int* ids;        // [T * topk]
  int pairs, topk, k, experts, chunks, k_atoms;
  int* chunk_counts;     // workspace [chunks][experts]
  int* counts;           // [experts]
  int* row_offsets;      // [experts + 1]
  int* atom_offsets;     // [experts + 1]
  int* src;              // [pairs]
  int* dst;              // [pairs]
  uint8_t* packed;       // [pairs][K/2] (rows >= row_offsets[E] untouched)
  uint8_t* sf_perm;      // [ceil(pairs/128) + min(E, pairs)][K/64][512] (bound)
};

__global__ void __launch_bounds__(32 * kMoeWarps) moe_count_kernel(const MoeParams p) {
  extern __shared__ int hist[];                       // [kMoeWarps][experts]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int* h = hist + warp * p.experts;
  for (int e = lane; e < p.experts; e += 32) h[e] = 0;
  __syncwarp();
  const int chunk = blockIdx.x * kMoeWarps + warp;
  if (chunk >= p.chunks) return;
  const int p0 = chunk * kMoeChunk, p1 = min(p0 + kMoeChunk, p.pairs);
  int ids[kMoeChunk / 32];                            // every load in flight before the first use
  #pragma unroll
  for (int s = 0; s < kMoeChunk / 32; ++s) {
    const int i = p0 + 32 * s + lane;
    ids[s] = i < p1 ? __ldg(p.ids + i) : -1;
  }
  #pragma unroll
  for (int s = 0; s < kMoeChunk / 32; ++s)
    if (ids[s] >= 0 && ids[s] < p.experts) atomicAdd(h + ids[s], 1);
  __syncwarp();
  int* out = p.chunk_counts + (size_t)chunk * p.experts;
  for (int e = lane; e < p.experts; e += 32) out[e] = h[e];
}

// Exclusive scan of v over the CTA's threads (blockDim.x <= 1024), via
// warp shuffles and one shared array of warp totals.
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = (blockDim.x + 31) >> 5;
  int x = v;
  #pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? warp_sums[lane] : 0;
    #pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;                              // inclusive warp prefix
  }
  __syncthreads();
  total = warp_sums[nwarps - 1];
  const int before = warp == 0 ? 0 : warp_sums[warp - 1];
  __syncthreads();                                    // warp_sums reusable after return
  return before + x - v;
}

__global__ void __launch_bounds__(kMoeMaxExperts) moe_scan_kernel(const MoeParams p) {
  __shared__ int warp_sums[32];
  const int e = threadIdx.x;
  int running = 0;
  if (e < p.experts) {
    // per expert: chunk_counts[c][e] <- pairs of expert e in chunks before c
    int c = 0;
    for (; c + 8 <= p.chunks; c += 8) {
      int v[8];
      #pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = p.chunk_counts[(size_t)(c + i) * p.experts + e];
      #pragma unroll
      for (int i = 0; i < 8; ++i) {
        p.chunk_counts[(size_t)(c + i) * p.experts + e] = running;
        running += v[i];
      }
    }
    for (; c < p.chunks; ++c) {
      const int v = p.chunk_counts[(size_t)c * p.experts + e];
      p.chunk_counts[(size_t)c * p.experts + e] = running;
      running += v;
    }
    p.counts[e] = running;
  }
  int rows_total, blocks_total;
  const int row_off = block_exclusive_scan(running, warp_sums, rows_total);
  const int atom_off = block_exclusive_scan((running + 127) / 128, warp_sums, blocks_total);
  if (e < p.experts) {
    p.row_offsets[e] = row_off;
    p.atom_offsets[e] = atom_off;
  }
  if (e == 0) {
    p.row_offsets[p.experts] = rows_total;
    p.atom_offsets[p.experts] = blocks_total;
  }
}

__global__ void __launch_bounds__(32 * kMoeWarps) moe_scatter_kernel(const MoeParams p) {
  extern __shared__ int next_row[];                   // [kMoeWarps][experts]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunk = blockIdx.x * kMoeWarps + warp;
  if (chunk >= p.chunks) return;                      // whole warps only: no block barrier below
  const int p0 = chunk * kMoeChunk, p1 = min(p0 + kMoeChunk, p.pairs);
  const uint32_t lt = (1u << lane) - 1u;
  int ids[kMoeChunk / 32];                            // every load in flight before the walk
  #pragma unroll
  for (int s = 0; s < kMoeChunk / 32; ++s) {
    const int i = p0 + 32 * s + lane;
    ids[s] = i < p1 ? __ldg(p.ids + i) : -1;
  }
  int* nr = next_row + warp * p.experts;
  const int* base = p.chunk_counts + (size_t)chunk * p.experts;
  for (int e = lane; e < p.experts; e += 32) nr[e] = p.row_offsets[e] + base[e];
  __syncwarp();
  #pragma unroll
  for (int s = 0; s < kMoeChunk / 32; ++s) {
    const int i = p0 + 32 * s + lane;
    const int e = ids[s];
    const bool valid = e >= 0 && e < p.experts;
    const int key = valid ? e : -1;
    const uint32_t same = __match_any_sync(0xffffffffu, key);
    int row = -1;
    if (valid) row = nr[e] + __popc(same & lt);
    __syncwarp();
    if (valid && (same & lt) == 0) nr[e] += __popc(same);   // the group's lowest lane advances it
    __syncwarp();
    if (i < p1) {
      p.dst[i] = row;
      if (valid) p.src[row] = i;
    }
  }
}

__global__ void __launch_bounds__(kQuantThreads, kQuantCtasPerSm) moe_quantize_kernel(const MoeParams p) {
  const int gb = blockIdx.y;                          // 128-row block over all experts
  // the expert owning block gb (atom_offsets[e] <= gb < atom_offsets[e + 1]):
  // every thread tests a few experts, one dependent load instead of a search
  __shared__ int s_expert;
  __shared__ ScaleTables tab;
  fill_scale_tables(tab);
  if (threadIdx.x == 0) s_expert = -1;
  __syncthreads();
  for (int i = threadIdx.x; i < p.experts; i += blockDim.x)
    if (__ldg(p.atom_offsets + i) <= gb && gb < __ldg(p.atom_offsets + i + 1)) s_expert = i;
  __syncthreads();
  const int e = s_expert;
  if (e < 0) return;                                  // past the last block: whole CTA exits
  const int local_block = gb - p.atom_offsets[e];
  const int row0 = p.row_offsets[e] + local_block * 128;
  const int valid_rows = min(128, p.row_offsets[e + 1] - row0);
  const int topk = p.topk;
  const int a1 = min(p.k_atoms, (int)(blockIdx.x + 1) * kMoeAtomsPerCta);
  #pragma unroll 1
  for (int atom = blockIdx.x * kMoeAtomsPerCta; atom < a1; ++atom) {   // not unrolled: measured faster
    uint8_t* atom_base = p.sf_perm + ((size_t)gb * p.k_atoms + atom) * 512;
    quantize_atom_block(
        tab, atom, atom_base,
        [&](int r) -> const float* {
          return r < valid_rows ? p.x + (size_t)(__ldg(p.src + row0 + r) / topk) * p.k : nullptr;
        },
        [&](int r) -> uint8_t* { return p.packed + (size_t)(row0 + r) * (p.k / 2); },
        [&](int) -> uint8_t* { return nullptr; });
  }
}

struct MoeCombineParams {
  const __half* c;       // [R][N]
  const int* dst;        // [T * topk]
  const float* w;        // [T * topk] or nullptr
  float* out;            // [T][N]
  int tokens, topk, n;
  int c_rows;            // rows of c: larger dst entries are treated as dropped
};

constexpr int kCombineThreads = 256;

// One CTA per (token, 2048-column span); each thread sums 8 consecutive
// columns over the token's choices.  kVec (N % 8 == 0, 16-byte aligned
// bases): 16-byte loads of C and 32-byte stores of out; else scalar.
template <bool kVec>
__global__ void __launch_bounds__(kCombineThreads) moe_combine_kernel(const MoeCombineParams p) {
  const int t = blockIdx.y;
  const int col = (blockIdx.x * kCombineThreads + threadIdx.x) * 8;
  if (col >= p.n) return;
  const int cols = min(8, p.n - col);
  float acc[8];
  #pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  for (int j = 0; j < p.topk; ++j) {
    const int row = __ldg(p.dst + (size_t)t * p.topk + j);
    if (row < 0 || row >= p.c_rows) continue;
    const float w = p.w ? __ldg(p.w + (size_t)t * p.topk + j) : 1.f;
    const __half* src = p.c + (size_t)row * p.n + col;
    if constexpr (kVec) {
      const uint4 raw = __ldcs(reinterpret_cast<const uint4*>(src));
      const __half2* h = reinterpret_cast<const __half2*>(&raw);
      #pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(h[i]);
        acc[2 * i] = __fadd_rn(acc[2 * i], __fmul_rn(w, f.x));
        acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], __fmul_rn(w, f.y));
      }
    } else {
      #pragma unroll
      for (int i = 0; i < 8; ++i)
        if (i < cols) acc[i] = __fadd_rn(acc[i], __fmul_rn(w, __half2float(src[i])));
    }
  }
  float* o = p.out + (size_t)t * p.n + col;
  if constexpr (kVec) {
    reinterpret_cast<float4*>(o)[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    reinterpret_cast<float4*>(o)[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  } else {
    #pragma unroll
    for (int i = 0; i < 8; ++i)
      if (i < cols) o[i] = acc[i];
  }
}

}  // namespace nvfp4
