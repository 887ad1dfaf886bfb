// Pieces shared by the dual and grouped NVFP4 GEMM kernels: the CTA-wide
// abort protocol for bounded waits, the fused SiLU-gate math and fp16 packing.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>
#include "ptx.cuh"

namespace nvfp4 {

constexpr int kBM = 128;        // UMMA M (cta_group::1)
constexpr int kBK = 256;        // K per pipeline stage: one 128-byte swizzled line per row
constexpr int kKStep = 64;      // K per tcgen05.mma kind::mxf4nvf4
constexpr int kSfAtom = 512;    // bytes of one scale atom: 128 rows x 4 scales (64 K)
constexpr int kSfStageBytes = kSfAtom * (kBK / kKStep);  // 2048: 4 atoms per stage

// Shared abort flag + global status word.  A role whose bounded wait runs out
// records why, raises the flag, and every other role's waits return early.
struct AbortCtl {
  volatile int* flag;       // shared memory
  unsigned* status;         // global memory (per-device status word)
  long long limit;          // clock64 cycles per wait

  __device__ __forceinline__ bool aborted() const { return *flag != 0; }
  __device__ __forceinline__ void raise(unsigned bit) const {
    atomicOr(status, bit);
    *flag = 1;
    __threadfence_block();
  }
  // Bounded wait that also gives up as soon as another role has aborted.
  __device__ __forceinline__ bool wait(uint32_t bar, uint32_t parity, unsigned bit) const {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
      #pragma unroll 1
      for (int i = 0; i < 32; ++i)
        if (mbar_try_wait(bar, parity)) return true;
      if (aborted()) return false;
      if (clock64() - t0 > limit) {
        raise(bit);
        return false;
      }
    }
  }
  // Same with cluster-scope acquire (for barriers other CTAs arrive on
  // after writing into this CTA's shared memory).
  __device__ __forceinline__ bool wait_cluster(uint32_t bar, uint32_t parity, unsigned bit) const {
    if (mbar_try_wait_cluster(bar, parity)) return true;
    const long long t0 = clock64();
    while (true) {
      #pragma unroll 1
      for (int i = 0; i < 32; ++i)
        if (mbar_try_wait_cluster(bar, parity)) return true;
      if (aborted()) return false;
      if (clock64() - t0 > limit) {
        raise(bit);
        return false;
      }
    }
  }
  // Used on the way out after an abort: wait for async work this thread
  // issued (bounded, no new status bits).
  __device__ __forceinline__ void drain(uint32_t bar, uint32_t parity) const {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
      if (clock64() - t0 > limit) return;
  }
  // The same for a stage barrier that also counts other warps' arrivals:
  // after an abort those may never come, so the phase may never complete;
  // the copies themselves land within microseconds, so give them ~30 us.
  __device__ __forceinline__ void drain_copies(uint32_t bar, uint32_t parity) const {
    const long long t0 = clock64();
    const long long cap = limit < (1LL << 16) ? limit : (1LL << 16);
    while (!mbar_try_wait(bar, parity))
      if (clock64() - t0 > cap) return;
  }
};

// silu(g) * u in fp32: g / (1 + e^-g) * u, using the fast exp and divide
// intrinsics (|rel err| ~1e-6, far inside the 1e-2 fp16 tolerance).
__device__ __forceinline__ float silu_gate(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void st_global_v4(void* p, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.global.v4.b32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

// Coalesced store of one 128-byte line per lane.
//
// On entry lane L holds, in w[0..31], the fp16 line of its own output row
// (row lane0_row + L, columns [col0, col0 + 64)), as sixteen-byte chunks
// w[4c..4c+3], c = 0..7.  Each group of 8 lanes transposes its 8x8 matrix
// of chunks with three xor-butterfly exchanges, after which chunk c of lane
// i holds chunk i of row 8*group + c; store c then writes four complete
// lines per warp instead of 32 sixteen-byte pieces of 32 different lines.
// `c_line0` points at (lane 0's row, col0); rows_left / cols_left bound the
// valid rows after lane 0's row and the valid columns after col0.
__device__ __forceinline__ void store_lines_coalesced(uint32_t (&w)[32], __half* c_line0,
                                                      size_t ld, int rows_left, int cols_left) {
  const int lane = (int)(threadIdx.x & 31u);
  const int i = lane & 7, grp = lane >> 3;
  #pragma unroll
  for (int s = 1; s < 8; s <<= 1) {
    const bool hi = (i & s) != 0;
    #pragma unroll
    for (int c = 0; c < 8; ++c) {
      if (c & s) continue;           // pair (c, c | s)
      #pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t send = hi ? w[4 * c + e] : w[4 * (c | s) + e];
        const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, s);
        if (hi) w[4 * c + e] = recv; else w[4 * (c | s) + e] = recv;
      }
    }
  }
  #pragma unroll
  for (int c = 0; c < 8; ++c) {
    const int r = 8 * grp + c;
    if (r < rows_left && 8 * i < cols_left)
      st_global_v4(c_line0 + (size_t)r * ld + 8 * i, w[4 * c], w[4 * c + 1], w[4 * c + 2],
                   w[4 * c + 3]);
  }
}

__device__ __forceinline__ void st_global_v8(void* p, const uint32_t* w) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]),
               "r"(w[1]), "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

// Same contract as store_lines_coalesced with 32-byte stores: a 4 x 4
// transpose of 32-byte chunks inside each group of four lanes, then each of
// four st.global.v8 writes eight whole 128-byte lines per warp.  Every row
// start must be 32-byte aligned (ld % 16 == 0 and c_line0 32-byte aligned)
// and cols_left a multiple of 16 when it is below 64.
__device__ __forceinline__ void store_lines_coalesced_v8(uint32_t (&w)[32], __half* c_line0,
                                                         size_t ld, int rows_left, int cols_left) {
  const int lane = (int)(threadIdx.x & 31u);
  const int i = lane & 3, grp = lane >> 2;
  #pragma unroll
  for (int s = 1; s < 4; s <<= 1) {
    const bool hi = (i & s) != 0;
    #pragma unroll
    for (int c = 0; c < 4; ++c) {
      if (c & s) continue;           // pair (c, c | s)
      #pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint32_t send = hi ? w[8 * c + e] : w[8 * (c | s) + e];
        const uint32_t recv = __shfl_xor_sync(0xffffffffu, send, s);
        if (hi) w[8 * c + e] = recv; else w[8 * (c | s) + e] = recv;
      }
    }
  }
  #pragma unroll
  for (int c = 0; c < 4; ++c) {
    const int r = 4 * grp + c;
    if (r < rows_left && 16 * i < cols_left) st_global_v8(c_line0 + (size_t)r * ld + 16 * i, &w[8 * c]);
  }
}

}  // namespace nvfp4
