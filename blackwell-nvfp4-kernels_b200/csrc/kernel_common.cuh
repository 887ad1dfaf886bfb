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
  // Used on the way out after an abort: wait for async work this thread
  // issued (bounded, no new status bits).
  __device__ __forceinline__ void drain(uint32_t bar, uint32_t parity) const {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity))
      if (clock64() - t0 > limit) return;
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

}  // namespace nvfp4
