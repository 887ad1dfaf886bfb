// NVFP4 quantise + scale swizzle on the device, sm_100a.
//
//   x fp32 [L][rows][K]  ->  packed e2m1 [L][rows][K/2]   (element 2i in the low nibble)
//                           scales as permuted 512-byte atoms [L][ceil(rows/128)][K/64][32][4][4]
//                           (optionally also the plain [L][rows][K/16] scale bytes)
//
// This is the producer step in front of both GEMMs: the reference builds its
// inputs on the host from raw bit patterns (nvfp4_dual_gemm/reference.py:113-187)
// and has no quantiser; the quantisation is the one the benchmark
// configurations define, the same as nvfp4_b200.formats.quantize_nvfp4:
//   scale = e4m3_rne(amax / 6)   (saturating at 448; CUDA's RNE fp8 conversion)
//   value = e2m1_rne(x / scale)  (the IEEE fp32 quotient; ties to the even code; saturating
//                                 at 6; a value rounding to zero keeps its sign)
//
// The quotient is formed without a division, by Markstein's method (P.
// Markstein, IBM J. Res. Dev. 34(1), 1990; "IA-64 and Elementary Functions",
// 2000): a quotient estimate from a correctly rounded reciprocal, refined by
// one fused multiply-add correction step.  With r = RN(1/s),
//   q0 = RN(x * r),  q1 = RN(q0 + RN(x - q0 * s) * r)   (two FMAs)
// Markstein's theorem gives RN(x / s) under conditions on the operands; here
// the equality is proven by exhaustion instead: q1 equals RN(x / s) for every
// fp32 x and every e4m3 scale s (s has one of 8
// mantissas; scaling x or s by a power of two scales every step exactly, so
// the exhaustive check over all 2^23 mantissas of x times the 8 mantissas of
// s covers all normal operands; tests/test_formats.py repeats it).  The
// residual is exact whenever it is nonzero, so it is computed rounding down:
// an exact zero then comes out as -0, which leaves q0 unchanged and gives
// x = +-0 the quotient +-0 that IEEE division gives.  x = +-inf makes the
// residual NaN: a block whose amax is infinite uses IEEE division.  The
// same two FMAs divide amax by 6 (mantissa 1.5, one of the 8 checked).
//   scale == 0 -> all values 0.
//
// HBM-bound: 4 bytes read and 0.5625 (+0.0625 plain scales) written per element.
#pragma once
#include <cuda_fp8.h>
#include <cstdint>

namespace nvfp4 {

struct QuantParams {
  const float* x;        // [L][rows][K]
  uint8_t* packed;       // [L][rows][K/2]
  uint8_t* sf_perm;      // [L][ceil(rows/128)][K/64][512]
  uint8_t* sf_plain;     // [L][rows][K/16] or null
  int rows, k, l;
  int row_blocks, k_atoms;
};

// Two fp32 values -> one byte of e2m1 codes (lo in the low nibble), rounded
// to nearest even and saturated to +-6 by the sm_100 conversion instruction
// (a value rounding to zero keeps its sign).
__device__ __forceinline__ uint32_t e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t, %1, %2;\n\t"
      "cvt.u32.u8 %0, t;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}

// One CTA of 256 threads per (128-row block, 64-deep K atom).  Lane j of a
// warp handles 8 consecutive values of row (4*step + j/8): a warp reads four
// whole 256-byte row segments per step (coalesced), the two lanes of a
// 16-element block combine their amax with one shuffle, each lane writes its
// 4 packed bytes, and the row's four scale bytes are gathered into one
// 4-byte word of the scale atom (byte (r%32)*16 + ((r/32)%4)*4 + block).
constexpr int kQuantThreads = 256;
// Resident CTAs per SM the quantise kernels are compiled for (a 64-register
// cap): the kernels are latency-bound on their loads, and four CTAs per SM
// measured best (three: 6% slower; five or six: spills, slower).
constexpr int kQuantCtasPerSm = 4;

// RN(x / s) for s one of the e4m3 values (or 6) and r = RN(1/s).
__device__ __forceinline__ float div_by_scale(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  return __fmaf_rn(__fmaf_rd(-q0, s, x), r, q0);
}

// Per-CTA tables over the 128 non-negative e4m3 codes: the scale's value and
// RN(1/value) (0 for code 0), one shared-memory load each instead of two
// conversions and an IEEE reciprocal per 8 values.
struct ScaleTables {
  float val[128];
  float rcp[128];
};

// Every thread of the CTA must call this, then __syncthreads() before use.
__device__ __forceinline__ void fill_scale_tables(ScaleTables& t) {
  for (int c = threadIdx.x; c < 128; c += blockDim.x) {
    const float v = __half2float(__half(__nv_cvt_fp8_to_halfraw((__nv_fp8_storage_t)c, __NV_E4M3)));
    t.val[c] = v;
    t.rcp[c] = v == 0.f ? 0.f : __frcp_rn(v);
  }
}

// The body shared by the plain quantiser and the MoE gather-quantiser: rows
// r = 0..127 of one 128-row block, one 64-deep K atom.  src(r) -> the fp32
// row (nullptr past the block's valid rows), packed(r) -> the packed row,
// plain(r) -> the plain-scale row or nullptr; atom_base -> the block's
// 512-byte scale atom for this K atom (padding rows get zero scales).
template <class Src, class Packed, class Plain>
__device__ __forceinline__ void quantize_atom_block(const ScaleTables& tab, int atom,
                                                    uint8_t* atom_base, Src src, Packed packed,
                                                    Plain plain) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int sub = lane & 7;                    // which 8 values of the 64-value row segment
  constexpr int kSteps = 128 / (4 * (kQuantThreads / 32));
  // all of this thread's loads first (4 x 32 bytes in flight per lane)
  float v[kSteps][8];
  const float* row_src[kSteps];
  #pragma unroll
  for (int step = 0; step < kSteps; ++step) {
    const int r = (step * (kQuantThreads / 32) + warp) * 4 + (lane >> 3);
    row_src[step] = src(r);
    if (row_src[step] != nullptr) {
      const float4* q = reinterpret_cast<const float4*>(row_src[step] + (size_t)atom * 64 + 8 * sub);
      const float4 f0 = __ldcs(q), f1 = __ldcs(q + 1);
      v[step][0] = f0.x, v[step][1] = f0.y, v[step][2] = f0.z, v[step][3] = f0.w;
      v[step][4] = f1.x, v[step][5] = f1.y, v[step][6] = f1.z, v[step][7] = f1.w;
    } else {
      #pragma unroll
      for (int e = 0; e < 8; ++e) v[step][e] = 0.f;
    }
  }
  #pragma unroll
  for (int step = 0; step < kSteps; ++step) {
    const int r = (step * (kQuantThreads / 32) + warp) * 4 + (lane >> 3);   // row in the block
    const bool valid = row_src[step] != nullptr;
    float amax = 0.f;
    #pragma unroll
    for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(v[step][e]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));   // the block's other half
    const bool finite = amax <= 3.402823466e38f;
    const float a6 = finite ? div_by_scale(amax, 6.0f, 1.0f / 6.0f) : amax;
    const __nv_fp8_storage_t s8 = __nv_cvt_float_to_fp8(a6, __NV_SATFINITE, __NV_E4M3);
    const float s = tab.val[s8];
    float q[8];
    if (s == 0.f) {
      #pragma unroll
      for (int e = 0; e < 8; ++e) q[e] = 0.f;
    } else if (finite) {
      const float rs = tab.rcp[s8];
      #pragma unroll
      for (int e = 0; e < 8; ++e) q[e] = div_by_scale(v[step][e], s, rs);
    } else {                                   // an infinite value in the block
      #pragma unroll
      for (int e = 0; e < 8; ++e) q[e] = __fdiv_rn(v[step][e], s);
    }
    uint32_t word = 0;
    #pragma unroll
    for (int e = 0; e < 4; ++e) word |= e2m1x2(q[2 * e], q[2 * e + 1]) << (8 * e);
    // scale bytes of blocks 0..3 of this row sit in lanes sub = 0, 2, 4, 6:
    // pairs first (sub 0: blocks 0,1; sub 4: blocks 2,3), then the halves
    const uint32_t pair = (uint32_t)s8 | (__shfl_down_sync(0xffffffffu, (uint32_t)s8, 2) << 8);
    const uint32_t sf_word = pair | (__shfl_down_sync(0xffffffffu, pair, 4) << 16);   // sub 0
    if (valid) {
      *reinterpret_cast<uint32_t*>(packed(r) + (size_t)atom * 32 + 4 * sub) = word;
      uint8_t* pl = plain(r);
      if (sub == 0 && pl != nullptr) *reinterpret_cast<uint32_t*>(pl + (size_t)atom * 4) = sf_word;
    }
    // rows past the valid ones leave zero scales in the atom's padding
    if (sub == 0)
      *reinterpret_cast<uint32_t*>(atom_base + (r % 32) * 16 + (r / 32) * 4) = valid ? sf_word : 0u;
  }
}

// One K atom per CTA (measured: several atoms per CTA, as the MoE quantiser
// uses, leave too few CTAs for the last wave on operand-sized inputs).
__global__ void __launch_bounds__(kQuantThreads, kQuantCtasPerSm) quantize_nvfp4_kernel(const QuantParams p) {
  __shared__ ScaleTables tab;
  fill_scale_tables(tab);
  __syncthreads();
  const int atom = blockIdx.x;                 // k-atom index (64 K per atom)
  const int rb = blockIdx.y;                   // 128-row block
  const int l = blockIdx.z;
  uint8_t* atom_base = p.sf_perm + (((size_t)l * p.row_blocks + rb) * p.k_atoms + atom) * 512;
  const size_t row0 = (size_t)l * p.rows + (size_t)rb * 128;
  const int valid_rows = min(128, p.rows - rb * 128);
  quantize_atom_block(
      tab, atom, atom_base,
      [&](int r) -> const float* { return r < valid_rows ? p.x + (row0 + r) * (size_t)p.k : nullptr; },
      [&](int r) -> uint8_t* { return p.packed + (row0 + r) * (size_t)(p.k / 2); },
      [&](int r) -> uint8_t* { return p.sf_plain ? p.sf_plain + (row0 + r) * (size_t)(p.k / 16) : nullptr; });
}

}  // namespace nvfp4
