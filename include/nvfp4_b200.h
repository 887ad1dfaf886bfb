/*
 * nvfp4_b200.h - C ABI of libnvfp4_b200.so, the B200 (sm_100a) kernels for the
 * two NVFP4 hot paths of kazim05/Blackwell-nvfp4-kernels.
 *
 * Plain pointers and sizes only (no torch or CUDA types): `stream` is a
 * cudaStream_t passed as void* (NULL = legacy default stream).  Every entry
 * point returns NVFP4_OK (0) or a negative status; no exception crosses the
 * ABI.  Launches are asynchronous on `stream`; device-side wait timeouts are
 * reported through nvfp4_device_status().  The calls work on the calling
 * thread's current device; several host threads may call at once, each on
 * its own stream; every call can be captured into a CUDA graph (the first
 * one on a stream included).
 *
 * Data layouts are those of the reference task (nvfp4_dual_gemm/reference.py,
 * nvfp4_group_gemm/reference.py):
 *   A  [M, K/2, L]  float4_e2m1fn_x2, K-major; batch l starts at l*M*K/2 bytes
 *   B  [N, K/2, L]  same
 *   SF permuted scale tensor [32, 4, ceil(MN/128), 4, K/64, L] float8_e4m3fn,
 *      i.e. contiguous 512-byte atoms [L][ceil(MN/128)][K/64][32][4][4]
 *   C  [M, N, L]    float16, row-major; batch l starts at l*M*N elements
 * Requirements: K % 256 == 0, N % 8 == 0, M >= 1, all pointers 16-byte aligned.
 */
#ifndef NVFP4_B200_H
#define NVFP4_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NVFP4_OK 0
#define NVFP4_ERR_INVALID_ARG (-1)   /* null pointer, negative size, bad count */
#define NVFP4_ERR_SHAPE (-2)         /* K % 256 != 0, N % 8 != 0, too large */
#define NVFP4_ERR_ALIGNMENT (-3)     /* a pointer is not 16-byte aligned */
#define NVFP4_ERR_CUDA (-4)          /* a CUDA runtime / driver call failed */
#define NVFP4_ERR_DEVICE (-5)        /* current device is not sm_100 */
#define NVFP4_ERR_TIMEOUT (-6)       /* a kernel's bounded wait ran out */

/* One problem of a grouped GEMM (one entry of the reference's
 * abc_list / sfasfb_reordered_list / problem_sizes). */
typedef struct nvfp4_group {
  const void* a;        /* [M, K/2, L] e2m1 x2 */
  const void* b;        /* [N, K/2, L] e2m1 x2 */
  const void* sfa_perm; /* permuted scales of A */
  const void* sfb_perm; /* permuted scales of B */
  void* c;              /* [M, N, L] fp16 */
  int32_t m, n, k, l;
} nvfp4_group;

/* C = silu(A . B1ᵀ) * (A . B2ᵀ), fp32 accumulation, fp16 output.
 * Replaces the host launcher torch.ops.<ns>.dual_gemm(A,B1,B2,SFA,SFB1,SFB2,C)
 * (nvfp4_dual_gemm/submission_v1.py:1305-1356) and the compiled CuTe call of
 * nvfp4_dual_gemm/submission_v4.py:1256-1284. */
int nvfp4_dual_gemm(const void* a, const void* b1, const void* b2, const void* sfa_perm,
                    const void* sfb1_perm, const void* sfb2_perm, void* c, int m, int n, int k,
                    int l, void* stream);

/* The dual GEMM above, for callers that may not allocate device memory at
 * call time (servers that hand the whole HBM budget to weights and KV caches
 * up front; hosts whose own memory manager must own every device byte).  It
 * allocates nothing: when the shape is split along K, the partial sums live
 * in a fixed array inside this library (20 MiB of partials + 16 KiB of
 * counters, held by every GPU that loads the library until exit), and shapes
 * whose split needs more are rejected with NVFP4_ERR_SHAPE.  The first call on
 * a device looks up that array's device address (also inside a stream
 * capture).  All calls share the one array: calls that overlap on
 * the GPU (e.g. on two streams at once) race.  No counterpart in the
 * reference. */
int nvfp4_dual_gemm_noalloc(const void* a, const void* b1, const void* b2, const void* sfa_perm,
                            const void* sfb1_perm, const void* sfb2_perm, void* c, int m, int n,
                            int k, int l, void* stream);

/* C_g = A_g . B_gᵀ for g in [0, num_groups) in one persistent launch (the host
 * splits tables larger than one launch's parameter block).  Groups with
 * M == 0 are skipped.  Replaces module.kernel_launch(As,Bs,SFAs,SFBs,Cs,
 * problem_sizes) (nvfp4_group_gemm/submission_v7.py:454-522). */
int nvfp4_grouped_gemm(const nvfp4_group* groups, int num_groups, void* stream);

/* Quantise fp32 x [L][rows][K] (K % 64 == 0) to NVFP4 on the device:
 * packed e2m1 [L][rows][K/2] (element 2i in the low nibble), the permuted
 * scale atoms [L][ceil(rows/128)][K/64][32][4][4] the GEMMs read (padding rows
 * get zero scales) and, if sf_plain is not NULL, the plain scales
 * [L][rows][K/16].  Per 16-element block: scale = e4m3_rne(amax/6), value =
 * e2m1_rne(x/scale) (ties to even, saturating), zero scale -> zero values.
 * No kernel counterpart in the reference: it is the host-side input
 * construction of nvfp4_dual_gemm/reference.py:113-187 moved on-device. */
int nvfp4_quantize(const float* x, int rows, int k, int l, void* packed, void* sf_perm,
                   void* sf_plain, void* stream);

/* MoE dispatch: routes `tokens` fp32 rows x [tokens][K] (K % 64 == 0, 16-byte
 * aligned) with `topk` expert choices each, expert_ids[t*topk + j] (choices
 * outside [0, num_experts) are dropped; num_experts <= 1024), into the
 * per-expert NVFP4 A operands of nvfp4_grouped_gemm, on the device:
 *   counts[e]            pairs routed to expert e
 *   row_offsets[e]       sum of counts[e' < e]; row_offsets[E] = rows used
 *   atom_offsets[e]      sum of ceil(counts[e'] / 128) for e' < e
 *   src[row]             pair index t*topk + j held by permuted row `row`
 *                        (rows of one expert in ascending pair order)
 *   dst[t*topk + j]      permuted row of that pair, -1 if dropped
 *   packed               [tokens*topk][K/2] e2m1 bytes, row r = x[src[r]/topk]
 *                        quantised exactly as nvfp4_quantize does
 *   sf_perm              expert e's permuted scale atoms [ceil(counts[e]/128)]
 *                        [K/64][512] from byte atom_offsets[e]*(K/64)*512
 *                        (padding rows zero); size nvfp4_moe_sf_bytes()
 * so that expert e's grouped-GEMM operand is A = packed + row_offsets[e]*K/2,
 * SFA = sf_perm + atom_offsets[e]*(K/64)*512, M = counts[e].  `workspace`
 * (nvfp4_moe_workspace_bytes(), 4-byte aligned) is scratch owned by the
 * call until it completes on `stream`.  Asynchronous; offsets stay on the
 * device.  No reference counterpart: the reference's grouped GEMM
 * (nvfp4_group_gemm/reference.py:39-74) takes the per-expert A_g as given;
 * this is the routing step that produces them. */
int nvfp4_moe_dispatch(const float* x, const int* expert_ids, int tokens, int topk, int k,
                       int num_experts, void* packed, void* sf_perm, int* counts,
                       int* row_offsets, int* atom_offsets, int* src, int* dst, void* workspace,
                       size_t workspace_bytes, void* stream);
size_t nvfp4_moe_workspace_bytes(int tokens, int topk, int num_experts);
/* Upper bound of the dispatch's scale bytes: (ceil(tokens*topk/128) +
 * min(num_experts, tokens*topk)) * (K/64) * 512. */
size_t nvfp4_moe_sf_bytes(int tokens, int topk, int k, int num_experts);

/* Grouped GEMM over a dispatch without a host round trip: for every expert
 * e < num_experts, C rows [row_offsets[e], +counts[e]) = A rows of the same
 * range . B_eᵀ (fp16 out, fp32 accumulate), with A = a_packed (the
 * dispatch's packed [a_rows][K/2] e2m1 rows), expert e's A scales the 128-row
 * atom blocks of sfa_atoms from block atom_offsets[e], and b[e] / sfb_perm[e]
 * (host arrays of device pointers) expert e's weights [N][K/2] and permuted
 * scales.  counts / row_offsets / atom_offsets are the dispatch's DEVICE
 * arrays: the kernel reads them when it runs, so dispatch, this GEMM and the
 * combine can be enqueued (or captured in a CUDA graph) without reading the
 * routing back.  c: fp16 [a_rows][N].  K % 256 == 0, N % 8 == 0.  Same
 * arithmetic per tile as nvfp4_grouped_gemm.  No reference counterpart: the
 * reference's grouped GEMM (nvfp4_group_gemm/submission_v7.py:454-522) takes
 * host problem sizes. */
int nvfp4_moe_grouped_gemm(const void* a_packed, int a_rows, const void* sfa_atoms,
                           const int* counts, const int* row_offsets, const int* atom_offsets,
                           const void* const* b, const void* const* sfb_perm, int num_experts,
                           int n, int k, void* c, void* stream);

/* MoE combine: out[t][n] = sum over j of weights[t*topk + j] *
 * c[dst[t*topk + j]][n] (fp32, j ascending, products and sums rounded
 * separately; pairs with dst < 0 or dst >= c_rows skipped; weights == NULL
 * means 1), with c the fp16 [c_rows][N] output of the grouped GEMM over the
 * dispatch's permuted rows and dst the dispatch's dst.  No reference
 * counterpart. */
int nvfp4_moe_combine(const void* c, int c_rows, const int* dst, const float* weights, int tokens,
                      int topk, int n, float* out, void* stream);

/* Synchronises `stream`, then reads and clears this device's status word.
 * Returns NVFP4_ERR_TIMEOUT if a kernel gave up on a wait (bits in *bits_out,
 * may be NULL), NVFP4_ERR_CUDA on a CUDA error, else NVFP4_OK.  No reference
 * counterpart: the reference kernels spin forever. */
int nvfp4_device_status(void* stream, unsigned* bits_out);

/* Launches a one-CTA kernel that waits on an mbarrier nothing ever completes,
 * bounded by `limit_cycles`; nvfp4_device_status() must then report
 * NVFP4_ERR_TIMEOUT.  Exercises the bounded-wait path without faulting.
 * No reference counterpart. */
int nvfp4_wait_selftest(long long limit_cycles, void* stream);

/* Status code -> static string.  Detail of the calling thread's last failure. */
const char* nvfp4_status_string(int status);
const char* nvfp4_last_error(void);

/* Library version: major*10000 + minor*100 + patch. */
int nvfp4_version(void);

/* Kernels this library has launched in this process so far (every entry
 * point, all devices).  Callers read it before and after a region to count
 * the region's launches.  No reference counterpart. */
unsigned long long nvfp4_launch_count(void);

#ifdef __cplusplus
}
#endif
#endif /* NVFP4_B200_H */
