// C ABI of libnvfp4_b200.so: argument validation, TMA descriptor encoding,
// tile-configuration choice and kernel launches for the NVFP4 dual and
// grouped GEMMs.  See include/nvfp4_b200.h for the contract.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <unistd.h>
#include <unordered_map>
#include <vector>

#include "../../include/nvfp4_b200.h"
#include "dual_gemm.cuh"
#include "dual_gemm_2sm.cuh"
#include "grouped_gemm.cuh"
#include "grouped_gemm_2sm.cuh"
#include "quantize.cuh"
#include "moe.cuh"

// Fixed split-K scratch of the allocation-free dual GEMM entry point
// (nvfp4_dual_gemm_noalloc): fp32 partial slots followed by one ticket
// counter per tile.  Every GPU that loads the library holds it until exit.
namespace nvfp4 {
constexpr size_t kNoAllocPartialBytes = size_t(20) << 20;   // 20 MiB of fp32 partial slots
constexpr size_t kNoAllocCounterInts = 4096;                // one ticket counter per tile
constexpr size_t kNoAllocScratchBytes = kNoAllocPartialBytes + kNoAllocCounterInts * sizeof(int);
}  // namespace nvfp4

static __device__ __align__(256) unsigned char g_noalloc_scratch[nvfp4::kNoAllocScratchBytes];

namespace nvfp4 {

// Per-device status word written by the kernels' bounded waits.
__device__ unsigned g_status_word;

__global__ void wait_selftest_kernel(unsigned* status, long long limit) {
  __shared__ uint64_t bar;
  __shared__ volatile int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  const AbortCtl ctl{&abort_flag, status, limit};
  if (threadIdx.x == 0) ctl.wait(smem_u32(&bar), 0, kDevTimeoutSelftest);  // nobody arrives
}

namespace {

thread_local char t_last_error[512] = "";

int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(t_last_error, sizeof(t_last_error), fmt, ap);
  va_end(ap);
  return code;
}

constexpr int kMaxDevices = 64;

// Split-K scratch of one stream: fp32 partial slots and per-tile counters.
// Kernels on one stream run in order, so a stream never races with itself;
// different streams get different scratch.
struct Workspace {
  float* partials = nullptr;
  size_t partial_bytes = 0;
  int* counters = nullptr;
  size_t counter_count = 0;
  bool zero_pending = false;   // new counters not yet zeroed by an uncaptured call
};

// One-time setup (context and symbol lookups, kernel attributes, workspace
// allocation) may run while this thread captures a stream into a CUDA graph:
// relaxed capture mode permits those calls for the scope of this guard.
struct RelaxedCapture {
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  RelaxedCapture() { cudaThreadExchangeStreamCaptureMode(&mode); }
  ~RelaxedCapture() { cudaThreadExchangeStreamCaptureMode(&mode); }
};

struct DeviceState {
  bool ready = false;
  int num_sms = 0;
  unsigned* status = nullptr;
  std::atomic<bool> smem_set[32] = {};  // one slot per kernel instantiation (any thread may set it)
  int max_clusters[5] = {};  // co-resident clusters of the cluster split-K kernel, by size
  std::unordered_map<cudaStream_t, Workspace> ws;
  unsigned char* noalloc_scratch = nullptr;   // device address of g_noalloc_scratch
};

std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

long long wait_limit_cycles() {
  static long long v = [] {
    const char* e = getenv("NVFP4_WAIT_LIMIT_CYCLES");
    long long x = e ? atoll(e) : 0;
    return x > 0 ? x : 4000000000LL;  // ~2 s at 2 GHz
  }();
  return v;
}

// Tuning knobs (NVFP4_* environment variables) read in one pass over the
// environment per call: a getenv per knob costs a full scan each, which at
// ~1 us of host time per call matters for microsecond-scale problems.  They
// are re-read on every call so a process can change them between calls.
struct Knobs {
  int dual_group_m = 32;   // NVFP4_DUAL_GROUP_M (measured: 16 -> 32 saves ~1.5% on 8192x14336x4096)
  int dual_splits = 0;     // NVFP4_DUAL_SPLITS (0 = automatic)
  int dual_bn = 0;         // NVFP4_DUAL_BN (64 / 128; 0 = automatic)
  int dual_kernel = 0;     // NVFP4_DUAL_KERNEL: 0 automatic, 1 pair (CTA-pair kernel), 2 single
  int dual_cluster = 0;    // NVFP4_DUAL_CLUSTER: 0 automatic, 1 off, 2 / 4 forced cluster split-K
  int grouped_bn = 0;      // NVFP4_GROUPED_BN (128 / 256; 0 = automatic)
  int grouped_kernel = 0;  // NVFP4_GROUPED_KERNEL: 0 automatic, 1 pair (CTA-pair kernel), 2 single
  bool pdl = true;         // NVFP4_PDL=0: launch the GEMMs without programmatic dependent launch
};

Knobs read_knobs() {
  Knobs k;
  for (char** e = environ; e && *e; ++e) {
    const char* v = *e;
    if (strncmp(v, "NVFP4_", 6) != 0) continue;
    v += 6;
    auto val = [&](const char* name) -> const char* {
      const size_t n = strlen(name);
      return (strncmp(v, name, n) == 0 && v[n] == '=') ? v + n + 1 : nullptr;
    };
    const char* x;
    if ((x = val("DUAL_GROUP_M"))) k.dual_group_m = atoi(x);
    else if ((x = val("DUAL_SPLITS"))) k.dual_splits = atoi(x);
    else if ((x = val("DUAL_BN"))) k.dual_bn = atoi(x);
    else if ((x = val("DUAL_KERNEL")))
      k.dual_kernel = strcmp(x, "pair") == 0 ? 1 : strcmp(x, "single") == 0 ? 2 : 0;
    else if ((x = val("DUAL_CLUSTER"))) k.dual_cluster = atoi(x);
    else if ((x = val("GROUPED_BN"))) k.grouped_bn = atoi(x);
    else if ((x = val("GROUPED_KERNEL")))
      k.grouped_kernel = strcmp(x, "pair") == 0 ? 1 : strcmp(x, "single") == 0 ? 2 : 0;
    else if ((x = val("PDL"))) k.pdl = atoi(x) != 0;
  }
  if (k.dual_group_m < 1) k.dual_group_m = 1;
  return k;
}

// Resolve per-device state (SM count, status-word address) once.
int get_device(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(NVFP4_ERR_DEVICE, "device index %d", dev);
  // A thread that has made no runtime call yet has no current context, and
  // the tensor-map encoder (a driver call) then fails: make the device's
  // primary context current for this thread once.
  thread_local int t_bound_dev = -1;
  if (t_bound_dev != dev) {
    RelaxedCapture relaxed;
    e = cudaSetDevice(dev);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "cudaSetDevice(%d): %s", dev, cudaGetErrorString(e));
    t_bound_dev = dev;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  DeviceState& d = g_dev[dev];
  if (!d.ready) {
    RelaxedCapture relaxed;
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (major != 10 || minor != 0)
      return fail(NVFP4_ERR_DEVICE, "device %d is sm_%d%d; this library is built for sm_100a",
                  dev, major, minor);
    e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "SM count: %s", cudaGetErrorString(e));
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_status_word);
    if (e != cudaSuccess)
      return fail(NVFP4_ERR_CUDA, "status word address: %s", cudaGetErrorString(e));
    d.status = static_cast<unsigned*>(p);
    if (!g_encode) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                           cudaEnableDefault, &q);
      if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !fn)
        return fail(NVFP4_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    d.ready = true;
  }
  *out = &d;
  return NVFP4_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// 3-D byte view [L][rows][K/2] of a packed e2m1 operand, box {128 B, box_rows, 1},
// 128-byte swizzle (the canonical K-major SW128 operand layout of tcgen05.mma).
int encode_operand_uncached(CUtensorMap* map, const void* base, int rows, int k, int l,
                            int box_rows) {
  const cuuint64_t dims[3] = {(cuuint64_t)(k / 2), (cuuint64_t)rows, (cuuint64_t)l};
  const cuuint64_t strides[2] = {(cuuint64_t)(k / 2), (cuuint64_t)rows * (cuuint64_t)(k / 2)};
  const cuuint32_t box[3] = {128u, (cuuint32_t)box_rows, 1u};
  const cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(NVFP4_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%d k=%d l=%d", (int)r,
                rows, k, l);
  return NVFP4_OK;
}

// Encoded descriptors are pure functions of (address, rows, K, L, box rows);
// repeated calls on the same tensors (the common case: weights, persistent
// activation buffers) reuse them instead of re-encoding.
struct MapKey {
  uintptr_t ptr;
  int rows, k, l, box;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && rows == o.rows && k == o.k && l == o.l && box == o.box;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& key) const {
    uint64_t h = key.ptr * 0x9E3779B97F4A7C15ull;
    h ^= ((uint64_t)(uint32_t)key.rows << 32 | (uint32_t)key.k) + 0x632BE59BD9B4E019ull + (h << 6);
    h ^= ((uint64_t)(uint32_t)key.l << 32 | (uint32_t)key.box) + (h >> 2);
    return (size_t)h;
  }
};
std::mutex g_map_mu;
std::unordered_map<MapKey, CUtensorMap, MapKeyHash> g_maps;
constexpr size_t kMaxCachedMaps = 8192;

template <typename Encode>
int cached_map(CUtensorMap* map, const MapKey& key, Encode encode) {
  {
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto it = g_maps.find(key);
    if (it != g_maps.end()) {
      *map = it->second;
      return NVFP4_OK;
    }
  }
  int rc = encode();
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_map_mu);
  if (g_maps.size() >= kMaxCachedMaps) g_maps.clear();
  g_maps.emplace(key, *map);
  return NVFP4_OK;
}

int encode_operand(CUtensorMap* map, const void* base, int rows, int k, int l, int box_rows) {
  const MapKey key{reinterpret_cast<uintptr_t>(base), rows, k, l, box_rows};
  return cached_map(map, key,
                    [&] { return encode_operand_uncached(map, base, rows, k, l, box_rows); });
}

// 2-D view [atoms][128 x 32-bit] of a permuted scale tensor (512-byte atoms),
// box {128, 4}: the four atoms of one 256-deep K step of one 128-row block.
int encode_sf_atoms_uncached(CUtensorMap* map, const void* base, int atoms) {
  const cuuint64_t dims[2] = {128u, (cuuint64_t)atoms};
  const cuuint64_t strides[1] = {(cuuint64_t)kSfAtom};
  const cuuint32_t box[2] = {128u, (cuuint32_t)(kBK / kKStep)};
  const cuuint32_t estr[2] = {1u, 1u};
  CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(NVFP4_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) for %d scale atoms", (int)r,
                atoms);
  return NVFP4_OK;
}

int encode_sf_atoms(CUtensorMap* map, const void* base, int atoms) {
  // k = -1 keeps these keys apart from the operand maps'
  const MapKey key{reinterpret_cast<uintptr_t>(base), atoms, -1, 0, kBK / kKStep};
  return cached_map(map, key, [&] { return encode_sf_atoms_uncached(map, base, atoms); });
}

std::atomic<unsigned long long> g_launches{0};

// Every kernel launch of the library ends here (and is counted).
int check_launch(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return NVFP4_OK;
}

template <typename Kern>
int set_smem_once(DeviceState* d, int slot, Kern kern, int bytes) {
  // two threads may both set the attribute the first time: it is idempotent
  if (d->smem_set[slot].load(std::memory_order_acquire)) return NVFP4_OK;
  RelaxedCapture relaxed;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess)
    return fail(NVFP4_ERR_CUDA, "cudaFuncSetAttribute(smem=%d): %s", bytes, cudaGetErrorString(e));
  d->smem_set[slot].store(true, std::memory_order_release);
  return NVFP4_OK;
}

// Grow (never shrink) the stream's split-K scratch; counters start at zero
// and every kernel leaves them at zero.  Growth may happen while the stream is
// being captured into a CUDA graph: the allocation then runs in relaxed
// capture mode, a buffer that is outgrown is kept (a graph captured earlier
// may still use it), and new counters are zeroed by a stream-ordered memset —
// a node of the graph when captured — on every call until an uncaptured call
// has zeroed them.
int get_workspace(DeviceState* d, cudaStream_t stream, size_t partial_bytes, size_t counters,
                  Workspace** out) {
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) cs = cudaStreamCaptureStatusNone;
  const bool capturing = cs != cudaStreamCaptureStatusNone;
  std::lock_guard<std::mutex> lk(g_mu);
  Workspace& w = d->ws[stream];
  if (w.partial_bytes < partial_bytes) {
    RelaxedCapture relaxed;
    float* p = nullptr;
    cudaError_t e = cudaMalloc(&p, partial_bytes);
    if (e != cudaSuccess)
      return fail(NVFP4_ERR_CUDA, "split-K workspace (%zu bytes): %s", partial_bytes,
                  cudaGetErrorString(e));
    w.partials = p;
    w.partial_bytes = partial_bytes;
  }
  if (w.counter_count < counters) {
    RelaxedCapture relaxed;
    int* p = nullptr;
    cudaError_t e = cudaMalloc(&p, counters * sizeof(int));
    if (e != cudaSuccess)
      return fail(NVFP4_ERR_CUDA, "split-K counters: %s", cudaGetErrorString(e));
    w.counters = p;
    w.counter_count = counters;
    w.zero_pending = true;
  }
  if (w.zero_pending) {
    cudaError_t e = cudaMemsetAsync(w.counters, 0, w.counter_count * sizeof(int), stream);
    if (e != cudaSuccess)
      return fail(NVFP4_ERR_CUDA, "split-K counters: %s", cudaGetErrorString(e));
    if (!capturing) w.zero_pending = false;
  }
  *out = &w;
  return NVFP4_OK;
}

// After a kernel gave up on a wait its counters may be mid-protocol: zero them.
void reset_workspaces(DeviceState* d) {
  std::lock_guard<std::mutex> lk(g_mu);
  for (auto& kv : d->ws)
    if (kv.second.counters) cudaMemset(kv.second.counters, 0, kv.second.counter_count * sizeof(int));
}

// Once per device, with that device current: the device address of the
// no-alloc scratch array (host code may not use the symbol itself as a pointer).
int noalloc_scratch(DeviceState* d, unsigned char** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!d->noalloc_scratch) {
    RelaxedCapture relaxed;
    void* ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || !ptr)
      return fail(NVFP4_ERR_CUDA, "no-alloc scratch address: %s", cudaGetErrorString(e));
    d->noalloc_scratch = static_cast<unsigned char*>(ptr);
  }
  *out = d->noalloc_scratch;
  return NVFP4_OK;
}

// Where a dual call's split-K scratch and tensor maps come from.  The
// ordinary entry point grows a per-stream workspace with cudaMalloc and keeps
// encoded descriptors in a host-side cache; the allocation-free one (`fixed`
// set) uses the library's fixed scratch array and encodes every descriptor
// on the stack.  Kernel and split choices are the same for both.
struct DualAlloc {
  unsigned char* fixed = nullptr;
};

int encode_dual_operand(const DualAlloc& al, CUtensorMap* map, const void* base, int rows, int k,
                        int l, int box_rows) {
  return al.fixed ? encode_operand_uncached(map, base, rows, k, l, box_rows)
                  : encode_operand(map, base, rows, k, l, box_rows);
}

// Workspace split-K scratch for `p.tiles` tiles x `p.splits` slots of
// `slot_bytes` each: the stream's cudaMalloc'd workspace, or the fixed array
// (rejected when too small; its counters are zeroed on `stream` first, since
// the array keeps whatever the previous call left there).
int dual_scratch(DeviceState* d, const DualAlloc& al, cudaStream_t stream, size_t slot_bytes,
                 DualParams& p) {
  const size_t need = (size_t)p.tiles * p.splits * slot_bytes;
  if (!al.fixed) {
    Workspace* w = nullptr;
    int rc = get_workspace(d, stream, need, (size_t)p.tiles, &w);
    if (rc) return rc;
    p.ws = w->partials;
    p.ws_ctr = w->counters;
    return NVFP4_OK;
  }
  if (need > kNoAllocPartialBytes || (size_t)p.tiles > kNoAllocCounterInts)
    return fail(NVFP4_ERR_SHAPE,
                "split-K needs %zu bytes of partials for %d tiles x %d splits; the fixed "
                "no-alloc scratch holds %zu bytes and %zu tiles",
                need, p.tiles, p.splits, kNoAllocPartialBytes, kNoAllocCounterInts);
  p.ws = reinterpret_cast<float*>(al.fixed);
  p.ws_ctr = reinterpret_cast<int*>(al.fixed + kNoAllocPartialBytes);
  cudaError_t e = cudaMemsetAsync(p.ws_ctr, 0, (size_t)p.tiles * sizeof(int), stream);
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "counter reset: %s", cudaGetErrorString(e));
  return NVFP4_OK;
}

// Number of K splits for the 128-wide dual kernel.  A split costs the
// partial-sum exchange through global memory (~5 us on B200), which measured
// slower than leaving SMs idle once there are at least a quarter as many
// tiles as SMs (e.g. 48 tiles: 18.4 us unsplit, 24.6 us in 2 splits, 28.7 us
// in 3).  Below that: enough work units to give every SM one, each split at
// least two 256-deep K blocks, at most 16.
int choose_splits(int tiles, int k_blocks, int num_sms) {
  if (4 * tiles >= num_sms) return 1;
  int s = num_sms / tiles;
  s = s < k_blocks / 2 ? s : k_blocks / 2;
  s = s < 16 ? s : 16;
  return s < 1 ? 1 : s;
}

// Programmatic dependent launch for the GEMM kernels on this thread's calls
// (set from the knobs at every entry point).  The kernels build their
// barriers and TMEM allocation while the previous kernel in the stream is
// still running and wait on griddepcontrol before touching global memory;
// each kernel is persistent (every CTA resident from the start), so letting
// the next one be scheduled early cannot starve it of SMs.
thread_local bool t_pdl = true;

// cudaLaunchKernelEx with programmatic stream serialization (when enabled)
// and an optional cluster dimension.
template <class Kern, class Params>
int launch_gemm(Kern kern, unsigned grid, int threads, int smem, cudaStream_t stream,
                const Params& p, int cluster, const char* what) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3((unsigned)threads, 1, 1);
  cfg.dynamicSmemBytes = (size_t)smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned n = 0;
  if (cluster > 0) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = (unsigned)cluster;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (t_pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "%s launch: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

// ---------------------------------------------------------------- dual GEMM
// Cluster split-K launch: grid = tiles * S CTAs in clusters of S (one unit
// per CTA), no workspace.
template <int kStages, int S>
int launch_dual_cluster(DeviceState* d, int slot, DualParams& p, cudaStream_t stream) {
  using Cfg = DualCfg<128, kStages, 8, 1>;
  auto kern = dual_gemm_kernel<128, kStages, 8, 1, true, S>;
  int rc = set_smem_once(d, slot, kern, Cfg::kSmemBytes);
  if (rc) return rc;
  p.splits = S;
  return launch_gemm(kern, (unsigned)(p.tiles * S), Cfg::kThreads, Cfg::kSmemBytes, stream, p, S,
                     "dual_gemm_kernel (cluster split-K)");
}

// How many S-CTA clusters of the cluster split-K kernel fit on the device at
// once (cached; 0 if the query fails).
template <int kStages, int S>
int max_active_clusters(DeviceState* d, int slot) {
  if (d->max_clusters[S]) return d->max_clusters[S];
  using Cfg = DualCfg<128, kStages, 8, 1>;
  auto kern = dual_gemm_kernel<128, kStages, 8, 1, true, S>;
  if (set_smem_once(d, slot, kern, Cfg::kSmemBytes)) return 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(S * d->num_sms), 1, 1);
  cfg.blockDim = dim3(Cfg::kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
    cudaGetLastError();
    n = 0;
  }
  d->max_clusters[S] = n > 0 ? n : -1;
  return n;
}

// Automatic split-K only when it takes at least kMinSplitSaving 256-deep K
// blocks off each CTA: the partial exchange and its barriers cost ~5-6 us
// (measured, unsplit vs split, us: 256x512x1024 11.9 / 16.3, 256x512x2048
// 13.3 / 16.7, 256x1024x4096 16.6 / 18.7, 128x2048x4096 18.1 / 19.1 (saving
// 2-12 blocks); 1536x512x7168 22.6 / 22.3, 512x768x7168 22.5 / 22.1,
// 128x7168x16384 49.6 / 44.6 (saving 14-32 blocks)).
constexpr int kMinSplitSaving = 14;
bool split_pays(int k_blocks, int splits) {
  return k_blocks - (k_blocks + splits - 1) / splits >= kMinSplitSaving;
}

template <int kBN, int kStages, int kEpiWarps, int kAccBufs>
int launch_dual(DeviceState* d, int slot, DualParams& p, int forced_splits, int cluster,
                const DualAlloc& al, cudaStream_t stream) {
  using Cfg = DualCfg<kBN, kStages, kEpiWarps, kAccBufs>;
  int rc = NVFP4_OK;
  p.n_blocks = (p.n + kBN - 1) / kBN;
  p.tiles = p.l * p.m_blocks * p.n_blocks;
  p.splits = 1;
  if constexpr (kBN == 128 && kEpiWarps == 8 && kAccBufs == 1) {
    // Cluster split-K when the tiles leave SMs idle, every split keeps at
    // least two 256-deep K blocks, and all clusters fit on the device at once
    // (partials cross the cluster instead of global memory).
    if (forced_splits < 1 && cluster != 1 && p.tiles < d->num_sms) {
      const int want = cluster == 2 || cluster == 4 ? cluster
                       : (4 * p.tiles <= d->num_sms ? 4 : 2);
      for (int S = want; S >= 2; S /= 2) {
        if (p.k_blocks < 2 * S) continue;
        if (cluster == 0 && !split_pays(p.k_blocks, S)) continue;
        const int fit = S == 4 ? max_active_clusters<kStages, 4>(d, 13)
                               : max_active_clusters<kStages, 2>(d, 12);
        if (p.tiles > fit) continue;
        return S == 4 ? launch_dual_cluster<kStages, 4>(d, 13, p, stream)
                      : launch_dual_cluster<kStages, 2>(d, 12, p, stream);
      }
    }
  }
  if (kBN == 128) {
    p.splits = choose_splits(p.tiles, p.k_blocks, d->num_sms);
    if (cluster == 0 && !split_pays(p.k_blocks, p.splits)) p.splits = 1;
    if (forced_splits >= 1) p.splits = forced_splits < p.k_blocks ? forced_splits : p.k_blocks;
  }
  if (p.splits > 1 &&
      (rc = dual_scratch(d, al, stream, (size_t)2 * kBN * kBM * sizeof(float), p)))
    return rc;
  const int units = p.tiles * p.splits;
  const int grid = units < d->num_sms ? units : d->num_sms;
  if (p.splits > 1) {
    auto kern = dual_gemm_kernel<kBN, kStages, kEpiWarps, kAccBufs, true>;
    if ((rc = set_smem_once(d, slot + 10, kern, Cfg::kSmemBytes))) return rc;
    return launch_gemm(kern, (unsigned)grid, Cfg::kThreads, Cfg::kSmemBytes, stream, p, 0,
                       "dual_gemm_kernel (split-K)");
  }
  auto kern = dual_gemm_kernel<kBN, kStages, kEpiWarps, kAccBufs, false>;
  if ((rc = set_smem_once(d, slot, kern, Cfg::kSmemBytes))) return rc;
  return launch_gemm(kern, (unsigned)grid, Cfg::kThreads, Cfg::kSmemBytes, stream, p, 0,
                     "dual_gemm_kernel");
}

// CTA-pair kernel: kBN-column tiles (128 or 64), two M=256 x N=kBN MMAs per
// 64-deep K step, one accumulator, scale atoms copied into TMEM by the MMA thread.
template <int kBN, int kStages>
int launch_dual_2sm(DeviceState* d, int slot, const void* a, const void* b1, const void* b2,
                    const void* sfa, const void* sfb1, const void* sfb2, void* c, int m, int n,
                    int k, int l, int group_m, const DualAlloc& al, cudaStream_t stream) {
  using Cfg = Dual2smCfg<kBN, kStages>;
  auto kern = dual_gemm_2sm_kernel<kBN, kStages>;
  int rc = set_smem_once(d, slot, kern, Cfg::kSmemBytes);
  if (rc) return rc;
  Dual2smParams p;
  memset(&p, 0, sizeof(p));
  p.c = static_cast<__half*>(c);
  p.m = m, p.n = n, p.k = k, p.l = l;
  p.mp_blocks = (m + 2 * kBM - 1) / (2 * kBM);
  p.n_blocks = (n + kBN - 1) / kBN;
  p.k_blocks = k / kBK;
  p.tiles = l * p.mp_blocks * p.n_blocks;
  p.sfa_blocks = (m + 127) / 128;
  p.sfb_blocks = (n + 127) / 128;
  p.group_m = group_m;
  p.c_lines32 = (n % 16 == 0) && (reinterpret_cast<uintptr_t>(c) % 32 == 0);
  p.status = d->status;
  p.wait_limit = wait_limit_cycles();
  // each CTA loads half of the tile's B1 rows and half of its B2 rows
  if ((rc = encode_dual_operand(al, &p.tmap_a, a, m, k, l, kBM))) return rc;
  if ((rc = encode_dual_operand(al, &p.tmap_b1, b1, n, k, l, kBN / 2))) return rc;
  if ((rc = encode_dual_operand(al, &p.tmap_b2, b2, n, k, l, kBN / 2))) return rc;
  const int rest_k = k / kKStep;
  const int a_atoms = l * p.sfa_blocks * rest_k, b_atoms = l * p.sfb_blocks * rest_k;
  auto enc = [&](CUtensorMap* map, const void* base, int atoms) {
    return al.fixed ? encode_sf_atoms_uncached(map, base, atoms) : encode_sf_atoms(map, base, atoms);
  };
  if ((rc = enc(&p.tmap_sfa, sfa, a_atoms))) return rc;
  if ((rc = enc(&p.tmap_sfb1, sfb1, b_atoms))) return rc;
  if ((rc = enc(&p.tmap_sfb2, sfb2, b_atoms))) return rc;
  const int pairs = p.tiles < d->num_sms / 2 ? p.tiles : d->num_sms / 2;
  return launch_gemm(kern, (unsigned)(2 * pairs), Cfg::kThreads, Cfg::kSmemBytes, stream, p, 0,
                     "dual_gemm_2sm_kernel");
}

// ---------------------------------------------------------------- grouped GEMM
template <int kBN, int kStages, int kEpiWarps, int kAccBufs, int kMaxGroups>
int launch_grouped_chunk(DeviceState* d, int slot, const nvfp4_group* gs, const int* idx, int count,
                         bool chained, cudaStream_t stream) {
  using Cfg = GroupedCfg<kBN, kStages, kEpiWarps, kAccBufs>;
  auto kern = grouped_gemm_kernel<kBN, kStages, kEpiWarps, kAccBufs, GroupedParams<kMaxGroups>>;
  int rc = set_smem_once(d, slot, kern, Cfg::kSmemBytes);
  if (rc) return rc;
  static thread_local GroupedParams<kMaxGroups> p;
  int tiles = 0;
  for (int i = 0; i < count; ++i) {
    const nvfp4_group& g = gs[idx[i]];
    GroupInfo& gi = p.g[i];
    gi.sfa = static_cast<const uint8_t*>(g.sfa_perm);
    gi.sfb = static_cast<const uint8_t*>(g.sfb_perm);
    gi.c = static_cast<__half*>(g.c);
    gi.m = g.m, gi.n = g.n, gi.k = g.k, gi.l = g.l;
    gi.m_blocks = (g.m + kBM - 1) / kBM;
    gi.n_blocks = (g.n + kBN - 1) / kBN;
    gi.tile_start = tiles;
    gi.lines32 = (g.n % 16 == 0) && (reinterpret_cast<uintptr_t>(g.c) % 32 == 0);
    tiles += g.l * gi.m_blocks * gi.n_blocks;
    if ((rc = encode_operand(&p.tmap_a[i], g.a, g.m, g.k, g.l, kBM))) return rc;
    if ((rc = encode_operand(&p.tmap_b[i], g.b, g.n, g.k, g.l, kBN))) return rc;
  }
  p.num_groups = count;
  p.tiles = tiles;
  p.chained = chained;
  p.status = d->status;
  p.wait_limit = wait_limit_cycles();
  const int grid = tiles < d->num_sms ? tiles : d->num_sms;
  return launch_gemm(kern, (unsigned)grid, Cfg::kThreads, Cfg::kSmemBytes, stream, p, 0,
                     "grouped_gemm_kernel");
}

// bn 256: 128x256 tiles (4 stages, 8 epilogue warps, one accumulator
// buffer); bn 128: 128x128 tiles (6 stages, 4 epilogue warps, two
// accumulator buffers).
template <int kMaxGroups>
int launch_grouped(DeviceState* d, const nvfp4_group* gs, const int* idx, int count, int bn,
                   bool chained, cudaStream_t stream) {
  const int base = kMaxGroups == 16 ? 4 : 6;
  if (bn == 256)
    return launch_grouped_chunk<256, 4, 8, 1, kMaxGroups>(d, base, gs, idx, count, chained, stream);
  return launch_grouped_chunk<128, 6, 4, 2, kMaxGroups>(d, base + 1, gs, idx, count, chained, stream);
}

// CTA-pair grouped kernel: 256x256 tiles, one M=256 x N=256 pair MMA per
// 64-deep K step, scale atoms copied into TMEM by the MMA thread; four tensor
// maps per group in the parameter block.
constexpr int kPairMaxGroups = 48;   // 48 x 4 maps + the table: ~27 KB of parameters
int launch_grouped_pair(DeviceState* d, const nvfp4_group* gs, const int* idx, int count,
                        bool chained, cudaStream_t stream) {
  using Cfg = GroupedPairCfg<5>;
  using P = GroupedPairParams<kPairMaxGroups>;
  auto kern = grouped_gemm_2sm_kernel<5, kPairMaxGroups>;
  int rc = set_smem_once(d, 16, kern, Cfg::kSmemBytes);
  if (rc) return rc;
  static thread_local P p;
  int tiles = 0;
  for (int i = 0; i < count; ++i) {
    const nvfp4_group& g = gs[idx[i]];
    GroupPairInfo& gi = p.g[i];
    gi.c = static_cast<__half*>(g.c);
    gi.m = g.m, gi.n = g.n, gi.k = g.k, gi.l = g.l;
    const int rem = g.m % (2 * kBM);
    gi.half = rem != 0 && rem <= kBM;   // the last pair block runs as a half tile
    gi.mp_blocks = (g.m + 2 * kBM - 1) / (2 * kBM);
    gi.n_blocks = (g.n + Cfg::kBN - 1) / Cfg::kBN;
    gi.sfa_blocks = (g.m + 127) / 128;
    gi.sfb_blocks = (g.n + 127) / 128;
    gi.tile_start = tiles;
    gi.lines32 = (g.n % 16 == 0) && (reinterpret_cast<uintptr_t>(g.c) % 32 == 0);
    tiles += g.l * gi.mp_blocks * gi.n_blocks;
    const int rest_k = g.k / kKStep;
    if ((rc = encode_operand(&p.tmap_a[i], g.a, g.m, g.k, g.l, kBM / 2))) return rc;
    if ((rc = encode_operand(&p.tmap_b[i], g.b, g.n, g.k, g.l, Cfg::kBN / 2))) return rc;
    if ((rc = encode_sf_atoms(&p.tmap_sfa[i], g.sfa_perm, g.l * gi.sfa_blocks * rest_k))) return rc;
    if ((rc = encode_sf_atoms(&p.tmap_sfb[i], g.sfb_perm, g.l * gi.sfb_blocks * rest_k))) return rc;
  }
  p.num_groups = count;
  p.tiles = tiles;
  p.chained = chained;
  p.status = d->status;
  p.wait_limit = wait_limit_cycles();
  const int pairs = tiles < d->num_sms / 2 ? tiles : d->num_sms / 2;
  return launch_gemm(kern, (unsigned)(2 * pairs), Cfg::kThreads, Cfg::kSmemBytes, stream, p, 0,
                     "grouped_gemm_2sm_kernel");
}

// MoE mode: up to kMoeMaxExpertsPerLaunch experts per launch, sizes read on
// the device; the grid is persistent over the upper bound of the tiles.
constexpr int kMoeMaxExpertsPerLaunch = 128;

template <int kBN, int kStages, int kEpiWarps, int kAccBufs>
int launch_moe_grouped_chunk(DeviceState* d, int slot, const void* a, int a_rows, const void* sfa,
                             const int* counts, const int* row_offsets, const int* atom_offsets,
                             const void* const* b, const void* const* sfb, int e0, int count,
                             int n, int k, void* c, cudaStream_t stream) {
  using Cfg = GroupedCfg<kBN, kStages, kEpiWarps, kAccBufs>;
  using P = MoeGemmParams<kMoeMaxExpertsPerLaunch>;
  auto kern = grouped_gemm_kernel<kBN, kStages, kEpiWarps, kAccBufs, P>;
  int rc = set_smem_once(d, slot, kern, Cfg::kSmemBytes);
  if (rc) return rc;
  static thread_local P p;
  if ((rc = encode_operand(&p.tmap_a, a, a_rows, k, 1, kBM))) return rc;
  for (int i = 0; i < count; ++i) {
    if ((rc = encode_operand(&p.tmap_b[i], b[e0 + i], n, k, 1, kBN))) return rc;
    p.sfb[i] = static_cast<const uint8_t*>(sfb[e0 + i]);
  }
  p.sfa = static_cast<const uint8_t*>(sfa);
  p.counts = counts, p.row_offsets = row_offsets, p.atom_offsets = atom_offsets;
  p.c = static_cast<__half*>(c);
  p.e0 = e0, p.experts = count, p.n = n, p.k = k;
  p.lines32 = (n % 16 == 0) && (reinterpret_cast<uintptr_t>(c) % 32 == 0);
  p.chained = 0;
  p.status = d->status;
  p.wait_limit = wait_limit_cycles();
  // tiles <= (ceil(rows / 128) + experts) * n_blocks whatever the routing
  const long long bound = ((long long)(a_rows + kBM - 1) / kBM + count) * ((n + kBN - 1) / kBN);
  const int grid = bound < d->num_sms ? (int)bound : d->num_sms;
  return launch_gemm(kern, (unsigned)grid, Cfg::kThreads, Cfg::kSmemBytes, stream, p, 0,
                     "grouped_gemm_kernel (MoE)");
}

}  // namespace
}  // namespace nvfp4

using namespace nvfp4;

namespace nvfp4 {
namespace {

int validate_dual(const void* a, const void* b1, const void* b2, const void* sfa,
                  const void* sfb1, const void* sfb2, const void* c, int m, int n, int k, int l) {
  if (!a || !b1 || !b2 || !sfa || !sfb1 || !sfb2 || !c)
    return fail(NVFP4_ERR_INVALID_ARG, "null pointer argument");
  if (m < 1 || n < 1 || k < 1 || l < 1)
    return fail(NVFP4_ERR_INVALID_ARG, "sizes must be positive (m=%d n=%d k=%d l=%d)", m, n, k, l);
  if (k % kBK != 0) return fail(NVFP4_ERR_SHAPE, "K=%d is not a multiple of 256", k);
  if (n % 8 != 0) return fail(NVFP4_ERR_SHAPE, "N=%d is not a multiple of 8", n);
  if ((long long)m * n * l >= (1LL << 40) || (long long)(m > n ? m : n) * k * l >= (1LL << 41))
    return fail(NVFP4_ERR_SHAPE, "problem too large");
  if (!aligned16(a) || !aligned16(b1) || !aligned16(b2) || !aligned16(sfa) || !aligned16(sfb1) ||
      !aligned16(sfb2) || !aligned16(c))
    return fail(NVFP4_ERR_ALIGNMENT, "all operands must be 16-byte aligned");
  return NVFP4_OK;
}

// Kernel choice and launch of one validated dual GEMM call (both entry points).
int run_dual(DeviceState* d, const void* a, const void* b1, const void* b2, const void* sfa,
             const void* sfb1, const void* sfb2, void* c, int m, int n, int k, int l,
             const DualAlloc& al, cudaStream_t stream) {
  int rc = NVFP4_OK;
  DualParams p;
  memset(&p, 0, sizeof(p));
  p.sfa = static_cast<const uint8_t*>(sfa);
  p.sfb1 = static_cast<const uint8_t*>(sfb1);
  p.sfb2 = static_cast<const uint8_t*>(sfb2);
  p.c = static_cast<__half*>(c);
  p.m = m, p.n = n, p.k = k, p.l = l;
  p.c_lines32 = (n % 16 == 0) && (reinterpret_cast<uintptr_t>(c) % 32 == 0);
  p.m_blocks = (m + kBM - 1) / kBM;
  p.k_blocks = k / kBK;
  const Knobs kn = read_knobs();
  t_pdl = kn.pdl;
  p.group_m = kn.dual_group_m;
  p.status = d->status;
  p.wait_limit = wait_limit_cycles();
  // Kernel choice: the CTA-pair kernel unless the single-CTA kernel's K
  // split pays.  Measured on one B200 (us per call, 15 distinct inputs back
  // to back after an L2 flush; pair 64-wide / pair 128-wide / single):
  //   pair 64-wide tiles when they make at most one CTA per SM:
  //     256x4096x7168 14.3 / 16.1 / 18.7, 256x3072x4096 10.2 / 11.6 / 12.3,
  //     256x2048x7168 12.2 / 15.1 / 17.1, 256x4096x14336 22.8 / 25.5 / 25.5,
  //     128x4096x7168 15.3 / 15.9 / 18.7, 256x512x1024 6.1 / 7.2 / 6.8;
  //   but with M <= 128 (one 128-row block: the pair's second CTA has no
  //     rows) and at least 48 K blocks the single-CTA kernel's cluster K
  //     split: 128x3584x16384 26.2 / 27.7 / 24.4, 128x1792x16384 20.6 / 26.4
  //     / 19.5, 128x896x16384 19.9 / 25.6 / 17.9 (with 28 K blocks the pair
  //     still wins: 128x2048x7168 12.2 / 15.0 / 15.1);
  //   otherwise the single-CTA kernel too when it would split K (at least 48
  //     K blocks) and the 128-wide pair tiles leave SMs idle:
  //     128x7168x16384 (configuration 2) 46.3 / 33.3 / 32.3;
  //   otherwise pair 128-wide tiles: 512x4096x7168 21.8 / 16.9 / 18.9,
  //     512x7168x2048 17.0 / 14.1 / 15.2, 1024x4096x7168 36.8 / 27.2 / 33.0,
  //     2048x4096x7168 62.4 / 48.6 / 60.2, 256x7168x2048 11.7 / 10.1 / 11.3,
  //     8192x14336x4096 (configuration 1) 507 / 352 / 427.
  // NVFP4_DUAL_KERNEL=pair|single forces the kernel (NVFP4_DUAL_BN=64|128 its
  // tile width; NVFP4_DUAL_BN alone: the single-CTA kernel at that width).
  const int pair_blocks = l * ((m + 2 * kBM - 1) / (2 * kBM));
  const int ctas64 = 2 * pair_blocks * ((n + 63) / 64);
  const int ctas128 = 2 * pair_blocks * ((n + 127) / 128);
  const bool forced_single = kn.dual_kernel == 2 || kn.dual_splits > 0 || kn.dual_cluster > 0;
  bool pair = kn.dual_kernel == 1;
  int pair_bn = kn.dual_bn == 64 || kn.dual_bn == 128 ? kn.dual_bn : 0;
  if (!pair && !forced_single && kn.dual_bn == 0) {
    const bool long_k = p.k_blocks >= 48, half_idle = m <= kBM;
    if (ctas64 <= d->num_sms && !(half_idle && long_k)) pair = true, pair_bn = 64;
    else if (!(long_k && (half_idle || ctas128 < d->num_sms))) pair = true, pair_bn = 128;
  }
  if (pair) {
    if (pair_bn == 0) pair_bn = ctas64 <= d->num_sms ? 64 : 128;
    if (pair_bn == 64)
      return launch_dual_2sm<64, 7>(d, 15, a, b1, b2, sfa, sfb1, sfb2, c, m, n, k, l,
                                    kn.dual_group_m, al, stream);
    return launch_dual_2sm<128, 5>(d, 14, a, b1, b2, sfa, sfb1, sfb2, c, m, n, k, l,
                                   kn.dual_group_m, al, stream);
  }
  // 128-wide tiles (one fused N=256 MMA per K step), split along K when
  // there are fewer tiles than SMs; 64-wide tiles only on request.
  int bn = 128;
  if (kn.dual_bn == 64 || kn.dual_bn == 128) bn = kn.dual_bn;
  if ((rc = encode_dual_operand(al, &p.tmap_a, a, m, k, l, kBM))) return rc;
  if ((rc = encode_dual_operand(al, &p.tmap_b1, b1, n, k, l, bn))) return rc;
  if ((rc = encode_dual_operand(al, &p.tmap_b2, b2, n, k, l, bn))) return rc;
  if (bn == 128)
    return launch_dual<128, 4, 8, 1>(d, 0, p, kn.dual_splits, kn.dual_cluster, al, stream);
  return launch_dual<64, 5, 4, 2>(d, 1, p, kn.dual_splits, kn.dual_cluster, al, stream);
}

}  // namespace
}  // namespace nvfp4

extern "C" int nvfp4_dual_gemm(const void* a, const void* b1, const void* b2, const void* sfa,
                               const void* sfb1, const void* sfb2, void* c, int m, int n, int k,
                               int l, void* stream_) {
  int rc = validate_dual(a, b1, b2, sfa, sfb1, sfb2, c, m, n, k, l);
  if (rc) return rc;
  DeviceState* d = nullptr;
  if ((rc = get_device(&d))) return rc;
  return run_dual(d, a, b1, b2, sfa, sfb1, sfb2, c, m, n, k, l, DualAlloc{},
                  static_cast<cudaStream_t>(stream_));
}


extern "C" int nvfp4_grouped_gemm(const nvfp4_group* groups, int num_groups, void* stream_) {
  if (!groups || num_groups < 0) return fail(NVFP4_ERR_INVALID_ARG, "bad group table");
  std::vector<int> live;
  live.reserve(num_groups);
  for (int i = 0; i < num_groups; ++i) {
    const nvfp4_group& g = groups[i];
    if (g.m < 0 || g.n < 1 || g.k < 1 || g.l < 1)
      return fail(NVFP4_ERR_INVALID_ARG, "group %d: bad sizes (m=%d n=%d k=%d l=%d)", i, g.m, g.n,
                  g.k, g.l);
    if (g.m == 0) continue;
    if (!g.a || !g.b || !g.sfa_perm || !g.sfb_perm || !g.c)
      return fail(NVFP4_ERR_INVALID_ARG, "group %d: null pointer", i);
    if (g.k % kBK != 0) return fail(NVFP4_ERR_SHAPE, "group %d: K=%d not a multiple of 256", i, g.k);
    if (g.n % 8 != 0) return fail(NVFP4_ERR_SHAPE, "group %d: N=%d not a multiple of 8", i, g.n);
    if ((long long)g.m * g.n * g.l >= (1LL << 40) ||
        (long long)(g.m > g.n ? g.m : g.n) * g.k * g.l >= (1LL << 41))
      return fail(NVFP4_ERR_SHAPE, "group %d: too large", i);
    if (!aligned16(g.a) || !aligned16(g.b) || !aligned16(g.sfa_perm) || !aligned16(g.sfb_perm) ||
        !aligned16(g.c))
      return fail(NVFP4_ERR_ALIGNMENT, "group %d: operands must be 16-byte aligned", i);
    live.push_back(i);
  }
  if (live.empty()) return NVFP4_OK;
  DeviceState* d = nullptr;
  int rc = get_device(&d);
  if (rc) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const int n = (int)live.size();
  // 128x256 tiles when every group is at least 256 wide, unless all the
  // 128x128 tiles fit in one wave: a 128-wide K block costs ~0.74 of a
  // 256-wide one (the copy path moves 36 instead of 54 KB), so a one-wave
  // grid of them finishes first (measured 149.7 vs 101.1 us on configuration
  // 3, twice the tiles, 0.74 per K block).
  int min_n = groups[live[0]].n;
  long long tiles128 = 0;
  for (int i : live) {
    const nvfp4_group& g = groups[i];
    min_n = g.n < min_n ? g.n : min_n;
    tiles128 += (long long)g.l * ((g.m + kBM - 1) / kBM) * ((g.n + 127) / 128);
  }
  int bn = min_n >= 256 && tiles128 > d->num_sms ? 256 : 128;
  const Knobs kn = read_knobs();
  t_pdl = kn.pdl;
  const int forced = kn.grouped_bn;
  if (forced == 128 || forced == 256) bn = forced;
  // The CTA-pair kernel (256x256 tiles) when every group has at least 24 K
  // blocks and 256 columns, and covering the groups in 256-row pair blocks
  // costs at most 1.5x the 128-row blocks' rows (a last block of <= 128 rows
  // runs as a half tile at ~0.95 of a full tile's time, so it counts as a
  // full block); it keeps one accumulator,
  // so with few K blocks per tile its exposed epilogue loses.  Measured on
  // one B200 (us per call, pair / single-CTA): configuration 3 88.9 / 95.4,
  // configuration 4 241.8 / 255.0, 8 groups of 64-248 rows x 4096 x 7168
  // 32.0 / 37.5 (padding 1.45x); with fewer K blocks 8 groups x 7168 x 2048
  // 26.1 / 22.3, [192, 320] x 3072 x 4096 11.6 / 10.3, [128, 384] x 4096 x
  // 1536 10.0 / 6.8.
  bool pair = kn.grouped_kernel == 1;
  if (kn.grouped_kernel == 0 && forced == 0) {
    long long rows128 = 0, rows256 = 0;
    bool long_k = min_n >= 256;
    for (int i : live) {
      const nvfp4_group& g = groups[i];
      long_k = long_k && g.k >= 24 * kBK;
      rows128 += (long long)g.l * ((g.m + 127) / 128) * 128 * g.n;
      rows256 += (long long)g.l * ((g.m + 255) / 256) * 256 * g.n;
    }
    pair = long_k && 2 * rows256 <= 3 * rows128;
  }
  if (pair) {
    // near-equal chunks of at most kPairMaxGroups groups
    const int chunks = (n + kPairMaxGroups - 1) / kPairMaxGroups;
    for (int c = 0, s = 0; c < chunks; ++c) {
      const int cnt = (n - s) / (chunks - c);
      if ((rc = launch_grouped_pair(d, groups, live.data() + s, cnt, s > 0, stream))) return rc;
      s += cnt;
    }
    return NVFP4_OK;
  }
  if (n <= 16) return launch_grouped<16>(d, groups, live.data(), n, bn, false, stream);
  // later chunks chained, as for the pair kernel
  for (int s = 0; s < n; s += 96) {
    const int cnt = n - s < 96 ? n - s : 96;
    if ((rc = launch_grouped<96>(d, groups, live.data() + s, cnt, bn, s > 0, stream))) return rc;
  }
  return NVFP4_OK;
}

extern "C" int nvfp4_device_status(void* stream_, unsigned* bits_out) {
  DeviceState* d = nullptr;
  int rc = get_device(&d);
  if (rc) return rc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "stream sync: %s", cudaGetErrorString(e));
  unsigned bits = 0;
  e = cudaMemcpy(&bits, d->status, sizeof(bits), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return fail(NVFP4_ERR_CUDA, "status read: %s", cudaGetErrorString(e));
  if (bits) {
    const unsigned zero = 0;
    cudaMemcpy(d->status, &zero, sizeof(zero), cudaMemcpyHostToDevice);
    reset_workspaces(d);
  }
  if (bits_out) *bits_out = bits;
  if (bits) return fail(NVFP4_ERR_TIMEOUT, "device status bits 0x%x (a bounded wait ran out)", bits);
  return NVFP4_OK;
}

extern "C" int nvfp4_wait_selftest(long long limit_cycles, void* stream_) {
  if (limit_cycles < 1) return fail(NVFP4_ERR_INVALID_ARG, "limit must be positive");
  DeviceState* d = nullptr;
  int rc = get_device(&d);
  if (rc) return rc;
  wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream_)>>>(d->status, limit_cycles);
  return check_launch("wait_selftest_kernel");
}

extern "C" const char* nvfp4_status_string(int s) {
  switch (s) {
    case NVFP4_OK: return "ok";
    case NVFP4_ERR_INVALID_ARG: return "invalid argument";
    case NVFP4_ERR_SHAPE: return "unsupported shape";
    case NVFP4_ERR_ALIGNMENT: return "misaligned pointer";
    case NVFP4_ERR_CUDA: return "CUDA error";
    case NVFP4_ERR_DEVICE: return "unsupported device";
    case NVFP4_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

extern "C" const char* nvfp4_last_error(void) { return t_last_error; }

extern "C" int nvfp4_version(void) { return 100; }

extern "C" unsigned long long nvfp4_launch_count(void) {
  return nvfp4::g_launches.load(std::memory_order_relaxed);
}

extern "C" int nvfp4_quantize(const float* x, int rows, int k, int l, void* packed,
                              void* sf_perm, void* sf_plain, void* stream_) {
  if (!x || !packed || !sf_perm) return fail(NVFP4_ERR_INVALID_ARG, "null pointer argument");
  if (rows < 1 || k < 1 || l < 1)
    return fail(NVFP4_ERR_INVALID_ARG, "sizes must be positive (rows=%d k=%d l=%d)", rows, k, l);
  if (k % 64 != 0) return fail(NVFP4_ERR_SHAPE, "K=%d is not a multiple of 64", k);
  const int row_blocks = (rows + 127) / 128;
  if (row_blocks > 65535 || l > 65535 || (long long)rows * k * l >= (1LL << 40))
    return fail(NVFP4_ERR_SHAPE, "problem too large");
  if (!aligned16(x) || !aligned16(packed) || !aligned16(sf_perm) ||
      (sf_plain && (reinterpret_cast<uintptr_t>(sf_plain) & 3u)))
    return fail(NVFP4_ERR_ALIGNMENT, "x/packed/sf_perm need 16-byte, sf_plain 4-byte alignment");
  DeviceState* d = nullptr;
  int rc = get_device(&d);
  if (rc) return rc;
  QuantParams p;
  p.x = x;
  p.packed = static_cast<uint8_t*>(packed);
  p.sf_perm = static_cast<uint8_t*>(sf_perm);
  p.sf_plain = static_cast<uint8_t*>(sf_plain);
  p.rows = rows, p.k = k, p.l = l;
  p.row_blocks = row_blocks;
  p.k_atoms = k / 64;
  const dim3 grid(p.k_atoms, row_blocks, l);
  quantize_nvfp4_kernel<<<grid, kQuantThreads, 0, static_cast<cudaStream_t>(stream_)>>>(p);
  return check_launch("quantize_nvfp4_kernel");
}

// ---------------------------------------------------------------------------
// MoE dispatch (route -> per-expert NVFP4 A operands) and combine.
// ---------------------------------------------------------------------------
extern "C" int nvfp4_moe_grouped_gemm(const void* a_packed, int a_rows, const void* sfa_atoms,
                                      const int* counts, const int* row_offsets,
                                      const int* atom_offsets, const void* const* b,
                                      const void* const* sfb_perm, int num_experts, int n, int k,
                                      void* c, void* stream_) {
  if (a_rows < 0 || num_experts < 1 || n < 1 || k < 1)
    return fail(NVFP4_ERR_INVALID_ARG, "bad sizes (rows=%d experts=%d n=%d k=%d)", a_rows,
                num_experts, n, k);
  if (k % kBK != 0) return fail(NVFP4_ERR_SHAPE, "K=%d is not a multiple of 256", k);
  if (n % 8 != 0) return fail(NVFP4_ERR_SHAPE, "N=%d is not a multiple of 8", n);
  if ((long long)a_rows * n >= (1LL << 40) || (long long)a_rows * k >= (1LL << 41))
    return fail(NVFP4_ERR_SHAPE, "problem too large");
  if (a_rows == 0) return NVFP4_OK;
  if (!a_packed || !sfa_atoms || !counts || !row_offsets || !atom_offsets || !b || !sfb_perm || !c)
    return fail(NVFP4_ERR_INVALID_ARG, "null pointer argument");
  if (!aligned16(a_packed) || !aligned16(sfa_atoms) || !aligned16(c))
    return fail(NVFP4_ERR_ALIGNMENT, "a/sfa/c must be 16-byte aligned");
  for (int e = 0; e < num_experts; ++e) {
    if (!b[e] || !sfb_perm[e]) return fail(NVFP4_ERR_INVALID_ARG, "expert %d: null weights", e);
    if (!aligned16(b[e]) || !aligned16(sfb_perm[e]))
      return fail(NVFP4_ERR_ALIGNMENT, "expert %d: weights must be 16-byte aligned", e);
  }
  DeviceState* d = nullptr;
  int rc = get_device(&d);
  if (rc) return rc;
  const cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const Knobs kn = read_knobs();
  t_pdl = kn.pdl;
  int bn = n >= 256 ? 256 : 128;
  if (kn.grouped_bn == 128 || kn.grouped_bn == 256) bn = kn.grouped_bn;
  for (int e0 = 0; e0 < num_experts; e0 += kMoeMaxExpertsPerLaunch) {
    const int cnt = num_experts - e0 < kMoeMaxExpertsPerLaunch ? num_experts - e0
                                                               : kMoeMaxExpertsPerLaunch;
    rc = bn == 256
             ? launch_moe_grouped_chunk<256, 4, 8, 1>(d, 22, a_packed, a_rows, sfa_atoms, counts,
                                                      row_offsets, atom_offsets, b, sfb_perm, e0,
                                                      cnt, n, k, c, stream)
             : launch_moe_grouped_chunk<128, 6, 4, 2>(d, 23, a_packed, a_rows, sfa_atoms, counts,
                                                      row_offsets, atom_offsets, b, sfb_perm, e0,
                                                      cnt, n, k, c, stream);
    if (rc) return rc;
  }
  return NVFP4_OK;
}

extern "C" size_t nvfp4_moe_workspace_bytes(int tokens, int topk, int num_experts) {
  if (tokens < 0 || topk < 1 || num_experts < 1) return 0;
  const long long pairs = (long long)tokens * topk;
  const long long chunks = (pairs + kMoeChunk - 1) / kMoeChunk;
  return (size_t)(chunks > 0 ? chunks : 1) * (size_t)num_experts * sizeof(int);
}

extern "C" size_t nvfp4_moe_sf_bytes(int tokens, int topk, int k, int num_experts) {
  if (tokens < 0 || topk < 1 || num_experts < 1 || k < 64) return 0;
  const long long pairs = (long long)tokens * topk;
  const long long blocks = (pairs + 127) / 128 + (pairs < num_experts ? pairs : num_experts);
  return (size_t)blocks * (size_t)(k / 64) * 512u;
}

extern "C" int nvfp4_moe_dispatch(const float* x, const int* expert_ids, int tokens, int topk,
                                  int k, int num_experts, void* packed, void* sf_perm, int* counts,
                                  int* row_offsets, int* atom_offsets, int* src, int* dst,
                                  void* workspace, size_t workspace_bytes, void* stream_) {
  if (tokens < 0 || topk < 1 || k < 1 || num_experts < 1)
    return fail(NVFP4_ERR_INVALID_ARG, "bad sizes (tokens=%d topk=%d k=%d experts=%d)", tokens,
                topk, k, num_experts);
  if (num_experts > kMoeMaxExperts)
    return fail(NVFP4_ERR_SHAPE, "%d experts (at most %d)", num_experts, kMoeMaxExperts);
  if (k % 64 != 0) return fail(NVFP4_ERR_SHAPE, "K=%d is not a multiple of 64", k);
  const long long pairs = (long long)tokens * topk;
  const long long max_blocks = (pairs + 127) / 128 + (pairs < num_experts ? pairs : num_experts);
  if (pairs >= (1LL << 31) / 2 || max_blocks > 65535 || pairs * (long long)k >= (1LL << 40))
    return fail(NVFP4_ERR_SHAPE, "problem too large");
  if (!counts || !row_offsets || !atom_offsets || !workspace ||
      (pairs > 0 && (!x || !expert_ids || !packed || !sf_perm || !src || !dst)))
    return fail(NVFP4_ERR_INVALID_ARG, "null pointer argument");
  if (workspace_bytes < nvfp4_moe_workspace_bytes(tokens, topk, num_experts))
    return fail(NVFP4_ERR_INVALID_ARG, "workspace too small (%zu < %zu bytes)", workspace_bytes,
                nvfp4_moe_workspace_bytes(tokens, topk, num_experts));
  if ((x && !aligned16(x)) || (packed && !aligned16(packed)) || (sf_perm && !aligned16(sf_perm)) ||
      (reinterpret_cast<uintptr_t>(workspace) & 3u))
    return fail(NVFP4_ERR_ALIGNMENT, "x/packed/sf_perm need 16-byte alignment");
  DeviceState* d = nullptr;
  int rc = get_device(&d);
  if (rc) return rc;
  const cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  MoeParams p;
  p.x = x, p.ids = expert_ids;
  p.pairs = (int)pairs, p.topk = topk, p.k = k, p.experts = num_experts;
  p.chunks = (int)((pairs + kMoeChunk - 1) / kMoeChunk);
  p.k_atoms = k / 64;
  p.chunk_counts = static_cast<int*>(workspace);
  p.counts = counts, p.row_offsets = row_offsets, p.atom_offsets = atom_offsets;
  p.src = src, p.dst = dst;
  p.packed = static_cast<uint8_t*>(packed);
  p.sf_perm = static_cast<uint8_t*>(sf_perm);
  const size_t hist_bytes = (size_t)kMoeWarps * num_experts * sizeof(int);
  const int chunk_ctas = (p.chunks + kMoeWarps - 1) / kMoeWarps;
  if (chunk_ctas > 0) {
    moe_count_kernel<<<chunk_ctas, 32 * kMoeWarps, hist_bytes, stream>>>(p);
    if ((rc = check_launch("moe_count_kernel"))) return rc;
  }
  const int scan_threads = (num_experts + 31) / 32 * 32;
  moe_scan_kernel<<<1, scan_threads, 0, stream>>>(p);
  if ((rc = check_launch("moe_scan_kernel"))) return rc;
  if (chunk_ctas > 0) {
    moe_scatter_kernel<<<chunk_ctas, 32 * kMoeWarps, hist_bytes, stream>>>(p);
    if ((rc = check_launch("moe_scatter_kernel"))) return rc;
    const dim3 grid((p.k_atoms + kMoeAtomsPerCta - 1) / kMoeAtomsPerCta, (unsigned)max_blocks, 1);
    moe_quantize_kernel<<<grid, kQuantThreads, 0, stream>>>(p);
    if ((rc = check_launch("moe_quantize_kernel"))) return rc;
  }
  return NVFP4_OK;
}

extern "C" int nvfp4_moe_combine(const void* c, int c_rows, const int* dst, const float* weights,
                                 int tokens, int topk, int n, float* out, void* stream_) {
  if (tokens < 0 || topk < 1 || n < 1 || c_rows < 0)
    return fail(NVFP4_ERR_INVALID_ARG, "bad sizes (tokens=%d topk=%d n=%d c_rows=%d)", tokens,
                topk, n, c_rows);
  if (tokens == 0) return NVFP4_OK;
  if (!c || !dst || !out) return fail(NVFP4_ERR_INVALID_ARG, "null pointer argument");
  if ((long long)tokens > 65535 * 1024LL || (long long)tokens * n >= (1LL << 40))
    return fail(NVFP4_ERR_SHAPE, "problem too large");
  if ((reinterpret_cast<uintptr_t>(c) & 1u) || (reinterpret_cast<uintptr_t>(out) & 3u) ||
      (reinterpret_cast<uintptr_t>(dst) & 3u) || (weights && (reinterpret_cast<uintptr_t>(weights) & 3u)))
    return fail(NVFP4_ERR_ALIGNMENT, "c needs 2-byte, dst/weights/out 4-byte alignment");
  DeviceState* d = nullptr;
  int rc = get_device(&d);
  if (rc) return rc;
  MoeCombineParams p;
  p.c = static_cast<const __half*>(c);
  p.dst = dst, p.w = weights, p.out = out;
  p.tokens = tokens, p.topk = topk, p.n = n, p.c_rows = c_rows;
  const int span = kCombineThreads * 8;
  const cudaStream_t stream = static_cast<cudaStream_t>(stream_);
  const bool vec = n % 8 == 0 && aligned16(c) && aligned16(out);
  // grid.y is limited to 65535: token rows beyond it go in further launches
  for (int t0 = 0; t0 < tokens; t0 += 65535) {
    MoeCombineParams q = p;
    const int nt = tokens - t0 < 65535 ? tokens - t0 : 65535;
    q.dst = p.dst + (size_t)t0 * topk;
    q.w = p.w ? p.w + (size_t)t0 * topk : nullptr;
    q.out = p.out + (size_t)t0 * n;
    q.tokens = nt;
    const dim3 grid((n + span - 1) / span, nt, 1);
    if (vec)
      moe_combine_kernel<true><<<grid, kCombineThreads, 0, stream>>>(q);
    else
      moe_combine_kernel<false><<<grid, kCombineThreads, 0, stream>>>(q);
    if ((rc = check_launch("moe_combine_kernel"))) return rc;
  }
  return NVFP4_OK;
}

// ---------------------------------------------------------------------------
// Dual GEMM without any allocation.
//
// For callers that must not allocate device memory at call time: inference
// servers that reserve the whole HBM budget up front for weights and KV
// caches and hand out no further bytes, and hosts whose memory manager owns
// every device allocation (so a library-side cudaMalloc is forbidden or
// would fragment its pool).  The kernel and split choices are those of
// nvfp4_dual_gemm; only a workspace split-K keeps its partial sums somewhere
// else: in the fixed array g_noalloc_scratch (declared at the top of this
// file) instead of the per-stream workspace that nvfp4_dual_gemm grows with
// cudaMalloc.  Tensor maps are encoded on the stack (the descriptor cache
// would allocate host memory).
// ---------------------------------------------------------------------------
extern "C" int nvfp4_dual_gemm_noalloc(const void* a, const void* b1, const void* b2,
                                       const void* sfa, const void* sfb1, const void* sfb2,
                                       void* c, int m, int n, int k, int l, void* stream_) {
  int rc = validate_dual(a, b1, b2, sfa, sfb1, sfb2, c, m, n, k, l);
  if (rc) return rc;
  DeviceState* d = nullptr;
  if ((rc = get_device(&d))) return rc;
  DualAlloc al;
  if ((rc = noalloc_scratch(d, &al.fixed))) return rc;
  return run_dual(d, a, b1, b2, sfa, sfb1, sfb2, c, m, n, k, l, al,
                  static_cast<cudaStream_t>(stream_));
}
