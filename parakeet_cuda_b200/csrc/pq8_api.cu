// C ABI of libpq8: argument checking, per-device state, tile-shape choice and
// kernel launches. See include/pq8.h for the contract of each entry point.
#include <cublas_v2.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <vector>

#include "pq8.h"
#include "pq8_device.cuh"
#include "pq8_gemm.cuh"
#include "pq8_gemv.cuh"
#include "pq8_block.cuh"
#include "pq8_tdt.cuh"
#include "pq8_decode.cuh"
#include "pq8_attention.cuh"

namespace pq8 {

__device__ int g_status;  // device-side error word (PQ8_ERR_LAYOUT / PQ8_ERR_TIMEOUT)

namespace {

constexpr int kMaxDevices = 64;

struct DeviceState {
  bool ready = false;
  int sms = 0;
  int* status = nullptr;
  // cudaFuncSetAttribute done, per kernel: slots 0-6 the GEMM tile
  // configurations (GemmConfig), 8-11 the GEMV (MT = 1, 2, 4, 8), 13 the
  // attention, 14-15 the streaming GEMV (MT = 1, 2), 16 the GEMM sequence
  // kernel, 17 the GEMV batch kernel
  bool attr_set[24] = {};
  // GEMV launches with clusters of 9-16 CTAs: how many such clusters the GPU
  // holds at once, per (rows per group, splits, K blocks per split); guarded by g_mutex
  std::map<long long, int> gemv_cluster_fit;
  cublasHandle_t blas = nullptr;  // attention GEMMs; created on first use, guarded by blas_mutex
  std::mutex blas_mutex;
};

std::mutex g_mutex;
DeviceState g_dev[kMaxDevices];

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

int to_code(cudaError_t e) { return e == cudaSuccess ? PQ8_OK : static_cast<int>(e); }

// Current device's state; checks compute capability 10.0 on first use.
int device_state(DeviceState** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return to_code(e);
  if (dev < 0 || dev >= kMaxDevices) return PQ8_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_mutex);
  DeviceState& s = g_dev[dev];
  if (!s.ready) {
    int major = 0, minor = 0;
    if ((e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev)) != cudaSuccess) return to_code(e);
    if ((e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev)) != cudaSuccess) return to_code(e);
    if (major != 10 || minor != 0) return PQ8_ERR_ARCH;
    if ((e = cudaDeviceGetAttribute(&s.sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return to_code(e);
    void* sym = nullptr;
    if ((e = cudaGetSymbolAddress(&sym, g_status)) != cudaSuccess) return to_code(e);
    s.status = static_cast<int*>(sym);
    s.ready = true;
  }
  *out = &s;
  return PQ8_OK;
}

int encode_fn(EncodeTiledFn* fn) {
  std::call_once(g_encode_once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<EncodeTiledFn>(p);
  });
  *fn = g_encode;
  return g_encode ? PQ8_OK : PQ8_ERR_DRIVER;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---------------------------------------------------------------- GEMM
template <int BN, int STAGES, int ASLOTS, int ACC, bool PAIR, int GROUPS, int WSTAGES>
int launch_gemm(DeviceState* ds, int cfg_id, const float* x, GemmParams p, cudaStream_t st) {
  using C = GemmCfg<BN, STAGES, ASLOTS, ACC, PAIR, GROUPS, 4, 32, WSTAGES>;
  if (p.k_splits < 1) p.k_splits = 1;
  if (p.k_splits > 1 && (!C::kSplitK || (p.k_splits != 2 && p.k_splits != 4 && p.k_splits != 8)))
    return PQ8_ERR_INVALID_ARGUMENT;
  EncodeTiledFn enc;
  int rc = encode_fn(&enc);
  if (rc) return rc;
  CUtensorMap tmap;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(p.k), static_cast<cuuint64_t>(p.m)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(p.k) * sizeof(float)};
  const cuuint32_t box[2] = {32, static_cast<cuuint32_t>(C::kRowsPerCta)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult cr = enc(&tmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(x), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return PQ8_ERR_DRIVER;
  // Output tensor map for the staged epilogue: TMA needs a 16-byte-aligned base
  // and row stride; other outputs are written with plain stores.
  CUtensorMap tmap_y;
  std::memset(&tmap_y, 0, sizeof(tmap_y));
  p.tma_store = (p.out_cols % 4 == 0) && aligned(p.y, 16);
  if (p.tma_store) {
    const cuuint64_t ydims[2] = {static_cast<cuuint64_t>(p.out_cols), static_cast<cuuint64_t>(p.m)};
    const cuuint64_t ystrides[1] = {static_cast<cuuint64_t>(p.out_cols) * sizeof(float)};
    const cuuint32_t ybox[2] = {static_cast<cuuint32_t>(p.epi == PQ8_EPI_GLU ? 64 : 128), 32};
    cr = enc(&tmap_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, p.y, ydims, ystrides, ybox, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (cr != CUDA_SUCCESS) return PQ8_ERR_DRIVER;
  }
  auto kernel = gemm_tc_kernel<BN, STAGES, ASLOTS, ACC, PAIR, GROUPS, 4, 32, WSTAGES, false>;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!ds->attr_set[cfg_id]) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
      if (e != cudaSuccess) return to_code(e);
      ds->attr_set[cfg_id] = true;
    }
  }
  p.m_tiles = (p.m + BN - 1) / BN;
  const int units = (PAIR ? (p.n_tiles + 1) / 2 : p.n_tiles) * p.m_tiles * p.k_splits;
  const int slots = PAIR ? ds->sms / 2 : ds->sms;
  // a split CTA runs exactly one tile (it stages partials in the activation
  // ring); the splits of a tile are consecutive CTAs and form one cluster
  if (p.k_splits > 1 && units > slots) return PQ8_ERR_INVALID_ARGUMENT;
  const int grid = std::min(units, slots) * C::kCtas;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmemBytes;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.k_splits > 1 ? p.k_splits : C::kCtas;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  // Programmatic dependent launch: set-up, weight fetch and conversion overlap
  // the tail of the previous kernel in the stream (the kernel waits for it
  // before reading activations or writing outputs).
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, tmap, tmap_y, p, static_cast<const uint8_t*>(nullptr));
  if (e != cudaSuccess) return to_code(e);
  return to_code(cudaGetLastError());
}

// Launch with programmatic dependent launch allowed: the kernel may start
// while the previous kernel in the stream finishes (it calls griddep_wait
// before reading that kernel's results).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// GEMM configurations: activation rows per tile (the MMA N), single CTA or a
// pair of CTAs sharing one MMA, accumulator buffers.
enum GemmConfig { kG256 = 0, kG192, kG128, kG64, kP256, kP192, kP128, kNumGemmConfigs };
struct GemmShape {
  int bn, pair, acc;
  // Time model, in units of one 32-wide K block of the BN = 192 tile:
  // a launch takes waves * KB * t + (waves - 1) * e + f, where e is the
  // epilogue a single accumulator serialises with the next tile and f the
  // per-launch fixed cost (pipeline fill, last epilogue). Fitted to B200
  // measurements of the encoder shapes at M = 3000.
  double t, e, f;
};
constexpr GemmShape kGemmShapes[kNumGemmConfigs] = {
    {256, 0, 1, 1.31, 3.6, 20.6}, {192, 0, 2, 1.00, 0.0, 26.4}, {128, 0, 2, 0.86, 0.0, 26.4},
    {64, 0, 2, 0.80, 0.0, 26.4},  {256, 1, 1, 1.04, 7.3, 29.1}, {192, 1, 2, 1.02, 0.0, 26.4},
    {128, 1, 2, 0.88, 0.0, 26.4}};

// The configuration with the least modelled time is chosen.
// PQ8_GEMM_CONFIG=<index> or PQ8_GEMM_BN=64|128|192|256 (single CTA) in the
// environment force a configuration; the tests use this to cover all of them.
int choose_gemm(int m, int n_tiles, int kb, int sms) {
  if (const char* force = std::getenv("PQ8_GEMM_CONFIG")) {
    const int v = std::atoi(force);
    if (v >= 0 && v < kNumGemmConfigs) return v;
  }
  if (const char* force = std::getenv("PQ8_GEMM_BN")) {
    switch (std::atoi(force)) {
      case 256: return kG256;
      case 192: return kG192;
      case 128: return kG128;
      case 64: return kG64;
      default: break;
    }
  }
  int best = kG256;
  double best_cost = -1;
  for (int c = 0; c < kNumGemmConfigs; ++c) {
    const GemmShape g = kGemmShapes[c];
    const long units = static_cast<long>(g.pair ? (n_tiles + 1) / 2 : n_tiles) * ((m + g.bn - 1) / g.bn);
    const long slots = g.pair ? sms / 2 : sms;
    const long waves = (units + slots - 1) / slots;
    const double cost = waves * kb * g.t + (waves - 1) * g.e + g.f;
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = c;
    }
  }
  return best;
}

// ---------------------------------------------------------------- GEMV
// Workspace layout. The counters (split-K tickets, joint completion counts,
// joint arg-max keys) live in a fixed area at the start that no plan uses for
// anything else: they reset themselves after every launch, so a workspace
// zeroed once stays valid across calls of any shape. (If the counters followed
// each plan's own data regions, a plan with more tiles would find its tickets
// on bytes an earlier plan had left its partial sums in.) Tickets fill the
// area from the start; then come the arg-max keys (row groups x 8 rows x 2
// parts) and, in the last 256 bytes, one completion counter per row group.
constexpr size_t kGemvCounterBytes = size_t(64) << 10;
constexpr size_t kGemvDoneOffset = kGemvCounterBytes - 256;
constexpr size_t kGemvKeyOffset = kGemvDoneOffset - 1024;
constexpr int kGemvMaxTickets = static_cast<int>(kGemvKeyOffset / sizeof(int));
static_assert((PQ8_GEMV_MAX_M + 7) / 8 * sizeof(int) <= kGemvCounterBytes - kGemvDoneOffset,
              "one completion counter per row group");
static_assert((PQ8_GEMV_MAX_M + 7) / 8 * 8 * 2 * sizeof(unsigned long long) <= kGemvDoneOffset - kGemvKeyOffset,
              "arg-max keys of every row group");

struct GemvPlan {
  bool ok;                       // false: more split tiles than the counter area holds
  int mt, groups, splits, kbps;  // rows per CTA, row groups (grid y), K splits, K blocks per split
  bool stream;   // weights brought in by bulk copies (HBM regime: few rows, long K range per CTA)
  bool cluster;  // the K splits of a tile reduce through a thread-block cluster's shared memory
  size_t off_tickets, off_done, off_keys, off_partial, total;
};

size_t round256(size_t v) { return (v + 255) & ~size_t(255); }

GemvPlan plan_gemv(int m, int n, int k, int sms) {
  GemvPlan g{};
  g.mt = m <= 1 ? 1 : m <= 2 ? 2 : m <= 4 ? 4 : 8;
  g.groups = (m + g.mt - 1) / g.mt;
  const int n_tiles = (n + kTileRows - 1) / kTileRows;
  const int units = n_tiles * g.groups;  // CTAs per K split
  const int kb = k / 32;
  const int max_kbps = kGemvXSmemFloats / (32 * g.mt);
  int splits = 0, kbps = 0;
  if (g.mt == 1) {
    // One wave of two streaming CTAs per SM, if that leaves every CTA a long
    // run of K blocks to stream (measured: worth it for one row; with two the
    // per-CTA arithmetic, not the bytes in flight, sets the pace).
    int s = std::max(1, (2 * sms) / n_tiles);
    int b = std::min((kb + s - 1) / s, max_kbps);
    if (b >= 8) {
      g.stream = true;
      kbps = b;
      splits = (kb + b - 1) / b;
    }
  }
  if (!g.stream) {
    // Fill the CTA slots of one wave (kGemvCtasPerSm per SM) without a second
    // wave. Up to kGemvMaxClusterSplits splits reduce inside a cluster; a K
    // range longer than the activation staging area may need more splits,
    // which reduce through the workspace.
    const int want = std::max(1, std::min({kb, (kGemvCtasPerSm * sms) / units, kGemvMaxClusterSplits}));
    kbps = std::min((kb + want - 1) / want, max_kbps);
    splits = (kb + kbps - 1) / kbps;
    g.cluster = splits > 1 && splits <= kGemvMaxClusterSplits;
  }
  g.splits = splits;
  g.kbps = kbps;
  g.ok = splits == 1 || g.cluster || units <= kGemvMaxTickets;
  g.off_tickets = 0;
  g.off_done = kGemvDoneOffset;
  g.off_keys = kGemvKeyOffset;
  size_t off = kGemvCounterBytes;
  g.off_partial = off;
  off += (splits > 1 && !g.cluster) ? round256(sizeof(float) * (size_t)units * splits * kTileRows * g.mt) : 0;
  g.total = off;
  return g;
}

template <int MT>
int gemv_cluster_fit(DeviceState* ds, const GemvParams& p, const GemvPlan& g, int* fit) {
  auto kernel = gemv_kernel<MT, false>;
  const long long key = (static_cast<long long>(MT) << 40) | (static_cast<long long>(g.splits) << 20) | g.kbps;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    auto it = ds->gemv_cluster_fit.find(key);
    if (it != ds->gemv_cluster_fit.end()) {
      *fit = it->second;
      return PQ8_OK;
    }
  }
  const int max_smem = static_cast<int>(sizeof(float) * kGemvXSmemFloats + 128 +
                                        sizeof(float) * kGemvMaxClusterSplits * kGemvThreads * MT);
  // The query enqueues nothing; relaxed capture mode lets it run while the
  // caller's stream is being captured into a graph (a shape's first call).
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
  if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  int n = 0;
  if (e == cudaSuccess) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.n_tiles * g.splits, g.groups);
    cfg.blockDim = dim3(kGemvThreads);
    cfg.dynamicSmemBytes = ((sizeof(float) * MT * g.kbps * 32 + 127) & ~size_t(127)) +
                           sizeof(float) * g.splits * kGemvThreads * MT;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = g.splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
  }
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (e != cudaSuccess) {  // no answer: keep the plan as it is (not cached)
    cudaGetLastError();
    *fit = 1 << 30;
    return PQ8_OK;
  }
  std::lock_guard<std::mutex> lock(g_mutex);
  ds->gemv_cluster_fit[key] = n;
  *fit = n;
  return PQ8_OK;
}

// Reduces a plan's non-portable cluster split to at most 8 CTAs when the
// GPU cannot hold all of the launch's clusters at once.
int gemv_limit_cluster(DeviceState* ds, const GemvParams& p, GemvPlan& g) {
  int fit = 0;
  const int rc = g.mt == 1 ? gemv_cluster_fit<1>(ds, p, g, &fit)
               : g.mt == 2 ? gemv_cluster_fit<2>(ds, p, g, &fit)
               : g.mt == 4 ? gemv_cluster_fit<4>(ds, p, g, &fit)
                           : gemv_cluster_fit<8>(ds, p, g, &fit);
  if (rc) return rc;
  const int clusters = p.n_tiles * g.groups;
  const int kb = p.k / 32;
  const int kbps = (kb + 7) / 8;
  if (fit < clusters && kbps <= kGemvXSmemFloats / (32 * g.mt)) {
    g.kbps = kbps;
    g.splits = (kb + kbps - 1) / kbps;  // 2..8: still a cluster reduction
  }
  return PQ8_OK;
}

int launch_gemv(DeviceState* ds, GemvParams p, void* ws, size_t ws_bytes, cudaStream_t st) {
  GemvPlan g = plan_gemv(p.m, p.n, p.k, ds->sms);
  if (!g.ok) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (g.cluster && g.splits > 8) {
    // Clusters of more than 8 CTAs (a non-portable size) only help while the
    // GPU holds every cluster of the launch at once; otherwise the launch
    // takes the largest portable split instead (measured on B200 at M = 1,
    // N = 4096, K = 1024, 32 clusters of 16: 5.95 us, against 3.34 in 8
    // splits). The cluster reduction needs no workspace, so the plan's size
    // is unchanged.
    int rc = gemv_limit_cluster(ds, p, g);
    if (rc) return rc;
  }
  if (ws == nullptr || ws_bytes < g.total) return PQ8_ERR_WORKSPACE;
  if (!aligned(ws, 256)) return PQ8_ERR_MISALIGNED;
  auto* base = static_cast<unsigned char*>(ws);
  p.splits = g.splits;
  p.kb_per_split = g.kbps;
  p.tickets = reinterpret_cast<int*>(base + g.off_tickets);
  p.done_count = reinterpret_cast<int*>(base + g.off_done);
  p.best_key = reinterpret_cast<unsigned long long*>(base + g.off_keys);
  p.partial = reinterpret_cast<float*>(base + g.off_partial);
  p.status = ds->status;
  const dim3 grid(p.n_tiles * g.splits, g.groups);
  size_t smem = sizeof(float) * g.mt * g.kbps * 32;
  if (g.stream) {
    smem = ((smem + 127) & ~size_t(127)) + kStreamRingBytes;
    auto kernel = g.mt == 1 ? gemv_kernel<1, true> : gemv_kernel<2, true>;
    const int attr_id = g.mt == 1 ? 14 : 15;
    {
      std::lock_guard<std::mutex> lock(g_mutex);
      if (!ds->attr_set[attr_id]) {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sizeof(float) * 2 * kGemvXSmemFloats + 128 +
                                                              kStreamRingBytes));
        if (e != cudaSuccess) return to_code(e);
        ds->attr_set[attr_id] = true;
      }
    }
    cudaError_t e = launch_pdl(kernel, grid, dim3(kStreamThreads), smem, st, p);
    if (e != cudaSuccess) return to_code(e);
    return to_code(cudaGetLastError());
  }
  auto kernel = g.mt == 1 ? gemv_kernel<1, false>
              : g.mt == 2 ? gemv_kernel<2, false>
              : g.mt == 4 ? gemv_kernel<4, false>
                          : gemv_kernel<8, false>;
  const int attr_id = 8 + (g.mt == 1 ? 0 : g.mt == 2 ? 1 : g.mt == 4 ? 2 : 3);
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!ds->attr_set[attr_id]) {
      // staged activations plus the cluster reduction's partial sums
      const int max_smem = static_cast<int>(sizeof(float) * kGemvXSmemFloats + 128 +
                                            sizeof(float) * kGemvMaxClusterSplits * kGemvThreads * g.mt);
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, max_smem);
      if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
      if (e != cudaSuccess) return to_code(e);
      ds->attr_set[attr_id] = true;
    }
  }
  p.cluster_reduce = g.cluster;
  if (g.cluster) smem = ((smem + 127) & ~size_t(127)) + sizeof(float) * g.splits * kGemvThreads * g.mt;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kGemvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = g.cluster ? g.splits : 1;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g.cluster ? 2 : 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, p);
  if (e != cudaSuccess) return to_code(e);
  return to_code(cudaGetLastError());
}

// ---------------------------------------------------------------- dequant
__global__ void dequant_kernel(const uint8_t* __restrict__ src, float* __restrict__ out, long long blocks) {
  const long long b = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (b >= blocks) return;
  const uint8_t* rec = src + b * 34;
  const float s = __half2float(__ushort_as_half(static_cast<uint16_t>(rec[0] | (rec[1] << 8))));
  float* o = out + b * 32;
#pragma unroll
  for (int i = 0; i < 32; ++i) o[i] = s * static_cast<float>(static_cast<int8_t>(rec[2 + i]));
}

// GGUF Q8_0 bytes already on the device -> packed records (the layout of
// pq8_pack_q8_0_part, pq8_pack.cpp). One thread per packed row of a tile
// (128 per CTA), kRepackChunk K blocks per CTA: each block's 34 bytes are read
// as 2-byte words (a block is 2-byte aligned) and written as two 16-byte value
// stores and one scale store, so a warp writes 512 contiguous bytes per store.
// Padding rows get zeros. The first part (k_offset 0) writes the header; a
// later part checks it and records PQ8_ERR_LAYOUT in the status word if it
// does not match.
constexpr int kRepackChunk = 8;
__global__ void repack_q8_0_kernel(const uint16_t* __restrict__ raw, int n, int kb_src, int kb_total, int kb_off,
                                   int layout, uint8_t* __restrict__ packed, int* status) {
  const int t = blockIdx.y, r = threadIdx.x;
  RowMap rm;
  const bool valid = map_row(layout, n, t * kTileRows + r, rm);
  if (blockIdx.x == 0 && t == 0) {
    auto* h = reinterpret_cast<PackedHeader*>(packed);
    const int n_tiles = gridDim.y, out_cols = layout == PQ8_LAYOUT_GLU ? n / 2 : layout == PQ8_LAYOUT_GATES4 ? n / 4 : n;
    if (kb_off == 0) {
      uint32_t word = 0;
      switch (r) {
        case 0: word = kMagic; break;
        case 1: word = 1; break;
        case 2: word = static_cast<uint32_t>(n); break;
        case 3: word = static_cast<uint32_t>(kb_total * 32); break;
        case 4: word = static_cast<uint32_t>(layout); break;
        case 5: word = static_cast<uint32_t>(n_tiles); break;
        case 6: word = static_cast<uint32_t>(kb_total); break;
        case 7: word = static_cast<uint32_t>(out_cols); break;
        default: break;
      }
      if (r < PQ8_HEADER_BYTES / 4) reinterpret_cast<uint32_t*>(packed)[r] = word;
    } else if (r == 0 && !(h->magic == kMagic && h->n == n && h->k == kb_total * 32 && h->layout == layout)) {
      atomicCAS(status, 0, PQ8_ERR_LAYOUT);
    }
  }
  const uint16_t* row = raw + static_cast<size_t>(valid ? rm.src : 0) * kb_src * 17;
  uint8_t* data = packed + PQ8_HEADER_BYTES;
  const int kb_end = min(kb_src, (blockIdx.x + 1) * kRepackChunk);
  for (int kb = blockIdx.x * kRepackChunk; kb < kb_end; ++kb) {
    uint4 lo = make_uint4(0, 0, 0, 0), hi = make_uint4(0, 0, 0, 0);
    uint16_t sc = 0;
    if (valid) {
      const uint16_t* b = row + static_cast<size_t>(kb) * 17;
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = b[1 + i];
      sc = b[0];
      lo = make_uint4(w[0] | w[1] << 16, w[2] | w[3] << 16, w[4] | w[5] << 16, w[6] | w[7] << 16);
      hi = make_uint4(w[8] | w[9] << 16, w[10] | w[11] << 16, w[12] | w[13] << 16, w[14] | w[15] << 16);
    }
    uint8_t* rec = data + (static_cast<size_t>(t) * kb_total + kb_off + kb) * kRecordBytes;
    *reinterpret_cast<uint4*>(rec + r * 16) = lo;
    *reinterpret_cast<uint4*>(rec + 2048 + r * 16) = hi;
    *reinterpret_cast<uint16_t*>(rec + kScaleOffset + r * 2) = sc;
  }
}

__global__ void round_tf32_kernel(uint32_t* __restrict__ x, long long n) {
  const long long n4 = n >> 2;
  uint4* x4 = reinterpret_cast<uint4*>(x);
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    uint4 v = x4[i];
    v.x = tf32_round_bits(v.x);
    v.y = tf32_round_bits(v.y);
    v.z = tf32_round_bits(v.z);
    v.w = tf32_round_bits(v.w);
    x4[i] = v;
  }
  for (long long i = (n4 << 2) + blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
       i += (long long)gridDim.x * blockDim.x)
    x[i] = tf32_round_bits(x[i]);
}

// x rounded to TF32 (as the GEMM's converters would round it) into y: one
// streaming pass; n4 float4s, both 16-byte aligned. Launched with
// programmatic dependent launch: x may be the previous kernel's output, and
// the GEMM that reads y may start its set-up while this pass runs.
__global__ void round_tf32_copy_kernel(const uint4* __restrict__ x, uint4* __restrict__ y, long long n4) {
  griddep_launch();
  griddep_wait();
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n4; i += (long long)gridDim.x * blockDim.x) {
    uint4 v = x[i];
    v.x = tf32_round_bits(v.x);
    v.y = tf32_round_bits(v.y);
    v.z = tf32_round_bits(v.z);
    v.w = tf32_round_bits(v.w);
    y[i] = v;
  }
}

int check_linear_args(const void* w, const float* x, const float* y, const float* resid, int m, int n, int k,
                      int epi) {
  if (m < 0 || n < 1) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (k <= 0 || k % 32) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (epi < PQ8_EPI_NONE || epi > PQ8_EPI_RESIDUAL) return PQ8_ERR_INVALID_ARGUMENT;
  if (epi == PQ8_EPI_GLU && n % 2) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (m == 0) return PQ8_OK;
  if (w == nullptr || x == nullptr || y == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (epi == PQ8_EPI_RESIDUAL && resid == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(w, 16)) return PQ8_ERR_MISALIGNED;
  return PQ8_OK;
}

}  // namespace
}  // namespace pq8

using namespace pq8;

extern "C" const char* pq8_error_string(int code) {
  switch (code) {
    case PQ8_OK: return "PQ8_OK";
    case PQ8_ERR_INVALID_ARGUMENT: return "PQ8_ERR_INVALID_ARGUMENT: NULL pointer, negative size or unknown enum";
    case PQ8_ERR_UNSUPPORTED_SHAPE: return "PQ8_ERR_UNSUPPORTED_SHAPE: K must be a positive multiple of 32";
    case PQ8_ERR_MISALIGNED: return "PQ8_ERR_MISALIGNED: pointer alignment requirement not met";
    case PQ8_ERR_ARCH: return "PQ8_ERR_ARCH: current device is not sm_100 (B200)";
    case PQ8_ERR_WORKSPACE: return "PQ8_ERR_WORKSPACE: workspace missing or too small";
    case PQ8_ERR_LAYOUT: return "PQ8_ERR_LAYOUT: packed weight header does not match n/k/layout";
    case PQ8_ERR_TIMEOUT: return "PQ8_ERR_TIMEOUT: a bounded wait inside a kernel expired";
    case PQ8_ERR_DRIVER: return "PQ8_ERR_DRIVER: CUDA driver entry point unavailable or tensor map rejected";
    case PQ8_ERR_LIBRARY: return "PQ8_ERR_LIBRARY: a cuBLAS call of the attention failed";
    default:
      if (code > 0 && code < 1000) return cudaGetErrorString(static_cast<cudaError_t>(code));
      return "unknown pq8 error";
  }
}

extern "C" int pq8_version(void) { return 100; }

extern "C" int pq8_dequant_q8_0(const void* gguf_blocks, float* out, long long n_elements, void* stream) {
  if (n_elements < 0 || n_elements % 32) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (n_elements == 0) return PQ8_OK;
  if (gguf_blocks == nullptr || out == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  const long long blocks = n_elements / 32;
  const int threads = 256;
  const long long grid = (blocks + threads - 1) / threads;
  dequant_kernel<<<static_cast<unsigned>(grid), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(gguf_blocks), out, blocks);
  return to_code(cudaGetLastError());
}

extern "C" int pq8_pack_q8_0_part_device(const void* gguf_blocks, int n, int k_src, int k_total, int k_offset,
                                         int layout, void* packed, void* stream) {
  if (gguf_blocks == nullptr || packed == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  size_t total = 0;
  int rc = pq8_packed_size(n, k_total, layout, &total);
  if (rc) return rc;
  if (k_src <= 0 || k_src % 32 || k_offset < 0 || k_offset % 32 || k_offset + k_src > k_total)
    return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (!aligned(gguf_blocks, 2) || !aligned(packed, 16)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  if ((rc = device_state(&ds))) return rc;
  const int n_tiles = (n + kTileRows - 1) / kTileRows, kb_src = k_src / 32;
  if (n_tiles > 65535) return PQ8_ERR_UNSUPPORTED_SHAPE;
  const dim3 grid((kb_src + kRepackChunk - 1) / kRepackChunk, n_tiles);
  repack_q8_0_kernel<<<grid, kTileRows, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(gguf_blocks), n, kb_src, k_total / 32, k_offset / 32, layout,
      static_cast<uint8_t*>(packed), ds->status);
  return to_code(cudaGetLastError());
}

extern "C" int pq8_pack_q8_0_device(const void* gguf_blocks, int n, int k, int layout, void* packed, void* stream) {
  return pq8_pack_q8_0_part_device(gguf_blocks, n, k, k, 0, layout, packed, stream);
}

extern "C" int pq8_round_tf32(float* x, long long n, void* stream) {
  if (n < 0) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (n == 0) return PQ8_OK;
  if (x == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(x, 16)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  const long long blocks = std::min<long long>((n / 4 + 255) / 256 + 1, 8LL * ds->sms);
  round_tf32_kernel<<<static_cast<unsigned>(blocks), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<uint32_t*>(x), n);
  return to_code(cudaGetLastError());
}

namespace pq8 {
namespace {

// The tile configuration with the least modelled time for this shape.
int launch_chosen(DeviceState* ds, const float* x, const GemmParams& p, cudaStream_t st) {
  switch (choose_gemm(p.m, p.n_tiles, p.k_blocks, ds->sms)) {
    case kG256: return launch_gemm<256, 4, 4, 1, false, 2, 7>(ds, kG256, x, p, st);
    case kG192: return launch_gemm<192, 5, 4, 2, false, 2, 8>(ds, kG192, x, p, st);
    case kG128: return launch_gemm<128, 7, 4, 2, false, 2, 8>(ds, kG128, x, p, st);
    case kG64: return launch_gemm<64, 10, 4, 2, false, 2, 8>(ds, kG64, x, p, st);
    case kP256: return launch_gemm<256, 7, 4, 1, true, 2, 8>(ds, kP256, x, p, st);
    case kP192: return launch_gemm<192, 8, 4, 2, true, 2, 8>(ds, kP192, x, p, st);
    default: return launch_gemm<128, 10, 4, 2, true, 2, 8>(ds, kP128, x, p, st);
  }
}

// The tensor-core kernel on a dense row-major FP32 weight [n, k] (k a multiple
// of 32, 16-byte aligned rows): the converters round the weights to TF32
// (nearest-even) instead of expanding Q8_0 records. Used for the stem's
// pointwise convolutions, whose weights are FP32 in the model.
int gemm_dense_f32(DeviceState* ds, const float* w, const float* x, float* y, int m, int n, int k, int flags,
                   cudaStream_t st) {
  GemmParams p{};
  p.w = reinterpret_cast<const uint8_t*>(w);
  p.w_f32 = 1;
  p.y = y;
  p.status = ds->status;
  p.m = m;
  p.n = n;
  p.k = k;
  p.epi = PQ8_EPI_NONE;
  p.alpha = 1.0f;
  p.flags = flags;
  p.layout = PQ8_LAYOUT_ROWS;
  p.out_cols = n;
  p.n_tiles = (n + kTileRows - 1) / kTileRows;
  p.k_blocks = k / 32;
  return launch_chosen(ds, x, p, st);
}

}  // namespace
}  // namespace pq8

extern "C" int pq8_gemm(const void* w, const float* x, float* y, const float* bias, const float* resid, int m, int n,
                        int k, int epilogue, float alpha, int flags, void* stream) {
  int rc = check_linear_args(w, x, y, resid, m, n, k, epilogue);
  if (rc || m == 0) return rc;
  if (!aligned(x, 16)) return PQ8_ERR_MISALIGNED;
  if (flags & ~(PQ8_FLAG_X_TF32 | PQ8_FLAG_OUT_TF32)) return PQ8_ERR_INVALID_ARGUMENT;
  DeviceState* ds;
  if ((rc = device_state(&ds))) return rc;
  GemmParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.y = y;
  p.bias = bias;
  p.resid = resid;
  p.status = ds->status;
  p.m = m;
  p.n = n;
  p.k = k;
  p.epi = epilogue;
  p.alpha = alpha;
  p.flags = flags;
  p.layout = epilogue == PQ8_EPI_GLU ? PQ8_LAYOUT_GLU : PQ8_LAYOUT_ROWS;
  p.out_cols = epilogue == PQ8_EPI_GLU ? n / 2 : n;
  p.n_tiles = (n + kTileRows - 1) / kTileRows;
  p.k_blocks = k / 32;
  return launch_chosen(ds, x, p, static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- GEMM sequences
// Every tile of a sequence runs in the single-CTA BN = 192 configuration with
// two accumulators (the epilogue of one tile overlaps the next tile's MMAs).
namespace pq8 {
namespace {

constexpr int kSeqBN = 192, kSeqStages = 6, kSeqSlots = 4, kSeqAcc = 2, kSeqWStages = 4;
using SeqCfg = GemmCfg<kSeqBN, kSeqStages, kSeqSlots, kSeqAcc, false, 2, 4, 32, kSeqWStages>;
constexpr int kSeqCfgId = 16;  // DeviceState::attr_set slot of the sequence kernel
constexpr size_t kSeqHeaderBytes = sizeof(SeqPlanHeader);

struct SeqLayout {
  size_t tasks_offset, counters_offset, start_offset, order_offset, total;
  int n_counters, total_tiles;
};

int seq_layout(const pq8_gemm_task* tasks, int count, SeqLayout* out) {
  if (tasks == nullptr || count < 1) return PQ8_ERR_INVALID_ARGUMENT;
  long long counters = 0, tiles = 0;
  for (int i = 0; i < count; ++i) {
    const pq8_gemm_task& t = tasks[i];
    int rc = check_linear_args(t.w, t.x, t.y, t.resid, t.m, t.n, t.k, t.epilogue);
    if (rc) return rc;
    if (t.m < 1) return PQ8_ERR_UNSUPPORTED_SHAPE;
    if (!aligned(t.x, 16)) return PQ8_ERR_MISALIGNED;
    if (t.flags & ~(PQ8_FLAG_X_TF32 | PQ8_FLAG_OUT_TF32)) return PQ8_ERR_INVALID_ARGUMENT;
    if (t.after >= i || t.after < -1 || t.after_window < 0) return PQ8_ERR_INVALID_ARGUMENT;
    // one activation-rounding mode per sequence (the converters and the scheduler share it)
    if ((t.flags & PQ8_FLAG_X_TF32) != (tasks[0].flags & PQ8_FLAG_X_TF32)) return PQ8_ERR_INVALID_ARGUMENT;
    const long long m_tiles = (t.m + kSeqBN - 1) / kSeqBN, n_tiles = (t.n + kTileRows - 1) / kTileRows;
    counters += m_tiles;
    tiles += m_tiles * n_tiles;
  }
  if (tiles > (1LL << 30) || counters > (1LL << 30)) return PQ8_ERR_UNSUPPORTED_SHAPE;
  // a tile's task, weight tile, row block and K blocks travel as 16-bit fields
  if (count > 0xFFFF) return PQ8_ERR_UNSUPPORTED_SHAPE;
  for (int i = 0; i < count; ++i)
    if ((tasks[i].m + kSeqBN - 1) / kSeqBN > 0xFFFF || (tasks[i].n + kTileRows - 1) / kTileRows > 0xFFFF ||
        tasks[i].k / 32 > 0xFFFF)
      return PQ8_ERR_UNSUPPORTED_SHAPE;
  out->tasks_offset = kSeqHeaderBytes;
  out->counters_offset = round256(kSeqHeaderBytes + sizeof(SeqTask) * static_cast<size_t>(count));
  out->n_counters = static_cast<int>(counters);
  out->total_tiles = static_cast<int>(tiles);
  out->start_offset = round256(out->counters_offset + sizeof(int) * static_cast<size_t>(counters));
  out->order_offset = round256(out->start_offset + sizeof(int) * (kSeqMaxCtas + 1));
  out->total = round256(out->order_offset + sizeof(uint64_t) * static_cast<size_t>(tiles));
  return PQ8_OK;
}

// The tile schedule of a sequence: which CTA runs which tile, in what order.
// List scheduling over a model of the launch: the CTA the model frees first
// takes, among the next kLookahead tiles not yet taken (in plan order: task
// after task, N units fastest), the first whose activation rows the model
// has ready by then, else the one ready soonest; a tile is a candidate only
// once every tile it depends on has been taken. The order in which tiles are
// taken is therefore one in which each comes after every tile it depends on,
// and every CTA's list follows it. The model (per-tile times measured in the
// sequence kernel): a tile occupies its CTA's tensor pipe for
// (2 + 0.41 x K blocks) us, starting no earlier than 1 us
// after its activation rows' producer row blocks completed; a row block
// completes 3 us (the epilogue) after its last tile's mainloop, or after its
// output's dependencies. Against taking every gridDim-th tile it evens out
// CTAs that drew long-K tiles (FFN down projections: 128 K blocks against 32)
// and fills dependency waits with tiles that have none.
// PQ8_SEQUENCE_SCHEDULE=strided in the environment gives CTA c tiles c,
// c + ctas, ... of the plan order instead (for comparison).
void seq_schedule(const std::vector<SeqTask>& host, int ctas, std::vector<int>& start, std::vector<uint64_t>& order) {
  constexpr double kTileFixed = 2.0, kPerBlock = 0.41, kEpilogue = 3.0, kLoad = 1.0;
  constexpr int kLookahead = 64;
  int n_counters = 0;
  long long total = 0;
  for (const SeqTask& t : host) {
    n_counters = std::max(n_counters, t.counter + t.p.m_tiles);
    total += static_cast<long long>(t.p.m_tiles) * t.n_units;
  }
  std::vector<double> done(n_counters, 0.0);
  std::vector<int> left(n_counters, 0);  // tiles of each row block not yet taken
  for (const SeqTask& t : host)
    for (int m = 0; m < t.p.m_tiles; ++m) left[t.counter + m] = t.n_units;
  // Latest completion of the producer row blocks a dependency list needs for
  // row block m_tile, or -1 while any of their tiles has not been taken.
  auto ready = [&](const SeqDep* deps, int nd, int m_tile) {
    double r = 0.0;
    for (int d = 0; d < nd; ++d) {
      const SeqTask& prod = host[deps[d].task];
      int lo = m_tile, hi = m_tile;
      if (deps[d].window > 0) {
        const int w = deps[d].window, r0 = m_tile * kSeqBN, r1 = r0 + kSeqBN - 1;
        lo = (r0 / w) * w / kSeqBN;
        hi = ((r1 / w) * w + w - 1) / kSeqBN;
      }
      hi = std::min(hi, prod.p.m_tiles - 1);
      for (int row = lo; row <= hi; ++row) {
        if (left[prod.counter + row] > 0) return -1.0;
        r = std::max(r, done[prod.counter + row]);
      }
    }
    return r;
  };
  // tiles in plan order: (task, row block, weight tile)
  std::vector<uint64_t> tiles;
  tiles.reserve(static_cast<size_t>(total));
  for (size_t i = 0; i < host.size(); ++i)
    for (int m = 0; m < host[i].p.m_tiles; ++m)
      for (int n = 0; n < host[i].n_units; ++n)
        tiles.push_back((static_cast<uint64_t>(i) << 48) | (static_cast<uint64_t>(n) << 32) |
                        (static_cast<uint64_t>(m) << 16) | static_cast<uint64_t>(host[i].p.k_blocks));
  const char* mode = std::getenv("PQ8_SEQUENCE_SCHEDULE");
  const bool strided = mode != nullptr && std::strcmp(mode, "strided") == 0;
  std::vector<std::vector<uint64_t>> lists(ctas);
  std::vector<char> taken(tiles.size(), 0);
  std::vector<std::pair<double, int>> heap;  // (time the CTA's tensor pipe is free, CTA), min-heap
  for (int c = 0; c < ctas; ++c) heap.push_back({0.0, c});
  auto later = [](const std::pair<double, int>& a, const std::pair<double, int>& b) { return a > b; };
  std::make_heap(heap.begin(), heap.end(), later);
  size_t first = 0;  // lowest tile not yet taken
  for (size_t k = 0; k < tiles.size(); ++k) {
    std::pop_heap(heap.begin(), heap.end(), later);
    auto [free_at, c] = heap.back();
    while (taken[first]) ++first;
    size_t pick = first;
    double pick_ready = 0.0;
    if (strided) {
      c = static_cast<int>(k % ctas);
      pick_ready = std::max(0.0, ready(host[tiles[k] >> 48].x_dep, host[tiles[k] >> 48].n_x_deps,
                                       static_cast<int>((tiles[k] >> 16) & 0xFFFF)));
      pick = k;
    } else {
      pick_ready = -1.0;
      int seen = 0;
      for (size_t j = first; j < tiles.size() && seen < kLookahead; ++j) {
        if (taken[j]) continue;
        ++seen;
        const SeqTask& t = host[tiles[j] >> 48];
        const int m = static_cast<int>((tiles[j] >> 16) & 0xFFFF);
        const double xr = ready(t.x_dep, t.n_x_deps, m);
        if (xr < 0.0 || ready(t.out_dep, t.n_out_deps, m) < 0.0) continue;  // a dependency not taken yet
        if (xr + kLoad <= free_at) {
          pick = j;
          pick_ready = xr;
          break;
        }
        if (pick_ready < 0.0 || xr < pick_ready) {
          pick = j;
          pick_ready = xr;
        }
      }
      if (pick_ready < 0.0) pick_ready = 0.0;  // (the first tile not taken always qualifies)
    }
    const uint64_t e = tiles[pick];
    const SeqTask& t = host[e >> 48];
    const int m = static_cast<int>((e >> 16) & 0xFFFF);
    const double end = std::max(free_at, pick_ready + kLoad) + kTileFixed + kPerBlock * t.p.k_blocks;
    const double out_ready = std::max(0.0, ready(t.out_dep, t.n_out_deps, m));
    heap.back() = {end, c};
    std::push_heap(heap.begin(), heap.end(), later);
    done[t.counter + m] = std::max(done[t.counter + m], std::max(end, out_ready) + kEpilogue);
    --left[t.counter + m];
    taken[pick] = 1;
    lists[c].push_back(e);
  }
  start.assign(ctas + 1, 0);
  order.clear();
  for (int c = 0; c < ctas; ++c) {
    start[c] = static_cast<int>(order.size());
    order.insert(order.end(), lists[c].begin(), lists[c].end());
  }
  start[ctas] = static_cast<int>(order.size());
}

// A buffer as the sequence sees it: rows of `width` floats starting at `base`.
struct Region {
  uintptr_t base;
  size_t bytes;
  int width;
};
bool overlaps(const Region& a, const Region& b) { return a.base < b.base + b.bytes && b.base < a.base + a.bytes; }

int add_dep(SeqDep* deps, int* n, int task, int window) {
  for (int i = 0; i < *n; ++i)
    if (deps[i].task == task && deps[i].window == window) return PQ8_OK;
  if (*n == kSeqMaxDeps) return PQ8_ERR_UNSUPPORTED_SHAPE;
  deps[(*n)++] = SeqDep{task, window};
  return PQ8_OK;
}

// Dependencies from the buffers each task reads (x, resid) and writes (y).
// A region is identified by its base address and row width; regions that
// overlap without being the same rows are refused (row blocks would not line
// up). For each region the last writer and the readers since are tracked:
// a reader depends on the last writer (read-after-write), a writer on the
// last writer (write-after-write) and on every reader since (write-after-read).
int seq_dependencies(const pq8_gemm_task* tasks, int count, std::vector<SeqTask>& out) {
  struct State {
    Region r;
    int writer;
    std::vector<int> readers;
  };
  std::vector<State> regions;
  auto find = [&](const Region& r, int* idx) -> int {
    for (size_t i = 0; i < regions.size(); ++i) {
      if (!overlaps(regions[i].r, r)) continue;
      if (regions[i].r.base != r.base || regions[i].r.width != r.width) return PQ8_ERR_UNSUPPORTED_SHAPE;
      if (r.bytes > regions[i].r.bytes) regions[i].r.bytes = r.bytes;
      *idx = static_cast<int>(i);
      return PQ8_OK;
    }
    regions.push_back(State{r, -1, {}});
    *idx = static_cast<int>(regions.size()) - 1;
    return PQ8_OK;
  };
  for (int j = 0; j < count; ++j) {
    const pq8_gemm_task& t = tasks[j];
    SeqTask& st = out[j];
    const int out_cols = t.epilogue == PQ8_EPI_GLU ? t.n / 2 : t.n;
    const Region rx{reinterpret_cast<uintptr_t>(t.x), sizeof(float) * (size_t)t.m * t.k, t.k};
    const Region ry{reinterpret_cast<uintptr_t>(t.y), sizeof(float) * (size_t)t.m * out_cols, out_cols};
    int ix, iy, ir = -1, rc;
    if ((rc = find(rx, &ix))) return rc;
    if ((rc = find(ry, &iy))) return rc;
    if (t.epilogue == PQ8_EPI_RESIDUAL) {
      const Region rr{reinterpret_cast<uintptr_t>(t.resid), ry.bytes, out_cols};
      if ((rc = find(rr, &ir))) return rc;
    }
    if (ix == iy) return PQ8_ERR_UNSUPPORTED_SHAPE;  // a GEMM cannot overwrite its own input rows
    if (regions[ix].writer >= 0 && (rc = add_dep(st.x_dep, &st.n_x_deps, regions[ix].writer, 0))) return rc;
    if (t.after >= 0 && (rc = add_dep(st.x_dep, &st.n_x_deps, t.after, t.after_window))) return rc;
    if (ir >= 0 && regions[ir].writer >= 0 && (rc = add_dep(st.out_dep, &st.n_out_deps, regions[ir].writer, 0)))
      return rc;
    if (regions[iy].writer >= 0 && (rc = add_dep(st.out_dep, &st.n_out_deps, regions[iy].writer, 0))) return rc;
    for (int rd : regions[iy].readers)
      if (rd != j && (rc = add_dep(st.out_dep, &st.n_out_deps, rd, 0))) return rc;
    regions[ix].readers.push_back(j);
    if (ir >= 0 && ir != iy) regions[ir].readers.push_back(j);
    regions[iy].writer = j;
    regions[iy].readers.clear();
  }
  return PQ8_OK;
}

}  // namespace
}  // namespace pq8

extern "C" int pq8_sequence_plan_size(const pq8_gemm_task* tasks, int count, size_t* bytes) {
  if (bytes == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  SeqLayout L;
  int rc = seq_layout(tasks, count, &L);
  if (rc) return rc;
  *bytes = L.total;
  return PQ8_OK;
}

extern "C" int pq8_sequence_plan(const pq8_gemm_task* tasks, int count, void* plan, size_t plan_bytes,
                                 void* stream) {
  SeqLayout L;
  int rc = seq_layout(tasks, count, &L);
  if (rc) return rc;
  if (plan == nullptr || plan_bytes < L.total) return PQ8_ERR_WORKSPACE;
  if (!aligned(plan, 256)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  if ((rc = device_state(&ds))) return rc;
  EncodeTiledFn enc;
  if ((rc = encode_fn(&enc))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  std::vector<SeqTask> host(count);
  std::memset(host.data(), 0, sizeof(SeqTask) * host.size());
  if ((rc = seq_dependencies(tasks, count, host))) return rc;
  int counter = 0;
  for (int i = 0; i < count; ++i) {
    const pq8_gemm_task& t = tasks[i];
    SeqTask& q = host[i];
    // the packed header must describe this task's weight (checked here, not per tile)
    PackedHeader h;
    cudaError_t e = cudaMemcpy(&h, t.w, sizeof(h), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return to_code(e);
    const int layout = t.epilogue == PQ8_EPI_GLU ? PQ8_LAYOUT_GLU : PQ8_LAYOUT_ROWS;
    const int n_tiles = (t.n + kTileRows - 1) / kTileRows;
    if (h.magic != kMagic || h.n != t.n || h.k != t.k || h.layout != layout || h.n_tiles != n_tiles)
      return PQ8_ERR_LAYOUT;
    GemmParams& p = q.p;
    p.w = static_cast<const uint8_t*>(t.w);
    p.y = t.y;
    p.bias = t.bias;
    p.resid = t.resid;
    p.status = ds->status;
    p.m = t.m;
    p.n = t.n;
    p.k = t.k;
    p.epi = t.epilogue;
    p.alpha = t.alpha;
    p.flags = t.flags;
    p.layout = layout;
    p.out_cols = t.epilogue == PQ8_EPI_GLU ? t.n / 2 : t.n;
    p.n_tiles = n_tiles;
    p.k_blocks = t.k / 32;
    p.m_tiles = (t.m + kSeqBN - 1) / kSeqBN;
    p.k_splits = 1;
    p.tma_store = (p.out_cols % 4 == 0) && aligned(t.y, 16);
    q.n_units = n_tiles;
    q.counter = counter;
    counter += p.m_tiles;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(t.k), static_cast<cuuint64_t>(t.m)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(t.k) * sizeof(float)};
    const cuuint32_t box[2] = {32, static_cast<cuuint32_t>(kSeqBN)};
    const cuuint32_t estr[2] = {1, 1};
    if (enc(&q.tmap_x, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(t.x), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return PQ8_ERR_DRIVER;
    if (p.tma_store) {
      const cuuint64_t ydims[2] = {static_cast<cuuint64_t>(p.out_cols), static_cast<cuuint64_t>(t.m)};
      const cuuint64_t ystrides[1] = {static_cast<cuuint64_t>(p.out_cols) * sizeof(float)};
      const cuuint32_t ybox[2] = {static_cast<cuuint32_t>(t.epilogue == PQ8_EPI_GLU ? 64 : 128), 32};
      if (enc(&q.tmap_y, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, t.y, ydims, ystrides, ybox, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
        return PQ8_ERR_DRIVER;
    }
  }
  if (ds->sms > kSeqMaxCtas) return PQ8_ERR_UNSUPPORTED_SHAPE;
  std::vector<int> start;
  std::vector<uint64_t> order;
  seq_schedule(host, ds->sms, start, order);
  std::vector<uint8_t> blob(L.total, 0);
  SeqPlanHeader hdr{};
  hdr.magic = kSeqMagic;
  hdr.count = count;
  hdr.total_tiles = L.total_tiles;
  hdr.n_counters = L.n_counters;
  hdr.bn = kSeqBN;
  hdr.finished = 0;
  hdr.tasks_offset = static_cast<long long>(L.tasks_offset);
  hdr.counters_offset = static_cast<long long>(L.counters_offset);
  hdr.ctas = ds->sms;
  hdr.start_offset = static_cast<long long>(L.start_offset);
  hdr.order_offset = static_cast<long long>(L.order_offset);
  std::memcpy(blob.data(), &hdr, sizeof(hdr));
  std::memcpy(blob.data() + L.tasks_offset, host.data(), sizeof(SeqTask) * host.size());
  std::memcpy(blob.data() + L.start_offset, start.data(), sizeof(int) * start.size());
  std::memcpy(blob.data() + L.order_offset, order.data(), sizeof(uint64_t) * order.size());
  cudaError_t e = cudaMemcpyAsync(plan, blob.data(), blob.size(), cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  return to_code(e);
}

extern "C" int pq8_sequence_run(const void* plan, void* stream) {
  if (plan == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(plan, 256)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  auto kernel = gemm_tc_kernel<kSeqBN, kSeqStages, kSeqSlots, kSeqAcc, false, 2, 4, 32, kSeqWStages, true>;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!ds->attr_set[kSeqCfgId]) {
      cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SeqCfg::kSmemBytes);
      if (e != cudaSuccess) return to_code(e);
      ds->attr_set[kSeqCfgId] = true;
    }
  }
  CUtensorMap unused;
  std::memset(&unused, 0, sizeof(unused));
  GemmParams p{};
  p.status = ds->status;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(ds->sms);  // one persistent CTA per SM; all must be resident (dependencies span CTAs)
  cfg.blockDim = dim3(SeqCfg::kThreads);
  cfg.dynamicSmemBytes = SeqCfg::kSmemBytes;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, unused, unused, p, static_cast<const uint8_t*>(plan));
  if (e != cudaSuccess) return to_code(e);
  return to_code(cudaGetLastError());
}

extern "C" int pq8_gemv_workspace_size(int m, int n, int k, size_t* bytes) {
  if (bytes == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (m < 1 || m > PQ8_GEMV_MAX_M || n < 1 || k <= 0 || k % 32) return PQ8_ERR_UNSUPPORTED_SHAPE;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  const GemvPlan g = plan_gemv(m, n, k, ds->sms);
  if (!g.ok) return PQ8_ERR_UNSUPPORTED_SHAPE;
  *bytes = g.total;
  return PQ8_OK;
}

extern "C" int pq8_workspace_init(void* workspace, size_t bytes, void* stream) {
  if (workspace == nullptr && bytes) return PQ8_ERR_INVALID_ARGUMENT;
  if (!bytes) return PQ8_OK;
  return to_code(cudaMemsetAsync(workspace, 0, bytes, static_cast<cudaStream_t>(stream)));
}

extern "C" int pq8_gemv(const void* w, const float* x, float* y, const float* bias, const float* resid, int m, int n,
                        int k, int epilogue, float alpha, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_linear_args(w, x, y, resid, m, n, k, epilogue);
  if (rc || m == 0) return rc;
  if (m > PQ8_GEMV_MAX_M) return PQ8_ERR_UNSUPPORTED_SHAPE;
  DeviceState* ds;
  if ((rc = device_state(&ds))) return rc;
  GemvParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.x0 = x;
  p.x_mode = kXPlain;
  p.x_vec4 = aligned(x, 16);
  p.y = y;
  p.bias = bias;
  p.resid = resid;
  p.alpha = alpha;
  p.epi = epilogue;
  p.m = m;
  p.n = n;
  p.k = k;
  p.layout = epilogue == PQ8_EPI_GLU ? PQ8_LAYOUT_GLU : PQ8_LAYOUT_ROWS;
  p.out_cols = epilogue == PQ8_EPI_GLU ? n / 2 : n;
  p.n_tiles = (n + kTileRows - 1) / kTileRows;
  p.k_blocks = k / 32;
  p.mode = kGemvLinear;
  return launch_gemv(ds, p, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

namespace pq8 {
namespace {

// Split K for pq8_linear's GEMM path: when BN = 128 tiles would fill at most
// half of the SMs, each tile's K blocks are shared by S = 2, 4 or 8 CTAs (S x
// tiles within the SM count, at least 4 K blocks each) launched as clusters
// of S, which exchange their partial sums through shared memory (no
// workspace). Measured on B200: a lone tile's pipeline runs ~0.4 us per K
// block and the exchange costs ~4 us, so a split must take at least 16 K
// blocks off each CTA (config 0, 128 x 4096 x 1024: 16.8 -> 14.3 us in 4
// splits; 128 x 1024 x 4096: 54 -> 17.6 us in 8; 256 x 4096 x 1024: 18.0 ->
// 17.0 us in 2; K = 640 in 2 splits would lose 0.8-1.6 us).
// PQ8_LINEAR_SPLITS=<S> forces S (rounded down to a power of two, within the
// same limits; 1 turns split K off).
int plan_split(int m, int n, int k, int sms, bool allow_force = true) {
  const long long units = static_cast<long long>((m + 127) / 128) * ((n + kTileRows - 1) / kTileRows);
  const int kb = k / 32;
  long long s = units * 2 > sms ? 1 : std::min<long long>({sms / units, kb / 4, 8});
  const char* force = allow_force ? std::getenv("PQ8_LINEAR_SPLITS") : nullptr;
  if (force) s = std::min<long long>({std::max(1, std::atoi(force)), sms / units, kb / 2, 8});
  int p2 = 1;
  while (p2 * 2 <= s) p2 *= 2;
  while (!force && p2 > 1 && kb - (kb + p2 - 1) / p2 < 16) p2 /= 2;
  // every split gets K blocks: splits of ceil(kb / S) blocks, the last one shorter
  while (p2 > 1 && (p2 - 1) * ((kb + p2 - 1) / p2) >= kb) p2 /= 2;
  return p2;
}

// pq8_linear's choice for PQ8_LINEAR_GEMV_MAX_M < m <= PQ8_GEMV_MAX_M, from
// B200 measurements of both kernels at 9-64 rows (N 1024-8197, K 640-4096,
// CUDA graphs of back-to-back calls, weights streamed from HBM): the GEMV
// costs ~4 us plus ~0.1 ns per multiply-add of its 8-row groups (FP32 FMA),
// twice that per multiply-add at K = 4096 (its K splits run long); the GEMM
// ~3.3 us plus ~0.4 us per 32-wide K block unsplit (one wave of tiles at
// these sizes), or ~9.5 us plus ~0.42 us per K block of one split when
// plan_split shares the K blocks among a cluster. Within ~1.3 us of the
// faster kernel at every measured point.
bool gemv_faster(int m, int n, int k, int sms) {
  const int kb = k / 32;
  const double macs = static_cast<double>((m + 7) / 8 * 8) * n * k;
  const double gemv = 4.0 + 1.0e-7 * macs * (1.0 + std::max(0, kb - 32) / 96.0);
  const int s = plan_split(m, n, k, sms, false);  // the policy's splits (PQ8_LINEAR_SPLITS does not steer this)
  const double gemm = s > 1 ? 9.5 + 0.42 * ((kb + s - 1) / s) : 3.3 + 0.4 * kb;
  return gemv < gemm;
}

}  // namespace
}  // namespace pq8

namespace pq8 {
namespace {
// Raw (not yet TF32-rounded) activations of at least this many rows are
// rounded once into pq8_linear's workspace before the GEMM instead of by
// every CTA's converter warps, which are the mainloop's bottleneck. Measured
// on B200 (graph replay): M = 3000, N = 4096, K = 1024 takes 82 us rounding
// in the GEMM against 48 us on rounded input; 3000 x 1024 x 4096 105 against
// 50 us; 441 x 1024 x 4096 25.6 against 20.6 us; config 0 (M = 128) 14.2
// against 12.8 us, about what a separate pass costs there.
constexpr int kPreRoundRows = 256;
size_t preround_bytes(int m, int k) {
  return m >= kPreRoundRows ? kGemvCounterBytes + round256(sizeof(float) * static_cast<size_t>(m) * k) : 0;
}
}  // namespace
}  // namespace pq8

extern "C" int pq8_linear(const void* w, const float* x, float* y, const float* bias, const float* resid, int m,
                          int n, int k, int epilogue, float alpha, int flags, void* workspace, size_t workspace_bytes,
                          void* stream) {
  if (m >= 1 && m <= PQ8_GEMV_MAX_M && k > 0 && k % 32 == 0 && n >= 1) {
    bool gemv = m <= PQ8_LINEAR_GEMV_MAX_M;
    if (!gemv) {
      DeviceState* ds;
      int rc = device_state(&ds);
      if (rc) return rc;
      gemv = gemv_faster(m, n, k, ds->sms);
    }
    if (gemv) return pq8_gemv(w, x, y, bias, resid, m, n, k, epilogue, alpha, workspace, workspace_bytes, stream);
  } else if (m >= 1 && m <= PQ8_LINEAR_GEMV_MAX_M) {
    return pq8_gemv(w, x, y, bias, resid, m, n, k, epilogue, alpha, workspace, workspace_bytes, stream);
  }
  if (m >= 1 && k > 0 && k % 32 == 0 && n >= 1) {
    DeviceState* ds;
    int rc = device_state(&ds);
    if (rc) return rc;
    if ((rc = check_linear_args(w, x, y, resid, m, n, k, epilogue))) return rc;
    if (!aligned(x, 16)) return PQ8_ERR_MISALIGNED;
    if (flags & ~(PQ8_FLAG_X_TF32 | PQ8_FLAG_OUT_TF32)) return PQ8_ERR_INVALID_ARGUMENT;
    const size_t pre = preround_bytes(m, k);
    if (!(flags & PQ8_FLAG_X_TF32) && pre > 0 && workspace != nullptr && workspace_bytes >= pre &&
        aligned(workspace, 256)) {
      // the activations, rounded once into the workspace (after its counter area)
      float* xr = reinterpret_cast<float*>(static_cast<unsigned char*>(workspace) + kGemvCounterBytes);
      const long long n4 = static_cast<long long>(m) * k / 4;
      const long long blocks = std::min<long long>((n4 + 255) / 256, 8LL * ds->sms);
      cudaError_t e = launch_pdl(round_tf32_copy_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0,
                                 static_cast<cudaStream_t>(stream), reinterpret_cast<const uint4*>(x),
                                 reinterpret_cast<uint4*>(xr), n4);
      if (e != cudaSuccess) return to_code(e);
      x = xr;
      flags |= PQ8_FLAG_X_TF32;
    }
    const int splits = plan_split(m, n, k, ds->sms);
    if (splits > 1) {
      GemmParams p{};
      p.w = static_cast<const uint8_t*>(w);
      p.y = y;
      p.bias = bias;
      p.resid = resid;
      p.status = ds->status;
      p.m = m;
      p.n = n;
      p.k = k;
      p.epi = epilogue;
      p.alpha = alpha;
      p.flags = flags;
      p.layout = epilogue == PQ8_EPI_GLU ? PQ8_LAYOUT_GLU : PQ8_LAYOUT_ROWS;
      p.out_cols = epilogue == PQ8_EPI_GLU ? n / 2 : n;
      p.n_tiles = (n + kTileRows - 1) / kTileRows;
      p.k_blocks = k / 32;
      p.k_splits = splits;
      return launch_gemm<128, 7, 4, 2, false, 2, 8>(ds, kG128, x, p, static_cast<cudaStream_t>(stream));
    }
  }
  return pq8_gemm(w, x, y, bias, resid, m, n, k, epilogue, alpha, flags, stream);
}

extern "C" int pq8_linear_workspace_size(int m, int n, int k, size_t* bytes) {
  if (bytes == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (m < 0 || n < 1 || k <= 0 || k % 32) return PQ8_ERR_UNSUPPORTED_SHAPE;
  *bytes = 0;
  if (m == 0) return PQ8_OK;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  if (m <= PQ8_GEMV_MAX_M) {
    const GemvPlan g = plan_gemv(m, n, k, ds->sms);
    if (g.ok) *bytes = g.total;
  }
  *bytes = std::max(*bytes, preround_bytes(m, k));  // raw activations rounded once (large M)
  return PQ8_OK;
}

extern "C" int pq8_lstm_layer(const void* w, const float* x, const uint16_t* embed_f16, const int* tokens,
                              const float* h, const float* c, const float* bias, float* h_out, float* c_out, int m,
                              int hidden, int in_k, void* workspace, size_t workspace_bytes, void* stream) {
  if (m < 1 || m > PQ8_GEMV_MAX_M || hidden < 1 || in_k <= 0 || in_k % 32 || hidden % 32)
    return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (w == nullptr || h == nullptr || c == nullptr || h_out == nullptr || c_out == nullptr)
    return PQ8_ERR_INVALID_ARGUMENT;
  if (embed_f16 == nullptr ? x == nullptr : tokens == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (h_out == h || c_out == c) return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(w, 16)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  GemvParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.x0 = x;
  p.x1 = h;
  p.embed = embed_f16;
  p.tokens = tokens;
  p.x_mode = embed_f16 ? kXEmbedConcat : kXConcat;
  p.x_vec4 = (embed_f16 ? aligned(embed_f16, 8) : aligned(x, 16)) && aligned(h, 16);
  p.k0 = in_k;
  p.bias = bias;
  p.m = m;
  p.n = 4 * hidden;
  p.k = in_k + hidden;
  p.layout = PQ8_LAYOUT_GATES4;
  p.out_cols = hidden;
  p.n_tiles = (p.n + kTileRows - 1) / kTileRows;
  p.k_blocks = p.k / 32;
  p.c_prev = c;
  p.h_out = h_out;
  p.c_out = c_out;
  p.hidden = hidden;
  p.mode = kGemvLstm;
  return launch_gemv(ds, p, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int pq8_joint_argmax(const void* w, const float* enc, const int* enc_rows, const float* pred,
                                const float* bias, float* logits, int* ids, int m, int n, int k, int vocab,
                                void* workspace, size_t workspace_bytes, void* stream) {
  if (m < 1 || m > PQ8_GEMV_MAX_M || n < 2 || k <= 0 || k % 32 || vocab < 1 || vocab >= n)
    return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (w == nullptr || enc == nullptr || pred == nullptr || ids == nullptr)
    return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(w, 16)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  GemvParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.x0 = enc;
  p.x0_rows = enc_rows;
  p.x1 = pred;
  p.x_mode = kXReluSum;
  p.x_vec4 = aligned(enc, 16) && aligned(pred, 16);
  p.y = logits;
  p.bias = bias;
  p.m = m;
  p.n = n;
  p.k = k;
  p.layout = PQ8_LAYOUT_ROWS;
  p.out_cols = n;
  p.n_tiles = (n + kTileRows - 1) / kTileRows;
  p.k_blocks = k / 32;
  p.ids = ids;
  p.vocab = vocab;
  p.mode = kGemvJoint;
  return launch_gemv(ds, p, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

extern "C" int pq8_tdt_commit(float* h, float* c, const float* h_new, const float* c_new, const int* mask, int m,
                              int layers, int hidden, void* stream) {
  if (m < 0 || layers < 1 || hidden < 1) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (m == 0) return PQ8_OK;
  if (h == nullptr || c == nullptr || h_new == nullptr || c_new == nullptr || mask == nullptr)
    return PQ8_ERR_INVALID_ARGUMENT;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  const long long total = (long long)layers * m * hidden;
  const int grid = (int)std::min<long long>((total + 255) / 256, 4LL * ds->sms);
  cudaError_t e = launch_pdl(tdt_commit_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), h, c,
                             h_new, c_new, mask, m, layers, hidden);
  if (e != cudaSuccess) return to_code(e);
  return to_code(cudaGetLastError());
}

extern "C" int pq8_tdt_control(const int* ids, const int* durations, int n_durations, int* state, int m,
                               int enc_stride, int* tokens, int* enc_rows, int* commit_mask, int* emitted,
                               int emitted_capacity, int* trace, int trace_capacity, int* remaining, void* stream) {
  if (m < 1 || m > 1024 || n_durations < 1 || enc_stride < 0 || emitted_capacity < 0 || trace_capacity < 0)
    return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (ids == nullptr || durations == nullptr || state == nullptr || tokens == nullptr || enc_rows == nullptr ||
      commit_mask == nullptr || remaining == nullptr || (emitted_capacity > 0 && emitted == nullptr) ||
      (trace_capacity > 0 && trace == nullptr))
    return PQ8_ERR_INVALID_ARGUMENT;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  const int threads = (m + 31) / 32 * 32;
  cudaError_t e = launch_pdl(tdt_control_kernel, dim3(1), dim3(threads), 0, static_cast<cudaStream_t>(stream), ids,
                             durations, n_durations, state, m, enc_stride, tokens, enc_rows, commit_mask, emitted,
                             emitted_capacity, trace, trace_capacity, remaining, ds->status);
  if (e != cudaSuccess) return to_code(e);
  return to_code(cudaGetLastError());
}

extern "C" int pq8_tdt_advance(const int* ids, const int* durations, int n_durations, int* state, int m,
                               int enc_stride, int* tokens, int* enc_rows, int* commit_mask, int* emitted,
                               int emitted_capacity, int* trace, int trace_capacity, int* remaining, float* h,
                               float* c, const float* h_new, const float* c_new, int layers, int hidden,
                               void* stream) {
  if (m < 1 || m > 1024 || n_durations < 1 || enc_stride < 0 || emitted_capacity < 0 || trace_capacity < 0 ||
      layers < 1 || hidden < 4 || hidden % 4)
    return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (ids == nullptr || durations == nullptr || state == nullptr || tokens == nullptr || enc_rows == nullptr ||
      commit_mask == nullptr || remaining == nullptr || (emitted_capacity > 0 && emitted == nullptr) ||
      (trace_capacity > 0 && trace == nullptr) || h == nullptr || c == nullptr || h_new == nullptr ||
      c_new == nullptr)
    return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(h, 16) || !aligned(c, 16) || !aligned(h_new, 16) || !aligned(c_new, 16)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  const long long vecs = (long long)layers * m * (hidden / 4);
  const int grid = (int)std::max<long long>(1, std::min<long long>((vecs + 255) / 256, ds->sms));
  cudaError_t e = launch_pdl(tdt_advance_kernel, dim3(grid), dim3(256), 0, static_cast<cudaStream_t>(stream), ids,
                             durations, n_durations, state, m, enc_stride, tokens, enc_rows, commit_mask, emitted,
                             emitted_capacity, trace, trace_capacity, remaining, h, c, h_new, c_new, layers, hidden,
                             ds->status);
  if (e != cudaSuccess) return to_code(e);
  return to_code(cudaGetLastError());
}

// ---------------------------------------------------------------- GEMV batch
namespace {

constexpr int kBatchKbPerCta = 32;             // K blocks one CTA streams (~139 KB of records)
constexpr uint32_t kBatchMagic = 0x42385150u;  // "PQ8B"
static_assert(sizeof(BatchPlanHeader) == 16, "plan header");
static_assert(sizeof(GemvTask) % 16 == 0, "task table entries stay 16-byte aligned");

struct BatchTaskShape {
  int n_tiles, kb, splits, kbps;
  size_t ws_bytes;
};
BatchTaskShape batch_task_shape(int n, int k) {
  BatchTaskShape b{};
  b.n_tiles = (n + kTileRows - 1) / kTileRows;
  b.kb = k / 32;
  b.splits = (b.kb + kBatchKbPerCta - 1) / kBatchKbPerCta;
  b.kbps = (b.kb + b.splits - 1) / b.splits;
  b.ws_bytes = round256(sizeof(int) * b.n_tiles) +
               (b.splits > 1 ? round256(sizeof(float) * (size_t)b.n_tiles * b.splits * kGemvThreads) : 0);
  return b;
}

int check_batch_task(const pq8_gemv_task& t) {
  if (t.w == nullptr || t.x == nullptr || t.y == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (t.n < 1 || t.k <= 0 || t.k % 32) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (t.epilogue < PQ8_EPI_NONE || t.epilogue > PQ8_EPI_RESIDUAL) return PQ8_ERR_INVALID_ARGUMENT;
  if (t.epilogue == PQ8_EPI_GLU && t.n % 2) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (t.epilogue == PQ8_EPI_RESIDUAL && t.resid == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(t.w, 16) || !aligned(t.x, 16)) return PQ8_ERR_MISALIGNED;
  return PQ8_OK;
}

}  // namespace

extern "C" int pq8_gemv_batch_sizes(const pq8_gemv_task* tasks, int count, size_t* plan_bytes,
                                    size_t* workspace_bytes) {
  if (tasks == nullptr || count < 1 || plan_bytes == nullptr || workspace_bytes == nullptr)
    return PQ8_ERR_INVALID_ARGUMENT;
  size_t ws = 0;
  for (int i = 0; i < count; ++i) {
    const int rc = check_batch_task(tasks[i]);
    if (rc) return rc;
    ws += batch_task_shape(tasks[i].n, tasks[i].k).ws_bytes;
  }
  *plan_bytes = sizeof(BatchPlanHeader) + sizeof(GemvTask) * static_cast<size_t>(count);
  *workspace_bytes = ws;
  return PQ8_OK;
}

extern "C" int pq8_gemv_batch_plan(const pq8_gemv_task* tasks, int count, void* plan, size_t plan_bytes,
                                   void* workspace, size_t workspace_bytes, int* ctas, void* stream) {
  size_t need_plan = 0, need_ws = 0;
  int rc = pq8_gemv_batch_sizes(tasks, count, &need_plan, &need_ws);
  if (rc) return rc;
  if (plan == nullptr || ctas == nullptr || workspace == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (plan_bytes < need_plan || workspace_bytes < need_ws) return PQ8_ERR_WORKSPACE;
  if (!aligned(plan, 16) || !aligned(workspace, 256)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  if ((rc = device_state(&ds))) return rc;
  std::vector<unsigned char> blob(need_plan, 0);
  BatchPlanHeader* hdr = reinterpret_cast<BatchPlanHeader*>(blob.data());
  GemvTask* table = reinterpret_cast<GemvTask*>(blob.data() + sizeof(BatchPlanHeader));
  auto* base = static_cast<unsigned char*>(workspace);
  size_t off = 0;
  long long total = 0;
  for (int i = 0; i < count; ++i) {
    const pq8_gemv_task& t = tasks[i];
    const BatchTaskShape b = batch_task_shape(t.n, t.k);
    GemvParams& p = table[i].p;
    p.w = static_cast<const uint8_t*>(t.w);
    p.x0 = t.x;
    p.x_mode = kXPlain;
    p.x_vec4 = 1;
    p.y = t.y;
    p.bias = t.bias;
    p.resid = t.resid;
    p.alpha = t.alpha;
    p.epi = t.epilogue;
    p.m = 1;
    p.n = t.n;
    p.k = t.k;
    p.layout = t.epilogue == PQ8_EPI_GLU ? PQ8_LAYOUT_GLU : PQ8_LAYOUT_ROWS;
    p.out_cols = t.epilogue == PQ8_EPI_GLU ? t.n / 2 : t.n;
    p.n_tiles = b.n_tiles;
    p.k_blocks = b.kb;
    p.splits = b.splits;
    p.kb_per_split = b.kbps;
    p.cluster_reduce = 0;
    p.tickets = reinterpret_cast<int*>(base + off);
    p.partial = reinterpret_cast<float*>(base + off + round256(sizeof(int) * b.n_tiles));
    p.mode = kGemvLinear;
    p.status = ds->status;
    off += b.ws_bytes;
    table[i].cta0 = static_cast<int>(total);
    total += static_cast<long long>(b.n_tiles) * b.splits;
  }
  if (total > (1ll << 30)) return PQ8_ERR_UNSUPPORTED_SHAPE;
  hdr->magic = kBatchMagic;
  hdr->count = count;
  hdr->ctas = static_cast<int>(total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(workspace, 0, need_ws, st);
  if (e == cudaSuccess) e = cudaMemcpyAsync(plan, blob.data(), need_plan, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return to_code(e);
  *ctas = static_cast<int>(total);
  return PQ8_OK;
}

extern "C" int pq8_gemv_batch_run(const void* plan, int ctas, void* stream) {
  if (plan == nullptr || ctas < 1) return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(plan, 16)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  // the task count is read by the kernel from the plan's header, not by the
  // host (so the launch stays capturable)
  const size_t smem = ((sizeof(float) * kBatchKbPerCta * 32 + 127) & ~size_t(127)) + kStreamRingBytes;
  {
    std::lock_guard<std::mutex> lock(g_mutex);
    if (!ds->attr_set[17]) {
      cudaError_t e = cudaFuncSetAttribute(gemv_batch_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return to_code(e);
      ds->attr_set[17] = true;
    }
  }
  const unsigned char* p = static_cast<const unsigned char*>(plan);
  cudaError_t e = launch_pdl(gemv_batch_kernel, dim3(static_cast<unsigned>(ctas)), dim3(kStreamThreads), smem,
                             static_cast<cudaStream_t>(stream),
                             reinterpret_cast<const GemvTask*>(p + sizeof(BatchPlanHeader)),
                             reinterpret_cast<const BatchPlanHeader*>(p));
  if (e != cudaSuccess) return to_code(e);
  return to_code(cudaGetLastError());
}

// ---------------------------------------------------------------- persistent TDT decode
namespace {

struct DecodeWorkspace {
  size_t keys, h, c, pred, total;
};

DecodeWorkspace decode_workspace(int m, int hidden, int joint_k) {
  DecodeWorkspace d{};
  size_t off = 256;  // barrier counter at 0, abort flag at 4
  d.keys = off;
  off += round256(3 * sizeof(unsigned long long) * 2 * m);
  d.h = off;
  off += round256(sizeof(float) * 4 * (size_t)m * hidden);
  d.c = off;
  off += round256(sizeof(float) * 4 * (size_t)m * hidden);
  d.pred = off;
  off += round256(sizeof(float) * (size_t)m * joint_k);
  d.total = off;
  return d;
}

}  // namespace

extern "C" int pq8_tdt_decode_workspace_size(int m, int hidden, int joint_k, size_t* bytes) {
  if (bytes == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (m < 1 || m > kDecodeMaxStreams || hidden < 32 || hidden % 32 || joint_k < 32 || joint_k % 32)
    return PQ8_ERR_UNSUPPORTED_SHAPE;
  *bytes = decode_workspace(m, hidden, joint_k).total;
  return PQ8_OK;
}

extern "C" int pq8_tdt_decode(const pq8_tdt_weights* w, const float* enc, int enc_stride, const int* durations,
                              int n_durations, int* state, int m, int* emitted, int emitted_capacity, int* trace,
                              int trace_capacity, int max_steps, int resume, int* steps_out, int* remaining,
                              void* workspace, size_t workspace_bytes, void* stream) {
  if (w == nullptr || enc == nullptr || durations == nullptr || state == nullptr || steps_out == nullptr ||
      remaining == nullptr || workspace == nullptr || (emitted_capacity > 0 && emitted == nullptr) ||
      (trace_capacity > 0 && trace == nullptr))
    return PQ8_ERR_INVALID_ARGUMENT;
  for (int l = 0; l < 2; ++l)
    if (w->lstm[l] == nullptr || w->lstm_bias[l] == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (w->pred == nullptr || w->pred_bias == nullptr || w->joint == nullptr || w->joint_bias == nullptr ||
      w->embed == nullptr)
    return PQ8_ERR_INVALID_ARGUMENT;
  const int H = w->hidden, E = w->embed_k, J = w->joint_k;
  if (m < 1 || m > kDecodeMaxStreams || H < 32 || H % 32 || E < 32 || E % 32 || J < 32 || J % 32 ||
      w->vocab < 1 || w->n_joint <= w->vocab || n_durations < 1 || enc_stride < 0 || max_steps < 0 ||
      emitted_capacity < 0 || trace_capacity < 0)
    return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (!aligned(enc, 16) || !aligned(workspace, 256)) return PQ8_ERR_MISALIGNED;
  for (int l = 0; l < 2; ++l)
    if (!aligned(w->lstm[l], 16)) return PQ8_ERR_MISALIGNED;
  if (!aligned(w->pred, 16) || !aligned(w->joint, 16) || !aligned(w->embed, 8)) return PQ8_ERR_MISALIGNED;
  const DecodeWorkspace d = decode_workspace(m, H, J);
  if (workspace_bytes < d.total) return PQ8_ERR_WORKSPACE;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  // one CTA per SM, and every CTA gets at least one row of every matrix
  const int grid = std::min({ds->sms, H, J, w->n_joint});
  auto ceil_div = [](int a, int b) { return (a + b - 1) / b; };
  const int kmax = std::max(E + H, std::max(2 * H, J));
  const DecodeLayout L = decode_layout(ceil_div(w->n_joint, grid), ceil_div(H, grid), ceil_div(J, grid), J / 32,
                                       (E + H) / 32, 2 * H / 32, H / 32, kmax, m);
  if (L.total > 227u * 1024u) return PQ8_ERR_UNSUPPORTED_SHAPE;
  cudaError_t e = cudaFuncSetAttribute(tdt_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L.total);
  if (e != cudaSuccess) return to_code(e);
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, tdt_decode_kernel, kDecodeThreads, L.total);
  if (e != cudaSuccess) return to_code(e);
  if (per_sm < 1) return PQ8_ERR_UNSUPPORTED_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* base = static_cast<unsigned char*>(workspace);
  // fresh: zero LSTM state, pred, keys and the barrier; resumed: keys and barrier only
  e = cudaMemsetAsync(base, 0, resume ? d.h : d.total, st);
  if (e != cudaSuccess) return to_code(e);
  DecodeParams p{};
  for (int l = 0; l < 2; ++l) {
    p.w_lstm[l] = static_cast<const uint8_t*>(w->lstm[l]);
    p.b_lstm[l] = w->lstm_bias[l];
  }
  p.w_pred = static_cast<const uint8_t*>(w->pred);
  p.b_pred = w->pred_bias;
  p.w_joint = static_cast<const uint8_t*>(w->joint);
  p.b_joint = w->joint_bias;
  p.embed = w->embed;
  p.enc = enc;
  p.durations = durations;
  p.state = state;
  p.emitted = emitted;
  p.trace = trace;
  p.steps_out = steps_out;
  p.remaining = remaining;
  p.barrier = reinterpret_cast<unsigned*>(base);
  p.abort = reinterpret_cast<int*>(base + 4);
  p.keys = reinterpret_cast<unsigned long long*>(base + d.keys);
  p.h = reinterpret_cast<float*>(base + d.h);
  p.c = reinterpret_cast<float*>(base + d.c);
  p.pred = reinterpret_cast<float*>(base + d.pred);
  p.status = ds->status;
  p.m = m;
  p.hidden = H;
  p.embed_k = E;
  p.joint_k = J;
  p.n_joint = w->n_joint;
  p.vocab = w->vocab;
  p.n_durations = n_durations;
  p.enc_stride = enc_stride;
  p.emitted_capacity = emitted_capacity;
  p.trace_capacity = trace_capacity;
  p.max_steps = max_steps;
  p.resume = resume ? 1 : 0;
  // all CTAs must be resident at once: a cooperative launch fails instead of
  // running with some of them waiting for an SM
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kDecodeThreads);
  cfg.dynamicSmemBytes = L.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, tdt_decode_kernel, p);
  if (e != cudaSuccess) return to_code(e);
  return to_code(cudaGetLastError());
}

extern "C" int pq8_device_status(int* status, void* stream) {
  if (status == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int value = 0;
  cudaError_t e = cudaMemcpyAsync(&value, ds->status, sizeof(int), cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e == cudaSuccess) e = cudaMemsetAsync(ds->status, 0, sizeof(int), st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return to_code(e);
  *status = value;
  return PQ8_OK;
}

// ---------------------------------------------------------------------------
// GEMV entry point that allocates nothing.
//
// Some callers cannot hand the library a workspace: a host that reserves all
// device memory up front in its own pool and forbids other allocations, or a
// latency-critical decode loop where a cudaMalloc would implicitly
// synchronize the device. For them the split-K partials and the arrival
// tickets live in this fixed-size array, which every GPU that loads the
// library holds until the process exits. All calls on a device share it:
// calls that overlap on the GPU (on different streams, or from several host
// threads) race on it, so they must be ordered, e.g. on one stream.
namespace pq8 {
namespace {

constexpr size_t kStaticScratchBytes = size_t(4) << 20;  // 4 MiB per device
__device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];

std::mutex g_static_mutex;
void* g_static_ptr[kMaxDevices] = {};

// Device address of g_static_scratch on the current device. In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
int static_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return to_code(e);
  if (dev < 0 || dev >= kMaxDevices) return PQ8_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_static_mutex);
  if (g_static_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess) return to_code(e);
    g_static_ptr[dev] = p;
  }
  *out = g_static_ptr[dev];
  return PQ8_OK;
}

}  // namespace
}  // namespace pq8

extern "C" int pq8_gemv_static(const void* w, const float* x, float* y, const float* bias, const float* resid, int m,
                               int n, int k, int epilogue, float alpha, void* stream) {
  int rc = check_linear_args(w, x, y, resid, m, n, k, epilogue);
  if (rc || m == 0) return rc;
  if (m > PQ8_GEMV_MAX_M) return PQ8_ERR_UNSUPPORTED_SHAPE;
  DeviceState* ds;
  if ((rc = device_state(&ds))) return rc;
  const GemvPlan plan = plan_gemv(m, n, k, ds->sms);
  if (plan.total > kStaticScratchBytes) return PQ8_ERR_WORKSPACE;  // shape needs more than the 4 MiB built in
  void* scratch = nullptr;
  if ((rc = static_scratch(&scratch))) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The array keeps whatever the previous call left; the counters must start at zero.
  cudaError_t e = cudaMemsetAsync(scratch, 0, kGemvCounterBytes, st);
  if (e != cudaSuccess) return to_code(e);
  GemvParams p{};
  p.w = static_cast<const uint8_t*>(w);
  p.x0 = x;
  p.x_mode = kXPlain;
  p.x_vec4 = aligned(x, 16);
  p.y = y;
  p.bias = bias;
  p.resid = resid;
  p.alpha = alpha;
  p.epi = epilogue;
  p.m = m;
  p.n = n;
  p.k = k;
  p.layout = epilogue == PQ8_EPI_GLU ? PQ8_LAYOUT_GLU : PQ8_LAYOUT_ROWS;
  p.out_cols = epilogue == PQ8_EPI_GLU ? n / 2 : n;
  p.n_tiles = (n + kTileRows - 1) / kTileRows;
  p.k_blocks = k / 32;
  p.mode = kGemvLinear;
  return launch_gemv(ds, p, scratch, kStaticScratchBytes, st);
}


// ---------------------------------------------------------------- the block around the linears
extern "C" int pq8_layer_norm(const float* x, const float* w, const float* b, float* y, int rows, int width,
                              int flags, void* stream) {
  if (rows < 0 || width <= 0 || width % 128 || width > 1024) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (rows == 0) return PQ8_OK;
  if (x == nullptr || w == nullptr || b == nullptr || y == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (flags & ~PQ8_FLAG_OUT_TF32) return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(b, 16) || !aligned(y, 16)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  const int round_out = (flags & PQ8_FLAG_OUT_TF32) ? 1 : 0;
  constexpr int kRowsPerCta = 8;  // warps per CTA, one row at a time each
  // a warp per row up to 64 warps per SM (all of them resident at once), so
  // a LayerNorm of up to ~9,000 rows costs one memory round trip per row
  const dim3 grid(static_cast<unsigned>(std::min<long long>((rows + kRowsPerCta - 1) / kRowsPerCta,
                                                            8LL * ds->sms)));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  void (*const kernels[8])(const float*, const float*, const float*, float*, int, int) = {
      layer_norm_kernel<1>, layer_norm_kernel<2>, layer_norm_kernel<3>, layer_norm_kernel<4>,
      layer_norm_kernel<5>, layer_norm_kernel<6>, layer_norm_kernel<7>, layer_norm_kernel<8>};
  cudaError_t e = launch_pdl(kernels[width / 128 - 1], grid, dim3(32 * kRowsPerCta), 0, st, x, w, b, y, rows,
                             round_out);
  if (e != cudaSuccess) return to_code(e);
  return to_code(cudaGetLastError());
}

extern "C" int pq8_conv_depthwise_bn_silu(const float* x, const uint16_t* w9_f16, const float* bn_weight,
                                          const float* bn_bias, const float* bn_mean, const float* bn_var, float* y,
                                          int windows, int t, int channels, int flags, void* stream) {
  if (windows < 0 || t < 0 || channels <= 0 || channels % 2 || channels > 4096 || windows > 65535)
    return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (windows == 0 || t == 0) return PQ8_OK;
  if (x == nullptr || w9_f16 == nullptr || bn_weight == nullptr || bn_bias == nullptr || bn_mean == nullptr ||
      bn_var == nullptr || y == nullptr)
    return PQ8_ERR_INVALID_ARGUMENT;
  if (x == y) return PQ8_ERR_INVALID_ARGUMENT;  // neighbouring rows are read after a row is written
  if (flags & ~PQ8_FLAG_OUT_TF32) return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(x, 16) || !aligned(y, 16) || !aligned(w9_f16, 2)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  const dim3 grid((t + kConvStrip - 1) / kConvStrip, windows, (channels / 2 + kConvThreads - 1) / kConvThreads);
  cudaError_t e = launch_pdl(conv_depthwise_bn_silu_kernel, grid, dim3(kConvThreads), 0,
                             static_cast<cudaStream_t>(stream), x, w9_f16, bn_weight, bn_bias, bn_mean, bn_var, y, t,
                             channels, (flags & PQ8_FLAG_OUT_TF32) ? 1 : 0);
  if (e != cudaSuccess) return to_code(e);
  return to_code(cudaGetLastError());
}

namespace pq8 {
namespace {
// Workspace of pq8_rel_attention: biased queries, content / positional scores,
// pointer tables of the batched GEMMs and cuBLAS's own workspace.
struct AttentionPlan {
  size_t qu, qv, ac, bd, ptrs, blas, total;
};
constexpr size_t kBlasWorkspace = size_t(32) << 20;
AttentionPlan plan_attention(int windows, int t) {
  AttentionPlan a{};
  const size_t rows = static_cast<size_t>(windows) * t, b = static_cast<size_t>(windows) * 8;
  size_t off = 0;
  a.qu = off;
  off += round256(rows * 1024 * sizeof(float));
  a.qv = off;
  off += round256(rows * 1024 * sizeof(float));
  a.ac = off;
  off += round256(b * t * t * sizeof(float));
  a.bd = off;
  off += round256(b * t * (2 * static_cast<size_t>(t) - 1) * sizeof(float));
  a.ptrs = off;
  off += round256(9 * b * sizeof(void*));
  a.blas = off;
  off += kBlasWorkspace;
  a.total = off;
  return a;
}
}  // namespace
}  // namespace pq8

extern "C" int pq8_attention_workspace_size(int windows, int t, size_t* bytes) {
  if (bytes == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (windows < 1 || t < 1 || t > 8192) return PQ8_ERR_UNSUPPORTED_SHAPE;
  *bytes = plan_attention(windows, t).total;
  return PQ8_OK;
}

extern "C" int pq8_rel_attention(const float* qkv, const float* pos, const float* pos_bias_u,
                                 const float* pos_bias_v, float* ctx, int windows, int t, int flags, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (windows < 1 || windows > 65535 || t < 1 || t > 8192) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (qkv == nullptr || pos == nullptr || pos_bias_u == nullptr || pos_bias_v == nullptr || ctx == nullptr)
    return PQ8_ERR_INVALID_ARGUMENT;
  if (flags & ~(PQ8_FLAG_OUT_TF32 | PQ8_ATTN_FP32)) return PQ8_ERR_INVALID_ARGUMENT;
  if (!aligned(qkv, 16) || !aligned(pos, 16) || !aligned(pos_bias_u, 16) || !aligned(pos_bias_v, 16) ||
      !aligned(ctx, 16))
    return PQ8_ERR_MISALIGNED;
  const AttentionPlan a = plan_attention(windows, t);
  if (workspace == nullptr || workspace_bytes < a.total) return PQ8_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!(flags & PQ8_FLAG_FP32_PRODUCTS)) {
    // Fused tensor-core kernel (tcgen05, accumulators in tensor memory).
    {
      std::lock_guard<std::mutex> lock(g_mutex);
      if (!ds->attr_set[13]) {
        cudaError_t e = cudaFuncSetAttribute(rel_attention_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kTcSmemBytes);
        if (e != cudaSuccess) return to_code(e);
        ds->attr_set[13] = true;
      }
    }
    const dim3 grid((t + kTcQ - 1) / kTcQ, 8, windows);  // kTcThreads threads: softmax and producer warps
    cudaError_t e = launch_pdl(rel_attention_tc_kernel, grid, dim3(kTcThreads), kTcSmemBytes, st, qkv, pos,
                               pos_bias_u, pos_bias_v, ctx, t, (flags & PQ8_FLAG_OUT_TF32) ? 1 : 0, ds->status);
    if (e != cudaSuccess) return to_code(e);
    return to_code(cudaGetLastError());
  }
  auto* base = static_cast<unsigned char*>(workspace);
  float* qu = reinterpret_cast<float*>(base + a.qu);
  float* qv = reinterpret_cast<float*>(base + a.qv);
  float* ac = reinterpret_cast<float*>(base + a.ac);
  float* bd = reinterpret_cast<float*>(base + a.bd);
  const int nb = windows * 8;
  void** ptrs = reinterpret_cast<void**>(base + a.ptrs);
  // nine tables of nb pointers: A, B, C of the content, positional and context products
  float** tables = reinterpret_cast<float**>(ptrs);

  const long long rows = static_cast<long long>(windows) * t;
  cudaError_t e = launch_pdl(attention_query_bias_kernel,
                             dim3(static_cast<unsigned>(std::min<long long>((rows * 256 + 255) / 256, 8LL * ds->sms))),
                             dim3(256), 0, st, qkv, pos_bias_u, pos_bias_v, qu, qv, rows);
  if (e != cudaSuccess) return to_code(e);
  attention_pointers_kernel<<<(nb + 127) / 128, 128, 0, st>>>(qkv, qu, qv, pos, ac, bd, ctx, windows, t, tables);
  if ((e = cudaGetLastError()) != cudaSuccess) return to_code(e);

  std::lock_guard<std::mutex> lock(ds->blas_mutex);
  if (ds->blas == nullptr && cublasCreate(&ds->blas) != CUBLAS_STATUS_SUCCESS) return PQ8_ERR_LIBRARY;
  cublasHandle_t h = ds->blas;
  if (cublasSetStream(h, st) != CUBLAS_STATUS_SUCCESS ||
      cublasSetWorkspace(h, base + a.blas, kBlasWorkspace) != CUBLAS_STATUS_SUCCESS)
    return PQ8_ERR_LIBRARY;
  const cublasComputeType_t ct = (flags & PQ8_ATTN_FP32) ? CUBLAS_COMPUTE_32F : CUBLAS_COMPUTE_32F_FAST_TF32;
  const float one = 1.0f, zero = 0.0f;
  // Column-major view of the row-major buffers: a row-major [r][c] matrix with
  // row stride ld is the column-major c x r matrix with leading dimension ld.
  // Content scores ac[i][j] = qu_i . k_j  (columns i, rows j).
  cublasStatus_t bs = cublasGemmBatchedEx(h, CUBLAS_OP_T, CUBLAS_OP_N, t, t, 128, &one,
                                          (const void* const*)(ptrs + 0 * nb), CUDA_R_32F, 3072,
                                          (const void* const*)(ptrs + 1 * nb), CUDA_R_32F, 1024, &zero,
                                          (void* const*)(ptrs + 2 * nb), CUDA_R_32F, t, nb, ct,
                                          CUBLAS_GEMM_DEFAULT);
  // Positional scores bd[i][p] = qv_i . pos_p over all 2t - 1 positional rows.
  if (bs == CUBLAS_STATUS_SUCCESS)
    bs = cublasGemmBatchedEx(h, CUBLAS_OP_T, CUBLAS_OP_N, 2 * t - 1, t, 128, &one,
                             (const void* const*)(ptrs + 3 * nb), CUDA_R_32F, 1024,
                             (const void* const*)(ptrs + 4 * nb), CUDA_R_32F, 1024, &zero,
                             (void* const*)(ptrs + 5 * nb), CUDA_R_32F, 2 * t - 1, nb, ct,
                             CUBLAS_GEMM_DEFAULT);
  if (bs != CUBLAS_STATUS_SUCCESS) return PQ8_ERR_LIBRARY;
  const long long n_rows = static_cast<long long>(nb) * t;
  const unsigned sm_grid = static_cast<unsigned>((n_rows + 7) / 8);
  const int lanes_j = (t + 31) / 32;  // shifted scores per lane
  if (lanes_j <= 4) rel_shift_softmax_kernel<4><<<sm_grid, 256, 0, st>>>(ac, bd, t, n_rows);
  else if (lanes_j <= 8) rel_shift_softmax_kernel<8><<<sm_grid, 256, 0, st>>>(ac, bd, t, n_rows);
  else if (lanes_j <= 12) rel_shift_softmax_kernel<12><<<sm_grid, 256, 0, st>>>(ac, bd, t, n_rows);
  else if (lanes_j <= 16) rel_shift_softmax_kernel<16><<<sm_grid, 256, 0, st>>>(ac, bd, t, n_rows);
  else rel_shift_softmax_kernel<0><<<sm_grid, 256, 0, st>>>(ac, bd, t, n_rows);
  if ((e = cudaGetLastError()) != cudaSuccess) return to_code(e);
  // Context ctx[i][h*128 + d] = sum_j prob[i][j] v_j[d], heads merged in place.
  bs = cublasGemmBatchedEx(h, CUBLAS_OP_N, CUBLAS_OP_N, 128, t, t, &one,
                           (const void* const*)(ptrs + 6 * nb), CUDA_R_32F, 3072,
                           (const void* const*)(ptrs + 7 * nb), CUDA_R_32F, t, &zero,
                           (void* const*)(ptrs + 8 * nb), CUDA_R_32F, 1024, nb, ct, CUBLAS_GEMM_DEFAULT);
  if (bs != CUBLAS_STATUS_SUCCESS) return PQ8_ERR_LIBRARY;
  if (flags & PQ8_FLAG_OUT_TF32) {
    const long long n = rows * 1024;
    round_tf32_kernel<<<static_cast<unsigned>(std::min<long long>((n / 4 + 255) / 256 + 1, 8LL * ds->sms)), 256, 0,
                        st>>>(reinterpret_cast<uint32_t*>(ctx), n);
  }
  return to_code(cudaGetLastError());
}

// ---------------------------------------------------------------- subsampling stem
namespace pq8 {
namespace {
struct StemPlan {
  int t1, t2, t3;
  size_t a, b, c, d, z, flat, blas, total;
};
StemPlan plan_stem(int windows, int frames) {
  StemPlan p{};
  p.t1 = (frames + 1) / 2;
  p.t2 = (p.t1 + 1) / 2;
  p.t3 = (p.t2 + 1) / 2;
  const size_t w = windows, ch = kStemChannels * sizeof(float);
  size_t off = 0;
  p.a = off;
  off += round256(w * p.t1 * 64 * ch);
  p.b = off;
  off += round256(w * p.t2 * 32 * ch);
  p.c = off;
  off += round256(w * p.t2 * 32 * ch);
  p.d = off;
  off += round256(w * p.t3 * 16 * ch);
  p.z = off;
  off += round256(w * p.t3 * 16 * ch);
  p.flat = off;
  off += round256(w * p.t3 * 4096 * sizeof(float));
  p.blas = off;
  off += kBlasWorkspace;
  p.total = off;
  return p;
}
unsigned stem_grid(long long positions, int sms) {
  return static_cast<unsigned>(std::max<long long>(1, std::min<long long>(positions, 16LL * sms)));
}
}  // namespace
}  // namespace pq8

extern "C" int pq8_stem_workspace_size(int windows, int frames, size_t* bytes) {
  if (bytes == nullptr) return PQ8_ERR_INVALID_ARGUMENT;
  if (windows < 1 || frames < 1) return PQ8_ERR_UNSUPPORTED_SHAPE;
  *bytes = plan_stem(windows, frames).total;
  return PQ8_OK;
}

extern "C" int pq8_stem(const float* mel, int windows, int frames, const float* w0, const float* b0, const float* w2,
                        const float* b2, const float* w3, const float* b3, const float* w5, const float* b5,
                        const float* w6, const float* b6, const void* w_out, const float* b_out, float* out, int flags,
                        void* workspace, size_t workspace_bytes, void* stream) {
  if (windows < 1 || windows > 65535 || frames < 1) return PQ8_ERR_UNSUPPORTED_SHAPE;
  if (mel == nullptr || w0 == nullptr || b0 == nullptr || w2 == nullptr || b2 == nullptr || w3 == nullptr ||
      b3 == nullptr || w5 == nullptr || b5 == nullptr || w6 == nullptr || b6 == nullptr || w_out == nullptr ||
      out == nullptr)
    return PQ8_ERR_INVALID_ARGUMENT;
  if (flags & ~PQ8_FLAG_FP32_PRODUCTS) return PQ8_ERR_INVALID_ARGUMENT;
  const StemPlan sp = plan_stem(windows, frames);
  if (workspace == nullptr || workspace_bytes < sp.total) return PQ8_ERR_WORKSPACE;
  if (!aligned(workspace, 256) || !aligned(out, 16) || !aligned(w3, 16) || !aligned(w6, 16))
    return PQ8_ERR_MISALIGNED;
  DeviceState* ds;
  int rc = device_state(&ds);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  auto* base = static_cast<unsigned char*>(workspace);
  float* a = reinterpret_cast<float*>(base + sp.a);
  float* b = reinterpret_cast<float*>(base + sp.b);
  float* c = reinterpret_cast<float*>(base + sp.c);
  float* d = reinterpret_cast<float*>(base + sp.d);
  float* z = reinterpret_cast<float*>(base + sp.z);
  float* flat = reinterpret_cast<float*>(base + sp.flat);
  // positions of the two pointwise products
  const long long p2 = static_cast<long long>(windows) * sp.t2 * 32, p3 = static_cast<long long>(windows) * sp.t3 * 16;
  const float* no_bias = nullptr;
  auto frame_tiles = [](int t) { return static_cast<unsigned>((t + kStemFrames - 1) / kStemFrames); };
  cudaError_t e = launch_pdl(stem_conv_first_kernel, dim3(frame_tiles(sp.t1), windows), dim3(kStemChannels),
                             sizeof(float) * (2 * kStemFrames + 1) * (128 + 2), st, mel, w0, b0, a, frames, 128, sp.t1,
                             64);
  if (e == cudaSuccess)
    e = launch_pdl(stem_depthwise_kernel, dim3(frame_tiles(sp.t2) * 32, windows), dim3(kStemChannels), 0, st,
                   static_cast<const float*>(a), no_bias, w2, b2, b, sp.t1, 64, sp.t2, 32);
  if (e != cudaSuccess) return to_code(e);
  if (!(flags & PQ8_FLAG_FP32_PRODUCTS)) {
    // pointwise 256 x 256 on the tensor cores: out[p][n] = sum_k in[p][k] w[n][k] (TF32 operands, FP32
    // accumulation; bias and ReLU applied by the reader)
    if ((rc = gemm_dense_f32(ds, w3, b, c, static_cast<int>(p2), 256, 256, 0, st))) return rc;
    e = launch_pdl(stem_depthwise_kernel, dim3(frame_tiles(sp.t3) * 16, windows), dim3(kStemChannels), 0, st,
                   static_cast<const float*>(c), b3, w5, b5, d, sp.t2, 32, sp.t3, 16);
    if (e != cudaSuccess) return to_code(e);
    if ((rc = gemm_dense_f32(ds, w6, d, z, static_cast<int>(p3), 256, 256, 0, st))) return rc;
  } else {
    // exactness reference: FP32 products through cuBLAS
    std::lock_guard<std::mutex> lock(ds->blas_mutex);
    if (ds->blas == nullptr && cublasCreate(&ds->blas) != CUBLAS_STATUS_SUCCESS) return PQ8_ERR_LIBRARY;
    cublasHandle_t h = ds->blas;
    if (cublasSetStream(h, st) != CUBLAS_STATUS_SUCCESS ||
        cublasSetWorkspace(h, base + sp.blas, kBlasWorkspace) != CUBLAS_STATUS_SUCCESS)
      return PQ8_ERR_LIBRARY;
    const cublasComputeType_t ct = CUBLAS_COMPUTE_32F;
    const float one = 1.0f, zero = 0.0f;
    if (cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, 256, static_cast<int>(p2), 256, &one, w3, CUDA_R_32F, 256, b,
                     CUDA_R_32F, 256, &zero, c, CUDA_R_32F, 256, ct, CUBLAS_GEMM_DEFAULT) != CUBLAS_STATUS_SUCCESS)
      return PQ8_ERR_LIBRARY;
    e = launch_pdl(stem_depthwise_kernel, dim3(frame_tiles(sp.t3) * 16, windows), dim3(kStemChannels), 0, st,
                   static_cast<const float*>(c), b3, w5, b5, d, sp.t2, 32, sp.t3, 16);
    if (e != cudaSuccess) return to_code(e);
    if (cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, 256, static_cast<int>(p3), 256, &one, w6, CUDA_R_32F, 256, d,
                     CUDA_R_32F, 256, &zero, z, CUDA_R_32F, 256, ct, CUBLAS_GEMM_DEFAULT) != CUBLAS_STATUS_SUCCESS)
      return PQ8_ERR_LIBRARY;
  }
  const long long rows = static_cast<long long>(windows) * sp.t3;
  e = launch_pdl(stem_flatten_kernel, dim3(stem_grid(rows, ds->sms)), dim3(kStemChannels), 0, st,
                 static_cast<const float*>(z), b6, flat, rows);
  if (e != cudaSuccess) return to_code(e);
  // the output linear, Q8_0 [1024, 4096] + bias, on the TF32-rounded flattened rows
  return pq8_gemm(w_out, flat, out, b_out, nullptr, static_cast<int>(rows), 1024, 4096, PQ8_EPI_NONE, 1.0f,
                  PQ8_FLAG_X_TF32, stream);
}
