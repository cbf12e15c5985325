// Q8_0 x FP32 GEMM on the 5th-generation tensor cores (tcgen05, kind::tf32).
//
// Y[m, j] = epilogue(sum_k X[m, k] * W[j, k] + bias[j]) for a packed Q8_0 W.
//
// Roles are swapped relative to the output: the MMA "M" dimension is 128
// weight rows (operand A, dequantised to TF32 by converter warps and written
// straight into tensor memory with tcgen05.st), the MMA "N" dimension is BN
// activation rows (operand B, FP32 tiles streamed by TMA into 128-byte
// swizzled shared memory, rounded to TF32 in place unless the caller says the
// producer already did). The accumulator D[weight row, activation row] lives
// in tensor memory; each epilogue thread owns one weight row, so a warp's
// stores cover 32 consecutive output columns of one activation row
// (coalesced 128-byte writes). Keeping the expanded weights out of shared
// memory leaves shared-memory bandwidth to the FP32 activations.
//
// Three pipelines are decoupled, so that no buffer is held across another
// pipeline's latency:
//   * STAGES activation stages in shared memory (TMA, freed by MMA completion);
//   * WSTAGES 4352-byte weight-record stages (bulk copies from a producer of
//     their own, freed as soon as a converter holds the record in registers),
//     so the records run ahead of the activations by the conversion latency;
//   * ASLOTS tensor-memory slots for the converted weights (filled by
//     converters, freed by MMA completion), bounding how far conversion runs
//     ahead of the MMA.
// GROUPS converter groups of 4 warps (one per TMEM lane quarter) work on
// alternate K blocks.
//
// With PAIR = true, two CTAs of a cluster share one MMA (tcgen05 cta_group::2,
// M = 256 weight rows): each CTA converts its own 128-row weight tile into its
// own tensor memory and loads only half of the activation tile (BN/2 rows), so
// each activation byte fetched from L2 serves 256 weight rows instead of 128.
// The leader CTA (cluster rank 0) issues the MMAs; the peer's converters and
// epilogue arrive on the leader's barriers remotely, and MMA completion is
// multicast to the barriers of both CTAs. No TMA multicast is used.
//
// Warp roles (one persistent CTA per SM):
//   warp 0       MMA issuer: 4 x tcgen05.mma (K = 8 each) per K block; owns
//                the tensor-memory allocation
//   warp 1       scheduler: waits on the accumulator and conversion barriers
//                and releases the MMA warp through a named-barrier rendezvous
//   warp 2       X producer: TMA loads of the activation tile
//   warp 3       W producer: bulk copies of the weight records
//   converters   GROUPS x 4 warps
//   epilogue     8 warps: 2 per lane quarter, each half of the columns
// The MMA of a K block is released once its weights are in tensor memory and
// its activation stage has landed (or been rounded in place).
#pragma once

#include <cuda.h>

#include "pq8_device.cuh"

namespace pq8 {

struct GemmParams {
  const uint8_t* w;  // packed weights (header first)
  float* y;
  const float* bias;
  const float* resid;
  int* status;
  int m, n, k;
  int epi;
  float alpha;
  int flags;
  int layout;
  int out_cols;
  int n_tiles, k_blocks, m_tiles;
  int tma_store;  // 1: epilogue stages chunks in shared memory and writes them with TMA stores
  int w_f32;      // 1: w is a dense row-major FP32 [n, k] matrix (no header), rounded to TF32 by the converters
  // Split K (single GEMMs, single-CTA tiles): each output tile's K blocks are
  // shared by k_splits (2, 4 or 8) CTAs launched as one cluster. Each stages
  // its raw accumulator in shared memory; after a cluster barrier every split
  // pushes each other split the rows that one finishes (CTA s: rows
  // [s, s + 1) * BN / k_splits of the tile) with bulk copies between the
  // CTAs' shared memories, and runs the epilogue on its rows' sums, added in
  // split order.
  int k_splits;
};

template <int BN_, int STAGES_, int ASLOTS_, int ACC_, bool PAIR_, int GROUPS_ = 2, int GROUP_WARPS_ = 4,
          int EPI_COLS_ = 32, int WSTAGES_ = 4>
struct GemmCfg {
  static constexpr int BN = BN_, STAGES = STAGES_, ASLOTS = ASLOTS_, ACC = ACC_, WSTAGES = WSTAGES_;
  static constexpr bool PAIR = PAIR_;
  static constexpr int kCtas = PAIR ? 2 : 1;
  static constexpr int kRowsPerCta = BN / kCtas;  // activation rows this CTA loads per stage
  static constexpr int kGroups = GROUPS_;          // converter groups working on alternate K blocks
  static constexpr int kGroupThreads = GROUP_WARPS_ * 32;
  static constexpr int kValuesPerThread = 32 / (GROUP_WARPS_ / 4);  // of the 32 K values of a row
  static constexpr int kEpiCols = EPI_COLS_;       // accumulator columns per tcgen05.ld
  // The single-warp roles come first: the MMA warp is warp 0, the oldest warp
  // of its sub-partition, which the warp schedulers favour among ready warps.
  static constexpr int kMmaWarp = 0;
  static constexpr int kSchedWarp = 1;  // waits on behalf of the MMA warp
  static constexpr int kTmaWarp = 2;    // activation producer
  static constexpr int kWWarp = 3;      // weight-record producer
  static constexpr int kConvWarp0 = 4;
  static constexpr int kConvWarps = kGroups * kGroupThreads / 32;
  static constexpr int kEpiWarp0 = kConvWarp0 + kConvWarps;
  static constexpr int kEpiWarps = 8;
  // K blocks per scheduler/MMA rendezvous: enough MMA work (>= 512 tensor
  // cycles at BN = 256) to cover the rendezvous latency, while converters
  // fill the other half of the tensor-memory slots.
  static constexpr int kRendezvousBlocks = (512 / BN) < (ASLOTS / 2) ? (512 / BN) : (ASLOTS / 2);
  static constexpr int kRendezvousBar = 3;  // named barrier id (1 and 2 are the epilogue halves')
  static constexpr int kThreads = (kEpiWarp0 + kEpiWarps) * 32;
  static constexpr int kXStageBytes = kRowsPerCta * 128;  // rows x 32 fp32
  static constexpr int kXOff = 0;
  static constexpr int kWOff = STAGES * kXStageBytes;
  // Epilogue staging: 2 column halves x 2 buffers x [32 activation rows][128 output columns] fp32.
  static constexpr int kOutChunkFloats = 32 * 128;
  static constexpr int kOutOff = kWOff + WSTAGES * kRecordBytes;
  static constexpr int kBarOff = kOutOff + 4 * kOutChunkFloats * 4;
  // Split K: a split CTA stages its accumulator ([BN activation rows][128
  // weight rows] fp32) and receives the other splits' partials of the rows it
  // finishes (as much again) in the activation and weight rings, idle by then
  // (it runs one tile).
  static constexpr int kSplitPartialBytes = BN * 128 * 4;
  static constexpr bool kSplitFits = !PAIR && kOutOff >= 2 * kSplitPartialBytes;
  static constexpr bool kSplitK = kSplitFits && BN == 128;  // the configuration split launches use
  static constexpr int kNumBars = 3 * STAGES + 2 * WSTAGES + 2 * ASLOTS + 2 * ACC + 1 + 2;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kUsedBytes = kMiscOff + 24;
  static constexpr int kAColBase = ACC * BN;
  static constexpr int kColsNeeded = ACC * BN + ASLOTS * 32;
  static constexpr int kTmemCols = kColsNeeded <= 32 ? 32 : kColsNeeded <= 64 ? 64 : kColsNeeded <= 128 ? 128
                                   : kColsNeeded <= 256 ? 256 : 512;
  // Reserve enough shared memory that no more CTAs share an SM than its
  // 512 tensor-memory columns can hold, so tcgen05.alloc never has to wait.
  static constexpr int kMinSmem = (512 / kTmemCols) <= 1 ? 120 * 1024 : (512 / kTmemCols) == 2 ? 80 * 1024 : 0;
  static constexpr int kSmemBytes = (kUsedBytes + 1024 > kMinSmem ? kUsedBytes + 1024 : kMinSmem);
  static_assert(kColsNeeded <= 512, "tensor memory overflow");
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be a multiple of 64 in [64, 256]");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory overflow");
  static_assert((kXStageBytes / 16) % kGroupThreads == 0, "X stage must split evenly over a group");
  static_assert(kRowsPerCta % 8 == 0, "activation rows per CTA must fill 8-row swizzle atoms");
  // A converter's parity wait on a weight-record stage must not pass on the
  // phase before last, i.e. the stage's previous record must have landed.
  // Either the same group consumed that record (WSTAGES a multiple of the
  // group count), or the group's previous tensor-memory slot wait proved
  // MMA(i - kGroups - ASLOTS) complete, and with it every record up to there
  // consumed (WSTAGES >= kGroups + ASLOTS).
  // Tensor-memory slots need no such rule: a group's previous slot wait saw
  // the slot's use before last complete (kGroups <= ASLOTS). Nor do activation
  // stages: the slot wait of block i proves every block up to i - ASLOTS
  // vouched for, which covers the stage's previous use when STAGES >= ASLOTS.
  static_assert(WSTAGES % kGroups == 0 || WSTAGES >= kGroups + ASLOTS, "weight-record stage reuse must be covered");
  static_assert(STAGES >= ASLOTS, "activation stage reuse is covered by the slot waits");
  static_assert(GROUP_WARPS_ == 4 || GROUP_WARPS_ == 8, "a converter group covers the 4 TMEM lane quarters");
  static_assert(kEpiCols == 32, "the staged epilogue writes 32 activation rows per chunk");
  static_assert(kRendezvousBlocks >= 1, "need at least two tensor-memory slots");
  static_assert(kGroups <= STAGES && kGroups <= WSTAGES && kGroups <= ASLOTS, "rings advance by kGroups at a time");
  static_assert(kConvWarp0 % 4 == 0 && kEpiWarp0 % 4 == 0, "converter and epilogue warps start on lane quarter 0");
};

__device__ __forceinline__ float silu_fast(float z) { return __fdividef(z, 1.0f + __expf(-z)); }


// True when every product q * s (|q| <= 128) of this fp16 scale is zero or a
// normal fp16 number: s = 0, or 2^-14 <= |s| <= 511 (exponent field 1..23).
__device__ __forceinline__ bool scale_fp16_exact(uint32_t sbits) {
  return (((sbits >> 10) & 31u) - 1u) < 23u || (sbits & 0x7FFFu) == 0;
}

// Expands 16 Q8_0 codes (one uint4 of int8) times their fp16 scale into TF32
// bit patterns, rounded to nearest-even.
// Fast path (scale_fp16_exact): the codes, biased to bytes b = q + 128, are
// placed under the fp16 exponent of 1024 (bits 0x64bb = 1024 + b, two per
// PRMT); one HSUB2 recovers q exactly and one HMUL2 forms q * s rounded to 11
// significant bits, which is TF32 precision, for two weights at a time. This
// halves the converter's instruction count against fp32 arithmetic, which
// matters because the converters share issue slots with the MMA-issuing warp.
// Other scales take fp32 arithmetic (q * s is exact in fp32) and round the
// product to nearest-even explicitly.
__device__ __forceinline__ void expand16_tf32(const uint4 q, uint32_t sbits, bool fast, uint32_t* a) {
  const uint32_t wd[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u, q.w ^ 0x80808080u};
  if (fast) {
    const __half hs = __ushort_as_half(static_cast<unsigned short>(sbits));
    const __half2 s2 = __halves2half2(hs, hs);
    const __half2 bias = __float2half2_rn(1152.0f);  // 1024 + 128
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      uint32_t d = __byte_perm(wd[i >> 1], 0x64646464u, (i & 1) ? 0x7362 : 0x5140);
      const __half2 hv = __hmul2(__hsub2(*reinterpret_cast<__half2*>(&d), bias), s2);
      const float2 f = __half22float2(hv);
      a[2 * i] = __float_as_uint(f.x);
      a[2 * i + 1] = __float_as_uint(f.y);
    }
  } else {
    const float sc = __half2float(__ushort_as_half(static_cast<unsigned short>(sbits)));
#pragma unroll
    for (int i = 0; i < 16; ++i) a[i] = tf32_rne_bits(__float_as_uint(i8_to_f32(wd[i >> 2], i & 3) * sc));
  }
}

// ---------------------------------------------------------------------------
// GEMM sequences: one persistent launch runs the tiles of many GEMMs.
//
// The host lays a plan out in device memory (pq8_sequence_plan): a header,
// one SeqTask per GEMM (its parameters, tensor maps and dependencies) and one
// completion counter per (task, 192-row block). The plan's schedule gives
// each CTA its list of tiles, all lists following one global order in which
// every tile comes after the tiles it depends on. Before a tile's
// activations are loaded, its X dependencies must have completed the row
// blocks the tile reads; before its epilogue reads the residual or writes the
// output, its output dependencies must have (write-after-read,
// write-after-write, and the residual's read-after-write). As every CTA runs
// its list in order, the earliest unfinished tile of the global order can
// always make progress while all CTAs are resident (one per SM). Counters
// are reset by the last CTA to finish.
constexpr uint32_t kSeqMagic = 0x51455350u;  // "PSEQ"
constexpr int kSeqMaxDeps = 4;

struct SeqDep {
  int task;    // producer task (earlier in the sequence)
  int window;  // 0: the same row block; W > 0: every row block of the producer that holds rows of the W-row
               // windows that this tile's rows belong to (e.g. attention over windows between two GEMMs)
};

struct alignas(128) SeqTask {
  CUtensorMap tmap_x;  // activations [m, k], box 32 x BN rows
  CUtensorMap tmap_y;  // output [m, out_cols] (when p.tma_store)
  GemmParams p;
  int n_units;   // tiles along N
  int counter;   // index of this task's first row-block counter
  int n_x_deps, n_out_deps;
  SeqDep x_dep[kSeqMaxDeps];
  SeqDep out_dep[kSeqMaxDeps];
};

// Tile schedule: CTA c runs tiles order[start[c]] ... order[start[c + 1] - 1],
// each entry (task << 48 | weight tile << 32 | row block << 16 | K blocks).
// Every CTA's list follows one global order in which each tile comes after
// every tile it depends on.
constexpr int kSeqMaxCtas = 1024;

struct alignas(128) SeqPlanHeader {
  uint32_t magic;
  int count;        // tasks
  int total_tiles;
  int n_counters;
  int bn;           // rows per tile (all tasks)
  int finished;     // CTAs done with this run (the last one resets the counters)
  long long tasks_offset, counters_offset;
  int ctas;         // CTAs the schedule is made for (the device's SM count)
  long long start_offset, order_offset;  // int start[ctas + 1]; uint64_t order[total_tiles]
};

__device__ __forceinline__ int ld_acquire(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// Wait (bounded, like mbar_wait) until counter >= target.
__device__ __forceinline__ bool wait_counter(const int* ctr, int target, volatile int* abort_flag, int* status) {
  if (ld_acquire(ctr) >= target) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i) {
      __nanosleep(128);
      if (ld_acquire(ctr) >= target) return true;
    }
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      if (status) atomicCAS(status, 0, PQ8_ERR_TIMEOUT);
      return false;
    }
  }
}

// Row blocks of dependency `d`'s producer that tile row block m_tile needs.
__device__ __forceinline__ void dep_range(const SeqTask& t, const SeqDep& d, int m_tile, int bn, int* lo, int* hi) {
  *lo = m_tile;
  *hi = m_tile;
  if (d.window > 0) {
    const int r0 = m_tile * bn, r1 = r0 + bn - 1;
    *lo = (r0 / d.window) * d.window / bn;
    *hi = ((r1 / d.window) * d.window + d.window - 1) / bn;
  }
  *hi = *hi < t.p.m_tiles - 1 ? *hi : t.p.m_tiles - 1;
}

// Wait for the row blocks that dependency `d` must have completed before tile
// rows [row0, row0 + bn) of the consumer may be used.
__device__ __forceinline__ bool wait_dep(const SeqTask* tasks, int* counters, const SeqDep& d, int m_tile, int bn,
                                         volatile int* abort_flag, int* status) {
  const SeqTask& t = tasks[d.task];
  int lo, hi;
  dep_range(t, d, m_tile, bn, &lo, &hi);
  const int target = 2 * t.n_units;  // each tile's two epilogue halves signal once
  for (int r = lo; r <= hi; ++r)
    if (!wait_counter(counters + t.counter + r, target, abort_flag, status)) return false;
  return true;
}


// Where a tile of the launch lies: its GEMM (sequences), weight tile, row block and K blocks.
struct TileRef {
  const SeqTask* task;  // sequences only
  int n_tile, m_tile, kb;
  int kb0 = 0, split = 0;  // split K: first K block and split index of this tile
};

// Tile `tile` of a single GEMM: output tiles N-unit major, their K splits
// fastest (the splits of a tile run side by side on consecutive CTAs).
template <int kCtas>
__device__ __forceinline__ TileRef single_tile(int tile, uint32_t rank, int m_tiles, int k_blocks, int splits) {
  const int s = tile % splits, out_tile = tile / splits;
  const int per = (k_blocks + splits - 1) / splits, kb0 = s * per;
  const int kb = k_blocks - kb0 < per ? k_blocks - kb0 : per;
  return {nullptr, (out_tile / m_tiles) * kCtas + static_cast<int>(rank), out_tile % m_tiles, kb, kb0, s};
}

// A role warp's view of its tiles (local index i = the CTA's i-th tile,
// tile blockIdx + i * grid). For a sequence, the lanes look up 32 tiles at
// once (lane j holds the entry of tile base + j) and each tile's entry is
// then two shuffles away: looking a task up in the plan is a chain of global
// loads, which at every tile boundary would otherwise stall the warp that has
// to start the next tile. The state is four registers; everything else is
// re-derived from kernel parameters and special registers. Every lane of the
// warp must call get() with the same index.
template <int kCtas, bool SEQ>
struct TileWindow;

template <int kCtas>
struct TileWindow<kCtas, false> {
  int m_tiles, k_blocks, splits;
  __device__ __forceinline__ TileRef get(int local, uint32_t rank, const uint8_t*) const {
    const int tile = static_cast<int>(blockIdx.x) / kCtas + local * static_cast<int>(gridDim.x / kCtas);
    return single_tile<kCtas>(tile, rank, m_tiles, k_blocks, splits);
  }
};

// Looks up the tile of lane (threadIdx & 31) of the window starting at local
// index `local`; out of line, so that its temporaries do not add to the
// register pressure of the role loops it is called from (once per 32 tiles).
__device__ __noinline__ void seq_window_entry(const uint8_t* plan, int local, uint32_t* task_n, uint32_t* m_kb) {
  const SeqPlanHeader* hdr = reinterpret_cast<const SeqPlanHeader*>(plan);
  const int* start = reinterpret_cast<const int*>(plan + hdr->start_offset);
  const int tile = start[blockIdx.x] + local + static_cast<int>(threadIdx.x & 31);
  if (tile >= start[blockIdx.x + 1]) return;
  const uint64_t e = reinterpret_cast<const uint64_t*>(plan + hdr->order_offset)[tile];
  *task_n = static_cast<uint32_t>(e >> 32);
  *m_kb = static_cast<uint32_t>(e);
}

template <int kCtas>
struct TileWindow<kCtas, true> {
  int base = -64;  // local index of lane 0's entry
  uint32_t e_task_n = 0, e_m_kb = 0;  // this lane's entry, two 16-bit fields each
  __device__ __forceinline__ TileRef get(int local, uint32_t, const uint8_t* plan) {
    const SeqTask* tasks = reinterpret_cast<const SeqTask*>(plan + sizeof(SeqPlanHeader));
    if (local - base >= 32) {
      base = local;
      seq_window_entry(plan, local, &e_task_n, &e_m_kb);
    }
    const int i = local - base;
    const uint32_t tn = __shfl_sync(0xffffffffu, e_task_n, i), mk = __shfl_sync(0xffffffffu, e_m_kb, i);
    return {tasks + (tn >> 16), static_cast<int>(tn & 0xFFFFu), static_cast<int>(mk >> 16),
            static_cast<int>(mk & 0xFFFFu)};
  }
};

// Per-thread lookup of a tile (the converters, the epilogue and the
// producers, which reach a tile boundary well before its data is needed).
template <int kCtas, bool SEQ>
struct TileCursor {
  int m_tiles, k_blocks, splits;  // single GEMM
  const uint64_t* order;          // sequence: the schedule's tile entries
  __device__ __forceinline__ TileRef at(int tile, uint32_t rank, const uint8_t* plan) {
    if constexpr (SEQ) {
      const SeqTask* tasks = reinterpret_cast<const SeqTask*>(plan + sizeof(SeqPlanHeader));
      const uint64_t e = __ldg(reinterpret_cast<const unsigned long long*>(order) + tile);
      return {tasks + static_cast<int>(e >> 48), static_cast<int>((e >> 32) & 0xFFFFu),
              static_cast<int>((e >> 16) & 0xFFFFu), static_cast<int>(e & 0xFFFFu)};
    } else {
      return single_tile<kCtas>(tile, rank, m_tiles, k_blocks, splits);
    }
  }
};

// A parameter of the tile's GEMM: the sequence task's, or the launch's own
// (read straight from the kernel parameters).
#define PQ8_TP(t, field) (SEQ ? (t).task->p.field : p.field)

template <int BN, int STAGES, int ASLOTS, int ACC, bool PAIR, int GROUPS = 2, int GROUP_WARPS = 4, int EPI_COLS = 32,
          int WSTAGES = 4, bool SEQ = false>
__global__ void __launch_bounds__(GemmCfg<BN, STAGES, ASLOTS, ACC, PAIR, GROUPS, GROUP_WARPS, EPI_COLS, WSTAGES>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_y,
                   const GemmParams p, const uint8_t* plan) {
  using C = GemmCfg<BN, STAGES, ASLOTS, ACC, PAIR, GROUPS, GROUP_WARPS, EPI_COLS, WSTAGES>;
  static_assert(!(SEQ && PAIR), "sequences run single-CTA tiles");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem + C::kXOff;
  uint8_t* ws = smem + C::kWOff;
  float* out_stage = reinterpret_cast<float*>(smem + C::kOutOff);
  uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + C::kBarOff);  // activation stage landed
  uint64_t* xempty = xfull + STAGES;                                  // activation stage read by the MMA
  uint64_t* wfull = xempty + STAGES;                                  // weight record landed
  uint64_t* wempty = wfull + WSTAGES;                                 // weight record taken by a converter
  uint64_t* conv = wempty + WSTAGES;
  uint64_t* afree = conv + ASLOTS;
  uint64_t* acc_full = afree + ASLOTS;
  uint64_t* acc_empty = acc_full + ACC;
  uint64_t* drain = acc_empty + ACC;
  uint64_t* red_full = drain + 1;  // [2 epilogue halves]: split K, the other splits' rows received
  uint64_t* xround = red_full + 2;  // activation stage rounded by the epilogue warps (epi_round_x)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);
  int* bad_flag = reinterpret_cast<int*>(smem + C::kMiscOff + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // The next kernel may launch now: its CTAs take SMs as this grid's CTAs
  // exit, set up and fetch and convert their (constant) weights, and wait for
  // this grid before touching activations or outputs.
  griddep_launch();
  const uint32_t rank = PAIR ? cluster_rank() : 0;  // 0 = leader (issues the MMAs)
  const bool leader = rank == 0;
  // Tiles of this launch: one GEMM (p), or every task of a sequence plan.
  // A single GEMM's CTA (pair) runs units blockIdx, blockIdx + grid, ...; a
  // sequence CTA runs its list of the plan's schedule, entries start[c] on.
  const SeqPlanHeader* hdr = SEQ ? reinterpret_cast<const SeqPlanHeader*>(plan) : nullptr;
  const SeqTask* tasks = SEQ ? reinterpret_cast<const SeqTask*>(plan + sizeof(SeqPlanHeader)) : nullptr;
  int* counters = SEQ ? reinterpret_cast<int*>(const_cast<uint8_t*>(plan) + hdr->counters_offset) : nullptr;
  const int* seq_start = SEQ ? reinterpret_cast<const int*>(plan + hdr->start_offset) : nullptr;
  const int task_count = SEQ ? hdr->count : 1;
  const int n_units = PAIR ? (p.n_tiles + 1) / 2 : p.n_tiles;
  const int unit0 = SEQ ? seq_start[blockIdx.x] : static_cast<int>(blockIdx.x) / C::kCtas;
  const int unit_stride = SEQ ? 1 : static_cast<int>(gridDim.x) / C::kCtas;
  const int num_tiles = SEQ ? seq_start[blockIdx.x + 1] : n_units * p.m_tiles * p.k_splits;
  int* const status = p.status;

  if (threadIdx.x == 0) {
    bool ok = true;
    if constexpr (!SEQ) {  // a sequence's headers are checked when its plan is made
      if (!p.w_f32) {
        const PackedHeader* h = reinterpret_cast<const PackedHeader*>(p.w);
        ok = h->magic == kMagic && h->n == p.n && h->k == p.k && h->layout == p.layout && h->n_tiles == p.n_tiles;
      }
    } else {
      ok = hdr->ctas == static_cast<int>(gridDim.x);  // the schedule is made for this many CTAs
    }
    *bad_flag = ok ? 0 : 1;
    *abort_flag = 0;
    if (!ok) atomicCAS(status, 0, PQ8_ERR_LAYOUT);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xempty[s], 1);
    }
    for (int s = 0; s < WSTAGES; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], GROUP_WARPS);
    }
    for (int a = 0; a < ASLOTS; ++a) {
      mbar_init(&conv[a], GROUP_WARPS * C::kCtas);  // one arrival per converter warp
      mbar_init(&afree[a], 1);
    }
    for (int a = 0; a < ACC; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], C::kEpiWarps * C::kCtas);  // one arrival per epilogue warp
    }
    mbar_init(drain, 1);
    mbar_init(&red_full[0], 1);
    mbar_init(&red_full[1], 1);
    for (int s = 0; s < STAGES; ++s) mbar_init(&xround[s], C::kEpiWarps);  // one arrival per epilogue warp
    fence_mbar_init();
  }
  if (warp == C::kTmaWarp && lane == 0 && !SEQ) {
    prefetch_tmap(&tmap_x);
    if (p.tma_store) prefetch_tmap(&tmap_y);
  }
  __syncthreads();
  // Both CTAs of a pair see the same header, so they leave together.
  if (*bad_flag) return;
  if constexpr (PAIR) cluster_sync();  // peer barriers initialised before any remote arrive
  if (warp == C::kMmaWarp) {
    if constexpr (PAIR) {
      tmem_alloc_pair(tmem_slot, C::kTmemCols);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tmem_slot, C::kTmemCols);
      tmem_relinquish();
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Arrivals that the leader's MMA waits for go to the leader's barriers.
  const uint32_t conv_remote = PAIR ? map_to_rank(conv, 0) : 0;
  const uint32_t acc_empty_remote = PAIR ? map_to_rank(acc_empty, 0) : 0;
  TileCursor<C::kCtas, SEQ> src{p.m_tiles, p.k_blocks, p.k_splits,
                                SEQ ? reinterpret_cast<const uint64_t*>(plan + hdr->order_offset) : nullptr};
  const int x_flags = SEQ ? (task_count > 0 ? tasks[0].p.flags : 0) : p.flags;
  // Activations not yet rounded to TF32 are rounded in shared memory as each
  // stage lands: by the epilogue warps when every CTA of a single-CTA launch
  // runs one tile (they have nothing to do before its epilogue, and the
  // converters are the mainloop's bottleneck), otherwise by the converters.
  // (All tasks of a sequence share the X rounding flag.)
  const bool round_x = !(x_flags & PQ8_FLAG_X_TF32);
  const bool epi_round_x = !SEQ && !PAIR && round_x && num_tiles <= unit_stride;
  bool mma_issued = false;

  if (warp >= C::kConvWarp0 && warp < C::kConvWarp0 + C::kConvWarps) {
    // ------------------------------------------------------------ converters
    const int cw = warp - C::kConvWarp0;               // converter warp index (kConvWarp0 % 4 == 0)
    const int grp = cw / (C::kGroupThreads / 32);
    const int gt = (threadIdx.x - C::kConvWarp0 * 32) % C::kGroupThreads;  // thread index within the group
    const int quarter = warp & 3;                      // TMEM lane quarter of this warp
    const int kpart = (cw >> 2) % (GROUP_WARPS / 4);   // which kValuesPerThread of the 32 K values
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    // Barrier checks are started early (non-blocking tests) and only waited
    // on when they had not completed, so their round trips overlap the
    // conversion arithmetic.
    constexpr uint32_t G = C::kGroups;
    Ring<STAGES> xr;
    Ring<WSTAGES> wr;
    Ring<ASLOTS> ar;
    xr.advance(grp);  // this group's first K block is block `grp`
    wr.advance(grp);
    ar.advance(grp);
    // Who vouches for this CTA's activation stage before the MMA: the
    // converters when they round it in place or when they are the pair peer's
    // (whose barriers the leader cannot see); otherwise the scheduler.
    const bool vouch_x = (round_x && !epi_round_x) || (PAIR && !leader);
    bool w_ready = false;
    int tile = unit0, local = 0;
    uint32_t tile_first = 0;  // index of the current tile's first K block
    bool has_w = false;
    uint32_t kb_tile = 0;
    int n_tile = 0, kb0_tile = 0;
    // dense FP32 weights (single GEMMs only): each converter thread reads its
    // row's 32 values of the K block from global memory instead of a record
    const bool w_f32 = !SEQ && p.w_f32 != 0;
    auto enter = [&]() {
      const TileRef t = src.at(tile, rank, plan);
      has_w = t.n_tile < PQ8_TP(t, n_tiles);
      kb_tile = static_cast<uint32_t>(t.kb);
      n_tile = t.n_tile;
      kb0_tile = t.kb0;
    };
    if (tile < num_tiles) enter();
    for (uint32_t it = grp;; it += G) {
      while (tile < num_tiles && it >= tile_first + kb_tile) {
        tile += unit_stride;
        ++local;
        tile_first += kb_tile;
        if (tile < num_tiles) enter();
      }
      if (tile >= num_tiles) break;
      const uint32_t stage = xr.idx, wst = wr.idx, slot = ar.idx;
      // The weight record is converted into registers and only then released:
      // the refill is an async-proxy write, which an mbarrier release does not
      // order after this warp's shared-memory loads, so the stage is handed
      // back once the conversion has consumed every loaded value. The
      // conversion runs before the tensor-memory slot is waited for.
      if (!w_ready && !mbar_wait(&wfull[wst], wr.phase, abort_flag, status)) goto conv_done;
      uint32_t a[C::kValuesPerThread];
      bool slot_ready;
      {
        constexpr int H = C::kValuesPerThread / 16;
        uint4 q[H];
        uint32_t sbits = 0;
        if (has_w && !w_f32) {
          const uint8_t* rec = ws + wst * kRecordBytes;
          sbits = *reinterpret_cast<const uint16_t*>(rec + kScaleOffset + row * 2);
#pragma unroll
          for (int h = 0; h < H; ++h)  // 16-value halves of the K block
            q[h] = *reinterpret_cast<const uint4*>(rec + (kpart * H + h) * 2048 + row * 16);
        }
        slot_ready = mbar_test_wait(smem_addr(&afree[slot]), ar.phase ^ 1u);
        if (has_w && w_f32) {
          const int wrow = n_tile * kTileRows + row;
          const uint32_t kb = it - tile_first + static_cast<uint32_t>(kb0_tile);
          const float4* src4 = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p.w) +
                                                               (size_t)wrow * p.k + kb * 32 +
                                                               kpart * C::kValuesPerThread);
#pragma unroll
          for (int i = 0; i < C::kValuesPerThread / 4; ++i) {
            const float4 v = wrow < p.n ? src4[i] : make_float4(0.f, 0.f, 0.f, 0.f);
            a[4 * i] = tf32_rne_bits(__float_as_uint(v.x));
            a[4 * i + 1] = tf32_rne_bits(__float_as_uint(v.y));
            a[4 * i + 2] = tf32_rne_bits(__float_as_uint(v.z));
            a[4 * i + 3] = tf32_rne_bits(__float_as_uint(v.w));
          }
        } else if (has_w) {
          const bool fast = scale_fp16_exact(sbits);
#pragma unroll
          for (int h = 0; h < H; ++h) expand16_tf32(q[h], sbits, fast, a + h * 16);
        } else {
          // Odd tile count: the peer of the last pair multiplies zeros.
#pragma unroll
          for (int i = 0; i < C::kValuesPerThread; ++i) a[i] = 0;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&wempty[wst]);
      if (!slot_ready && !mbar_wait(&afree[slot], ar.phase ^ 1u, abort_flag, status)) goto conv_done;
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < C::kValuesPerThread / 16; ++h) {
        const int khalf = kpart * (C::kValuesPerThread / 16) + h;
        uint32_t part[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) part[i] = a[h * 16 + i];
        tmem_st16(tmem + lane_base + C::kAColBase + slot * 32 + khalf * 16, part);
      }
      if (vouch_x) {
        if (!mbar_wait(&xfull[stage], xr.phase, abort_flag, status)) goto conv_done;
        if (round_x) {
          uint4* xv = reinterpret_cast<uint4*>(xs + stage * C::kXStageBytes);
          constexpr int kPer = C::kXStageBytes / 16 / C::kGroupThreads;
          uint4 v[kPer];
#pragma unroll
          for (int i = 0; i < kPer; ++i) v[i] = xv[gt + C::kGroupThreads * i];
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            v[i].x = tf32_round_bits(v[i].x);
            v[i].y = tf32_round_bits(v[i].y);
            v[i].z = tf32_round_bits(v[i].z);
            v[i].w = tf32_round_bits(v[i].w);
            xv[gt + C::kGroupThreads * i] = v[i];
          }
          if constexpr (PAIR) fence_proxy_async_cluster();
          else fence_proxy_async_smem();
        }
      }
      xr.advance(G);
      wr.advance(G);
      ar.advance(G);
      // Next record of this group: start its check now.
      w_ready = mbar_test_wait(smem_addr(&wfull[wr.idx]), wr.phase);
      tmem_wait_st();
      tc_fence_before();
      // every lane's tensor-memory stores are complete and fenced: one arrival per warp
      __syncwarp();
      if (lane == 0) {
        if (PAIR && !leader) mbar_arrive_cluster(conv_remote + slot * 8);
        else mbar_arrive(&conv[slot]);
      }
    }
  conv_done:;
  } else if (warp >= C::kEpiWarp0) {
    // -------------------------------------------------------------- epilogue
    // Each half (4 warps, one per TMEM lane quarter) handles half of the BN
    // activation rows, 32 at a time. With TMA stores, a chunk is written to a
    // shared-memory buffer laid out as the output tile and stored by one thread;
    // the accumulator is released as soon as it has been read, so the global
    // writes drain while the next tile is being multiplied.
    const int q = warp & 3;                        // TMEM lane quarter
    const int half = (warp - C::kEpiWarp0) >> 2;  // which half of the BN columns
    const int r = q * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(q * 32) << 16;
    const bool elected = q == 0 && lane == 0;      // issues this half's TMA stores
    constexpr int E = C::kEpiCols;
    constexpr int kChunks = BN / E / 2;            // E-column chunks per half
    int chunk_seq = 0;                             // chunks issued by this half (selects the buffer)
    // Split K: this CTA's split (its rank in the cluster), the activation rows
    // of the tile this half finishes, and whether the half has passed the
    // cluster barrier that publishes the partials (every thread of the cluster
    // passes it exactly once, also when giving up).
    // (Split launches use the BN = 128 configuration only.)
    const bool split = !SEQ && C::kSplitK && p.k_splits > 1;
    // rows [split_off, split_off + split_rows) of the tile; derived where used
    auto split_rows = [&]() { return BN / p.k_splits / 2; };
    auto split_off = [&]() { return static_cast<int>(cluster_rank()) * (BN / p.k_splits) + half * split_rows(); };
    bool published = false;
    bool received = false;  // this half's receive barrier waited for (it must be, before the CTA exits)
    int local = 0;
    griddep_wait();  // the residual and the output may be in use by the previous kernel
    if (epi_round_x && unit0 < num_tiles) {
      // This CTA's one tile: round each activation stage to TF32 as it lands
      // (the scheduler waits for xround before the MMA reads the stage).
      constexpr int kEpiThreads = C::kEpiWarps * 32;
      constexpr int kPer = C::kXStageBytes / 16 / kEpiThreads;
      static_assert(C::kXStageBytes / 16 % kEpiThreads == 0, "X stage must split evenly over the epilogue");
      const int et = static_cast<int>(threadIdx.x) - C::kEpiWarp0 * 32;
      const int KB = src.at(unit0, rank, plan).kb;
      Ring<STAGES> xr;
      for (int kb = 0; kb < KB; ++kb, xr.advance(1)) {
        if (!mbar_wait(&xfull[xr.idx], xr.phase, abort_flag, status)) break;
        uint4* xv = reinterpret_cast<uint4*>(xs + xr.idx * C::kXStageBytes);
        uint4 v[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) v[i] = xv[et + kEpiThreads * i];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          v[i].x = tf32_round_bits(v[i].x);
          v[i].y = tf32_round_bits(v[i].y);
          v[i].z = tf32_round_bits(v[i].z);
          v[i].w = tf32_round_bits(v[i].w);
          xv[et + kEpiThreads * i] = v[i];
        }
        fence_proxy_async_smem();  // the rounded values, read by the tensor cores
        __syncwarp();
        if (lane == 0) mbar_arrive(&xround[xr.idx]);
      }
    }
    for (int tile = unit0; tile < num_tiles; tile += unit_stride, ++local) {
      const TileRef t = src.at(tile, rank, plan);
      const int n_tile = t.n_tile, m_tile = t.m_tile;
      const int m = PQ8_TP(t, m), n = PQ8_TP(t, n), out_cols = PQ8_TP(t, out_cols), layout = PQ8_TP(t, layout);
      const int epi = PQ8_TP(t, epi), flags = PQ8_TP(t, flags);
      const float alpha = PQ8_TP(t, alpha);
      const bool tma_store = !split && PQ8_TP(t, tma_store) != 0;
      const float* const bias = PQ8_TP(t, bias);
      const void* ty = SEQ ? static_cast<const void*>(&t.task->tmap_y) : static_cast<const void*>(&tmap_y);
      const bool glu = epi == PQ8_EPI_GLU;
      const int box_cols = glu ? 64 : 128;           // output columns of one tile
      const int c_local = glu ? q * 16 + (lane & 15) : r;
      const int acc = local % ACC;
      RowMap rm;
      const bool valid = map_row(layout, n, n_tile * kTileRows + r, rm);
      const float b = (bias != nullptr && valid) ? bias[rm.src] : 0.0f;
      const bool store_lane = valid && (!glu || lane < 16);
      float* ycol = PQ8_TP(t, y) + rm.col;
      const float* rcol = PQ8_TP(t, resid) + rm.col;
      const bool resid = epi == PQ8_EPI_RESIDUAL;
      bool dep_ok = true;
      if constexpr (SEQ) {
        // write-after-read, write-after-write and the residual's producer
        const int nd = t.task->n_out_deps;
        for (int d = 0; d < nd && dep_ok; ++d)
          dep_ok = wait_dep(tasks, counters, t.task->out_dep[d], m_tile, BN, abort_flag, status);
        if (!dep_ok) break;
      }
      // Residual rows are loaded into out[] one chunk ahead: the tile's first
      // chunk before the accumulator is waited for, each next chunk as soon as
      // the previous one has been staged, so their latency is off the critical
      // path (they are other rows than any store still in flight).
      float out[E];
      auto load_resid = [&](int m0) {
#pragma unroll
        for (int j = 0; j < E; ++j)
          out[j] = (store_lane && m0 + j < m) ? rcol[(size_t)(m0 + j) * out_cols] : 0.0f;
      };
      if (resid) load_resid(split ? m_tile * BN + split_off() : m_tile * BN + half * kChunks * E);
      if (!mbar_wait(&acc_full[acc], (local / ACC) & 1, abort_flag, status)) break;
      tc_fence_after();
      if (split) {
        // Split K: each half stages its chunks of this split's raw accumulator
        // at the start of the idle activation ring ([BN activation rows][128
        // weight rows]), releases the accumulator, and its elected thread sets
        // the bytes its receive area expects. Then all splits of the tile meet
        // at the cluster barrier: every mainloop is done, so every receive area
        // is free, and every expectation is set.
        float* const stage = reinterpret_cast<float*>(xs);
#pragma unroll 1
        for (int cc = 0; cc < kChunks; ++cc) {
          const int c = half * kChunks + cc;
          uint32_t v[E];
          tmem_ld32(tmem + lane_base + acc * BN + c * E, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < E; ++j) stage[(c * E + j) * kTileRows + r] = __uint_as_float(v[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[acc]);
        fence_proxy_async_smem();  // the staged values, read by the bulk-copy unit
        if (elected)
          mbar_expect_tx(&red_full[half], static_cast<uint32_t>((p.k_splits - 1) * split_rows() * kTileRows * 4));
        __syncwarp();
        cluster_sync();
        published = true;
        // The first epilogue warp pushes every other split (d) the rows it
        // finishes, one bulk copy per (d, epilogue half of d), into d's receive
        // area ([half][source split][rows][128], after the staging area).
        if (half == 0 && q == 0) {
          const int S = p.k_splits, R = split_rows();
          const int me = static_cast<int>(cluster_rank());
          for (int i = lane; i < 2 * (S - 1); i += 32) {
            const int d = (me + 1 + (i >> 1)) % S, h2 = i & 1;
            const float* src = stage + (d * (BN / S) + h2 * R) * kTileRows;
            const uint32_t dst = map_to_rank(stage + BN * kTileRows, static_cast<uint32_t>(d)) +
                                 static_cast<uint32_t>((h2 * S + me) * R * kTileRows * 4);
            bulk_s2s_cluster(dst, src, static_cast<uint32_t>(R * kTileRows * 4),
                             map_to_rank(&red_full[h2], static_cast<uint32_t>(d)));
          }
        }
      }
      const int n_chunks = split ? 1 : kChunks;
#pragma unroll 1
      for (int cc = 0; cc < n_chunks; ++cc, ++chunk_seq) {
        const int c = half * kChunks + cc;
        const int m0 = m_tile * BN + (split ? split_off() : c * E);
        if (m0 >= m) break;
        uint32_t v[E];
        if (split) {
          // this half's split_rows rows, summed over the splits' partials in
          // split order (onto +0, which leaves the first partial's values as
          // they are): this split's from its staging area, the others' from
          // the receive area once they have landed
          const int rows = split_rows(), me = static_cast<int>(cluster_rank());
          if (!mbar_wait(&red_full[half], 0, abort_flag, status)) break;
          received = true;
          const float* const own = reinterpret_cast<const float*>(xs) + (m0 - m_tile * BN) * kTileRows + r;
          const float* const recv = reinterpret_cast<const float*>(xs) + BN * kTileRows +
                                    half * p.k_splits * rows * kTileRows + r;
#pragma unroll
          for (int j = 0; j < E; ++j) v[j] = 0u;
#pragma unroll 1
          for (int sp = 0; sp < p.k_splits; ++sp) {
            const float* src = sp == me ? own : recv + sp * rows * kTileRows;
#pragma unroll
            for (int j = 0; j < E; ++j)
              if (j < rows) v[j] = __float_as_uint(__uint_as_float(v[j]) + src[j * kTileRows]);
          }
        } else {
          tmem_ld32(tmem + lane_base + acc * BN + c * E, v);
          tmem_wait_ld();
        }
        const int cnt = min(split ? split_rows() : E, m - m0);  // warp-uniform
        if (resid) {
#pragma unroll
          for (int j = 0; j < E; ++j) out[j] = fmaf(alpha, __uint_as_float(v[j]) + b, out[j]);
        } else if (glu) {
#pragma unroll
          for (int j = 0; j < E; ++j) {
            const float z = __uint_as_float(v[j]) + b;
            const float gate = __shfl_down_sync(0xffffffffu, z, 16);
            out[j] = __fdividef(z, 1.0f + __expf(-gate));
          }
        } else if (epi == PQ8_EPI_SILU) {
#pragma unroll
          for (int j = 0; j < E; ++j) out[j] = silu_fast(__uint_as_float(v[j]) + b);
        } else if (epi == PQ8_EPI_RELU) {
#pragma unroll
          for (int j = 0; j < E; ++j) out[j] = fmaxf(__uint_as_float(v[j]) + b, 0.0f);
        } else {
#pragma unroll
          for (int j = 0; j < E; ++j) out[j] = __uint_as_float(v[j]) + b;
        }
        if (flags & PQ8_FLAG_OUT_TF32) {
#pragma unroll
          for (int j = 0; j < E; ++j) out[j] = tf32_round(out[j]);
        }
        if (tma_store) {
          float* stage = out_stage + (half * 2 + (chunk_seq & 1)) * C::kOutChunkFloats;
          // the store issued from this buffer two chunks ago must have read it
          if (elected) bulk_wait_group_read<1>();
          named_barrier_sync(1 + half, 128);
          if (!glu || lane < 16) {
#pragma unroll
            for (int j = 0; j < E; ++j) stage[j * box_cols + c_local] = out[j];
          }
          fence_proxy_async_smem();
          named_barrier_sync(1 + half, 128);
          // rows past M and columns past the output width are clipped by the TMA unit
          if (elected) {
            tma_store_2d(ty, stage, n_tile * box_cols, m0);
            bulk_commit_group();
          }
        } else if (store_lane) {
          float* yp = ycol + (size_t)m0 * out_cols;
#pragma unroll
          for (int j = 0; j < E; ++j)
            if (j < cnt) yp[(size_t)j * out_cols] = out[j];
        }
        if (resid && cc + 1 < kChunks) load_resid(m0 + E);
      }
      if (!split) {
        tc_fence_before();
        __syncwarp();  // every lane's accumulator loads are complete: one arrival per warp
        if (lane == 0) {
          if (PAIR && !leader) mbar_arrive_cluster(acc_empty_remote + acc * 8);
          else mbar_arrive(&acc_empty[acc]);
        }
      }
      if constexpr (SEQ) {
        // This half's rows of the tile are written: signal them (once per half).
        if (tma_store) {
          if (elected) {
            bulk_wait_group_all();
            fence_proxy_async_global();
            red_release_add(counters + t.task->counter + m_tile, 1);
          }
        } else {
          __threadfence();
          named_barrier_sync(1 + half, 128);
          if (elected) red_release_add(counters + t.task->counter + m_tile, 1);
        }
      }
    }
    if (elected) bulk_wait_group_all();
    if (split && !published) {  // gave up before the partials were published
      __syncwarp();
      cluster_sync();
    }
    // never leave the other splits' copies landing in this CTA's shared memory
    if (split && published && !received) mbar_drain(&red_full[half], 0);
  } else if (warp == C::kTmaWarp) {
    // ----------------------------------------------------- activation producer
    if (lane == 0) {
      griddep_wait();  // the activations may come from the previous kernel
      uint32_t issued = 0;
      Ring<STAGES> xr;
      for (int tile = unit0; tile < num_tiles; tile += unit_stride) {
        const TileRef t = src.at(tile, rank, plan);
        const int row0 = t.m_tile * BN + static_cast<int>(rank) * C::kRowsPerCta;
        const void* tx = SEQ ? static_cast<const void*>(&t.task->tmap_x) : static_cast<const void*>(&tmap_x);
        if constexpr (SEQ) {
          const int nd = t.task->n_x_deps;
          bool ok = true;
          for (int d = 0; d < nd && ok; ++d)
            ok = wait_dep(tasks, counters, t.task->x_dep[d], t.m_tile, BN, abort_flag, status);
          if (!ok) goto x_done;
          fence_proxy_async_global();  // the producers' rows, read by the tensor-copy unit
        }
        for (int kb = 0; kb < t.kb; ++kb, ++issued, xr.advance(1)) {
          if (!mbar_wait(&xempty[xr.idx], xr.phase ^ 1u, abort_flag, status)) goto x_done;
          mbar_expect_tx(&xfull[xr.idx], C::kXStageBytes);
          tma_load_2d(xs + xr.idx * C::kXStageBytes, tx, (t.kb0 + kb) * 32, row0, &xfull[xr.idx]);
        }
      }
    x_done:
      // Never leave the CTA with copies still landing in its shared memory.
      for (uint32_t j = issued > STAGES ? issued - STAGES : 0; j < issued; ++j)
        mbar_drain(&xfull[j % STAGES], (j / STAGES) & 1);
    }
  } else if (warp == C::kWWarp) {
    // -------------------------------------------------- weight-record producer
    if (lane == 0) {
      uint32_t issued = 0;
      Ring<WSTAGES> wr;
      for (int tile = unit0; tile < num_tiles; tile += unit_stride) {
        const TileRef t = src.at(tile, rank, plan);
        // dense FP32 weights are read by the converters themselves
        const bool has_w = t.n_tile < PQ8_TP(t, n_tiles) && !(!SEQ && p.w_f32);
        const uint8_t* wt = PQ8_TP(t, w) + PQ8_HEADER_BYTES +
                            ((size_t)t.n_tile * PQ8_TP(t, k_blocks) + t.kb0) * kRecordBytes;
        for (int kb = 0; kb < t.kb; ++kb, ++issued, wr.advance(1)) {
          if (!mbar_wait(&wempty[wr.idx], wr.phase ^ 1u, abort_flag, status)) goto w_done;
          if (has_w) {
            mbar_expect_tx(&wfull[wr.idx], kRecordBytes);
            bulk_g2s(ws + wr.idx * kRecordBytes, wt + (size_t)kb * kRecordBytes, kRecordBytes, &wfull[wr.idx]);
          } else {
            mbar_arrive(&wfull[wr.idx]);
          }
        }
      }
    w_done:
      for (uint32_t j = issued > WSTAGES ? issued - WSTAGES : 0; j < issued; ++j)
        mbar_drain(&wfull[j % WSTAGES], (j / WSTAGES) & 1);
    }
  } else if (warp == C::kSchedWarp) {
    // ------------------------------------------------------------- scheduler
    // Does every barrier wait the MMA warp depends on (accumulator free,
    // K blocks converted) and releases it through a two-warp rendezvous
    // every RK K blocks. The MMA warp itself never touches shared memory in
    // its loop: on this part a shared-memory access (an mbarrier test
    // included) by the warp that issues tcgen05.mma is held behind the MMAs
    // that warp has queued, so each wait there costs a drain of the tensor
    // pipe. The OR of the rendezvous carries an abort flag, so both warps
    // always meet the same number of times.
    if (leader) {
      constexpr int RK = C::kRendezvousBlocks;
      // The leader's activation stages are vouched for here unless its
      // converters round them in place (landed, or rounded by the epilogue
      // warps).
      const bool sched_x = !round_x || epi_round_x;
      uint64_t* const xready = epi_round_x ? xround : xfull;
      Ring<ASLOTS> ar;
      Ring<STAGES> xr;
      bool bad = false;
      int local = 0;
      for (int tile = unit0; tile < num_tiles && !bad; tile += unit_stride, ++local) {
        const int KB = src.at(tile, rank, plan).kb;
        const int acc = local % ACC;
        if (lane == 0) bad = !mbar_wait(&acc_empty[acc], ((local / ACC) & 1) ^ 1, abort_flag, status);
        for (int kb0 = 0; kb0 < KB; kb0 += RK) {
          const int nb = KB - kb0 < RK ? KB - kb0 : RK;
          if (lane == 0)
            for (int b = 0; b < nb && !bad; ++b) {
              bad = !mbar_wait(&conv[ar.idx], ar.phase, abort_flag, status);
              if (sched_x) bad = bad || !mbar_wait(&xready[xr.idx], xr.phase, abort_flag, status);
              ar.advance(1);
              xr.advance(1);
            }
          bad = __shfl_sync(0xffffffffu, bad, 0);
          if (rendezvous_or(C::kRendezvousBar, bad)) {
            bad = true;
            break;
          }
        }
      }
    }
  } else if (warp == C::kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    // Whole warp: meets the scheduler once per RK K blocks; lane 0 issues.
    // The operands advance incrementally (descriptor start address, slot
    // column, barrier addresses) to keep the issuing lane's instruction
    // stream short. A sequence's tiles differ in their K-block counts; the
    // tile window reads those of the warp's next 32 tiles at once, since a
    // memory access by this warp would wait behind the MMAs it has queued.
    if (leader) {
      constexpr uint32_t idesc = idesc_tf32(128 * C::kCtas, BN);
      constexpr int RK = C::kRendezvousBlocks;
      constexpr uint32_t kStageDesc = C::kXStageBytes >> 4;  // descriptor start-address units per stage
      const uint64_t desc0 = smem_desc_sw128(smem_addr(xs));
      const uint32_t desc_lo0 = static_cast<uint32_t>(desc0), desc_hi = static_cast<uint32_t>(desc0 >> 32);
      const uint32_t xempty0 = smem_addr(xempty), afree0 = smem_addr(afree);
      const uint32_t a0 = tmem + C::kAColBase;
      int stage = 0, slot = 0;
      bool stop = false;
      int local = 0;
      TileWindow<C::kCtas, SEQ> win{};
      if constexpr (!SEQ) win = TileWindow<C::kCtas, SEQ>{p.m_tiles, p.k_blocks, p.k_splits};
      for (int tile = unit0; tile < num_tiles && !stop; tile += unit_stride, ++local) {
        const int KB = win.get(local, rank, plan).kb;
        const int acc = local % ACC;
        const uint32_t d = tmem + acc * BN;
        for (int kb0 = 0; kb0 < KB; kb0 += RK) {
          const int nb = KB - kb0 < RK ? KB - kb0 : RK;
          if (rendezvous_or(C::kRendezvousBar, false)) {  // the scheduler gave up
            stop = true;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
#pragma unroll
            for (int b = 0; b < RK; ++b) {
              if (b < nb) {
                const uint32_t lo = desc_lo0 + static_cast<uint32_t>(stage) * kStageDesc;
                const uint32_t a = a0 + static_cast<uint32_t>(slot) * 32;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  const uint64_t bdesc = (static_cast<uint64_t>(desc_hi) << 32) | (lo + 2 * j);
                  const uint32_t accumulate = (kb0 + b + j) != 0;
                  if constexpr (PAIR) mma_tf32_ts_pair(d, a + j * 8, bdesc, idesc, accumulate);
                  else mma_tf32_ts(d, a + j * 8, bdesc, idesc, accumulate);
                }
                if constexpr (PAIR) {
                  mma_commit_pair_addr(xempty0 + stage * 8, 0x3);
                  mma_commit_pair_addr(afree0 + slot * 8, 0x3);
                } else {
                  mma_commit_addr(xempty0 + stage * 8);
                  mma_commit_addr(afree0 + slot * 8);
                }
                stage = stage + 1 == STAGES ? 0 : stage + 1;
                slot = slot + 1 == ASLOTS ? 0 : slot + 1;
              }
            }
            if (kb0 + nb == KB) {
              if constexpr (PAIR) mma_commit_pair(&acc_full[acc], 0x3);
              else mma_commit(&acc_full[acc]);
            }
          }
          __syncwarp();
          mma_issued = true;
        }
      }
      if (stop && mma_issued && lane == 0) {
        // Wait (bounded) for the MMAs already issued before the CTA tears down.
        if constexpr (PAIR) mma_commit_pair(drain, 0x1);
        else mma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
  }

  // Split K: the warps other than the epilogue's take part in the cluster
  // barrier that publishes the partials (with nothing to publish) ...
  const bool split_cluster = !SEQ && C::kSplitK && p.k_splits > 1;
  if (split_cluster && warp < C::kEpiWarp0) {
    __syncwarp();
    cluster_arrive_relaxed();
  }
  __syncthreads();
  // The peer must not exit (freeing shared memory the leader's MMAs read) and the
  // tensor memory must not be freed before both CTAs are done.
  if constexpr (PAIR) cluster_sync();
  if (split_cluster) {
    // ... and no split leaves (the bulk copies out of its shared memory still
    // running) before every split has received all of its rows.
    if (warp < C::kEpiWarp0) cluster_wait();
    cluster_sync();
  }
  if (warp == C::kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, C::kTmemCols);
    else tmem_dealloc(tmem, C::kTmemCols);
  }
  if constexpr (SEQ) {
    // The last CTA to finish resets the counters for the next run of the plan.
    int* finished = const_cast<int*>(&hdr->finished);
    __shared__ int last_cta;
    if (threadIdx.x == 0) {
      __threadfence();
      last_cta = atomicAdd(finished, 1) == static_cast<int>(gridDim.x) - 1;
    }
    __syncthreads();
    if (last_cta) {
      __threadfence();
      for (int i = threadIdx.x; i < hdr->n_counters; i += blockDim.x) counters[i] = 0;
      if (threadIdx.x == 0) *finished = 0;
      __threadfence();
    }
  }
}

#undef PQ8_TP

}  // namespace pq8
