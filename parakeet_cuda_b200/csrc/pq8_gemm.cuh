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
  static constexpr int kNumBars = 2 * STAGES + 2 * WSTAGES + 2 * ASLOTS + 2 * ACC + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kUsedBytes = kMiscOff + 16;
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

template <int BN, int STAGES, int ASLOTS, int ACC, bool PAIR, int GROUPS = 2, int GROUP_WARPS = 4, int EPI_COLS = 32,
          int WSTAGES = 4>
__global__ void __launch_bounds__(GemmCfg<BN, STAGES, ASLOTS, ACC, PAIR, GROUPS, GROUP_WARPS, EPI_COLS, WSTAGES>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_y,
                   const GemmParams p) {
  using C = GemmCfg<BN, STAGES, ASLOTS, ACC, PAIR, GROUPS, GROUP_WARPS, EPI_COLS, WSTAGES>;
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
  const int unit0 = blockIdx.x / C::kCtas;          // first work unit of this CTA (pair)
  const int unit_stride = gridDim.x / C::kCtas;

  if (threadIdx.x == 0) {
    const PackedHeader* h = reinterpret_cast<const PackedHeader*>(p.w);
    const bool ok = h->magic == kMagic && h->n == p.n && h->k == p.k && h->layout == p.layout &&
                    h->n_tiles == p.n_tiles;
    *bad_flag = ok ? 0 : 1;
    *abort_flag = 0;
    if (!ok) atomicCAS(p.status, 0, PQ8_ERR_LAYOUT);
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
    fence_mbar_init();
  }
  if (warp == C::kTmaWarp && lane == 0) {
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

  // Work units: 128 * kCtas weight rows x BN activation rows.
  const int n_units = PAIR ? (p.n_tiles + 1) / 2 : p.n_tiles;
  const int num_tiles = n_units * p.m_tiles;
  const int KB = p.k_blocks;
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
    const bool round_x = !(p.flags & PQ8_FLAG_X_TF32);
    // Who vouches for this CTA's activation stage before the MMA: the
    // converters when they round it in place or when they are the pair peer's
    // (whose barriers the leader cannot see); otherwise the scheduler.
    const bool vouch_x = round_x || (PAIR && !leader);
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
    bool w_ready = false;
    int tile = unit0;
    uint32_t tile_first = 0;  // index of the current tile's first K block
    bool has_w = tile < num_tiles && (tile / p.m_tiles) * C::kCtas + static_cast<int>(rank) < p.n_tiles;
    for (uint32_t it = grp;; it += G) {
      while (it >= tile_first + KB) {
        tile += unit_stride;
        tile_first += KB;
        has_w = (tile / p.m_tiles) * C::kCtas + static_cast<int>(rank) < p.n_tiles;
      }
      if (tile >= num_tiles) break;
      const uint32_t stage = xr.idx, wst = wr.idx, slot = ar.idx;
      // The weight record is converted into registers and only then released:
      // the refill is an async-proxy write, which an mbarrier release does not
      // order after this warp's shared-memory loads, so the stage is handed
      // back once the conversion has consumed every loaded value. The
      // conversion runs before the tensor-memory slot is waited for.
      if (!w_ready && !mbar_wait(&wfull[wst], wr.phase, abort_flag, p.status)) goto conv_done;
      uint32_t a[C::kValuesPerThread];
      bool slot_ready;
      {
        constexpr int H = C::kValuesPerThread / 16;
        uint4 q[H];
        uint32_t sbits = 0;
        if (has_w) {
          const uint8_t* rec = ws + wst * kRecordBytes;
          sbits = *reinterpret_cast<const uint16_t*>(rec + kScaleOffset + row * 2);
#pragma unroll
          for (int h = 0; h < H; ++h)  // 16-value halves of the K block
            q[h] = *reinterpret_cast<const uint4*>(rec + (kpart * H + h) * 2048 + row * 16);
        }
        slot_ready = mbar_test_wait(smem_addr(&afree[slot]), ar.phase ^ 1u);
        if (has_w) {
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
      if (!slot_ready && !mbar_wait(&afree[slot], ar.phase ^ 1u, abort_flag, p.status)) goto conv_done;
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
        if (!mbar_wait(&xfull[stage], xr.phase, abort_flag, p.status)) goto conv_done;
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
    const bool glu = p.epi == PQ8_EPI_GLU;
    const int box_cols = glu ? 64 : 128;           // output columns of one tile
    const int c_local = glu ? q * 16 + (lane & 15) : r;
    constexpr int E = C::kEpiCols;
    constexpr int kChunks = BN / E / 2;            // E-column chunks per half
    int chunk_seq = 0;                             // chunks issued by this half (selects the buffer)
    int local = 0;
    griddep_wait();  // the residual and the output may be in use by the previous kernel
    for (int tile = unit0; tile < num_tiles; tile += unit_stride, ++local) {
      const int n_tile = (tile / p.m_tiles) * C::kCtas + static_cast<int>(rank), m_tile = tile % p.m_tiles;
      const int acc = local % ACC;
      RowMap rm;
      const bool valid = map_row(p.layout, p.n, n_tile * kTileRows + r, rm);
      const float b = (p.bias != nullptr && valid) ? p.bias[rm.src] : 0.0f;
      const bool store_lane = valid && (!glu || lane < 16);
      float* ycol = p.y + rm.col;
      const float* rcol = p.resid + rm.col;
      const bool resid = p.epi == PQ8_EPI_RESIDUAL;
      // Residual rows are loaded into out[] one chunk ahead: the tile's first
      // chunk before the accumulator is waited for, each next chunk as soon as
      // the previous one has been staged, so their latency is off the critical
      // path (they are other rows than any store still in flight).
      float out[E];
      auto load_resid = [&](int m0) {
#pragma unroll
        for (int j = 0; j < E; ++j)
          out[j] = (store_lane && m0 + j < p.m) ? rcol[(size_t)(m0 + j) * p.out_cols] : 0.0f;
      };
      if (resid) load_resid(m_tile * BN + half * kChunks * E);
      if (!mbar_wait(&acc_full[acc], (local / ACC) & 1, abort_flag, p.status)) break;
      tc_fence_after();
#pragma unroll 1
      for (int cc = 0; cc < kChunks; ++cc, ++chunk_seq) {
        const int c = half * kChunks + cc;
        const int m0 = m_tile * BN + c * E;
        if (m0 >= p.m) break;
        uint32_t v[E];
        tmem_ld32(tmem + lane_base + acc * BN + c * E, v);
        tmem_wait_ld();
        const int cnt = min(E, p.m - m0);  // warp-uniform
        if (resid) {
#pragma unroll
          for (int j = 0; j < E; ++j) out[j] = fmaf(p.alpha, __uint_as_float(v[j]) + b, out[j]);
        } else if (glu) {
#pragma unroll
          for (int j = 0; j < E; ++j) {
            const float z = __uint_as_float(v[j]) + b;
            const float gate = __shfl_down_sync(0xffffffffu, z, 16);
            out[j] = __fdividef(z, 1.0f + __expf(-gate));
          }
        } else if (p.epi == PQ8_EPI_SILU) {
#pragma unroll
          for (int j = 0; j < E; ++j) out[j] = silu_fast(__uint_as_float(v[j]) + b);
        } else if (p.epi == PQ8_EPI_RELU) {
#pragma unroll
          for (int j = 0; j < E; ++j) out[j] = fmaxf(__uint_as_float(v[j]) + b, 0.0f);
        } else {
#pragma unroll
          for (int j = 0; j < E; ++j) out[j] = __uint_as_float(v[j]) + b;
        }
        if (p.flags & PQ8_FLAG_OUT_TF32) {
#pragma unroll
          for (int j = 0; j < E; ++j) out[j] = tf32_round(out[j]);
        }
        if (p.tma_store) {
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
            tma_store_2d(&tmap_y, stage, n_tile * box_cols, m0);
            bulk_commit_group();
          }
        } else if (store_lane) {
          float* yp = ycol + (size_t)m0 * p.out_cols;
#pragma unroll
          for (int j = 0; j < E; ++j)
            if (j < cnt) yp[(size_t)j * p.out_cols] = out[j];
        }
        if (resid && cc + 1 < kChunks) load_resid(m0 + E);
      }
      tc_fence_before();
      __syncwarp();  // every lane's accumulator loads are complete: one arrival per warp
      if (lane == 0) {
        if (PAIR && !leader) mbar_arrive_cluster(acc_empty_remote + acc * 8);
        else mbar_arrive(&acc_empty[acc]);
      }
    }
    if (p.tma_store && elected) bulk_wait_group_all();
  } else if (warp == C::kTmaWarp) {
    // ----------------------------------------------------- activation producer
    if (lane == 0) {
      griddep_wait();  // the activations may come from the previous kernel
      uint32_t issued = 0;
      Ring<STAGES> xr;
      for (int tile = unit0; tile < num_tiles; tile += unit_stride) {
        const int m_tile = tile % p.m_tiles;
        const int row0 = m_tile * BN + static_cast<int>(rank) * C::kRowsPerCta;
        for (int kb = 0; kb < KB; ++kb, ++issued, xr.advance(1)) {
          if (!mbar_wait(&xempty[xr.idx], xr.phase ^ 1u, abort_flag, p.status)) goto x_done;
          mbar_expect_tx(&xfull[xr.idx], C::kXStageBytes);
          tma_load_2d(xs + xr.idx * C::kXStageBytes, &tmap_x, kb * 32, row0, &xfull[xr.idx]);
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
        const int n_tile = (tile / p.m_tiles) * C::kCtas + static_cast<int>(rank);
        const bool has_w = n_tile < p.n_tiles;
        const uint8_t* wt = p.w + PQ8_HEADER_BYTES + (size_t)n_tile * KB * kRecordBytes;
        for (int kb = 0; kb < KB; ++kb, ++issued, wr.advance(1)) {
          if (!mbar_wait(&wempty[wr.idx], wr.phase ^ 1u, abort_flag, p.status)) goto w_done;
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
    // K blocks converted) and releases it through a two-warp rendezvous. The
    // MMA warp itself never touches shared memory in its loop: on this part a
    // shared-memory access (an mbarrier test included) by the warp that issues
    // tcgen05.mma is held behind the MMAs that warp has queued, so each wait
    // there costs a drain of the tensor pipe.
    if (leader) {
      constexpr int RK = C::kRendezvousBlocks;
      // The leader's activation stages are vouched for here unless its
      // converters round them in place.
      const bool sched_x = (p.flags & PQ8_FLAG_X_TF32) != 0;
      Ring<ASLOTS> ar;
      Ring<STAGES> xr;
      bool bad = false;
      int local = 0;
      for (int tile = unit0; tile < num_tiles && !bad; tile += unit_stride, ++local) {
        const int acc = local % ACC;
        if (lane == 0) bad = !mbar_wait(&acc_empty[acc], ((local / ACC) & 1) ^ 1, abort_flag, p.status);
        for (int kb0 = 0; kb0 < KB; kb0 += RK) {
          const int nb = KB - kb0 < RK ? KB - kb0 : RK;
          if (lane == 0)
            for (int b = 0; b < nb && !bad; ++b) {
              bad = !mbar_wait(&conv[ar.idx], ar.phase, abort_flag, p.status);
              if (sched_x) bad = bad || !mbar_wait(&xfull[xr.idx], xr.phase, abort_flag, p.status);
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
    // stream short.
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
      for (int tile = unit0; tile < num_tiles && !stop; tile += unit_stride, ++local) {
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

  __syncthreads();
  // The peer must not exit (freeing shared memory the leader's MMAs read) and the
  // tensor memory must not be freed before both CTAs are done.
  if constexpr (PAIR) cluster_sync();
  if (warp == C::kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    if constexpr (PAIR) tmem_dealloc_pair(tmem, C::kTmemCols);
    else tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace pq8
