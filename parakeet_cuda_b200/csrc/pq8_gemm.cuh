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
// Two pipelines are decoupled: STAGES shared-memory stages (activation tile +
// 4352-byte weight record, filled by TMA, freed by MMA completion) let the
// loads run far ahead, and ASLOTS tensor-memory slots for the converted
// weights (filled by converters, freed by MMA completion) bound how far the
// conversion runs ahead. Weight conversion latency sets the pace, so each
// 32-wide K block is converted by 8 warps (16 values per thread) and two
// converter groups work on alternate K blocks.
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
//   warps 0-15   converters: 2 groups x 8 warps (two per TMEM lane quarter,
//                one per half of the K block)
//   warps 16-23  epilogue: 2 per lane quarter, each half of the columns
//   warp 24      producer: TMA (activation tile) + bulk copy (weight record)
//   warp 25      MMA issuer: 4 x tcgen05.mma (K = 8 each) per K block; owns
//                the tensor-memory allocation
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
          int EPI_COLS_ = 32>
struct GemmCfg {
  static constexpr int BN = BN_, STAGES = STAGES_, ASLOTS = ASLOTS_, ACC = ACC_;
  static constexpr bool PAIR = PAIR_;
  static constexpr int kCtas = PAIR ? 2 : 1;
  static constexpr int kRowsPerCta = BN / kCtas;  // activation rows this CTA loads per stage
  static constexpr int kGroups = GROUPS_;          // converter groups working on alternate K blocks
  static constexpr int kGroupThreads = GROUP_WARPS_ * 32;
  static constexpr int kValuesPerThread = 32 / (GROUP_WARPS_ / 4);  // of the 32 K values of a row
  static constexpr int kEpiCols = EPI_COLS_;       // accumulator columns per tcgen05.ld
  static constexpr int kConvWarps = kGroups * kGroupThreads / 32;
  static constexpr int kEpiWarp0 = kConvWarps;
  static constexpr int kEpiWarps = 8;
  static constexpr int kTmaWarp = kEpiWarp0 + kEpiWarps;
  static constexpr int kMmaWarp = kTmaWarp + 1;
  static constexpr int kThreads = (kMmaWarp + 1) * 32;
  static constexpr int kXStageBytes = kRowsPerCta * 128;  // rows x 32 fp32
  static constexpr int kXOff = 0;
  static constexpr int kWOff = STAGES * kXStageBytes;
  // Epilogue staging: 2 column halves x 2 buffers x [32 activation rows][128 output columns] fp32.
  static constexpr int kOutChunkFloats = 32 * 128;
  static constexpr int kOutOff = kWOff + STAGES * kRecordBytes;
  static constexpr int kBarOff = kOutOff + 4 * kOutChunkFloats * 4;
  static constexpr int kNumBars = 2 * STAGES + 2 * ASLOTS + 2 * ACC + 1;
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
  static_assert(ASLOTS % kGroups == 0, "each converter group owns whole tensor-memory slots");
  static_assert(GROUP_WARPS_ == 4 || GROUP_WARPS_ == 8, "a converter group covers the 4 TMEM lane quarters");
  static_assert(kEpiCols == 32, "the staged epilogue writes 32 activation rows per chunk");
};

// Bounded wait used on the teardown path: ignores the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(a, parity)) {
    if (global_timer_ns() - t0 > kWaitLimitNs) return;
  }
}

__device__ __forceinline__ float silu_fast(float z) { return __fdividef(z, 1.0f + __expf(-z)); }

template <int BN, int STAGES, int ASLOTS, int ACC, bool PAIR, int GROUPS = 2, int GROUP_WARPS = 4, int EPI_COLS = 32>
__global__ void __launch_bounds__(GemmCfg<BN, STAGES, ASLOTS, ACC, PAIR, GROUPS, GROUP_WARPS, EPI_COLS>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_y,
                   const GemmParams p) {
  using C = GemmCfg<BN, STAGES, ASLOTS, ACC, PAIR, GROUPS, GROUP_WARPS, EPI_COLS>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem + C::kXOff;
  uint8_t* ws = smem + C::kWOff;
  float* out_stage = reinterpret_cast<float*>(smem + C::kOutOff);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* conv = empty + STAGES;
  uint64_t* afree = conv + ASLOTS;
  uint64_t* acc_full = afree + ASLOTS;
  uint64_t* acc_empty = acc_full + ACC;
  uint64_t* drain = acc_empty + ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);
  int* bad_flag = reinterpret_cast<int*>(smem + C::kMiscOff + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
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
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < ASLOTS; ++a) {
      mbar_init(&conv[a], C::kGroupThreads * C::kCtas);
      mbar_init(&afree[a], 1);
    }
    for (int a = 0; a < ACC; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], C::kEpiWarps * 32 * C::kCtas);
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

  if (warp < C::kConvWarps) {
    // ------------------------------------------------------------ converters
    const int grp = warp / (C::kGroupThreads / 32);
    const int gt = threadIdx.x % C::kGroupThreads;     // thread index within the group
    const int quarter = warp & 3;                      // TMEM lane quarter of this warp
    const int kpart = (warp >> 2) % (GROUP_WARPS / 4); // which kValuesPerThread of the 32 K values
    const int row = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const bool round_x = !(p.flags & PQ8_FLAG_X_TF32);
    uint32_t it = 0;
    for (int tile = unit0; tile < num_tiles; tile += unit_stride) {
      const bool has_w = (tile / p.m_tiles) * C::kCtas + static_cast<int>(rank) < p.n_tiles;
      for (int kb = 0; kb < KB; ++kb, ++it) {
        if (static_cast<int>(it % C::kGroups) != grp) continue;
        const int stage = it % STAGES;
        const int slot = it % ASLOTS;
        if (!mbar_wait(&full[stage], (it / STAGES) & 1, abort_flag, p.status)) goto conv_done;
        if (!mbar_wait(&afree[slot], ((it / ASLOTS) & 1) ^ 1, abort_flag, p.status)) goto conv_done;
        {
          const uint8_t* rec = ws + stage * kRecordBytes;
          const float sc = has_w ? __half2float(*reinterpret_cast<const __half*>(rec + kScaleOffset + row * 2)) : 0.f;
#pragma unroll
          for (int h = 0; h < C::kValuesPerThread / 16; ++h) {
            const int khalf = kpart * (C::kValuesPerThread / 16) + h;  // 16-value half of the K block
            uint32_t a[16];
            if (has_w) {
              const uint4 q = *reinterpret_cast<const uint4*>(rec + khalf * 2048 + row * 16);
              const uint32_t wd[4] = {q.x ^ 0x80808080u, q.y ^ 0x80808080u, q.z ^ 0x80808080u,
                                      q.w ^ 0x80808080u};
#pragma unroll
              for (int i = 0; i < 16; ++i)
                a[i] = tf32_round_bits(__float_as_uint(i8_to_f32(wd[i >> 2], i & 3) * sc));
            } else {
              // Odd tile count: the peer of the last pair multiplies zeros.
#pragma unroll
              for (int i = 0; i < 16; ++i) a[i] = 0;
            }
            tmem_st16(tmem + lane_base + C::kAColBase + slot * 32 + khalf * 16, a);
          }
        }
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
        tmem_wait_st();
        tc_fence_before();
        if (PAIR && !leader) mbar_arrive_cluster(conv_remote + slot * 8);
        else mbar_arrive(&conv[slot]);
      }
    }
  conv_done:;
  } else if (warp < C::kEpiWarp0 + C::kEpiWarps) {
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
    for (int tile = unit0; tile < num_tiles; tile += unit_stride, ++local) {
      const int n_tile = (tile / p.m_tiles) * C::kCtas + static_cast<int>(rank), m_tile = tile % p.m_tiles;
      const int acc = local % ACC;
      if (!mbar_wait(&acc_full[acc], (local / ACC) & 1, abort_flag, p.status)) break;
      tc_fence_after();
      RowMap rm;
      const bool valid = map_row(p.layout, p.n, n_tile * kTileRows + r, rm);
      const float b = (p.bias != nullptr && valid) ? p.bias[rm.src] : 0.0f;
      const bool store_lane = valid && (!glu || lane < 16);
      float* ycol = p.y + rm.col;
      const float* rcol = p.resid + rm.col;
#pragma unroll 1
      for (int cc = 0; cc < kChunks; ++cc, ++chunk_seq) {
        const int c = half * kChunks + cc;
        const int m0 = m_tile * BN + c * E;
        if (m0 >= p.m) break;
        uint32_t v[E];
        tmem_ld32(tmem + lane_base + acc * BN + c * E, v);
        tmem_wait_ld();
        const int cnt = min(E, p.m - m0);  // warp-uniform
        float out[E];
        if (p.epi == PQ8_EPI_RESIDUAL) {
#pragma unroll
          for (int j = 0; j < E; ++j)
            out[j] = (store_lane && j < cnt) ? rcol[(size_t)(m0 + j) * p.out_cols] : 0.0f;
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
      }
      tc_fence_before();
      if (PAIR && !leader) mbar_arrive_cluster(acc_empty_remote + acc * 8);
      else mbar_arrive(&acc_empty[acc]);
    }
    if (p.tma_store && elected) bulk_wait_group_all();
  } else if (warp == C::kTmaWarp) {
    // -------------------------------------------------------------- producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int tile = unit0; tile < num_tiles; tile += unit_stride) {
        const int n_tile = (tile / p.m_tiles) * C::kCtas + static_cast<int>(rank), m_tile = tile % p.m_tiles;
        const bool has_w = n_tile < p.n_tiles;
        const uint8_t* wt = p.w + PQ8_HEADER_BYTES + (size_t)n_tile * KB * kRecordBytes;
        const int row0 = m_tile * BN + static_cast<int>(rank) * C::kRowsPerCta;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int stage = it % STAGES;
          if (!mbar_wait(&empty[stage], ((it / STAGES) & 1) ^ 1, abort_flag, p.status)) goto tma_done;
          mbar_expect_tx(&full[stage], C::kXStageBytes + (has_w ? kRecordBytes : 0));
          tma_load_2d(xs + stage * C::kXStageBytes, &tmap_x, kb * 32, row0, &full[stage]);
          if (has_w)
            bulk_g2s(ws + stage * kRecordBytes, wt + (size_t)kb * kRecordBytes, kRecordBytes, &full[stage]);
        }
      }
    tma_done:
      // Never leave the CTA with copies still landing in its shared memory.
      for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; ++j) mbar_drain(&full[j % STAGES], (j / STAGES) & 1);
    }
  } else {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t idesc = idesc_tf32(128 * C::kCtas, BN);
      uint32_t it = 0;
      int local = 0;
      for (int tile = unit0; tile < num_tiles; tile += unit_stride, ++local) {
        const int acc = local % ACC;
        if (!mbar_wait(&acc_empty[acc], ((local / ACC) & 1) ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int stage = it % STAGES;
          const int slot = it % ASLOTS;
          if (!mbar_wait(&conv[slot], (it / ASLOTS) & 1, abort_flag, p.status)) goto mma_done;
          tc_fence_after();
          const uint64_t bdesc = smem_desc_sw128(smem_addr(xs + stage * C::kXStageBytes));
          const uint32_t a = tmem + C::kAColBase + slot * 32;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if constexpr (PAIR) mma_tf32_ts_pair(d, a + j * 8, bdesc + 2 * j, idesc, (kb | j) != 0);
            else mma_tf32_ts(d, a + j * 8, bdesc + 2 * j, idesc, (kb | j) != 0);
          }
          mma_issued = true;
          if constexpr (PAIR) {
            mma_commit_pair(&empty[stage], 0x3);
            mma_commit_pair(&afree[slot], 0x3);
          } else {
            mma_commit(&empty[stage]);
            mma_commit(&afree[slot]);
          }
        }
        if constexpr (PAIR) mma_commit_pair(&acc_full[acc], 0x3);
        else mma_commit(&acc_full[acc]);
      }
    mma_done:
      if (*abort_flag && mma_issued) {
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
