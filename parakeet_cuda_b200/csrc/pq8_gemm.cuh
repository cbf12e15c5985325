// Q8_0 x FP32 GEMM on the 5th-generation tensor cores (tcgen05, kind::tf32).
//
// Y[m, j] = epilogue(sum_k X[m, k] * W[j, k] + bias[j]) for a packed Q8_0 W.
//
// Roles are swapped relative to the output: the MMA "M" dimension is 128
// weight rows (operand A, dequantised to TF32 by converter warps and written
// straight into tensor memory with tcgen05.st), the MMA "N" dimension is BN
// activation rows (operand B, FP32 tiles streamed by TMA into 128-byte
// swizzled shared memory and rounded to TF32 in place). The accumulator
// D[weight row, activation row] lives in tensor memory; each epilogue thread
// owns one weight row, so a warp's stores cover 32 consecutive output columns
// of one activation row (coalesced 128-byte writes). Keeping the expanded
// weights out of shared memory leaves shared-memory bandwidth to the FP32
// activations, which dominate it.
//
// Warp roles (448 threads, one persistent CTA per SM):
//   warps 0-7  converters: W record -> TF32 -> TMEM (A slot); X stage -> TF32 in place
//   warps 8-11 epilogue:   TMEM accumulator -> bias/activation/residual/GLU -> global
//   warp 12    producer:   TMA (X tile) + bulk copy (4352-byte W record) per K block
//   warp 13    MMA issuer: 4 x tcgen05.mma (K = 8 each) per 32-wide K block; TMEM owner
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
};

template <int BN_, int STAGES_, int ACC_>
struct GemmCfg {
  static constexpr int BN = BN_, STAGES = STAGES_, ACC = ACC_;
  static constexpr int kConvWarps = 8;
  static constexpr int kEpiWarp0 = 8;
  static constexpr int kTmaWarp = 12;
  static constexpr int kMmaWarp = 13;
  static constexpr int kThreads = 14 * 32;
  static constexpr int kXStageBytes = BN * 128;  // BN rows x 32 fp32
  static constexpr int kXOff = 0;
  static constexpr int kWOff = STAGES * kXStageBytes;
  static constexpr int kBarOff = kWOff + STAGES * kRecordBytes;
  static constexpr int kNumBars = 3 * STAGES + 2 * ACC + 1;
  static constexpr int kMiscOff = kBarOff + kNumBars * 8;
  static constexpr int kUsedBytes = kMiscOff + 16;
  static constexpr int kAColBase = ACC * BN;
  static constexpr int kColsNeeded = ACC * BN + STAGES * 32;
  static constexpr int kTmemCols = kColsNeeded <= 32 ? 32 : kColsNeeded <= 64 ? 64 : kColsNeeded <= 128 ? 128
                                   : kColsNeeded <= 256 ? 256 : 512;
  // Reserve enough shared memory that no more CTAs share an SM than its
  // 512 tensor-memory columns can hold, so tcgen05.alloc never has to wait.
  static constexpr int kMinSmem = (512 / kTmemCols) <= 1 ? 120 * 1024 : (512 / kTmemCols) == 2 ? 80 * 1024 : 0;
  static constexpr int kSmemBytes = (kUsedBytes + 1024 > kMinSmem ? kUsedBytes + 1024 : kMinSmem);
  static_assert(kColsNeeded <= 512, "tensor memory overflow");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN must be a multiple of 32 in [32, 256]");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory overflow");
};

// Bounded wait used on the teardown path: ignores the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(a, parity)) {
    if (global_timer_ns() - t0 > kWaitLimitNs) return;
  }
}

template <int BN, int STAGES, int ACC>
__global__ void __launch_bounds__(GemmCfg<BN, STAGES, ACC>::kThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const GemmParams p) {
  using C = GemmCfg<BN, STAGES, ACC>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* xs = smem + C::kXOff;
  uint8_t* ws = smem + C::kWOff;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kBarOff);
  uint64_t* conv = full + STAGES;
  uint64_t* empty = conv + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + ACC;
  uint64_t* drain = acc_empty + ACC;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + C::kMiscOff);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kMiscOff + 4);
  int* bad_flag = reinterpret_cast<int*>(smem + C::kMiscOff + 8);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    const PackedHeader* h = reinterpret_cast<const PackedHeader*>(p.w);
    const bool ok = h->magic == kMagic && h->n == p.n && h->k == p.k && h->layout == p.layout &&
                    h->n_tiles == p.n_tiles;
    *bad_flag = ok ? 0 : 1;
    *abort_flag = 0;
    if (!ok) atomicCAS(p.status, 0, PQ8_ERR_LAYOUT);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], C::kConvWarps * 32);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < ACC; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == C::kTmaWarp && lane == 0) prefetch_tmap(&tmap_x);
  __syncthreads();
  if (*bad_flag) return;
  if (warp == C::kMmaWarp) {
    tmem_alloc(tmem_slot, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  const int num_tiles = p.n_tiles * p.m_tiles;
  const int KB = p.k_blocks;
  bool mma_issued = false;

  if (warp < C::kConvWarps) {
    // ------------------------------------------------------------ converters
    const int ct = threadIdx.x;  // 0..255
    const int row = ct & 127, half = ct >> 7;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const bool round_x = !(p.flags & PQ8_FLAG_X_TF32);
    uint32_t it = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      for (int kb = 0; kb < KB; ++kb, ++it) {
        const int stage = it % STAGES;
        const uint32_t phase = (it / STAGES) & 1;
        if (!mbar_wait(&full[stage], phase, abort_flag, p.status)) goto conv_done;
        {
          const uint8_t* rec = ws + stage * kRecordBytes;
          const uint4 qv = *reinterpret_cast<const uint4*>(rec + half * 2048 + row * 16);
          const float sc = __half2float(*reinterpret_cast<const __half*>(rec + kScaleOffset + row * 2));
          const uint32_t wd[4] = {qv.x ^ 0x80808080u, qv.y ^ 0x80808080u, qv.z ^ 0x80808080u,
                                  qv.w ^ 0x80808080u};
          uint32_t a[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) a[i] = tf32_round_bits(__float_as_uint(i8_to_f32(wd[i >> 2], i & 3) * sc));
          tmem_st16(tmem + lane_base + C::kAColBase + stage * 32 + half * 16, a);
        }
        if (round_x) {
          uint4* xv = reinterpret_cast<uint4*>(xs + stage * C::kXStageBytes);
#pragma unroll 4
          for (int i = ct; i < C::kXStageBytes / 16; i += C::kConvWarps * 32) {
            uint4 v = xv[i];
            v.x = tf32_round_bits(v.x);
            v.y = tf32_round_bits(v.y);
            v.z = tf32_round_bits(v.z);
            v.w = tf32_round_bits(v.w);
            xv[i] = v;
          }
          fence_proxy_async_smem();
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&conv[stage]);
      }
    }
  conv_done:;
  } else if (warp < C::kEpiWarp0 + 4) {
    // -------------------------------------------------------------- epilogue
    const int ew = warp - C::kEpiWarp0;  // TMEM lane quarter (== warp % 4)
    const int r = ew * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(ew * 32) << 16;
    int local = 0;
    for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const int n_tile = tile / p.m_tiles, m_tile = tile % p.m_tiles;
      const int acc = local % ACC;
      if (!mbar_wait(&acc_full[acc], (local / ACC) & 1, abort_flag, p.status)) break;
      tc_fence_after();
      RowMap rm;
      const bool valid = map_row(p.layout, p.n, n_tile * kTileRows + r, rm);
      const float b = (p.bias != nullptr && valid) ? p.bias[rm.src] : 0.0f;
      const bool store_lane = valid && (p.epi != PQ8_EPI_GLU || lane < 16);
      float* ycol = p.y + rm.col;
      const float* rcol = p.resid + rm.col;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int m0 = m_tile * BN + c * 32;
        if (m0 >= p.m) break;
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + acc * BN + c * 32, v);
        tmem_wait_ld();
        const int cnt = min(32, p.m - m0);  // warp-uniform
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if (j >= cnt) break;
          const float z = __uint_as_float(v[j]) + b;
          float out;
          if (p.epi == PQ8_EPI_GLU) {
            const float gate = __shfl_down_sync(0xffffffffu, z, 16);
            out = z * sigmoidf_(gate);
          } else if (p.epi == PQ8_EPI_RESIDUAL) {
            out = rcol[(size_t)(m0 + j) * p.out_cols] + p.alpha * z;
          } else {
            out = apply_act(z, p.epi);
          }
          if (p.flags & PQ8_FLAG_OUT_TF32) out = tf32_round(out);
          if (store_lane) ycol[(size_t)(m0 + j) * p.out_cols] = out;
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
    }
  } else if (warp == C::kTmaWarp) {
    // -------------------------------------------------------------- producer
    if (lane == 0) {
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
        const int n_tile = tile / p.m_tiles, m_tile = tile % p.m_tiles;
        const uint8_t* wt = p.w + PQ8_HEADER_BYTES + (size_t)n_tile * KB * kRecordBytes;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int stage = it % STAGES;
          const uint32_t phase = (it / STAGES) & 1;
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, p.status)) goto tma_done;
          mbar_expect_tx(&full[stage], C::kXStageBytes + kRecordBytes);
          tma_load_2d(xs + stage * C::kXStageBytes, &tmap_x, kb * 32, m_tile * BN, &full[stage]);
          bulk_g2s(ws + stage * kRecordBytes, wt + (size_t)kb * kRecordBytes, kRecordBytes, &full[stage]);
        }
      }
    tma_done:
      // Never leave the CTA with copies still landing in its shared memory.
      for (uint32_t j = it > STAGES ? it - STAGES : 0; j < it; ++j) mbar_drain(&full[j % STAGES], (j / STAGES) & 1);
    }
  } else {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_tf32(128, BN);
      uint32_t it = 0;
      int local = 0;
      for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
        const int acc = local % ACC;
        if (!mbar_wait(&acc_empty[acc], ((local / ACC) & 1) ^ 1, abort_flag, p.status)) break;
        tc_fence_after();
        const uint32_t d = tmem + acc * BN;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int stage = it % STAGES;
          const uint32_t phase = (it / STAGES) & 1;
          if (!mbar_wait(&conv[stage], phase, abort_flag, p.status)) goto mma_done;
          tc_fence_after();
          const uint64_t bdesc = smem_desc_sw128(smem_addr(xs + stage * C::kXStageBytes));
          const uint32_t a = tmem + C::kAColBase + stage * 32;
#pragma unroll
          for (int j = 0; j < 4; ++j) mma_tf32_ts(d, a + j * 8, bdesc + 2 * j, idesc, (kb | j) != 0);
          mma_issued = true;
          mma_commit(&empty[stage]);
        }
        mma_commit(&acc_full[acc]);
      }
    mma_done:
      if (*abort_flag && mma_issued) {
        mma_commit(drain);
        mbar_drain(drain, 0);
      }
    }
  }

  __syncthreads();
  if (warp == C::kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
}

}  // namespace pq8
