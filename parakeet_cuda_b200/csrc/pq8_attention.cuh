// Fused relative-position attention on the 5th-generation tensor cores
// (parakeet_cuda/reference.py:51-58; rel_scores and softmax in
// runtime.cu:122-137, the three batched products in gpu.py:92-100).
//
// One CTA per (window, head, 128 queries), 128 threads: thread r owns query
// row r, which is also TMEM lane r of every accumulator. Per tile of 64 keys:
//   S  = (Q + u) K^T         128 x 64   tcgen05.mma kind::f16, TMEM cols [0, 64)
//   BD = (Q + v) Band^T      128 x 192  (three MMAs of 64 positions each), TMEM cols [64, 256)
// where Band holds the 192 positional rows t-1+j-i the tile's (i, j) pairs
// need: query i and key j read band column j - i + 127. Each thread loads its
// row of S and a 96-column window of BD (the window of its warp's 32 rows),
// moves its own 64 band columns into place with a 5-stage register barrel
// shift (offset 31 - lane), and runs the online softmax over the row in
// registers. The probabilities go to shared memory as FP16 (the A operand of
//   O += P V^T               128 x 128  TMEM cols [256, 384)
// and O is rescaled in TMEM when a row's maximum grows.
//
// Operands are staged as FP16 (the 11-bit significand TF32 keeps; FP32
// accumulation) in the canonical K-major 128-byte-swizzled layout: row r of
// a tile is 128 bytes per 64 elements, its 16-byte chunk c stored at chunk
// c ^ (r % 8), atoms of 8 rows 1024 bytes apart. V is staged transposed
// (rows = head dimensions, K = keys). The positional band is a ring of three
// 64-row slabs: consecutive key tiles share two of them, so after the first
// tile one slab is staged per tile. One thread issues the MMAs; tcgen05
// commits signal completion on mbarriers that every thread waits on (bounded
// waits, PQ8_ERR_TIMEOUT in the device status word).
#pragma once

#include "pq8_device.cuh"

namespace pq8 {

constexpr int kTcQ = 128, kTcKeys = 64, kTcD = 128;
constexpr int kTcThreads = 128;
constexpr int kTcQuOff = 0;                        // [2 atoms][128 rows][128 B]
constexpr int kTcQvOff = kTcQuOff + 2 * 128 * 128;
constexpr int kTcKOff = kTcQvOff + 2 * 128 * 128;  // [2 atoms][64 keys][128 B]
constexpr int kTcVtOff = kTcKOff + 2 * 64 * 128;   // [128 dims][128 B = 64 keys]
constexpr int kTcBandOff = kTcVtOff + 128 * 128;   // 3 slabs x [2 atoms][64 rows][128 B]
constexpr int kTcSlabBytes = 2 * 64 * 128;
constexpr int kTcPOff = kTcBandOff + 3 * kTcSlabBytes;  // [128 rows][128 B = 64 keys]
constexpr int kTcBarOff = kTcPOff + 128 * 128;
constexpr int kTcSmemBytes = kTcBarOff + 64 + 1024;  // + 1024-byte alignment slack
constexpr uint32_t kTcColS = 0, kTcColBd = 64, kTcColO = 256, kTcTmemCols = 512;

// Instruction descriptor: kind::f16 with FP16 A and B (both K-major), FP32 accumulate, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16, one CTA. Issued by one thread.
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Each thread of the warp writes 32 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
      "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
      "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a 128-byte-swizzled atom column.
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// 8 floats (two float4) as one 16-byte FP16 chunk.
__device__ __forceinline__ uint4 pack_h8(const float4 a, const float4 b) {
  return make_uint4(pack_h2(a.x, a.y), pack_h2(a.z, a.w), pack_h2(b.x, b.y), pack_h2(b.z, b.w));
}

// Rows [0, rows) x 128 dimensions of an FP32 source (row r at src(r), NULL =
// zero row) into a K-major FP16 tile of `rows` rows (two atom columns of 64
// dimensions). Every load of a thread is issued before any store.
template <int ROWS, typename SrcFn>
__device__ __forceinline__ void stage_kmajor(uint8_t* tile, SrcFn src) {
  constexpr int kItems = ROWS * 16 / kTcThreads;  // (row, 8-dimension chunk) per thread
  float4 va[kItems], vb[kItems];
#pragma unroll
  for (int q = 0; q < kItems; ++q) {
    const int item = q * kTcThreads + static_cast<int>(threadIdx.x);
    const int r = item >> 4, c16 = item & 15;
    const float* s = src(r);
    if (s != nullptr) {
      va[q] = *reinterpret_cast<const float4*>(s + c16 * 8);
      vb[q] = *reinterpret_cast<const float4*>(s + c16 * 8 + 4);
    } else {
      va[q] = vb[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
  }
#pragma unroll
  for (int q = 0; q < kItems; ++q) {
    const int item = q * kTcThreads + static_cast<int>(threadIdx.x);
    const int r = item >> 4, c16 = item & 15;
    *reinterpret_cast<uint4*>(tile + (c16 >> 3) * (ROWS * 128) + sw128(r, c16 & 7)) = pack_h8(va[q], vb[q]);
  }
}

__global__ void __launch_bounds__(kTcThreads, 1)
    rel_attention_tc_kernel(const float* __restrict__ qkv, const float* __restrict__ pos,
                            const float* __restrict__ pos_bias_u, const float* __restrict__ pos_bias_v,
                            float* __restrict__ ctx, int t, int round_out, int* status) {
  griddep_launch();
  extern __shared__ uint8_t att_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(att_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(sm);
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + kTcBarOff);
  uint64_t* bar_pv = bar_s + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_s + 3);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int i0 = blockIdx.x * kTcQ, h = blockIdx.y, win = blockIdx.z;
  const size_t row_base = static_cast<size_t>(win) * t;
  const int n_pos = 2 * t - 1;

  if (tid == 0) {
    mbar_init(bar_s, 1);
    mbar_init(bar_pv, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTcTmemCols);
    tmem_relinquish();
  }
  griddep_wait();  // qkv comes from the previous kernel

  // Queries with each positional bias (rows past t are zero).
  {
    constexpr int kItems = kTcQ * 16 / kTcThreads;
    float4 xa[kItems], xb[kItems];
#pragma unroll
    for (int q = 0; q < kItems; ++q) {
      const int item = q * kTcThreads + tid, r = item >> 4, c16 = item & 15;
      if (i0 + r < t) {
        const float* s = qkv + (row_base + i0 + r) * 3072 + h * kTcD + c16 * 8;
        xa[q] = *reinterpret_cast<const float4*>(s);
        xb[q] = *reinterpret_cast<const float4*>(s + 4);
      } else {
        xa[q] = xb[q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
    }
#pragma unroll
    for (int q = 0; q < kItems; ++q) {
      const int item = q * kTcThreads + tid, r = item >> 4, c16 = item & 15;
      const float* u = pos_bias_u + h * kTcD + c16 * 8;
      const float* v = pos_bias_v + h * kTcD + c16 * 8;
      const float4 ua = *reinterpret_cast<const float4*>(u), ub = *reinterpret_cast<const float4*>(u + 4);
      const float4 va = *reinterpret_cast<const float4*>(v), vb = *reinterpret_cast<const float4*>(v + 4);
      const float4 a = xa[q], b = xb[q];
      const uint32_t off = (c16 >> 3) * (kTcQ * 128) + sw128(r, c16 & 7);
      *reinterpret_cast<uint4*>(sm + kTcQuOff + off) =
          pack_h8(make_float4(a.x + ua.x, a.y + ua.y, a.z + ua.z, a.w + ua.w),
                  make_float4(b.x + ub.x, b.y + ub.y, b.z + ub.z, b.w + ub.w));
      *reinterpret_cast<uint4*>(sm + kTcQvOff + off) =
          pack_h8(make_float4(a.x + va.x, a.y + va.y, a.z + va.z, a.w + va.w),
                  make_float4(b.x + vb.x, b.y + vb.y, b.z + vb.z, b.w + vb.w));
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;

  // Positional slab s holds positions p0 + 64 s + [0, 64): the tile of keys
  // j0 = 64 kt uses slabs kt, kt + 1, kt + 2 (band column c = j - i + 127).
  const int p0 = t - 128 - i0;
  auto stage_slab = [&](int s) {
    stage_kmajor<64>(sm + kTcBandOff + (s % 3) * kTcSlabBytes, [&](int r) -> const float* {
      const int p = p0 + 64 * s + r;
      return (p >= 0 && p < n_pos) ? pos + static_cast<size_t>(p) * 1024 + h * kTcD : nullptr;
    });
  };

  const float kScaleLog2 = 1.4426950408889634f * rsqrtf(128.0f);  // 1/sqrt(128) in base 2
  float m_row = -INFINITY, l_row = 0.0f;
  const int n_tiles = (t + kTcKeys - 1) / kTcKeys;
  bool ok = true;
  int kt = 0, s_issued = 0, pv_issued = 0;  // commits issued (thread 0)
  for (; kt < n_tiles; ++kt) {
    const int j0 = kt * kTcKeys;
    // The previous tile's context product has read V and P.
    if (kt > 0 && !mbar_wait(bar_pv, (kt - 1) & 1, abort_flag, status)) {
      ok = false;
      break;
    }
    // Keys, V transposed, and the new positional slab(s).
    stage_kmajor<64>(sm + kTcKOff, [&](int r) -> const float* {
      return j0 + r < t ? qkv + (row_base + j0 + r) * 3072 + 1024 + h * kTcD : nullptr;
    });
    {
      // thread: dimensions 4 (tid % 32) .. +3 of key chunk 4 q + tid / 32 (keys
      // 8 kc .. 8 kc + 7), q = 0, 1; a warp reads 512 contiguous bytes per key
      float4 vv[2][8];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int kc = 4 * q + (tid >> 5);
        const int d = (tid & 31) * 4;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int j = j0 + kc * 8 + e;
          vv[q][e] = j < t ? *reinterpret_cast<const float4*>(qkv + (row_base + j) * 3072 + 2048 + h * kTcD + d)
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int kc = 4 * q + (tid >> 5);
        const int d = (tid & 31) * 4;
        const float4* v = vv[q];
        *reinterpret_cast<uint4*>(sm + kTcVtOff + sw128(d + 0, kc)) =
            make_uint4(pack_h2(v[0].x, v[1].x), pack_h2(v[2].x, v[3].x), pack_h2(v[4].x, v[5].x),
                       pack_h2(v[6].x, v[7].x));
        *reinterpret_cast<uint4*>(sm + kTcVtOff + sw128(d + 1, kc)) =
            make_uint4(pack_h2(v[0].y, v[1].y), pack_h2(v[2].y, v[3].y), pack_h2(v[4].y, v[5].y),
                       pack_h2(v[6].y, v[7].y));
        *reinterpret_cast<uint4*>(sm + kTcVtOff + sw128(d + 2, kc)) =
            make_uint4(pack_h2(v[0].z, v[1].z), pack_h2(v[2].z, v[3].z), pack_h2(v[4].z, v[5].z),
                       pack_h2(v[6].z, v[7].z));
        *reinterpret_cast<uint4*>(sm + kTcVtOff + sw128(d + 3, kc)) =
            make_uint4(pack_h2(v[0].w, v[1].w), pack_h2(v[2].w, v[3].w), pack_h2(v[4].w, v[5].w),
                       pack_h2(v[6].w, v[7].w));
      }
    }
    if (kt == 0) {
      stage_slab(0);
      stage_slab(1);
    }
    stage_slab(kt + 2);
    fence_proxy_async_smem();  // generic-proxy stores, read by the tensor cores
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      constexpr uint32_t id_s = idesc_f16(128, 64);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t koff = (kk & 3) * 32;  // 16 dimensions = 32 bytes into the atom row
        const uint64_t a = smem_desc_sw128(sbase + kTcQuOff + (kk >> 2) * (kTcQ * 128) + koff);
        const uint64_t b = smem_desc_sw128(sbase + kTcKOff + (kk >> 2) * (64 * 128) + koff);
        mma_f16_ss(tmem + kTcColS, a, b, id_s, kk > 0);
      }
#pragma unroll
      for (int sl = 0; sl < 3; ++sl) {
        const uint32_t slab = sbase + kTcBandOff + ((kt + sl) % 3) * kTcSlabBytes;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t koff = (kk & 3) * 32;
          const uint64_t a = smem_desc_sw128(sbase + kTcQvOff + (kk >> 2) * (kTcQ * 128) + koff);
          const uint64_t b = smem_desc_sw128(slab + (kk >> 2) * (64 * 128) + koff);
          mma_f16_ss(tmem + kTcColBd + 64 * sl, a, b, id_s, kk > 0);
        }
      }
      mma_commit(bar_s);
      ++s_issued;
    }
    if (!mbar_wait(bar_s, kt & 1, abort_flag, status)) {
      ok = false;
      break;
    }
    tc_fence_after();

    // Scores of this thread's row: S plus its band columns j - r + 127.
    float z[64];
    {
      uint32_t raw[32];
      tmem_ld32(tmem + lane_base + kTcColS, raw);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) z[j] = __uint_as_float(raw[j]);
      tmem_ld32(tmem + lane_base + kTcColS + 32, raw);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) z[32 + j] = __uint_as_float(raw[j]);
    }
    {
      // the warp's 96-column window starts at band column 96 - 32 warp; this
      // row's 64 columns start 31 - lane further on
      float a[96];
      uint32_t raw[32];
#pragma unroll
      for (int c = 0; c < 3; ++c) {
        tmem_ld32(tmem + lane_base + kTcColBd + 96 - 32 * warp + 32 * c, raw);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) a[32 * c + j] = __uint_as_float(raw[j]);
      }
      const int o = 31 - lane;
#pragma unroll
      for (int k = 0; k < 80; ++k) a[k] = (o & 16) ? a[k + 16] : a[k];
#pragma unroll
      for (int k = 0; k < 72; ++k) a[k] = (o & 8) ? a[k + 8] : a[k];
#pragma unroll
      for (int k = 0; k < 68; ++k) a[k] = (o & 4) ? a[k + 4] : a[k];
#pragma unroll
      for (int k = 0; k < 66; ++k) a[k] = (o & 2) ? a[k + 2] : a[k];
#pragma unroll
      for (int k = 0; k < 65; ++k) a[k] = (o & 1) ? a[k + 1] : a[k];
      float tile_max = -INFINITY;
#pragma unroll
      for (int j = 0; j < 64; ++j) {
        const float s = (j0 + j < t) ? (z[j] + a[j]) * kScaleLog2 : -INFINITY;
        z[j] = s;
        tile_max = fmaxf(tile_max, s);
      }
      const float m_new = fmaxf(m_row, tile_max);
      const float alpha = exp2f(m_row - m_new);  // 0 on the first tile (m_row = -inf)
      m_row = m_new;
      float sum = 0.0f;
      uint32_t ph[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float pa = exp2f(z[2 * j] - m_new), pb = exp2f(z[2 * j + 1] - m_new);
        sum += pa + pb;
        ph[j] = pack_h2(pa, pb);
      }
      l_row = l_row * alpha + sum;
      // probabilities: row tid of the P tile, 8 chunks of 8 keys
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(sm + kTcPOff + sw128(tid, c)) =
            make_uint4(ph[4 * c], ph[4 * c + 1], ph[4 * c + 2], ph[4 * c + 3]);
      // rescale the context accumulated so far (the previous product has completed)
      if (kt > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          tmem_ld32(tmem + lane_base + kTcColO + 32 * c, raw);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) raw[j] = __float_as_uint(__uint_as_float(raw[j]) * alpha);
          tmem_st32(tmem + lane_base + kTcColO + 32 * c, raw);
        }
        tmem_wait_st();
      }
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      constexpr uint32_t id_o = idesc_f16(128, 128);
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t a = smem_desc_sw128(sbase + kTcPOff + kk * 32);
        const uint64_t b = smem_desc_sw128(sbase + kTcVtOff + kk * 32);
        mma_f16_ss(tmem + kTcColO, a, b, id_o, (kt > 0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(bar_pv);
      ++pv_issued;
    }
  }
  if (ok && mbar_wait(bar_pv, (n_tiles - 1) & 1, abort_flag, status)) {
    tc_fence_after();
    const int i = i0 + tid;
    const float inv = 1.0f / l_row;
    float* out = ctx + (row_base + i) * 1024 + h * kTcD;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t raw[32];
      tmem_ld32(tmem + lane_base + kTcColO + 32 * c, raw);
      tmem_wait_ld();
      if (i < t) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float4 v = make_float4(__uint_as_float(raw[j]) * inv, __uint_as_float(raw[j + 1]) * inv,
                                 __uint_as_float(raw[j + 2]) * inv, __uint_as_float(raw[j + 3]) * inv);
          if (round_out) v = make_float4(tf32_round(v.x), tf32_round(v.y), tf32_round(v.z), tf32_round(v.w));
          *reinterpret_cast<float4*>(out + 32 * c + j) = v;
        }
      }
    }
  } else if (tid == 0) {
    // never leave with MMAs in flight: wait (bounded) for the last commits issued
    if (s_issued > 0) mbar_drain(bar_s, (s_issued - 1) & 1);
    if (pv_issued > 0) mbar_drain(bar_pv, (pv_issued - 1) & 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTcTmemCols);
}

}  // namespace pq8
