// Fused relative-position attention on the 5th-generation tensor cores
// (parakeet_cuda/reference.py:51-58; rel_scores and softmax in
// runtime.cu:122-137, the three batched products in gpu.py:92-100).
//
// One CTA per (window, head, 128 queries); TMEM lane r is query row r of
// every accumulator. Per tile of 64 keys:
//   S  = (Q + u) K^T         128 x 64   tcgen05.mma kind::f16, TMEM cols [0, 64)
//   BD = (Q + v) Band^T      128 x 192  (three MMAs of 64 positions each), TMEM cols [64, 256)
//   O += P V^T               128 x 128  TMEM cols [256, 384)
// Band holds the 192 positional rows t-1+j-i the tile's (i, j) pairs need:
// query i and key j read band column j - i + 127.
//
// Warp roles (256 threads):
//   * warps 0-3, the softmax warps: thread r owns row r. It loads its row of
//     S and the 96-column BD window of its warp's 32 rows, releases the
//     accumulators, moves its own 64 band columns into place with a 5-stage
//     register barrel shift (offset 31 - lane), runs the online softmax over
//     the row in registers, rescales O in TMEM when the row maximum grows,
//     and writes the probabilities to shared memory as FP16;
//   * warps 4-7, the producers: stage the next tile (K and V^T double
//     buffered, the band as a ring of three 64-row slabs, mirrored so that a
//     tile's three are contiguous: consecutive tiles share two, so one slab
//     is staged per tile) while the softmax warps work
//     on the current one; their first thread issues the MMAs (S and BD of
//     tile k once it is staged and the softmax warps have read tile k - 1's
//     accumulators; P V^T of tile k - 1 once its probabilities are written).
//
// Operands are staged as FP16 (the 11-bit significand TF32 keeps; FP32
// accumulation) in the canonical K-major 128-byte-swizzled layout: row r of
// a tile is 128 bytes per 64 elements, its 16-byte chunk c stored at chunk
// c ^ (r % 8), atoms of 8 rows 1024 bytes apart. V is staged transposed
// (rows = head dimensions, K = keys). tcgen05 commits and warp arrivals meet
// on mbarriers; every wait is bounded (PQ8_ERR_TIMEOUT in the device status
// word).
#pragma once

#include "pq8_device.cuh"

namespace pq8 {

constexpr int kTcQ = 128, kTcKeys = 64, kTcD = 128;
constexpr int kTcThreads = 256, kTcRoleThreads = 128;
constexpr int kTcQuOff = 0;                              // [2 atoms][128 rows][128 B]
constexpr int kTcQvOff = kTcQuOff + 2 * 128 * 128;
constexpr int kTcKOff = kTcQvOff + 2 * 128 * 128;        // 2 buffers x [2 atoms][64 keys][128 B]
constexpr int kTcKBytes = 2 * 64 * 128;
constexpr int kTcVtOff = kTcKOff + 2 * kTcKBytes;        // 2 buffers x [128 dims][128 B = 64 keys]
constexpr int kTcVtBytes = 128 * 128;
// The positional band: [2 atom planes][5 slots x 64 rows][128 B]. Slab s
// (64 positions) lives in slot s % 3 and, for s % 3 < 2, also in slot
// 3 + s % 3, so the three slabs of any tile occupy three consecutive slots
// (from slot k % 3): one N = 192 operand.
constexpr int kTcBandOff = kTcVtOff + 2 * kTcVtBytes;
constexpr int kTcBandSlots = 5;
constexpr int kTcPlaneBytes = kTcBandSlots * 64 * 128;
constexpr int kTcPOff = kTcBandOff + 2 * kTcPlaneBytes;  // [128 rows][128 B = 64 keys]
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

__global__ void __launch_bounds__(kTcThreads, 1)
    rel_attention_tc_kernel(const float* __restrict__ qkv, const float* __restrict__ pos,
                            const float* __restrict__ pos_bias_u, const float* __restrict__ pos_bias_v,
                            float* __restrict__ ctx, int t, int round_out, int* status) {
  griddep_launch();
  extern __shared__ uint8_t att_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(att_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_addr(sm);
  uint64_t* bar_s = reinterpret_cast<uint64_t*>(sm + kTcBarOff);  // S and BD of a tile done (commit)
  uint64_t* bar_pv = bar_s + 1;                                    // P V^T of a tile done (commit)
  uint64_t* s_free = bar_s + 2;  // the softmax warps have read a tile's S and BD (one arrival per warp)
  uint64_t* p_full = bar_s + 3;  // a tile's probabilities written and O rescaled (one arrival per warp)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_s + 4);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(bar_s + 5);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int i0 = blockIdx.x * kTcQ, h = blockIdx.y, win = blockIdx.z;
  const size_t row_base = static_cast<size_t>(win) * t;
  const int n_tiles = (t + kTcKeys - 1) / kTcKeys;

  if (tid == 0) {
    mbar_init(bar_s, 2);  // the S and the positional-band issuers' commits
    mbar_init(bar_pv, 1);
    mbar_init(s_free, 4);
    mbar_init(p_full, 4);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(tmem_slot, kTcTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= 4) {
    // ------------------------------------------------------------ producers
    const int pt = tid - kTcRoleThreads;
    griddep_wait();  // qkv comes from the previous kernel
    {
      // queries with each positional bias (rows past t are zero)
      constexpr int kItems = kTcQ * 16 / kTcRoleThreads;
      float4 xa[kItems], xb[kItems];
#pragma unroll
      for (int q = 0; q < kItems; ++q) {
        const int item = q * kTcRoleThreads + pt, r = item >> 4, c16 = item & 15;
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
        const int item = q * kTcRoleThreads + pt, r = item >> 4, c16 = item & 15;
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
    // Positional slab s holds positions p0 + 64 s + [0, 64): the tile of keys
    // j0 = 64 k uses slabs k, k + 1, k + 2 (band column c = j - i + 127).
    const int p0 = t - 128 - i0, n_pos = 2 * t - 1;
    // slab sl into its slot (and mirror slot), rows r of both atom planes
    auto store_slab = [&](int sl, int item, uint4 val) {
      const int r = item >> 4, c16 = item & 15;
      uint8_t* plane = sm + kTcBandOff + (c16 >> 3) * kTcPlaneBytes;
      const int slot = sl % 3;
      *reinterpret_cast<uint4*>(plane + sw128(slot * 64 + r, c16 & 7)) = val;
      if (slot < 2) *reinterpret_cast<uint4*>(plane + sw128((3 + slot) * 64 + r, c16 & 7)) = val;
    };
    // slabs 0 and 1 (the first tile's other two come with it): all 32 loads
    // of a thread in flight at once
    {
      float4 ba[2][8], bb[2][8];
#pragma unroll
      for (int sl = 0; sl < 2; ++sl)
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const int item = q * kTcRoleThreads + pt, r = item >> 4, c16 = item & 15;
          const int pp = p0 + 64 * sl + r;
          if (pp >= 0 && pp < n_pos) {
            const float* src = pos + static_cast<size_t>(pp) * 1024 + h * kTcD + c16 * 8;
            ba[sl][q] = *reinterpret_cast<const float4*>(src);
            bb[sl][q] = *reinterpret_cast<const float4*>(src + 4);
          } else {
            ba[sl][q] = bb[sl][q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          }
        }
#pragma unroll
      for (int sl = 0; sl < 2; ++sl)
#pragma unroll
        for (int q = 0; q < 8; ++q) store_slab(sl, q * kTcRoleThreads + pt, pack_h8(ba[sl][q], bb[sl][q]));
    }
    // MMA issue (thread pt = 0). A wait that runs out stops the issue; the
    // thread keeps meeting the other producers at their named barrier, and
    // all of them leave at the next tile's (bounded) wait, which then fails.
    bool failed = false;
    int s_issued = 0, pv_issued = 0;
    auto issue_pv = [&](int k) {
      constexpr uint32_t id_o = idesc_f16(128, 128);
      const uint32_t vt = sbase + kTcVtOff + (k & 1) * kTcVtBytes;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const uint64_t a = smem_desc_sw128(sbase + kTcPOff + kk * 32);
        const uint64_t b = smem_desc_sw128(vt + kk * 32);
        mma_f16_ss(tmem + kTcColO, a, b, id_o, (k > 0 || kk > 0) ? 1u : 0u);
      }
      mma_commit(bar_pv);
      ++pv_issued;
    };
    const float* const v_rows = qkv + row_base * 3072 + 2048 + h * kTcD;
    const int vd = (pt & 31) * 4;
    // A tile's operands: every global load of a thread (K: 8 row chunks, V:
    // 2 x 8 keys of 4 dimensions, the new band slab: 8 row chunks) is issued
    // before the waits for the buffers they go to, and converted and stored
    // after them, so the staging costs about one memory round trip.
    float4 kr[8][2], vr[2][8], br[8][2];
    auto load_tile = [&](int k) {
      const int j0 = k * kTcKeys;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int item = q * kTcRoleThreads + pt, r = item >> 4, c16 = item & 15;
        if (j0 + r < t) {
          const float* src = qkv + (row_base + j0 + r) * 3072 + 1024 + h * kTcD + c16 * 8;
          kr[q][0] = *reinterpret_cast<const float4*>(src);
          kr[q][1] = *reinterpret_cast<const float4*>(src + 4);
        } else {
          kr[q][0] = kr[q][1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        const int pp = p0 + 64 * (k + 2) + r;
        if (pp >= 0 && pp < n_pos) {
          const float* src = pos + static_cast<size_t>(pp) * 1024 + h * kTcD + c16 * 8;
          br[q][0] = *reinterpret_cast<const float4*>(src);
          br[q][1] = *reinterpret_cast<const float4*>(src + 4);
        } else {
          br[q][0] = br[q][1] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int kc = 4 * q + (pt >> 5);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const int j = j0 + kc * 8 + e;
          vr[q][e] = j < t ? *reinterpret_cast<const float4*>(v_rows + (size_t)j * 3072 + vd)
                           : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
      }
    };
    int k = 0;
    for (; k < n_tiles; ++k) {
      load_tile(k);  // in flight during the waits below
      // tile k - 2's products are done (its K and V^T buffers are free), and
      // tile k - 1's scores (slab k + 2 replaces slab k - 1 in its slots)
      if (k >= 2 && !mbar_wait(bar_pv, (k - 2) & 1, abort_flag, status)) break;
      if (k >= 1 && !mbar_wait(bar_s, (k - 1) & 1, abort_flag, status)) break;
      uint8_t* const kt_s = sm + kTcKOff + (k & 1) * kTcKBytes;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int item = q * kTcRoleThreads + pt, r = item >> 4, c16 = item & 15;
        *reinterpret_cast<uint4*>(kt_s + (c16 >> 3) * (64 * 128) + sw128(r, c16 & 7)) = pack_h8(kr[q][0], kr[q][1]);
        store_slab(k + 2, item, pack_h8(br[q][0], br[q][1]));
      }
      uint8_t* const vt_s = sm + kTcVtOff + (k & 1) * kTcVtBytes;
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int kc = 4 * q + (pt >> 5);
        const float4* v = vr[q];
        *reinterpret_cast<uint4*>(vt_s + sw128(vd + 0, kc)) = make_uint4(
            pack_h2(v[0].x, v[1].x), pack_h2(v[2].x, v[3].x), pack_h2(v[4].x, v[5].x), pack_h2(v[6].x, v[7].x));
        *reinterpret_cast<uint4*>(vt_s + sw128(vd + 1, kc)) = make_uint4(
            pack_h2(v[0].y, v[1].y), pack_h2(v[2].y, v[3].y), pack_h2(v[4].y, v[5].y), pack_h2(v[6].y, v[7].y));
        *reinterpret_cast<uint4*>(vt_s + sw128(vd + 2, kc)) = make_uint4(
            pack_h2(v[0].z, v[1].z), pack_h2(v[2].z, v[3].z), pack_h2(v[4].z, v[5].z), pack_h2(v[6].z, v[7].z));
        *reinterpret_cast<uint4*>(vt_s + sw128(vd + 3, kc)) = make_uint4(
            pack_h2(v[0].w, v[1].w), pack_h2(v[2].w, v[3].w), pack_h2(v[4].w, v[5].w), pack_h2(v[6].w, v[7].w));
      }
      fence_proxy_async_smem();  // generic-proxy stores, read by the tensor cores
      named_barrier_sync(1, kTcRoleThreads);
      // Two issuing threads in different warps: pt 0 issues S (and the
      // context products), pt 32 the positional band, each committing to
      // bar_s (two arrivals), so the two chains of MMA issues overlap.
      if (pt == 32 && !failed) {
        if (k > 0 && !mbar_wait(s_free, (k - 1) & 1, abort_flag, status)) failed = true;
        if (!failed) {
          tc_fence_after();
          constexpr uint32_t id_bd = idesc_f16(128, 192);
          const uint32_t band = sbase + kTcBandOff + (k % 3) * (64 * 128);  // slots k % 3 .. + 2
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t koff = (kk & 3) * 32;
            const uint64_t a = smem_desc_sw128(sbase + kTcQvOff + (kk >> 2) * (kTcQ * 128) + koff);
            const uint64_t b = smem_desc_sw128(band + (kk >> 2) * kTcPlaneBytes + koff);
            mma_f16_ss(tmem + kTcColBd, a, b, id_bd, kk > 0);
          }
          mma_commit(bar_s);
          ++s_issued;
        }
      }
      if (pt == 0 && !failed) {
        if (k > 0 && !mbar_wait(s_free, (k - 1) & 1, abort_flag, status)) failed = true;
        if (!failed) {
          tc_fence_after();
          constexpr uint32_t id_s = idesc_f16(128, 64);
          const uint32_t kb = sbase + kTcKOff + (k & 1) * kTcKBytes;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t koff = (kk & 3) * 32;  // 16 dimensions = 32 bytes into the atom row
            const uint64_t a = smem_desc_sw128(sbase + kTcQuOff + (kk >> 2) * (kTcQ * 128) + koff);
            const uint64_t b = smem_desc_sw128(kb + (kk >> 2) * (64 * 128) + koff);
            mma_f16_ss(tmem + kTcColS, a, b, id_s, kk > 0);
          }
          mma_commit(bar_s);
          ++s_issued;
          if (k > 0) {
            if (!mbar_wait(p_full, (k - 1) & 1, abort_flag, status)) {
              failed = true;
            } else {
              tc_fence_after();
              issue_pv(k - 1);
            }
          }
        }
      }
    }
    if (pt == 32 && (failed || k < n_tiles) && s_issued > 0) mbar_drain(bar_s, (s_issued - 1) & 1);
    if (pt == 0) {
      if (!failed && k == n_tiles) {
        if (!mbar_wait(p_full, (n_tiles - 1) & 1, abort_flag, status)) {
          failed = true;
        } else {
          tc_fence_after();
          issue_pv(n_tiles - 1);
        }
      }
      if (failed || k < n_tiles) {
        // never leave with MMAs in flight: wait (bounded) for the last commits issued
        if (s_issued > 0) mbar_drain(bar_s, (s_issued - 1) & 1);
        if (pv_issued > 0) mbar_drain(bar_pv, (pv_issued - 1) & 1);
      }
    }
  } else {
    // -------------------------------------------------------- softmax warps
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const float kScaleLog2 = 1.4426950408889634f * rsqrtf(128.0f);  // 1/sqrt(128) in base 2
    float m_row = -INFINITY, l_row = 0.0f;
    bool ok = true;
    for (int k = 0; k < n_tiles; ++k) {
      const int j0 = k * kTcKeys;
      if (!mbar_wait(bar_s, k & 1, abort_flag, status)) {
        ok = false;
        break;
      }
      tc_fence_after();
      // this row of S, and the warp's 96-column window of BD, which starts
      // at band column 96 - 32 warp (this row's 64 columns start 31 - lane
      // on): five loads in flight, one wait
      uint32_t zr[64], ar[96];
      tmem_ld32(tmem + lane_base + kTcColS, *reinterpret_cast<uint32_t(*)[32]>(zr));
      tmem_ld32(tmem + lane_base + kTcColS + 32, *reinterpret_cast<uint32_t(*)[32]>(zr + 32));
#pragma unroll
      for (int c = 0; c < 3; ++c)
        tmem_ld32(tmem + lane_base + kTcColBd + 96 - 32 * warp + 32 * c,
                  *reinterpret_cast<uint32_t(*)[32]>(ar + 32 * c));
      tmem_wait_ld();
      float z[64], a[96];
#pragma unroll
      for (int j = 0; j < 64; ++j) z[j] = __uint_as_float(zr[j]);
#pragma unroll
      for (int j = 0; j < 96; ++j) a[j] = __uint_as_float(ar[j]);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(s_free);  // the next tile's S and BD may be computed
      const int o = 31 - lane;
#pragma unroll
      for (int q = 0; q < 80; ++q) a[q] = (o & 16) ? a[q + 16] : a[q];
#pragma unroll
      for (int q = 0; q < 72; ++q) a[q] = (o & 8) ? a[q + 8] : a[q];
#pragma unroll
      for (int q = 0; q < 68; ++q) a[q] = (o & 4) ? a[q + 4] : a[q];
#pragma unroll
      for (int q = 0; q < 66; ++q) a[q] = (o & 2) ? a[q + 2] : a[q];
#pragma unroll
      for (int q = 0; q < 65; ++q) a[q] = (o & 1) ? a[q + 1] : a[q];
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
      if (k > 0) {
        // the previous tile's product has read P and accumulated into O
        if (!mbar_wait(bar_pv, (k - 1) & 1, abort_flag, status)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.0f)) {
          uint32_t raw[32];
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
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(sm + kTcPOff + sw128(tid, c)) =
            make_uint4(ph[4 * c], ph[4 * c + 1], ph[4 * c + 2], ph[4 * c + 3]);
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
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
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, kTcTmemCols);
}

}  // namespace pq8
