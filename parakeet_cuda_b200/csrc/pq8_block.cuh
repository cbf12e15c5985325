// The FastConformer block around the Q8_0 linears (parakeet_cuda/reference.py:33-66):
// LayerNorm, the conv module's depthwise convolution with BatchNorm and SiLU,
// the relative-position attention (fused; with FP32 products the three
// batched products go to cuBLAS around the bias / shift-softmax kernels), and
// the subsampling stem. The linears are pq8_gemm.
//
// LayerNorm, the depthwise convolution and the stem's stages are HBM-bound:
// each reads its input once and writes its output once, coalesced across
// channels.
#pragma once

#include <cuda_fp16.h>

#include "pq8_device.cuh"

namespace pq8 {

constexpr float kLayerNormEps = 1e-5f;  // reference.py:8, runtime.cu:46

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float4 tf32_round4(float4 v) {
  return make_float4(tf32_round(v.x), tf32_round(v.y), tf32_round(v.z), tf32_round(v.w));
}
__device__ __forceinline__ float silu_exact(float z) { return z / (1.0f + expf(-z)); }

// LayerNorm over rows of width 128 * V: a warp per row at a time, V float4
// per lane (a warp reads 512 contiguous bytes per access). The weight and
// bias are loaded once per warp, before waiting for the previous kernel, and
// the warp walks rows with a grid stride, so only the row itself is on the
// critical path. Two passes over the values held in registers: mean, then the
// mean of squared deviations (runtime.cu:38-48 sums the deviations the same
// way). Optionally rounds the output to TF32 (to nearest, ties away) so that
// the GEMM reading it skips its own rounding pass (PQ8_FLAG_X_TF32).
template <int V>
__global__ void layer_norm_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                  const float* __restrict__ b, float* __restrict__ y, int rows, int round_out) {
  griddep_launch();
  const int lane = threadIdx.x & 31;
  constexpr int kWidth = 128 * V;
  float4 g[V], h[V];
  const float4* w4 = reinterpret_cast<const float4*>(w);
  const float4* b4 = reinterpret_cast<const float4*>(b);
#pragma unroll
  for (int i = 0; i < V; ++i) {
    g[i] = w4[i * 32 + lane];
    h[i] = b4[i * 32 + lane];
  }
  griddep_wait();  // x is the previous kernel's output
  const int warps = gridDim.x * (blockDim.x >> 5);
  for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < rows; row += warps) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * kWidth);
    float4 v[V];
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      v[i] = xr[i * 32 + lane];
      s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
    const float mean = warp_sum(s) * (1.0f / kWidth);
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < V; ++i) {
      v[i].x -= mean;
      v[i].y -= mean;
      v[i].z -= mean;
      v[i].w -= mean;
      q += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
    }
    const float inv = rsqrtf(warp_sum(q) * (1.0f / kWidth) + kLayerNormEps);
    float4* yr = reinterpret_cast<float4*>(y + static_cast<size_t>(row) * kWidth);
#pragma unroll
    for (int i = 0; i < V; ++i) {
      float4 o = make_float4(v[i].x * inv * g[i].x + h[i].x, v[i].y * inv * g[i].y + h[i].y,
                             v[i].z * inv * g[i].z + h[i].z, v[i].w * inv * g[i].w + h[i].w);
      if (round_out) o = tf32_round4(o);
      yr[i * 32 + lane] = o;
    }
  }
}

// Conv module middle (reference.py:60-63, runtime.cu:63-71): depthwise
// convolution with 9 taps over the frames of each window (4 zero rows beyond
// either end of a window), BatchNorm with running statistics, SiLU. x, y:
// [windows * t, C]. A CTA of 256 threads covers 512 channels (2 per thread) of
// a strip of kConvStrip frames of one window (grid: strips x windows x C /
// 512). Each thread issues the loads of all kConvStrip + 8 rows it needs
// before using any of them, so a strip costs one memory round trip.
constexpr int kConvStrip = 16;
constexpr int kConvThreads = 256;
__global__ void __launch_bounds__(kConvThreads)
    conv_depthwise_bn_silu_kernel(const float* __restrict__ x, const uint16_t* __restrict__ w9_f16,
                                  const float* __restrict__ gamma, const float* __restrict__ beta,
                                  const float* __restrict__ mean, const float* __restrict__ var,
                                  float* __restrict__ y, int t, int channels, int round_out) {
  griddep_launch();
  const int c2 = blockIdx.z * kConvThreads + threadIdx.x;  // channels 2 c2, 2 c2 + 1
  const bool active = 2 * c2 < channels;
  const int win = blockIdx.y;
  const int r0 = blockIdx.x * kConvStrip;
  const size_t base = static_cast<size_t>(win) * t;
  const int c2n = channels >> 1;
  float wk[2][9], sc[2], sh[2];
  if (active) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int ch = 2 * c2 + c;
#pragma unroll
      for (int k = 0; k < 9; ++k) wk[c][k] = __half2float(__ushort_as_half(w9_f16[static_cast<size_t>(ch) * 9 + k]));
      sc[c] = gamma[ch] * rsqrtf(var[ch] + kLayerNormEps);
      sh[c] = beta[ch] - mean[ch] * sc[c];
    }
  }
  griddep_wait();  // x is the previous kernel's output
  if (!active) return;
  const float2* x2 = reinterpret_cast<const float2*>(x);
  float2* y2 = reinterpret_cast<float2*>(y);
  float2 in[kConvStrip + 8];
#pragma unroll
  for (int k = 0; k < kConvStrip + 8; ++k) {
    const int r = r0 - 4 + k;
    in[k] = (r >= 0 && r < t) ? x2[(base + r) * c2n + c2] : make_float2(0.0f, 0.0f);
  }
#pragma unroll
  for (int q = 0; q < kConvStrip; ++q) {
    if (r0 + q >= t) break;
    float a0 = 0.0f, a1 = 0.0f;
#pragma unroll
    for (int k = 0; k < 9; ++k) {
      a0 = fmaf(in[q + k].x, wk[0][k], a0);
      a1 = fmaf(in[q + k].y, wk[1][k], a1);
    }
    float2 o = make_float2(silu_exact(a0 * sc[0] + sh[0]), silu_exact(a1 * sc[1] + sh[1]));
    if (round_out) o = make_float2(tf32_round(o.x), tf32_round(o.y));
    y2[(base + r0 + q) * c2n + c2] = o;
  }
}

// Queries with the two positional biases (reference.py:51-53): qu = q + u,
// qv = q + v per head, from the packed QKV projection [rows, 3 * 1024].
__global__ void attention_query_bias_kernel(const float* __restrict__ qkv, const float* __restrict__ u,
                                            const float* __restrict__ v, float* __restrict__ qu,
                                            float* __restrict__ qv, long long rows) {
  griddep_launch();
  griddep_wait();
  const long long n4 = rows * 256;  // 1024 / 4 float4 per row
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < n4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = i >> 8;
    const int c = static_cast<int>(i & 255);
    const float4 q = reinterpret_cast<const float4*>(qkv)[row * 768 + c];
    const float4 bu = reinterpret_cast<const float4*>(u)[c], bv = reinterpret_cast<const float4*>(v)[c];
    reinterpret_cast<float4*>(qu)[i] = make_float4(q.x + bu.x, q.y + bu.y, q.z + bu.z, q.w + bu.w);
    reinterpret_cast<float4*>(qv)[i] = make_float4(q.x + bv.x, q.y + bv.y, q.z + bv.z, q.w + bv.w);
  }
}

// Shifted scores and softmax, one warp per (window, head, query) row, in
// place over the content scores: s[j] = (ac[i][j] + bd[i][t - 1 + j - i]) /
// sqrt(128), then softmax over j (reference.py:54-57; rel_scores and softmax,
// runtime.cu:122-137). ac: [windows * heads, t, t]; bd: [windows * heads, t,
// 2t - 1]. With J > 0 each lane keeps its J = ceil(t / 32) shifted scores in
// registers, so both score rows are read once; J == 0 is the general
// three-pass form (max, sum, write) for long windows.
template <int J>
__global__ void rel_shift_softmax_kernel(float* __restrict__ ac, const float* __restrict__ bd, int t,
                                         long long n_rows) {
  const long long row = blockIdx.x * static_cast<long long>(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= n_rows) return;
  const int i = static_cast<int>(row % t);
  float* s = ac + row * t;
  const float* p = bd + row * (2LL * t - 1) + (t - 1 - i);  // p[j] = bd[i][t - 1 + j - i]
  const float scale = rsqrtf(128.0f);
  if constexpr (J > 0) {
    float v[J];
    float m = -INFINITY;
#pragma unroll
    for (int q = 0; q < J; ++q) {
      const int j = lane + 32 * q;
      v[q] = j < t ? (s[j] + p[j]) * scale : -INFINITY;
      m = fmaxf(m, v[q]);
    }
    m = warp_max(m);
    float sum = 0.0f;
#pragma unroll
    for (int q = 0; q < J; ++q) {
      v[q] = expf(v[q] - m);  // exp(-inf) = 0 for the lanes past t
      sum += v[q];
    }
    const float inv = 1.0f / warp_sum(sum);
#pragma unroll
    for (int q = 0; q < J; ++q) {
      const int j = lane + 32 * q;
      if (j < t) s[j] = v[q] * inv;
    }
  } else {
    float m = -INFINITY;
    for (int j = lane; j < t; j += 32) m = fmaxf(m, (s[j] + p[j]) * scale);
    m = warp_max(m);
    float sum = 0.0f;
    for (int j = lane; j < t; j += 32) sum += expf((s[j] + p[j]) * scale - m);
    const float inv = 1.0f / warp_sum(sum);
    for (int j = lane; j < t; j += 32) s[j] = expf((s[j] + p[j]) * scale - m) * inv;
  }
}

// ---------------------------------------------------------------------------
// Fused relative-position attention, flash style: one CTA per (window, head,
// 64 queries), 4 warps of 16 queries. Per tile of 64 keys a warp computes
//   positional scores  Qv . P_band^T  (16 x 80 positions: the diagonals its
//                       queries need, P_band = positional rows t-1+j-i),
//   content scores     Qu . K^T       (16 x 64),
// adds the positional scores along the shift through a per-warp scratch,
// scales by 1/sqrt(128), updates an online softmax and accumulates
//   context          P . V            (16 x 128)
// on the tensor cores with mma.sync m16n8k16 (FP16 operands, the 11-bit
// significand TF32 keeps; FP32 accumulation). Q, K, V and the positional
// projection are read from their FP32 buffers and converted when staged, so
// no score or probability touches HBM.
constexpr int kAttQ = 64, kAttK = 64, kAttD = 128;
constexpr int kAttBand = 128;             // positional rows of one (query tile, key tile): 2 * 64 - 1, padded
constexpr int kAttLd = kAttD + 8;         // fp16 row stride of K, V and the band (16-byte pad)
constexpr int kAttWarpBand = 80;          // band columns one warp needs (16 queries x 64 keys)
constexpr int kAttScratchLd = kAttWarpBand + 4;
constexpr size_t kAttSmemBytes = sizeof(__half) * (2 * kAttK * kAttLd + kAttBand * kAttLd) +
                                 sizeof(float) * 4 * 16 * kAttScratchLd;

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// B fragment (16 x 8, k = rows of a row-major [k][n] shared-memory tile) via
// ldmatrix with transpose: lanes 0-15 give the addresses of rows k0 .. k0+15
// at column n0 (16-byte aligned); lane l receives M[k0+2(l%4)+{0,1}][n0+l/4]
// and M[k0+8+2(l%4)+{0,1}][n0+l/4].
__device__ __forceinline__ void ldmatrix_x2_trans(uint32_t& b0, uint32_t& b1, const __half* row_addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0, %1}, [%2];"
               : "=r"(b0), "=r"(b1)
               : "r"(smem_addr(row_addr)));
}

__global__ void __launch_bounds__(128)
    rel_attention_fused_kernel(const float* __restrict__ qkv, const float* __restrict__ pos,
                               const float* __restrict__ pos_bias_u, const float* __restrict__ pos_bias_v,
                               float* __restrict__ ctx, int t, int round_out) {
  griddep_launch();
  extern __shared__ __align__(16) unsigned char att_smem[];
  __half* k_s = reinterpret_cast<__half*>(att_smem);               // [64 keys][136]
  __half* v_s = k_s + kAttK * kAttLd;                               // [64 keys][136]
  __half* band_s = v_s + kAttK * kAttLd;                            // [128 band rows][136]
  float* scratch = reinterpret_cast<float*>(band_s + kAttBand * kAttLd);  // [4 warps][16][84]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, q = lane & 3;
  const int i0 = blockIdx.x * kAttQ, h = blockIdx.y, win = blockIdx.z;
  const size_t row_base = static_cast<size_t>(win) * t;
  float* my_scratch = scratch + warp * 16 * kAttScratchLd;
  const int q0w = 48 - 16 * warp;  // first band column this warp needs
  griddep_wait();  // qkv and pos come from the previous kernels

  // Query fragments (rows 16 warp + g, + 8) with each positional bias, 8 k-steps of 16.
  uint32_t qu[8][4], qv[8][4];
  {
    const int ra = min(i0 + 16 * warp + g, t - 1), rb = min(i0 + 16 * warp + g + 8, t - 1);
    const float* qa = qkv + (row_base + ra) * 3072 + h * kAttD;
    const float* qb = qkv + (row_base + rb) * 3072 + h * kAttD;
    const float* u = pos_bias_u + h * kAttD;
    const float* v = pos_bias_v + h * kAttD;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int d = ks * 16 + 2 * q + 8 * half;
        const float2 xa = *reinterpret_cast<const float2*>(qa + d), xb = *reinterpret_cast<const float2*>(qb + d);
        const float2 bu = *reinterpret_cast<const float2*>(u + d), bv = *reinterpret_cast<const float2*>(v + d);
        qu[ks][2 * half] = pack_half2(xa.x + bu.x, xa.y + bu.y);
        qu[ks][2 * half + 1] = pack_half2(xb.x + bu.x, xb.y + bu.y);
        qv[ks][2 * half] = pack_half2(xa.x + bv.x, xa.y + bv.y);
        qv[ks][2 * half + 1] = pack_half2(xb.x + bv.x, xb.y + bv.y);
      }
    }
  }
  float o[16][4];
#pragma unroll
  for (int n = 0; n < 16; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m_row[2] = {-INFINITY, -INFINITY}, l_row[2] = {0.0f, 0.0f};
  const float kScaleLog2 = 1.4426950408889634f * rsqrtf(128.0f);  // 1/sqrt(128) in base 2

  for (int j0 = 0; j0 < t; j0 += kAttK) {
    // The positional band is a ring of 128 rows: band row b of this tile is in
    // slot (ring + b) % 128, and the first 64 rows of a tile are the last 64 of
    // the tile before, so after the first tile only 64 rows are loaded.
    const int ring = j0 & (kAttBand - 1);
    __syncthreads();  // the previous tile's operands are no longer read
    // Stage K, V [key][d] and the positional band [row][d] as FP16.
    for (int idx = tid; idx < kAttK * (kAttD / 4); idx += 128) {
      const int key = idx >> 5, d = (idx & 31) * 4, j = j0 + key;
      float4 kv = make_float4(0.0f, 0.0f, 0.0f, 0.0f), vv = kv;
      if (j < t) {
        const float* r = qkv + (row_base + j) * 3072 + h * kAttD + d;
        kv = *reinterpret_cast<const float4*>(r + 1024);
        vv = *reinterpret_cast<const float4*>(r + 2048);
      }
      *reinterpret_cast<uint2*>(k_s + key * kAttLd + d) = make_uint2(pack_half2(kv.x, kv.y), pack_half2(kv.z, kv.w));
      *reinterpret_cast<uint2*>(v_s + key * kAttLd + d) = make_uint2(pack_half2(vv.x, vv.y), pack_half2(vv.z, vv.w));
    }
    const int pb = t - 64 + j0 - i0;  // position of band row 0 (query i0 + 63, key j0)
    const int first_row = j0 == 0 ? 0 : kAttBand - kAttK;  // rows not already in the ring
    for (int idx = tid + first_row * (kAttD / 4); idx < kAttBand * (kAttD / 4); idx += 128) {
      const int r = idx >> 5, d = (idx & 31) * 4, p = pb + r;
      float4 pv = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      if (p >= 0 && p < 2 * t - 1) pv = *reinterpret_cast<const float4*>(pos + static_cast<size_t>(p) * 1024 + h * kAttD + d);
      *reinterpret_cast<uint2*>(band_s + ((ring + r) & (kAttBand - 1)) * kAttLd + d) =
          make_uint2(pack_half2(pv.x, pv.y), pack_half2(pv.z, pv.w));
    }
    __syncthreads();

    // Positional scores of this warp's 16 queries over its 80 band columns, to the scratch.
    {
      float bd[10][4];
#pragma unroll
      for (int n = 0; n < 10; ++n) bd[n][0] = bd[n][1] = bd[n][2] = bd[n][3] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
#pragma unroll
        for (int n = 0; n < 10; ++n) {
          const __half* br = band_s + ((ring + q0w + 8 * n + g) & (kAttBand - 1)) * kAttLd + ks * 16 + 2 * q;
          mma_16816(bd[n], qv[ks], *reinterpret_cast<const uint32_t*>(br), *reinterpret_cast<const uint32_t*>(br + 8));
        }
#pragma unroll
      for (int n = 0; n < 10; ++n) {
        *reinterpret_cast<float2*>(my_scratch + g * kAttScratchLd + 8 * n + 2 * q) = make_float2(bd[n][0], bd[n][1]);
        *reinterpret_cast<float2*>(my_scratch + (g + 8) * kAttScratchLd + 8 * n + 2 * q) =
            make_float2(bd[n][2], bd[n][3]);
      }
      __syncwarp();
    }
    // Content scores, plus the positional score on the shifted diagonal: for
    // query row r (0..15 in the warp) and key column c, band column c - r + 15.
    float sc[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) sc[n][0] = sc[n][1] = sc[n][2] = sc[n][3] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks)
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const __half* kr = k_s + (8 * n + g) * kAttLd + ks * 16 + 2 * q;
        mma_16816(sc[n], qu[ks], *reinterpret_cast<const uint32_t*>(kr), *reinterpret_cast<const uint32_t*>(kr + 8));
      }
    float tile_max[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 8; ++n)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = g + 8 * (e >> 1), c = 8 * n + 2 * q + (e & 1);
        const float z = (sc[n][e] + my_scratch[r * kAttScratchLd + c - r + 15]) * kScaleLog2;
        sc[n][e] = (j0 + c < t) ? z : -INFINITY;
        tile_max[e >> 1] = fmaxf(tile_max[e >> 1], sc[n][e]);
      }
    float alpha[2];
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      tile_max[rr] = fmaxf(tile_max[rr], __shfl_xor_sync(0xffffffffu, tile_max[rr], 1));
      tile_max[rr] = fmaxf(tile_max[rr], __shfl_xor_sync(0xffffffffu, tile_max[rr], 2));
      const float m_new = fmaxf(m_row[rr], tile_max[rr]);
      alpha[rr] = exp2f(m_row[rr] - m_new);  // 0 on the first tile (m_row = -inf)
      m_row[rr] = m_new;
      l_row[rr] *= alpha[rr];
    }
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
    // Probabilities (unnormalised) as the A operand of the context product.
    uint32_t pa[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = exp2f(sc[n][0] - m_row[0]), p1 = exp2f(sc[n][1] - m_row[0]);
      const float p2 = exp2f(sc[n][2] - m_row[1]), p3 = exp2f(sc[n][3] - m_row[1]);
      l_row[0] += p0 + p1;
      l_row[1] += p2 + p3;
      pa[n >> 1][(n & 1) * 2] = pack_half2(p0, p1);
      pa[n >> 1][(n & 1) * 2 + 1] = pack_half2(p2, p3);
    }
    const int lrow = lane & 15;  // ldmatrix row address of this lane (lanes 16-31: ignored, kept valid)
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int n = 0; n < 16; ++n) {
        uint32_t b0, b1;
        ldmatrix_x2_trans(b0, b1, v_s + (kk * 16 + lrow) * kAttLd + 8 * n);
        mma_16816(o[n], pa[kk], b0, b1);
      }
    __syncwarp();  // the scratch is rewritten by the next tile
  }
  // Row sums across the 4 lanes of a row, normalise, write heads merged.
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    l_row[rr] += __shfl_xor_sync(0xffffffffu, l_row[rr], 1);
    l_row[rr] += __shfl_xor_sync(0xffffffffu, l_row[rr], 2);
  }
  const float inv[2] = {1.0f / l_row[0], 1.0f / l_row[1]};
#pragma unroll
  for (int rr = 0; rr < 2; ++rr) {
    const int i = i0 + 16 * warp + g + 8 * rr;
    if (i >= t) continue;
    float* out = ctx + (row_base + i) * 1024 + h * kAttD;
#pragma unroll
    for (int n = 0; n < 16; ++n) {
      float a = o[n][2 * rr] * inv[rr], b = o[n][2 * rr + 1] * inv[rr];
      if (round_out) {
        a = tf32_round(a);
        b = tf32_round(b);
      }
      *reinterpret_cast<float2*>(out + 8 * n + 2 * q) = make_float2(a, b);
    }
  }
}

// Pointer tables for the batched attention GEMMs, one entry per (window,
// head) b = 8 w + h, nine tables of nb entries: A, B, C of the content scores
// (K, Q + u, scores), of the positional scores (pos, Q + v, scores) and of the
// context (V, probabilities, context).
__global__ void attention_pointers_kernel(const float* qkv, const float* qu, const float* qv, const float* pos,
                                          float* ac, float* bd, float* ctx, int windows, int t, float** tables) {
  const int nb = windows * 8;
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= nb) return;
  const int w = b >> 3, h = b & 7;
  const size_t row0 = static_cast<size_t>(w) * t;
  float* const p[9] = {const_cast<float*>(qkv) + row0 * 3072 + 1024 + h * 128,
                       const_cast<float*>(qu) + row0 * 1024 + h * 128,
                       ac + static_cast<size_t>(b) * t * t,
                       const_cast<float*>(pos) + h * 128,
                       const_cast<float*>(qv) + row0 * 1024 + h * 128,
                       bd + static_cast<size_t>(b) * t * (2 * static_cast<size_t>(t) - 1),
                       const_cast<float*>(qkv) + row0 * 3072 + 2048 + h * 128,
                       ac + static_cast<size_t>(b) * t * t,
                       ctx + row0 * 1024 + h * 128};
#pragma unroll
  for (int i = 0; i < 9; ++i) tables[i * nb + b] = p[i];
}

// ---------------------------------------------------------------------------
// Subsampling stem (reference.py:11-30; conv_first, conv_dw2, flatten_stem in
// runtime.cu:73-101). Windows are independent: every stage pads each window's
// own edges. Activations are [window][time][frequency][256 channels]; a CTA of
// 256 threads gives thread c channel c (so its 9 taps stay in registers) and
// walks output positions, reading its inputs coalesced across channels.
constexpr int kStemChannels = 256;

// Output frames per CTA (first stage) or per thread (depthwise stages).
constexpr int kStemFrames = 8;

// First stage: 3x3, stride 2, one input plane -> 256 channels, + bias, ReLU.
// A CTA covers kStemFrames output frames x all f_out frequencies of one window:
// it stages the 2 kStemFrames + 1 mel rows they read in shared memory, then
// thread c computes channel c at every position (taps read as broadcasts) and
// the CTA writes 1 KB per position.
__global__ void __launch_bounds__(kStemChannels)
    stem_conv_first_kernel(const float* __restrict__ mel, const float* __restrict__ w9,
                           const float* __restrict__ bias, float* __restrict__ out, int t_in, int f_in, int t_out,
                           int f_out) {
  griddep_launch();
  extern __shared__ float rows_s[];  // [2 kStemFrames + 1][f_in + 2], zero-padded
  const int c = threadIdx.x;
  const int win = blockIdx.y, t0 = blockIdx.x * kStemFrames;
  float wk[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) wk[k] = w9[c * 9 + k];
  const float b = bias[c];
  griddep_wait();
  const int width = f_in + 2;
  const float* m = mel + static_cast<size_t>(win) * t_in * f_in;
  for (int i = c; i < (2 * kStemFrames + 1) * width; i += kStemChannels) {
    const int rr = i / width, jf = i % width - 1, it = 2 * t0 - 1 + rr;
    rows_s[i] = (it >= 0 && it < t_in && jf >= 0 && jf < f_in) ? m[static_cast<size_t>(it) * f_in + jf] : 0.0f;
  }
  __syncthreads();
  const int t1 = min(t_out, t0 + kStemFrames);
  for (int t = t0; t < t1; ++t) {
    const float* r0 = rows_s + (2 * (t - t0)) * width;  // input row 2t - 1
    float* o = out + ((static_cast<size_t>(win) * t_out + t) * f_out) * kStemChannels + c;
    for (int f = 0; f < f_out; ++f) {
      float acc = b;
#pragma unroll
      for (int kt = 0; kt < 3; ++kt)
#pragma unroll
        for (int kf = 0; kf < 3; ++kf) acc = fmaf(r0[kt * width + 2 * f + kf], wk[kt * 3 + kf], acc);
      o[static_cast<size_t>(f) * kStemChannels] = fmaxf(acc, 0.0f);
    }
  }
}

// Depthwise stage: 3x3 per channel, stride 2, + bias. With bias_in != NULL the
// input is the raw output of the previous pointwise convolution and becomes
// ReLU(x + bias_in) on load (the previous stage's bias and ReLU, fused here);
// padding taps contribute zero either way. Thread c of a CTA computes channel
// c of kStemFrames consecutive output frames at one frequency: it issues the
// loads of all 3 x (2 kStemFrames + 1) input taps it needs before using any.
__global__ void __launch_bounds__(kStemChannels)
    stem_depthwise_kernel(const float* __restrict__ in, const float* __restrict__ bias_in,
                          const float* __restrict__ w9, const float* __restrict__ bias, float* __restrict__ out,
                          int t_in, int f_in, int t_out, int f_out) {
  griddep_launch();
  const int c = threadIdx.x;
  const int f = blockIdx.x % f_out, t0 = (blockIdx.x / f_out) * kStemFrames, win = blockIdx.y;
  float wk[9];
#pragma unroll
  for (int k = 0; k < 9; ++k) wk[k] = w9[c * 9 + k];
  const float b = bias[c];
  const bool relu_in = bias_in != nullptr;
  const float bi = relu_in ? bias_in[c] : 0.0f;
  griddep_wait();
  const float* x = in + static_cast<size_t>(win) * t_in * f_in * kStemChannels + c;
  constexpr int kRows = 2 * kStemFrames + 1;
  float v[kRows][3];
#pragma unroll
  for (int rr = 0; rr < kRows; ++rr) {
    const int it = 2 * t0 - 1 + rr;
#pragma unroll
    for (int kf = 0; kf < 3; ++kf) {
      const int jf = 2 * f + kf - 1;
      v[rr][kf] = (it >= 0 && it < t_in && jf >= 0 && jf < f_in)
                      ? x[(static_cast<size_t>(it) * f_in + jf) * kStemChannels]
                      : 0.0f;
    }
  }
  if (relu_in) {
#pragma unroll
    for (int rr = 0; rr < kRows; ++rr) {
      const int it = 2 * t0 - 1 + rr;
#pragma unroll
      for (int kf = 0; kf < 3; ++kf) {
        const int jf = 2 * f + kf - 1;
        const bool inside = it >= 0 && it < t_in && jf >= 0 && jf < f_in;
        v[rr][kf] = inside ? fmaxf(v[rr][kf] + bi, 0.0f) : 0.0f;
      }
    }
  }
  float* o = out + ((static_cast<size_t>(win) * t_out) * f_out + f) * kStemChannels + c;
#pragma unroll
  for (int q = 0; q < kStemFrames; ++q) {
    const int t = t0 + q;
    if (t >= t_out) break;
    float acc = b;
#pragma unroll
    for (int kt = 0; kt < 3; ++kt)
#pragma unroll
      for (int kf = 0; kf < 3; ++kf) acc = fmaf(v[2 * q + kt][kf], wk[kt * 3 + kf], acc);
    o[static_cast<size_t>(t) * f_out * kStemChannels] = acc;
  }
}

// ReLU(z + bias) of the last pointwise convolution, flattened channel-major:
// flat[row][c * 16 + f] = relu(z[row][f][c] + bias[c]), TF32-rounded for the
// output linear. One CTA per row through a padded shared-memory tile.
__global__ void __launch_bounds__(kStemChannels)
    stem_flatten_kernel(const float* __restrict__ z, const float* __restrict__ bias, float* __restrict__ flat,
                        long long rows) {
  griddep_launch();
  __shared__ float tile[16][kStemChannels + 1];
  const int c = threadIdx.x;
  const float b = bias[c];
  griddep_wait();
  for (long long row = blockIdx.x; row < rows; row += gridDim.x) {
    const float* zr = z + row * 16 * kStemChannels;
#pragma unroll
    for (int f = 0; f < 16; ++f) tile[f][c] = fmaxf(zr[f * kStemChannels + c] + b, 0.0f);
    __syncthreads();
    float* fr = flat + row * 16 * kStemChannels;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int j = i * kStemChannels + c;  // output index c' * 16 + f'
      fr[j] = tf32_round(tile[j & 15][j >> 4]);
    }
    __syncthreads();
  }
}

}  // namespace pq8
