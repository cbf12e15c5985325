// The FastConformer block around the Q8_0 linears (parakeet_cuda/reference.py:33-66):
// LayerNorm, the conv module's depthwise convolution with BatchNorm and SiLU,
// the relative-position attention with FP32 products (the three batched
// products on cuBLAS around the bias / shift-softmax kernels; the fused
// tensor-core attention is pq8_attention.cuh), and the subsampling stem. The
// linears are pq8_gemm.
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
