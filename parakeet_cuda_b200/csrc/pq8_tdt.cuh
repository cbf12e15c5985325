// Greedy TDT control on the device: one thread per stream applies the result
// of one joint call (token, duration index) exactly as the reference's host
// loop does (parakeet_cuda/decoder.py:78-97):
//   * a blank with duration 0 advances one frame;
//   * a non-blank token is emitted, becomes the predictor's next input, and
//     its candidate LSTM state is committed;
//   * at most kMaxSymbols joint calls per frame: the 10th call without a frame
//     advance moves on by one frame.
// It then prepares the next step (predictor input, encoder row of the next
// joint call, commit mask) so that a decode step is a fixed sequence of
// launches (predict, joint, control, commit) that can be captured in a CUDA
// graph and replayed without the host reading anything per step.
#pragma once

#include "pq8_device.cuh"

namespace pq8 {

constexpr int kTdtBlank = 8192;
constexpr int kTdtMaxSymbols = 10;
// Per-stream state words (int[m][kTdtStateWords]).
enum TdtState { kTdtFrames = 0, kTdtT, kTdtSymbols, kTdtPrevious, kTdtEmitted, kTdtCalls, kTdtDone, kTdtStateWords = 8 };

// Applies one joint result to stream i (ids[2i], ids[2i+1]) and writes the
// stream's inputs of the next step. Returns whether the stream is still live.
__device__ __forceinline__ bool tdt_control_stream(int i, const int* __restrict__ ids,
                                                   const int* __restrict__ durations, int n_durations,
                                                   int* __restrict__ state, int enc_stride, int* __restrict__ tokens,
                                                   int* __restrict__ enc_rows, int* __restrict__ commit_mask,
                                                   int* __restrict__ emitted, int emitted_capacity,
                                                   int* __restrict__ trace, int trace_capacity, int* status) {
  int* s = state + i * kTdtStateWords;
  const int frames = s[kTdtFrames];
  int t = s[kTdtT], symbols = s[kTdtSymbols], previous = s[kTdtPrevious];
  int n_emitted = s[kTdtEmitted], n_calls = s[kTdtCalls], done = s[kTdtDone];
  int commit = 0;
  if (!done) {
    const int token = ids[2 * i];
    const int d = ids[2 * i + 1];
    int skip = (d >= 0 && d < n_durations) ? durations[d] : 0;
    if (d < 0 || d >= n_durations) atomicCAS(status, 0, PQ8_ERR_INVALID_ARGUMENT);
    if (token == kTdtBlank && skip == 0) skip = 1;
    if (n_calls < trace_capacity) {
      int* tr = trace + (static_cast<size_t>(i) * trace_capacity + n_calls) * 3;
      tr[0] = t;
      tr[1] = token;
      tr[2] = skip;
    } else {
      atomicCAS(status, 0, PQ8_ERR_WORKSPACE);
    }
    ++n_calls;
    if (token != kTdtBlank) {
      commit = 1;
      if (n_emitted < emitted_capacity) {
        int* em = emitted + (static_cast<size_t>(i) * emitted_capacity + n_emitted) * 3;
        em[0] = token;
        em[1] = t;
        em[2] = skip;
      } else {
        atomicCAS(status, 0, PQ8_ERR_WORKSPACE);
      }
      ++n_emitted;
      previous = token;
    }
    ++symbols;
    t += skip;
    if (skip) {
      symbols = 0;
    } else if (symbols == kTdtMaxSymbols) {
      ++t;
      symbols = 0;
    }
    done = t >= frames;
    s[kTdtT] = t;
    s[kTdtSymbols] = symbols;
    s[kTdtPrevious] = previous;
    s[kTdtEmitted] = n_emitted;
    s[kTdtCalls] = n_calls;
    s[kTdtDone] = done;
  }
  commit_mask[i] = commit;
  tokens[i] = previous;
  enc_rows[i] = i * enc_stride + (frames > 0 ? min(t, frames - 1) : 0);
  return !done;
}

// One block; m <= blockDim.x.
__global__ void tdt_control_kernel(const int* __restrict__ ids, const int* __restrict__ durations, int n_durations,
                                   int* __restrict__ state, int m, int enc_stride, int* __restrict__ tokens,
                                   int* __restrict__ enc_rows, int* __restrict__ commit_mask,
                                   int* __restrict__ emitted, int emitted_capacity, int* __restrict__ trace,
                                   int trace_capacity, int* __restrict__ remaining, int* status) {
  griddep_launch();
  griddep_wait();  // the joint's ids and the previous step's state
  const int i = threadIdx.x;
  const bool live = i < m && tdt_control_stream(i, ids, durations, n_durations, state, enc_stride, tokens, enc_rows,
                                                commit_mask, emitted, emitted_capacity, trace, trace_capacity,
                                                status);
  const int n_live = __syncthreads_count(live);
  if (threadIdx.x == 0) *remaining = n_live;
}

// Control and commit in one launch. Block 0 applies the joint results of all
// m streams (tdt_control_stream); every block copies the candidate LSTM state
// (h_new, c_new -> h, c; float[layers][m][hidden]) of the rows whose joint
// token is not blank, over a grid-stride range of float4s. The commit test
// reads only the joint's ids, never the state block 0 is updating, so the
// blocks need no ordering; a stream already done may adopt a candidate too,
// which no result depends on. hidden % 4 == 0.
__global__ void tdt_advance_kernel(const int* __restrict__ ids, const int* __restrict__ durations, int n_durations,
                                   int* __restrict__ state, int m, int enc_stride, int* __restrict__ tokens,
                                   int* __restrict__ enc_rows, int* __restrict__ commit_mask,
                                   int* __restrict__ emitted, int emitted_capacity, int* __restrict__ trace,
                                   int trace_capacity, int* __restrict__ remaining, float* __restrict__ h,
                                   float* __restrict__ c, const float* __restrict__ h_new,
                                   const float* __restrict__ c_new, int layers, int hidden, int* status) {
  griddep_launch();
  griddep_wait();  // the joint's ids, the candidates and the previous step's state
  if (blockIdx.x == 0) {
    __shared__ int n_live;
    if (threadIdx.x == 0) n_live = 0;
    __syncthreads();
    int mine = 0;
    for (int i = threadIdx.x; i < m; i += blockDim.x)
      mine += tdt_control_stream(i, ids, durations, n_durations, state, enc_stride, tokens, enc_rows, commit_mask,
                                 emitted, emitted_capacity, trace, trace_capacity, status);
    if (mine) atomicAdd(&n_live, mine);
    __syncthreads();
    if (threadIdx.x == 0) *remaining = n_live;
  }
  const int row_vec = hidden / 4;
  const long long total = (long long)layers * m * row_vec;
  for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < total;
       v += (long long)gridDim.x * blockDim.x) {
    const int row = (int)((v / row_vec) % m);
    if (ids[2 * row] != kTdtBlank) {
      reinterpret_cast<float4*>(h)[v] = reinterpret_cast<const float4*>(h_new)[v];
      reinterpret_cast<float4*>(c)[v] = reinterpret_cast<const float4*>(c_new)[v];
    }
  }
}

}  // namespace pq8
