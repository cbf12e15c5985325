// The whole greedy TDT decode of up to kDecodeMaxStreams streams in one
// persistent launch (pq8_tdt_decode).
//
// The reference runs the loop on the host (parakeet_cuda/decoder.py:78-97):
// per joint call it launches the joint (decoder.py:66-72), reads the ids
// back, and after an emitted token commits the LSTM state and runs the
// prediction network (decoder.py:50-64: two LSTM layers and joint.pred).
// Here one cooperative grid (one CTA per SM, all co-resident) does all of it:
//   * every CTA copies its slice of the four Q8_0 weights (joint rows, the
//     four gates of a range of hidden units of both LSTM layers, joint.pred
//     rows; about 95 KB at the model's shapes) into shared memory once and
//     keeps them there for the whole decode, so a step reads no weights
//     from HBM;
//   * a step is one joint phase (ReLU(enc + pred) against the CTA's joint
//     rows, per-stream arg-max folded with 64-bit atomic keys), a grid
//     barrier, then the control rules of tdt_control_stream applied by every
//     CTA to its own copy of the streams' state (CTA 0 alone writes the
//     records), and, only when some stream emitted a token, the prediction
//     network for those streams (LSTM 0, barrier, LSTM 1, barrier, pred,
//     barrier);
//   * LSTM states live in two slots per stream: the committed one and the
//     candidate; committing a candidate flips the stream's slot index, so
//     nothing is copied.
// Grid barriers are a monotonically growing arrival counter (release add,
// acquire poll) with bounded waits: a CTA that waits kWaitLimitNs, or sees
// another CTA's abort, records PQ8_ERR_TIMEOUT and leaves, and every other
// CTA then leaves at its next barrier.
#pragma once

#include "pq8_device.cuh"
#include "pq8_gemv.cuh"
#include "pq8_tdt.cuh"

namespace pq8 {

constexpr int kDecodeThreads = 256;
constexpr int kDecodeMaxStreams = 64;
constexpr int kDecodeGroup = 16;  // streams per matrix-vector pass (activation rows staged at once)

// One Q8_0 matrix slice resident in shared memory: rows [0, rows) of the
// CTA's share, K blocks [0, kb). Values in two planes ([kb][row][16 B] for K
// positions 0-15 and 16-31 of the block: a warp's 16-byte loads of
// consecutive rows are contiguous), fp16 scales [kb][row].
struct SmemQ8 {
  uint32_t q0, q1, sc;  // byte offsets in dynamic shared memory
  int rows, kb;
};

struct DecodeParams {
  const uint8_t* w_lstm[2];
  const float* b_lstm[2];  // b_ih + b_hh, float[4 * hidden] in gate order i, f, g, o
  const uint8_t* w_pred;
  const float* b_pred;
  const uint8_t* w_joint;
  const float* b_joint;
  const uint16_t* embed;  // fp16 [vocab][embed_k]
  const float* enc;       // stream i, frame t: row i * enc_stride + t of [.][joint_k]
  const int* durations;
  int* state;  // int[m][kTdtStateWords]; word 7 = committed LSTM slot (kept for a resumed decode)
  int* emitted;
  int* trace;
  int* steps_out;  // joint steps run by this launch
  int* remaining;  // streams not done at the end
  // workspace
  float* h;  // [2 layers][2 slots][m][hidden]
  float* c;
  float* pred;                 // [m][joint_k]
  unsigned long long* keys;    // [3 buffers][m][2]
  unsigned* barrier;           // arrival counter
  int* abort;
  int* status;
  int m, hidden, embed_k, joint_k, n_joint, vocab, n_durations, enc_stride;
  int emitted_capacity, trace_capacity, max_steps, resume;
};

__device__ __forceinline__ void red_release_add_u32(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier: every CTA adds 1 to the counter and waits until it reaches
// `target` (advanced by gridDim.x per barrier). Returns false (and the CTA
// must leave) when the wait ran out or another CTA aborted.
__device__ __forceinline__ bool grid_barrier(const DecodeParams& p, unsigned& target, int* flag_s) {
  __syncthreads();
  if (threadIdx.x == 0) {
    target += gridDim.x;
    int ok = 1;
    __threadfence();  // the CTA's writes (ordered before this thread by the barrier above)
    red_release_add_u32(p.barrier, 1u);
    if (static_cast<int>(ld_acquire_u32(p.barrier) - target) < 0) {
      const uint64_t t0 = global_timer_ns();
      while (true) {
        bool arrived = false;
#pragma unroll 1
        for (int i = 0; i < 64; ++i) {
          if (static_cast<int>(ld_acquire_u32(p.barrier) - target) >= 0) {
            arrived = true;
            break;
          }
        }
        if (arrived) break;
        if (*reinterpret_cast<volatile int*>(p.abort)) {
          ok = 0;
          break;
        }
        if (global_timer_ns() - t0 > kWaitLimitNs) {
          atomicExch(p.abort, 1);
          atomicCAS(p.status, 0, PQ8_ERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    *flag_s = ok;
  }
  __syncthreads();
  return *flag_s != 0;
}

// Copies packed rows prow(r) of a packed weight (K blocks [0, kb)) into a
// shared-memory slice; rows past the matrix (prow < 0) are zero.
template <typename RowFn>
__device__ void load_slice(uint8_t* smem, const SmemQ8& s, const uint8_t* w, int kb_total, RowFn prow) {
  const uint8_t* data = w + PQ8_HEADER_BYTES;
  for (int i = threadIdx.x; i < s.rows * s.kb; i += blockDim.x) {
    const int r = i % s.rows, kb = i / s.rows;
    const int pr = prow(r);
    uint4 a = make_uint4(0, 0, 0, 0), b = a;
    uint16_t sc = 0;
    if (pr >= 0) {
      const uint8_t* rec = data + ((size_t)(pr >> 7) * kb_total + kb) * kRecordBytes;
      const int rr = pr & 127;
      a = *reinterpret_cast<const uint4*>(rec + rr * 16);
      b = *reinterpret_cast<const uint4*>(rec + 2048 + rr * 16);
      sc = *reinterpret_cast<const uint16_t*>(rec + kScaleOffset + rr * 2);
    }
    reinterpret_cast<uint4*>(smem + s.q0)[kb * s.rows + r] = a;
    reinterpret_cast<uint4*>(smem + s.q1)[kb * s.rows + r] = b;
    reinterpret_cast<uint16_t*>(smem + s.sc)[kb * s.rows + r] = sc;
  }
}

// Activation rows staged for a pass over a slice: the row count rounded up
// to 1, 2, 4, 8 or 16 (the matrix-vector product's template width).
__device__ __forceinline__ int group_rows(int mc) {
  return mc <= 1 ? 1 : mc <= 2 ? 2 : mc <= 4 ? 4 : mc <= 8 ? 8 : 16;
}

// xs[j][k] = load(j, k) (a float4 at k, k % 4 == 0) for rows j < mc and 0
// for rows mc .. group_rows(mc) - 1. A thread issues all its loads of a
// chunk (up to kStageUnroll float4s) before it stores any of them, so one
// staging costs about one memory round trip, not one per element.
constexpr int kStageUnroll = 10;  // (16 rows x 1280 floats: two chunks of loads)
template <typename LoadFn>
__device__ __forceinline__ void stage_rows(float* xs, int K, int mc, LoadFn load) {
  const int k4 = K / 4, n4 = group_rows(mc) * k4;
  for (int base = 0; base < n4; base += kDecodeThreads * kStageUnroll) {
    float4 v[kStageUnroll];
#pragma unroll
    for (int q = 0; q < kStageUnroll; ++q) {
      const int i = base + q * kDecodeThreads + static_cast<int>(threadIdx.x);
      const int j = i / k4;
      v[q] = (i < n4 && j < mc) ? load(j, (i - j * k4) * 4) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int q = 0; q < kStageUnroll; ++q) {
      const int i = base + q * kDecodeThreads + static_cast<int>(threadIdx.x);
      if (i < n4) reinterpret_cast<float4*>(xs)[i] = v[q];
    }
  }
}

// zs[r][j] (stride kDecodeGroup) = sum over K of slice row r times staged
// activation row j, for j < MT (xs is [MT][K], K = 32 * s.kb). The K blocks
// are split over the threads (S ranges per row), and the S partial sums of a
// row are added in range order, so the result does not depend on timing.
template <int MT>
__device__ __forceinline__ void slice_matvec(uint8_t* smem, const SmemQ8& s, const float* xs, float* part, float* zs) {
  const int R = s.rows, KB = s.kb, K = KB * 32;
  const int S = max(1, min(kDecodeThreads / R, KB));
  const int per = (KB + S - 1) / S;
  const int t = threadIdx.x;
  if (t < S * R) {
    const int r = t % R, sl = t / R;
    float acc[MT];
#pragma unroll
    for (int j = 0; j < MT; ++j) acc[j] = 0.0f;
    const uint4* q0 = reinterpret_cast<const uint4*>(smem + s.q0);
    const uint4* q1 = reinterpret_cast<const uint4*>(smem + s.q1);
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(smem + s.sc);
    const int kb1 = min(KB, (sl + 1) * per);
    // narrow passes unroll two K blocks so the next block's shared-memory loads
    // overlap this block's arithmetic (same order of additions)
#pragma unroll(MT <= 4 ? 2 : 1)
    for (int kb = sl * per; kb < kb1; ++kb)
      gemv_block<MT>(q0[kb * R + r], q1[kb * R + r], sc[kb * R + r], xs + kb * 32, K, acc);
#pragma unroll
    for (int j = 0; j < MT; ++j) part[(sl * R + r) * kDecodeGroup + j] = acc[j];
  }
  __syncthreads();
  for (int i = t; i < R * MT; i += kDecodeThreads) {
    const int idx = (i / MT) * kDecodeGroup + i % MT;
    // partials added in range order; four loads in flight per group of adds
    const float* pp = part + idx;
    const int step = R * kDecodeGroup;
    float z = 0.0f;
    int q = 0;
    for (; q + 4 <= S; q += 4) {
      const float a = pp[q * step], b = pp[(q + 1) * step], c = pp[(q + 2) * step], d = pp[(q + 3) * step];
      z += a;
      z += b;
      z += c;
      z += d;
    }
    for (; q < S; ++q) z += pp[q * step];
    zs[idx] = z;
  }
  __syncthreads();
}

// slice_matvec at the width staged for mc rows.
__device__ __forceinline__ void slice_matvec_rows(uint8_t* smem, const SmemQ8& s, const float* xs, float* part,
                                                  float* zs, int mc) {
  switch (group_rows(mc)) {
    case 1: slice_matvec<1>(smem, s, xs, part, zs); break;
    case 2: slice_matvec<2>(smem, s, xs, part, zs); break;
    case 4: slice_matvec<4>(smem, s, xs, part, zs); break;
    case 8: slice_matvec<8>(smem, s, xs, part, zs); break;
    default: slice_matvec<16>(smem, s, xs, part, zs); break;
  }
}

// Shared-memory layout of one CTA: the four weight slices, then the staged
// activations (kDecodeGroup rows of kmax floats), the partial sums, the
// reduced sums and the streams' control state. The host sizes the launch
// with the largest share (ceil(n / grid) rows of each matrix).
struct DecodeLayout {
  SmemQ8 joint, lstm[2], pred;
  uint32_t xs, part, zs, ctl, bias, total;
};

__host__ __device__ inline uint32_t decode_align16(uint32_t v) { return (v + 15u) & ~15u; }

__host__ __device__ inline DecodeLayout decode_layout(int rows_joint, int units, int rows_pred, int kb_joint,
                                                      int kb_lstm0, int kb_lstm1, int kb_pred, int kmax, int m) {
  DecodeLayout L;
  uint32_t off = 0;
  auto slice = [&](SmemQ8& s, int rows, int kb) {
    s.rows = rows;
    s.kb = kb;
    s.q0 = off;
    off = decode_align16(off + 16u * rows * kb);
    s.q1 = off;
    off = decode_align16(off + 16u * rows * kb);
    s.sc = off;
    off = decode_align16(off + 2u * rows * kb);
  };
  slice(L.joint, rows_joint, kb_joint);
  slice(L.lstm[0], 4 * units, kb_lstm0);
  slice(L.lstm[1], 4 * units, kb_lstm1);
  slice(L.pred, rows_pred, kb_pred);
  const int rmax = rows_joint > 4 * units ? (rows_joint > rows_pred ? rows_joint : rows_pred)
                                          : (4 * units > rows_pred ? 4 * units : rows_pred);
  L.xs = off;
  off = decode_align16(off + 4u * kDecodeGroup * kmax);
  L.part = off;
  off = decode_align16(off + 4u * kDecodeGroup * (rmax > kDecodeThreads ? rmax : kDecodeThreads));
  L.zs = off;
  off = decode_align16(off + 4u * kDecodeGroup * rmax);
  L.ctl = off;
  off = decode_align16(off + 4u * (kTdtStateWords * m + 2 * kDecodeMaxStreams + 8));
  L.bias = off;  // the biases of the CTA's rows: joint, LSTM 0 and 1 (gate-major), pred
  off = decode_align16(off + 4u * (rows_joint + 8 * units + rows_pred));
  L.total = off;
  return L;
}

// The reference's rules for one joint result (decoder.py:84-97; the same as
// tdt_control_stream): st = {frames, t, symbols, previous, emitted, calls,
// done, slot}. Returns 1 when the token is emitted (the candidate state is
// committed). CTA 0 writes the trace and emitted records.
__device__ __forceinline__ int decode_rules(int* st, int b, int token, int d, const DecodeParams& p, bool record) {
  int skip = (d >= 0 && d < p.n_durations) ? p.durations[d] : 0;
  if (record && (d < 0 || d >= p.n_durations)) atomicCAS(p.status, 0, PQ8_ERR_INVALID_ARGUMENT);
  if (token == kTdtBlank && skip == 0) skip = 1;
  const int t = st[kTdtT];
  if (record) {
    const int n_calls = st[kTdtCalls];
    if (n_calls < p.trace_capacity) {
      int* tr = p.trace + ((size_t)b * p.trace_capacity + n_calls) * 3;
      tr[0] = t;
      tr[1] = token;
      tr[2] = skip;
    } else {
      atomicCAS(p.status, 0, PQ8_ERR_WORKSPACE);
    }
  }
  ++st[kTdtCalls];
  int emit = 0;
  if (token != kTdtBlank) {
    emit = 1;
    if (record) {
      const int n_em = st[kTdtEmitted];
      if (n_em < p.emitted_capacity) {
        int* em = p.emitted + ((size_t)b * p.emitted_capacity + n_em) * 3;
        em[0] = token;
        em[1] = t;
        em[2] = skip;
      } else {
        atomicCAS(p.status, 0, PQ8_ERR_WORKSPACE);
      }
    }
    ++st[kTdtEmitted];
    st[kTdtPrevious] = token;
  }
  int symbols = st[kTdtSymbols] + 1, tn = t + skip;
  if (skip) {
    symbols = 0;
  } else if (symbols == kTdtMaxSymbols) {
    ++tn;
    symbols = 0;
  }
  st[kTdtT] = tn;
  st[kTdtSymbols] = symbols;
  st[kTdtDone] = tn >= st[kTdtFrames];
  return emit;
}

// list[0..count) = the streams b < m whose flag is set, in stream order
// (warps 0 and 1 ballot; every thread of the CTA calls it and gets the count).
__device__ __forceinline__ int decode_compact(const int* flags, int m, int* list, int* counts) {
  const int t = threadIdx.x;
  unsigned mask = 0;
  bool f = false;
  if (t < kDecodeMaxStreams) {  // whole warps
    f = t < m && flags[t] != 0;
    mask = __ballot_sync(0xffffffffu, f);
    if ((t & 31) == 0) counts[t >> 5] = __popc(mask);
  }
  __syncthreads();
  if (f) list[(t >= 32 ? counts[0] : 0) + __popc(mask & ((1u << (t & 31)) - 1u))] = t;
  __syncthreads();
  return counts[0] + counts[1];
}

// Balanced share [lo, hi) of n items for CTA `cta` of `ctas`.
__host__ __device__ inline void decode_share(int n, int cta, int ctas, int& lo, int& hi) {
  lo = static_cast<int>(static_cast<long long>(n) * cta / ctas);
  hi = static_cast<int>(static_cast<long long>(n) * (cta + 1) / ctas);
}

__global__ void __launch_bounds__(kDecodeThreads, 1) tdt_decode_kernel(const DecodeParams p) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int G = gridDim.x, cta = blockIdx.x, t = threadIdx.x;
  const int H = p.hidden, E = p.embed_k, KJ = p.joint_k, m = p.m;
  int j0, j1, u0, u1, p0, p1;
  decode_share(p.n_joint, cta, G, j0, j1);
  decode_share(H, cta, G, u0, u1);
  decode_share(KJ, cta, G, p0, p1);
  const int U = u1 - u0;
  const int kmax = max(E + H, max(2 * H, KJ));
  const DecodeLayout L = decode_layout(j1 - j0, U, p1 - p0, KJ / 32, (E + H) / 32, 2 * H / 32, H / 32, kmax, m);
  float* xs = reinterpret_cast<float*>(smem + L.xs);
  float* part = reinterpret_cast<float*>(smem + L.part);
  float* zs = reinterpret_cast<float*>(smem + L.zs);
  int* ctl = reinterpret_cast<int*>(smem + L.ctl);  // [m][kTdtStateWords]
  int* flags = ctl + kTdtStateWords * m;             // [kDecodeMaxStreams]
  int* list = flags + kDecodeMaxStreams;             // [kDecodeMaxStreams]
  int* misc = list + kDecodeMaxStreams;              // counts[4], barrier flag
  int* flag_s = misc + 4;

  // Headers: every CTA reads the same ones, so all leave together on a mismatch.
  if (t == 0) {
    auto hdr_ok = [](const uint8_t* w, int n, int k, int layout) {
      const PackedHeader* h = reinterpret_cast<const PackedHeader*>(w);
      return h->magic == kMagic && h->n == n && h->k == k && h->layout == layout;
    };
    const bool ok = hdr_ok(p.w_joint, p.n_joint, KJ, PQ8_LAYOUT_ROWS) && hdr_ok(p.w_pred, KJ, H, PQ8_LAYOUT_ROWS) &&
                    hdr_ok(p.w_lstm[0], 4 * H, E + H, PQ8_LAYOUT_GATES4) &&
                    hdr_ok(p.w_lstm[1], 4 * H, 2 * H, PQ8_LAYOUT_GATES4);
    if (!ok) atomicCAS(p.status, 0, PQ8_ERR_LAYOUT);
    *flag_s = ok;
  }
  __syncthreads();
  if (!*flag_s) return;

  // Resident weight slices. LSTM slice row g * U + ul is gate g of hidden
  // unit u0 + ul: packed row (u / 32) * 128 + g * 32 + u % 32 (GATES4).
  load_slice(smem, L.joint, p.w_joint, KJ / 32, [&](int r) { return j0 + r; });
  load_slice(smem, L.pred, p.w_pred, H / 32, [&](int r) { return p0 + r; });
  for (int l = 0; l < 2; ++l) {
    const int kbt = (l == 0 ? E + H : 2 * H) / 32;
    load_slice(smem, L.lstm[l], p.w_lstm[l], kbt, [&](int r) {
      const int g = r / U, u = u0 + r % U;
      return (u >> 5) * 128 + g * 32 + (u & 31);
    });
  }
  // The biases of the CTA's rows, read once (the phases' epilogues read them
  // right after their products, where a global load would be a round trip).
  float* bj = reinterpret_cast<float*>(smem + L.bias);  // [j1 - j0]
  float* bl = bj + (j1 - j0);                           // [2][4][U]: gate g of unit u0 + ul
  float* bp = bl + 8 * U;                               // [p1 - p0]
  for (int i = t; i < j1 - j0; i += kDecodeThreads) bj[i] = p.b_joint[j0 + i];
  for (int i = t; i < 8 * U; i += kDecodeThreads) bl[i] = p.b_lstm[i / (4 * U)][(i / U) % 4 * H + u0 + i % U];
  for (int i = t; i < p1 - p0; i += kDecodeThreads) bp[i] = p.b_pred[p0 + i];
  for (int i = t; i < m * kTdtStateWords; i += kDecodeThreads) ctl[i] = p.state[i];
  __syncthreads();
  if (!p.resume && t < m) ctl[t * kTdtStateWords + 7] = 0;  // committed slot of a fresh decode
  unsigned target = 0;
  const size_t HS = (size_t)m * H;  // floats per (layer, slot) state block
  auto hbuf = [&](int l, int slot, int b) { return p.h + ((size_t)(l * 2 + slot)) * HS + (size_t)b * H; };
  auto cbuf = [&](int l, int slot, int b) { return p.c + ((size_t)(l * 2 + slot)) * HS + (size_t)b * H; };

  // Prediction network for streams list[0..count): candidate state (slot
  // committed ^ 1) from the committed state and the stream's last token,
  // then pred = joint.pred(h1 candidate).
  auto predict = [&](int count) -> bool {
    for (int l = 0; l < 2; ++l) {
      const SmemQ8 sl = l == 0 ? L.lstm[0] : L.lstm[1];  // a copy: no dynamic index into L
      const int K = sl.kb * 32;
      for (int g0 = 0; g0 < count; g0 += kDecodeGroup) {
        const int mc = min(kDecodeGroup, count - g0);
        // the committed cell state of the cell update below, loaded alongside the staging
        float c_pre = 0.0f;
        if (t < U * mc) {
          const int b = list[g0 + t / U];
          c_pre = __ldcg(cbuf(l, ctl[b * kTdtStateWords + 7], b) + u0 + t % U);
        }
        stage_rows(xs, K, mc, [&](int j, int k) {
          const int b = list[g0 + j], cm = ctl[b * kTdtStateWords + 7];
          if (l == 0) {
            if (k >= E) return __ldcg(reinterpret_cast<const float4*>(hbuf(0, cm, b) + (k - E)));
            const uint2 hv = *reinterpret_cast<const uint2*>(
                p.embed + (size_t)ctl[b * kTdtStateWords + kTdtPrevious] * E + k);
            const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&hv.x));
            const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&hv.y));
            return make_float4(lo.x, lo.y, hi.x, hi.y);
          }
          return k < H ? __ldcg(reinterpret_cast<const float4*>(hbuf(0, cm ^ 1, b) + k))
                       : __ldcg(reinterpret_cast<const float4*>(hbuf(1, cm, b) + (k - H)));
        });
        __syncthreads();
        slice_matvec_rows(smem, sl, xs, part, zs, mc);
        for (int i = t; i < U * mc; i += kDecodeThreads) {
          const int ul = i % U, j = i / U, u = u0 + ul;
          const int b = list[g0 + j], cm = ctl[b * kTdtStateWords + 7];
          const float* bias = bl + l * 4 * U + ul;
          const float gi = zs[(0 * U + ul) * kDecodeGroup + j] + bias[0 * U];
          const float gf = zs[(1 * U + ul) * kDecodeGroup + j] + bias[1 * U];
          const float gg = zs[(2 * U + ul) * kDecodeGroup + j] + bias[2 * U];
          const float go = zs[(3 * U + ul) * kDecodeGroup + j] + bias[3 * U];
          const float si = 1.0f / (1.0f + expf(-gi)), sf = 1.0f / (1.0f + expf(-gf));
          const float so = 1.0f / (1.0f + expf(-go));
          const float cn = sf * (i == t ? c_pre : __ldcg(cbuf(l, cm, b) + u)) + si * tanhf(gg);
          cbuf(l, cm ^ 1, b)[u] = cn;
          hbuf(l, cm ^ 1, b)[u] = so * tanhf(cn);
        }
      }
      if (!grid_barrier(p, target, flag_s)) return false;
    }
    {
      const SmemQ8& sp = L.pred;
      const int K = H;
      for (int g0 = 0; g0 < count; g0 += kDecodeGroup) {
        const int mc = min(kDecodeGroup, count - g0);
        stage_rows(xs, K, mc, [&](int j, int k) {
          const int b = list[g0 + j];
          return __ldcg(reinterpret_cast<const float4*>(hbuf(1, ctl[b * kTdtStateWords + 7] ^ 1, b) + k));
        });
        __syncthreads();
        slice_matvec_rows(smem, sp, xs, part, zs, mc);
        for (int i = t; i < sp.rows * mc; i += kDecodeThreads) {
          const int r = i % sp.rows, j = i / sp.rows;
          p.pred[(size_t)list[g0 + j] * KJ + p0 + r] = zs[r * kDecodeGroup + j] + bp[r];
        }
      }
    }
    return grid_barrier(p, target, flag_s);
  };

  int steps = 0;
  bool ok = true;
  if (!p.resume) {
    for (int i = t; i < kDecodeMaxStreams; i += kDecodeThreads) flags[i] = i < m;
    const int count = decode_compact(flags, m, list, misc);
    ok = predict(count);
  }
  while (ok && steps < p.max_steps) {
    // streams still decoding
    for (int i = t; i < kDecodeMaxStreams; i += kDecodeThreads) flags[i] = i < m && !ctl[i * kTdtStateWords + kTdtDone];
    const int live = decode_compact(flags, m, list, misc);
    if (live == 0) break;
    const int buf = steps % 3;
    unsigned long long* keys = p.keys + (size_t)buf * m * 2;
    // Joint: ReLU(enc row + pred) against this CTA's rows, arg-max per stream.
    const SmemQ8& sj = L.joint;
    for (int g0 = 0; g0 < live; g0 += kDecodeGroup) {
      const int mc = min(kDecodeGroup, live - g0);
      stage_rows(xs, KJ, mc, [&](int j, int k) {
        const int b = list[g0 + j];
        const int* st = ctl + b * kTdtStateWords;
        const int frames = st[kTdtFrames];
        const int row = b * p.enc_stride + (frames > 0 ? min(st[kTdtT], frames - 1) : 0);
        const float4 e = *reinterpret_cast<const float4*>(p.enc + (size_t)row * KJ + k);
        const float4 q = __ldcg(reinterpret_cast<const float4*>(p.pred + (size_t)b * KJ + k));
        return make_float4(fmaxf(e.x + q.x, 0.0f), fmaxf(e.y + q.y, 0.0f), fmaxf(e.z + q.z, 0.0f),
                           fmaxf(e.w + q.w, 0.0f));
      });
      __syncthreads();
      slice_matvec_rows(smem, sj, xs, part, zs, mc);
      const int warp = t >> 5, lane = t & 31;
      for (int jw = warp; jw < mc; jw += kDecodeThreads / 32) {  // warp w: streams list[g0 + w], + 8, ...
        float v0 = -INFINITY, v1 = -INFINITY;
        int i0 = INT_MAX, i1 = INT_MAX;
        for (int r = lane; r < sj.rows; r += 32) {
          const int row = j0 + r;
          const float z = zs[r * kDecodeGroup + jw] + bj[r];
          if (row < p.vocab) argmax_merge(v0, i0, z, row);
          else argmax_merge(v1, i1, z, row);
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) {
          argmax_merge(v0, i0, __shfl_down_sync(0xffffffffu, v0, off), __shfl_down_sync(0xffffffffu, i0, off));
          argmax_merge(v1, i1, __shfl_down_sync(0xffffffffu, v1, off), __shfl_down_sync(0xffffffffu, i1, off));
        }
        if (lane == 0) {
          const int b = list[g0 + jw];
          if (i0 != INT_MAX) atomicMax(keys + b * 2 + 0, argmax_key(v0, i0));
          if (i1 != INT_MAX) atomicMax(keys + b * 2 + 1, argmax_key(v1, i1));
        }
      }
      __syncthreads();  // zs and xs are reused by the next group
    }
    if (!grid_barrier(p, target, flag_s)) {
      ok = false;
      break;
    }
    // the key buffer of the step before last has been read by every CTA
    if (cta == 0)
      for (int i = t; i < m * 2; i += kDecodeThreads) p.keys[(size_t)((steps + 2) % 3) * m * 2 + i] = 0ull;
    // Control: every CTA applies the rules to its copy of the state.
    if (t < m) {
      int emit = 0;
      int* st = ctl + t * kTdtStateWords;
      if (!st[kTdtDone]) {
        const unsigned long long k0 = __ldcg(keys + t * 2), k1 = __ldcg(keys + t * 2 + 1);
        const int i0 = k0 ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k0)) : 0;
        const int i1 = k1 ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(k1)) - p.vocab : 0;
        emit = decode_rules(st, t, i0, i1, p, cta == 0);
        if (emit) st[7] ^= 1;  // the candidate becomes the committed state
      }
      flags[t] = emit;
    }
    ++steps;
    __syncthreads();
    const int count = decode_compact(flags, m, list, misc);
    if (count > 0 && !predict(count)) {
      ok = false;
      break;
    }
  }
  if (ok && cta == 0) {
    __syncthreads();
    for (int i = t; i < m * kTdtStateWords; i += kDecodeThreads) p.state[i] = ctl[i];
    if (t == 0) {
      int live = 0;
      for (int b = 0; b < m; ++b) live += !ctl[b * kTdtStateWords + kTdtDone];
      *p.remaining = live;
      *p.steps_out = steps;
    }
  }
}

}  // namespace pq8
