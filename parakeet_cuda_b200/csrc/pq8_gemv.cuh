// Decoder-regime contraction (m <= 64 activation rows): an HBM-streaming,
// split-K GEMV over the packed Q8_0 records, with the TDT tails fused.
//
// One CTA of 128 threads handles one 128-row weight tile over a range of K
// blocks; thread r owns tile row r, so the reduction over K is thread-local
// and needs no shuffles. Each thread streams its row's 2 x 16 bytes of int8
// values and its fp16 scale per K block with 128-bit non-allocating loads
// (a warp reads 512 contiguous bytes per instruction). The activations of
// the CTA's K range are staged once in shared memory and read as broadcasts.
//
// When a tile's K range is split over S <= 16 CTAs, the splits form one
// thread-block cluster that reduces and scatters: CTA j finishes the tile
// rows r with (r % 16) % S == j (so a GLU pair r, r + 16 and the four LSTM
// gates r % 32 + 32 g of one hidden unit stay together). Every CTA stores each
// row's partial sums into the shared memory of that row's owner, one cluster
// barrier publishes them, and each owner adds its rows' partials in split
// order and runs the epilogue for them. The partial sums thus spread over all
// SMs of the cluster instead of converging on one. With more splits, each CTA
// writes its partials to the workspace and the last CTA to arrive (atomic
// ticket) adds them in split order; tickets reset themselves, so a zeroed
// workspace stays valid across calls. Either way the result does not depend
// on CTA timing.
//
// Modes: plain linear (bias / ReLU / SiLU / GLU / residual epilogues), one
// LSTM layer (GATES4 layout: the four gates of 32 hidden units per tile are
// combined in shared memory and the cell update runs in the epilogue), and
// the TDT joint (ReLU(enc + pred) staged as the activation; each CTA folds its
// rows' arg-max into one 64-bit key per (row, part) with an atomic maximum,
// which the last CTA to finish decodes).
//
// A CTA handles MT <= 8 activation rows; larger m runs ceil(m / 8) row groups
// as the grid's y dimension of one launch (rows [8y, 8y + 8)), each with its
// own slice of every workspace region, so that the groups' tiles run
// concurrently instead of one launch after another. The weights are re-read
// per group, from L2 for decoder-sized matrices.
#pragma once

#include <float.h>
#include <limits.h>

#include "pq8_device.cuh"

namespace pq8 {

enum GemvMode { kGemvLinear = 0, kGemvLstm = 1, kGemvJoint = 2 };
enum XMode { kXPlain = 0, kXConcat = 1, kXReluSum = 2, kXEmbedConcat = 3 };

struct GemvParams {
  const uint8_t* w;
  const float* x0;
  const float* x1;
  const uint16_t* embed;
  const int* tokens;
  const int* x0_rows;  // optional row indices into x0 (joint: frame of each stream)
  int x_mode;
  int x_vec4;  // activation pointers allow 16-byte loads (embedding: 8-byte)
  int k0;  // width of the first segment in concat modes
  float* y;
  const float* bias;
  const float* resid;
  float alpha;
  int epi;
  int m, n, k, layout, out_cols, n_tiles, k_blocks, splits, kb_per_split;
  int cluster_reduce;  // the splits of a tile form one thread-block cluster (rank = split)
  float* partial;  // [row groups][n_tiles][splits][128][MT]
  int* tickets;    // [row groups][n_tiles]
  int* done_count; // joint: [row groups] CTAs finished
  unsigned long long* best_key;  // joint: [row groups][MT][2] arg-max keys (argmax_key)
  const float* c_prev;
  float* h_out;
  float* c_out;
  int hidden;
  int* ids;
  int vocab;
  int mode;
  int* status;
};

constexpr int kGemvThreads = 128;
constexpr int kGemvXSmemFloats = 10240;  // at most 40 KB of staged activations per CTA
constexpr int kGemvMaxClusterSplits = 16;  // cluster size (non-portable above 8)
constexpr int kGemvCtasPerSm = 4;          // resident CTAs per SM (launch bounds; 128 registers)
// Streamed weights (HBM regime): a producer warp copies the CTA's records in
// chunks of kStreamChunk records into a ring of kStreamRing chunks.
constexpr int kStreamChunk = 4;
constexpr int kStreamRing = 4;
constexpr int kStreamRingBytes = kStreamRing * kStreamChunk * kRecordBytes;
// Streaming CTAs run two groups of 128 compute threads (alternate records of
// each chunk, combined before the epilogue) and one producer warp.
constexpr int kStreamCompute = 2 * kGemvThreads;
constexpr int kStreamThreads = kStreamCompute + 32;

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ uint16_t ldg_u16(const void* p) {
  uint16_t v;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
  return v;
}

// Activation element (row m, column kg) for the staged modes.
__device__ __forceinline__ float load_x(const GemvParams& p, int m, int kg) {
  switch (p.x_mode) {
    case kXConcat:
      return kg < p.k0 ? p.x0[(size_t)m * p.k0 + kg] : p.x1[(size_t)m * (p.k - p.k0) + (kg - p.k0)];
    case kXReluSum: {
      const size_t row = p.x0_rows ? (size_t)p.x0_rows[m] : (size_t)m;
      return fmaxf(p.x0[row * p.k + kg] + p.x1[(size_t)m * p.k + kg], 0.0f);
    }
    case kXEmbedConcat:
      return kg < p.k0 ? __half2float(__ushort_as_half(p.embed[(size_t)p.tokens[m] * p.k0 + kg]))
                       : p.x1[(size_t)m * (p.k - p.k0) + (kg - p.k0)];
    default:
      return p.x0[(size_t)m * p.k + kg];
  }
}

__device__ __forceinline__ float4 ldg_f4(const float* p) { return *reinterpret_cast<const float4*>(p); }

// Four consecutive activation elements (row m, columns kg..kg+3; kg % 4 == 0,
// so a group never straddles a concat boundary, k0 % 32 == 0). x0_row is the
// resolved row of x0 (joint: the stream's frame; embedding: the token).
__device__ __forceinline__ float4 load_x4(const GemvParams& p, int m, int x0_row, int kg) {
  switch (p.x_mode) {
    case kXConcat:
      return kg < p.k0 ? ldg_f4(p.x0 + (size_t)m * p.k0 + kg) : ldg_f4(p.x1 + (size_t)m * (p.k - p.k0) + (kg - p.k0));
    case kXReluSum: {
      const float4 a = ldg_f4(p.x0 + (size_t)x0_row * p.k + kg), b = ldg_f4(p.x1 + (size_t)m * p.k + kg);
      return make_float4(fmaxf(a.x + b.x, 0.0f), fmaxf(a.y + b.y, 0.0f), fmaxf(a.z + b.z, 0.0f),
                         fmaxf(a.w + b.w, 0.0f));
    }
    case kXEmbedConcat: {
      if (kg >= p.k0) return ldg_f4(p.x1 + (size_t)m * (p.k - p.k0) + (kg - p.k0));
      const uint2 h = *reinterpret_cast<const uint2*>(p.embed + (size_t)x0_row * p.k0 + kg);
      const float2 lo = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
      const float2 hi = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
      return make_float4(lo.x, lo.y, hi.x, hi.y);
    }
    default:
      return ldg_f4(p.x0 + (size_t)m * p.k + kg);
  }
}

// (value, index) as one 64-bit key whose unsigned order is the arg-max order
// of argmax_merge: larger value first, then the lower index. -0 counts as +0
// (they compare equal); a NaN never wins (key 0, as in a strict greater-than
// scan). The value's bits are mapped to an order-preserving unsigned integer.
__device__ __forceinline__ unsigned long long argmax_key(float v, int i) {
  if (v != v) return 0ull;
  uint32_t b = __float_as_uint(v + 0.0f);
  b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return (static_cast<unsigned long long>(b) << 32) | (0xFFFFFFFFu - static_cast<uint32_t>(i));
}

// (value, index) arg-max with ties to the lowest index.
__device__ __forceinline__ void argmax_merge(float& v, int& i, float ov, int oi) {
  if (ov > v || (ov == v && oi < i)) {
    v = ov;
    i = oi;
  }
}

// acc[m] += scale * sum_j q_j * x[m][j] over one 32-wide K block of this thread's row.
// Packed f32x2 arithmetic (sm_100): two lanes of FP32 per instruction.
__device__ __forceinline__ uint64_t f32x2_pack(float lo, float hi) {
  uint64_t v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "f"(lo), "f"(hi));
  return v;
}
__device__ __forceinline__ uint64_t f32x2_add(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t f32x2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float f32x2_sum(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}

// One 32-wide K block of one row against MT activation rows: the codes become
// floats by placing the biased byte under 2^23 (PRMT) and subtracting
// 2^23 + 128, two at a time with packed f32x2 adds; the products accumulate
// in packed f32x2 FMAs (even and odd K positions in the two halves), so the
// GEMV spends about 2 instructions per weight and row instead of 3. The block
// sum is scaled once.
template <int MT>
__device__ __forceinline__ void gemv_block(const uint4 q0, const uint4 q1, uint16_t scale_bits, const float* xk,
                                           int nk, float (&acc)[MT]) {
  const float sc = __half2float(__ushort_as_half(scale_bits));
  const uint32_t wd[8] = {q0.x ^ 0x80808080u, q0.y ^ 0x80808080u, q0.z ^ 0x80808080u, q0.w ^ 0x80808080u,
                          q1.x ^ 0x80808080u, q1.y ^ 0x80808080u, q1.z ^ 0x80808080u, q1.w ^ 0x80808080u};
  const uint64_t minus_bias = f32x2_pack(-8388736.0f, -8388736.0f);
  uint64_t inner[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) inner[m] = 0;  // (+0, +0)
#pragma unroll
  for (int j = 0; j < 32; j += 4) {
    const uint32_t w = wd[j >> 2];
    const uint64_t q01 = f32x2_add(f32x2_pack(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540)),
                                              __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541))),
                                   minus_bias);
    const uint64_t q23 = f32x2_add(f32x2_pack(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7542)),
                                              __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7543))),
                                   minus_bias);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      const float4 xv = *reinterpret_cast<const float4*>(xk + m * nk + j);
      inner[m] = f32x2_fma(q01, f32x2_pack(xv.x, xv.y), inner[m]);
      inner[m] = f32x2_fma(q23, f32x2_pack(xv.z, xv.w), inner[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = fmaf(sc, f32x2_sum(inner[m]), acc[m]);
}

// Barrier among the 128 compute threads (named barrier 1 when the producer
// warp of the streaming variant has left).
template <bool STREAM>
__device__ __forceinline__ void compute_sync() {
  if constexpr (STREAM) named_barrier_sync(1, kGemvThreads);
  else __syncthreads();
}

// STREAM: the weight records are brought in by bulk copies from a producer
// warp (tens of KB in flight per CTA without holding them in registers, which
// is what HBM streaming at M = 1 needs), and two groups of 128 threads
// consume alternate records of each chunk; otherwise each thread loads its
// row's bytes itself, U K blocks ahead (small launches where latency matters
// more than bytes in flight).
template <int MT, bool STREAM>
__device__ __forceinline__ void gemv_cta(const GemvParams& p, const int bx, const int by) {
  static_assert(MT * 2 * 8 <= kGemvThreads, "the joint tail gives 8 threads to each (row, part) pair");
  extern __shared__ __align__(128) float xs[];
  __shared__ float gate_s[MT][4][32];
  __shared__ float red_v[4][MT][2];
  __shared__ int red_i[4][MT][2];
  __shared__ int ticket_s;
  __shared__ uint64_t full[kStreamRing], empty[kStreamRing];
  __shared__ int abort_s;
  __shared__ float comb[STREAM ? MT : 1][kGemvThreads];  // second group's sums

  const int t = bx / p.splits, split = bx % p.splits;
  const int r = threadIdx.x, lane = r & 31, warp = r >> 5;
  // Row group: activation rows [row0, row0 + mg) of the launch's p.m rows.
  const int row0 = by * MT;
  const int mg = min(MT, p.m - row0);
  const size_t grp_sel = by;
  float* const partial = p.partial + grp_sel * ((size_t)p.n_tiles * p.splits * kGemvThreads * MT);
  int* const tickets = p.tickets + grp_sel * p.n_tiles;
  int* const done_count = p.done_count + grp_sel;
  // Rows this CTA finishes: all, or in a cluster of S splits those with (r % 16) % S == split.
  const int own_s = (!STREAM && p.cluster_reduce) ? p.splits : 1;
  const int own_j = own_s > 1 ? split : 0;
  const bool own = ((r & 15) % own_s) == own_j;
  unsigned long long* const best_key = p.best_key + grp_sel * (MT * 2);
  // (the last splits of a power-of-two cluster may have an empty K range)
  const int kb0 = min(p.k_blocks, split * p.kb_per_split);
  const int kb1 = min(p.k_blocks, kb0 + p.kb_per_split);
  const int nk = (kb1 - kb0) * 32;

  // Programmatic dependent launch: the next kernel in the stream may start its
  // own weight prefetch now; it waits for this grid before touching anything
  // this grid writes.
  griddep_launch();
  // Cluster split-K stores into the leader's shared memory only once every
  // CTA of the cluster is known to have started (first barrier phase).
  if (!STREAM && p.cluster_reduce) cluster_arrive_relaxed();
  if (r == 0 && bx == 0 && by == 0) {
    const PackedHeader* h = reinterpret_cast<const PackedHeader*>(p.w);
    if (!(h->magic == kMagic && h->n == p.n && h->k == p.k && h->layout == p.layout && h->n_tiles == p.n_tiles))
      atomicCAS(p.status, 0, PQ8_ERR_LAYOUT);
  }
  const uint8_t* tile_base = p.w + PQ8_HEADER_BYTES + (size_t)t * p.k_blocks * kRecordBytes;
  const int nrec = kb1 - kb0;
  const int chunks = (nrec + kStreamChunk - 1) / kStreamChunk;
  uint8_t* ring = reinterpret_cast<uint8_t*>(xs) + ((MT * nk * 4 + 127) & ~127);

  // Weights do not depend on the previous kernel: their first loads (the first
  // ring of chunks, or the first U blocks of this thread's row) are issued
  // before waiting for it, so they overlap its tail.
  constexpr int U = MT <= 2 ? 4 : 2;                 // K blocks per batch of loads
  constexpr bool kDoubleBuffer = !STREAM && MT <= 4;  // next batch in flight during the arithmetic
  uint4 qa[U], qb[U];
  uint16_t sh[U];
  auto load_batch = [&](int kb, uint4(&a)[U], uint4(&b)[U], uint16_t(&sc)[U]) {
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (kb + u < kb1) {
        const uint8_t* rec = tile_base + (size_t)(kb + u) * kRecordBytes;
        a[u] = ldg_stream(rec + r * 16);
        b[u] = ldg_stream(rec + 2048 + r * 16);
        sc[u] = ldg_u16(rec + kScaleOffset + r * 2);
      }
  };
  Ring<kStreamRing> pr;  // producer position (STREAM)
  int issued = 0;
  if constexpr (STREAM) {
    if (r == kStreamCompute) {
      for (int i = 0; i < kStreamRing; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], kStreamCompute / 32);  // one arrival per compute warp
      }
      abort_s = 0;
      fence_mbar_init();
      // the first ring of chunks needs no free slot
      for (; issued < min(chunks, kStreamRing); ++issued, pr.advance(1)) {
        const int n_in = min(kStreamChunk, nrec - issued * kStreamChunk);
        const uint32_t bytes = static_cast<uint32_t>(n_in * kRecordBytes);
        mbar_expect_tx(&full[pr.idx], bytes);
        bulk_g2s(ring + pr.idx * (kStreamChunk * kRecordBytes),
                 tile_base + (size_t)(kb0 + issued * kStreamChunk) * kRecordBytes, bytes, &full[pr.idx]);
      }
    }
  } else {
    load_batch(kb0, qa, qb, sh);
  }
  griddep_wait();

  // Stage the activations of this CTA's K range: xs[m * nk + kk]. The
  // indirect rows (joint frame, embedding token) are resolved once; each
  // thread then keeps kStageUnroll independent 16-byte loads in flight.
  __shared__ int x0row_s[MT];
  if (r < MT) {
    const int row = row0 + r;
    int v = row;
    if (r < mg) {
      if (p.x_mode == kXReluSum && p.x0_rows != nullptr) v = p.x0_rows[row];
      else if (p.x_mode == kXEmbedConcat) v = p.tokens[row];
    }
    x0row_s[r] = v;
  }
  __syncthreads();
  constexpr int kStagers = STREAM ? kStreamCompute : kGemvThreads;
  if (r < kStagers) {
    if (p.x_vec4) {
      constexpr int kStageUnroll = 4;
      const int nk4 = nk >> 2, n4 = MT * nk4;
      float4* xs4 = reinterpret_cast<float4*>(xs);
      for (int i0 = r; i0 < n4; i0 += kStageUnroll * kStagers) {
        float4 v[kStageUnroll];
#pragma unroll
        for (int u = 0; u < kStageUnroll; ++u) {
          const int i = i0 + u * kStagers;
          v[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          if (i < n4) {
            const int m = i / nk4, kk = (i - m * nk4) * 4;
            if (m < mg) v[u] = load_x4(p, row0 + m, x0row_s[m], kb0 * 32 + kk);
          }
        }
#pragma unroll
        for (int u = 0; u < kStageUnroll; ++u)
          if (i0 + u * kStagers < n4) xs4[i0 + u * kStagers] = v[u];
      }
    } else {
      for (int i = r; i < MT * nk; i += kStagers) {
        const int m = i / nk, kk = i - m * nk;
        xs[i] = (m < mg) ? load_x(p, row0 + m, kb0 * 32 + kk) : 0.0f;
      }
    }
  }
  __syncthreads();

  if constexpr (STREAM) {
    if (r >= kStreamCompute) {
      // ------------------------------------------------ producer warp
      if (lane == 0) {
        for (; issued < chunks; ++issued, pr.advance(1)) {
          if (!mbar_wait(&empty[pr.idx], pr.phase ^ 1u, &abort_s, p.status)) break;
          const int n_in = min(kStreamChunk, nrec - issued * kStreamChunk);
          const uint32_t bytes = static_cast<uint32_t>(n_in * kRecordBytes);
          mbar_expect_tx(&full[pr.idx], bytes);
          bulk_g2s(ring + pr.idx * (kStreamChunk * kRecordBytes),
                   tile_base + (size_t)(kb0 + issued * kStreamChunk) * kRecordBytes, bytes, &full[pr.idx]);
        }
        // Never leave the CTA with copies still landing in its shared memory.
        for (int j = issued > kStreamRing ? issued - kStreamRing : 0; j < issued; ++j)
          mbar_drain(&full[j % kStreamRing], (j / kStreamRing) & 1);
      }
      return;  // the compute warps synchronise among themselves from here on
    }
  }

  float acc[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc[m] = 0.0f;

  if constexpr (STREAM) {
    const int row = r & (kGemvThreads - 1), grp = r / kGemvThreads;  // group 1 takes the odd records
    Ring<kStreamRing> cr;
    for (int j = 0; j < chunks; ++j, cr.advance(1)) {
      if (!mbar_wait(&full[cr.idx], cr.phase, &abort_s, p.status)) break;
      const uint8_t* cs = ring + cr.idx * (kStreamChunk * kRecordBytes);
      const int n_in = min(kStreamChunk, nrec - j * kStreamChunk);
      for (int u = grp; u < n_in; u += 2) {
        const uint8_t* rec = cs + u * kRecordBytes;
        gemv_block<MT>(*reinterpret_cast<const uint4*>(rec + row * 16),
                       *reinterpret_cast<const uint4*>(rec + 2048 + row * 16),
                       *reinterpret_cast<const uint16_t*>(rec + kScaleOffset + row * 2),
                       xs + (j * kStreamChunk + u) * 32, nk, acc);
      }
      // the chunk's values have been consumed by this warp's arithmetic
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[cr.idx]);
    }
    // Second group hands its sums to the first, which runs the epilogue.
    if (grp == 1) {
#pragma unroll
      for (int m = 0; m < MT; ++m) comb[m][row] = acc[m];
    }
    named_barrier_sync(2, kStreamCompute);
    if (grp == 1) return;
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] += comb[m][row];
  } else {
    // Batches of U K blocks (U x 34 bytes of weights per thread in flight);
    // with double buffering the next batch is requested before this one's
    // arithmetic. The blocks are summed in K order either way.
    for (int kb = kb0; kb < kb1; kb += U) {
      if constexpr (kDoubleBuffer) {
        uint4 na[U], nb[U];
        uint16_t nsh[U];
        if (kb + U < kb1) load_batch(kb + U, na, nb, nsh);
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (kb + u < kb1) gemv_block<MT>(qa[u], qb[u], sh[u], xs + (kb + u - kb0) * 32, nk, acc);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          qa[u] = na[u];
          qb[u] = nb[u];
          sh[u] = nsh[u];
        }
      } else {
#pragma unroll
        for (int u = 0; u < U; ++u)
          if (kb + u < kb1) gemv_block<MT>(qa[u], qb[u], sh[u], xs + (kb + u - kb0) * 32, nk, acc);
        if (kb + U < kb1) load_batch(kb + U, qa, qb, sh);
      }
    }
  }

  if (!STREAM && p.cluster_reduce) {
    // part_s[split][r][MT] in the owner's shared memory, after the largest
    // staged-activation area of the launch.
    float* part_s = xs + ((MT * p.kb_per_split * 32 + 31) & ~31);
    const uint32_t dst =
        map_to_rank(part_s + ((size_t)split * kGemvThreads + r) * MT, static_cast<uint32_t>((r & 15) % own_s));
    cluster_wait();  // all CTAs of the cluster are running
    if constexpr (MT == 1) {
      st_cluster_f32(dst, acc[0]);
    } else if constexpr (MT == 2) {
      st_cluster_f32x2(dst, acc[0], acc[1]);
    } else {
#pragma unroll
      for (int m = 0; m < MT; m += 4) st_cluster_f32x4(dst + 16 * (m / 4), acc[m], acc[m + 1], acc[m + 2], acc[m + 3]);
    }
    cluster_sync();  // second phase: release the stores / acquire everyone's
    if (own) {
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
      for (int s = 0; s < own_s; ++s) {
        const float* part = part_s + ((size_t)s * kGemvThreads + r) * MT;
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[m] += part[m];
      }
    }
  } else if (p.splits > 1) {
    float* mine = partial + (((size_t)t * p.splits + split) * kGemvThreads + r) * MT;
#pragma unroll
    for (int m = 0; m < MT; ++m) __stcg(mine + m, acc[m]);
    __threadfence();
    compute_sync<STREAM>();
    if (r == 0) ticket_s = atomicAdd(&tickets[t], 1);
    compute_sync<STREAM>();
    if (ticket_s != p.splits - 1) return;
    __threadfence();
#pragma unroll
    for (int m = 0; m < MT; ++m) acc[m] = 0.0f;
#pragma unroll 4
    for (int s = 0; s < p.splits; ++s) {
      const float* part = partial + (((size_t)t * p.splits + s) * kGemvThreads + r) * MT;
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[m] += __ldcg(part + m);
    }
    if (r == 0) tickets[t] = 0;
  }

  RowMap rm;
  const bool valid = map_row(p.layout, p.n, t * kTileRows + r, rm);
  const float b = (p.bias != nullptr && valid) ? p.bias[rm.src] : 0.0f;

  if (p.mode == kGemvLinear) {
    // The residual rows are all read before any output is written (y may
    // alias resid), so they cost one memory round trip, not one per row.
    float res[MT];
#pragma unroll
    for (int m = 0; m < MT; ++m)
      res[m] = (p.epi == PQ8_EPI_RESIDUAL && valid && own && m < mg)
                   ? p.resid[(size_t)(row0 + m) * p.out_cols + rm.col]
                   : 0.0f;
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m >= mg) break;
      const size_t row = row0 + m;
      const float z = acc[m] + b;
      float out;
      if (p.epi == PQ8_EPI_GLU) {
        const float gate = __shfl_down_sync(0xffffffffu, z, 16);
        out = z * sigmoidf_(gate);
      } else if (p.epi == PQ8_EPI_RESIDUAL) {
        out = valid ? res[m] + p.alpha * z : 0.0f;
      } else {
        out = apply_act(z, p.epi);
      }
      if (valid && own && (p.epi != PQ8_EPI_GLU || lane < 16)) p.y[row * p.out_cols + rm.col] = out;
    }
    return;
  }

  if (p.mode == kGemvLstm) {
    // Tile row r holds gate (r / 32) of hidden unit t*32 + r%32.
#pragma unroll
    for (int m = 0; m < MT; ++m) gate_s[m][warp][lane] = acc[m] + b;
    compute_sync<STREAM>();
    // Cell update: warp w takes rows w, w + 4, ... of the group, lane = hidden
    // unit; all c_prev values are loaded before any state is written.
    constexpr int kRowsPerWarp = (MT + 3) / 4;
    const int u = t * 32 + lane;
    const bool unit = u < p.hidden && ((lane & 15) % own_s) == own_j;  // this CTA finishes unit u
    float cp[kRowsPerWarp];
#pragma unroll
    for (int j = 0; j < kRowsPerWarp; ++j) {
      const int m = warp + 4 * j;
      cp[j] = (m < mg && unit) ? p.c_prev[(size_t)(row0 + m) * p.hidden + u] : 0.0f;
    }
#pragma unroll
    for (int j = 0; j < kRowsPerWarp; ++j) {
      const int m = warp + 4 * j;
      if (m < mg && unit) {
        const size_t row = row0 + m;
        const float gi = gate_s[m][0][lane], gf = gate_s[m][1][lane];
        const float gg = gate_s[m][2][lane], go = gate_s[m][3][lane];
        const float si = 1.0f / (1.0f + expf(-gi)), sf = 1.0f / (1.0f + expf(-gf));
        const float so = 1.0f / (1.0f + expf(-go));
        const float c = sf * cp[j] + si * tanhf(gg);
        p.c_out[row * p.hidden + u] = c;
        p.h_out[row * p.hidden + u] = so * tanhf(c);
      }
    }
    return;
  }

  // Joint: logits, then per-tile arg-max partials for tokens / durations.
  float bv[MT][2];
  int bi[MT][2];
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    const float z = acc[m] + b;
    if (p.y != nullptr && valid && own && m < mg) p.y[(size_t)(row0 + m) * p.n + rm.src] = z;
    const bool tok = valid && own && rm.src < p.vocab, dur = valid && own && rm.src >= p.vocab;
    bv[m][0] = tok ? z : -INFINITY;
    bi[m][0] = tok ? rm.src : INT_MAX;
    bv[m][1] = dur ? z : -INFINITY;
    bi[m][1] = dur ? rm.src : INT_MAX;
  }
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      float v = bv[m][part];
      int i = bi[m][part];
#pragma unroll
      for (int off = 16; off; off >>= 1) {
        const float ov = __shfl_down_sync(0xffffffffu, v, off);
        const int oi = __shfl_down_sync(0xffffffffu, i, off);
        argmax_merge(v, i, ov, oi);
      }
      if (lane == 0) {
        red_v[warp][m][part] = v;
        red_i[warp][m][part] = i;
      }
    }
  compute_sync<STREAM>();
  if (r < MT * 2) {
    const int m = r >> 1, part = r & 1;
    float v = red_v[0][m][part];
    int i = red_i[0][m][part];
    for (int w = 1; w < 4; ++w) argmax_merge(v, i, red_v[w][m][part], red_i[w][m][part]);
    if (m < mg && i != INT_MAX) atomicMax(best_key + m * 2 + part, argmax_key(v, i));
  }
  __threadfence();
  compute_sync<STREAM>();
  if (r == 0) ticket_s = atomicAdd(done_count, 1);
  compute_sync<STREAM>();
  const int n_slots = p.n_tiles * own_s;
  if (ticket_s != n_slots - 1) return;
  __threadfence();
  // Last CTA of the row group: decode the keys (the atomics resolved in L2)
  // and reset them for the next call.
  if (r < MT * 2) {
    const int m = r >> 1, part = r & 1;
    if (m < mg) {
      const unsigned long long key = __ldcg(best_key + m * 2 + part);
      const int i = key ? static_cast<int>(0xFFFFFFFFu - static_cast<uint32_t>(key)) : -1;
      p.ids[(row0 + m) * 2 + part] = i < 0 ? 0 : i - (part ? p.vocab : 0);
      best_key[m * 2 + part] = 0ull;
    }
  }
  if (r == 0) *done_count = 0;
}

template <int MT, bool STREAM>
__global__ void __launch_bounds__(STREAM ? kStreamThreads : kGemvThreads, STREAM ? 2 : kGemvCtasPerSm)
    gemv_kernel(const GemvParams p) {
  gemv_cta<MT, STREAM>(p, static_cast<int>(blockIdx.x), static_cast<int>(blockIdx.y));
}

// Many independent M = 1 products in one launch (pq8_gemv_batch_run): task i
// owns CTAs [cta0, cta0 + ctas) of the grid, and each CTA runs the streaming
// GEMV of its task as if it were CTA blockIdx.x - cta0 of that task's own
// launch. One launch keeps HBM streaming across matrices of a few MB each,
// which as separate launches are bound by launch and ramp-up latency.
struct GemvTask {
  GemvParams p;
  int cta0;
  int pad[3];
};

// Header of a batch plan (the task table follows it).
struct BatchPlanHeader {
  uint32_t magic;
  int count, ctas, pad;
};

__global__ void __launch_bounds__(kStreamThreads, 2)
    gemv_batch_kernel(const GemvTask* tasks, const BatchPlanHeader* hdr) {
  __shared__ GemvParams ps;
  __shared__ int bx_s;
  if (threadIdx.x == 0) {
    const int count = hdr->count;
    int lo = 0, hi = count - 1;  // last task with cta0 <= blockIdx.x
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (tasks[mid].cta0 <= static_cast<int>(blockIdx.x)) lo = mid;
      else hi = mid - 1;
    }
    ps = tasks[lo].p;
    bx_s = static_cast<int>(blockIdx.x) - tasks[lo].cta0;
  }
  __syncthreads();
  gemv_cta<1, true>(ps, bx_s, 0);
}

// TDT commit: rows whose mask is set take the candidate LSTM state
// (decoder.py:74-75 swaps the buffers of its single stream).
__global__ void tdt_commit_kernel(float* __restrict__ h, float* __restrict__ c, const float* __restrict__ hn,
                                  const float* __restrict__ cn, const int* __restrict__ mask, int m, int layers,
                                  int hidden) {
  griddep_launch();
  griddep_wait();  // the mask and the candidates come from the kernels before
  const long long total = (long long)layers * m * hidden;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int row = (int)((i / hidden) % m);
    if (mask[row]) {
      h[i] = hn[i];
      c[i] = cn[i];
    }
  }
}

}  // namespace pq8
