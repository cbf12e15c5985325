// Device-side building blocks shared by the pq8 kernels (sm_100a only):
// PTX wrappers for mbarriers, TMA / bulk copies and tcgen05 (tensor memory +
// 5th-generation tensor-core MMA), bounded waits, and the Q8_0 value helpers.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "pq8.h"

namespace pq8 {

// ---------------------------------------------------------------------------
// Packed weight header (first PQ8_HEADER_BYTES of every packed tensor).
struct PackedHeader {
  uint32_t magic;     // kMagic
  uint32_t version;   // 1
  int32_t n;          // source rows
  int32_t k;          // columns (multiple of 32)
  int32_t layout;     // PQ8_LAYOUT_*
  int32_t n_tiles;    // tiles of 128 packed rows
  int32_t k_blocks;   // k / 32
  int32_t out_cols;   // n, n/2 (GLU) or n/4 (GATES4)
};
constexpr uint32_t kMagic = 0x50385150u;  // "PQ8P"
constexpr int kTileRows = PQ8_TILE_ROWS;
constexpr int kRecordBytes = PQ8_RECORD_BYTES;
constexpr int kScaleOffset = 4096;  // fp16 scales follow the 128 x 32 int8 values

// Bounded waits: a wait that has not completed after this many nanoseconds
// sets the CTA's abort flag and the device status word, and returns false.
constexpr uint64_t kWaitLimitNs = 4000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking test of phase `parity` (acquire, CTA scope): lets a thread
// start the check for its next phase before it needs the answer.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar`. Gives up (returns false) when the CTA's
// abort flag is raised or after kWaitLimitNs, raising the flag and recording
// PQ8_ERR_TIMEOUT in the device status word.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* status) {
  const uint32_t a = smem_addr(bar);
  if (mbar_try_wait(a, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 32; ++i)
      if (mbar_try_wait(a, parity)) return true;
    if (*abort_flag) return false;
    if (global_timer_ns() - t0 > kWaitLimitNs) {
      *abort_flag = 1;
      if (status) atomicCAS(status, 0, PQ8_ERR_TIMEOUT);
      return false;
    }
  }
}

// Bounded wait used on the teardown path: ignores the abort flag.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_addr(bar);
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(a, parity)) {
    if (global_timer_ns() - t0 > kWaitLimitNs) return;
  }
}

// Position in a ring of SIZE buffers and the parity of the pass over it,
// advanced without divisions (the roles' loops run on issue-starved warps,
// where a division by a non-power-of-two constant is a long dependent chain).
template <int SIZE>
struct Ring {
  uint32_t idx = 0, phase = 0;
  __device__ __forceinline__ void advance(uint32_t n) {  // n <= SIZE
    idx += n;
    if (idx >= SIZE) {
      idx -= SIZE;
      phase ^= 1u;
    }
  }
};

// ---------------------------------------------------------------------------
// Bulk / tensor copies (global -> shared, completion counted on an mbarrier)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_addr(dst)),
      "l"(tmap), "r"(c0), "r"(c1), "r"(smem_addr(bar))
      : "memory");
}
// Shared -> global tensor store (asynchronous; completion tracked by bulk groups).
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(tmap), "r"(c0),
               "r"(c1), "r"(smem_addr(src))
               : "memory");
}
// Shared -> global bulk copy (bytes a multiple of 16, both addresses 16-byte
// aligned; completion tracked by bulk groups).
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_addr(src)),
               "r"(bytes)
               : "memory");
}
// Shared -> shared bulk copy into a CTA of the cluster: dst and mbar are that
// CTA's addresses (from map_to_rank), src this CTA's; bytes a multiple of 16,
// both addresses 16-byte aligned. Completion is counted on the destination's
// mbarrier (complete_tx).
__device__ __forceinline__ void bulk_s2s_cluster(uint32_t dst, const void* src, uint32_t bytes, uint32_t mbar) {
  asm volatile("cp.async.bulk.shared::cluster.shared::cta.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   dst),
               "r"(smem_addr(src)), "r"(bytes), "r"(mbar)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups are still reading their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_group_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Barrier over `count` threads (a multiple of 32) using hardware barrier `id` (1..15).
__device__ __forceinline__ void named_barrier_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
// Programmatic dependent launch. A kernel launched with programmatic stream
// serialization may start while the previous kernel in the stream is still
// running; griddep_wait blocks until that kernel has completed and its memory
// is visible (a no-op without the launch attribute). griddep_launch lets the
// next kernel start launching as soon as every CTA of this one has called it.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Two-warp rendezvous on named barrier `id` (64 threads) that also ORs one
// flag across both warps. Both warps must call it the same number of times.
__device__ __forceinline__ bool rendezvous_or(int id, bool flag) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred q, p;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.or.pred p, %2, 64, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(flag)), "r"(id)
      : "memory");
  return out != 0;
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}
// Make generic-proxy shared-memory writes visible to the async proxy (tensor core reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory and MMA
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T, kind::tf32, one CTA. Issued by one thread.
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once all tcgen05 operations issued so far by this thread have completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_addr(bar))
               : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Each thread of the warp writes 16 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
// Each thread of the warp reads 16 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
// Each thread of the warp reads 32 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile written by TMA
// with 128-byte swizzling: 8-row x 128-byte swizzle atoms stacked at a
// 1024-byte stride (SBO), version 1 (sm_100), layout SWIZZLE_128B (2).
// Commit variants taking the barrier's shared-window address (no conversion
// per call; used by the MMA warp, whose instruction count is on the critical path).
__device__ __forceinline__ void mma_commit_addr(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mma_commit_pair_addr(uint32_t bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"(cta_mask)
      : "memory");
}
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}
// Instruction descriptor: kind::tf32, A and B TF32 K-major, FP32 accumulate, M x N.
__host__ __device__ constexpr uint32_t idesc_tf32(int m, int n) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// ---------------------------------------------------------------------------
// Numeric helpers

// Round an FP32 bit pattern to TF32 (10 explicit mantissa bits), to nearest,
// ties away from zero; Inf/NaN keep their exponent. The tensor core reads only
// the 19 high bits of each 32-bit operand, so the 13 low bits are cleared.
__device__ __forceinline__ uint32_t tf32_round_bits(uint32_t u) {
  return ((u & 0x7F800000u) == 0x7F800000u) ? u : ((u + 0x1000u) & 0xFFFFE000u);
}
__device__ __forceinline__ float tf32_round(float f) { return __uint_as_float(tf32_round_bits(__float_as_uint(f))); }
// fp32 bits -> TF32 bits, round to nearest, ties to even (finite inputs).
__device__ __forceinline__ uint32_t tf32_rne_bits(uint32_t u) {
  return (u + 0xFFFu + ((u >> 13) & 1u)) & 0xFFFFE000u;
}

// Signed int8 lane `i` (0..3) of a 32-bit word as an exact float: the biased
// byte (q + 128) is placed in the mantissa of 2^23 and the bias removed.
__device__ __forceinline__ float i8_to_f32(uint32_t biased_word, int i) {
  const uint32_t sel = 0x7540u | (uint32_t)i;  // bytes: [i], 0, 0, 0x4B
  return __uint_as_float(__byte_perm(biased_word, 0x4B000000u, sel)) - 8388736.0f;  // 2^23 + 128
}

__device__ __forceinline__ float sigmoidf_(float v) { return 1.0f / (1.0f + __expf(-v)); }

__device__ __forceinline__ float apply_act(float z, int epi) {
  if (epi == PQ8_EPI_RELU) return fmaxf(z, 0.0f);
  if (epi == PQ8_EPI_SILU) return z * sigmoidf_(z);
  return z;
}

// Source row and output column of packed row `p` (tile-local row r = p % 128).
// Returns false for padding rows.
struct RowMap {
  int src;  // source row in the GGUF tensor
  int col;  // output column (ROWS: = src; GLU: pair index; GATES4: hidden unit)
};
__device__ __forceinline__ bool map_row(int layout, int n, int p, RowMap& rm) {
  const int t = p >> 7, r = p & 127;
  if (layout == PQ8_LAYOUT_ROWS) {
    rm.src = p;
    rm.col = p;
    return p < n;
  }
  if (layout == PQ8_LAYOUT_GLU) {
    const int h = n >> 1, w = r >> 5, l = r & 31;
    const int j = t * 64 + w * 16 + (l & 15);
    rm.col = j;
    rm.src = (l < 16) ? j : h + j;
    return j < h;
  }
  const int h = n >> 2, g = r >> 5, u = t * 32 + (r & 31);
  rm.col = u;
  rm.src = g * h + u;
  return u < h;
}

}  // namespace pq8

// ---------------------------------------------------------------------------
// Pairs of CTAs (cluster of 2) sharing one tcgen05 MMA (cta_group::2)
namespace pq8 {

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Split cluster barrier: arrive without ordering (e.g. "this CTA has started"),
// wait later.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// Shared-memory address of the same variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void* p, uint32_t rank) {
  uint32_t out;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_addr(p)), "r"(rank));
  return out;
}
// Stores into another CTA's shared memory (address from map_to_rank).
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_f32x2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void st_cluster_f32x4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
// Arrive on a barrier of another CTA of the cluster (address from map_to_rank).
// Default (CTA-scope release) semantics: a cluster-scope release here made the
// arriving thread wait for all of its SM's outstanding memory traffic,
// including in-flight TMA loads, which cost ~2000 cycles per arrival.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Waits on barriers that also receive arrivals from the peer CTA.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                  int* status) {
  return mbar_wait(bar, parity, abort_flag, status);
}
__device__ __forceinline__ void fence_proxy_async_cluster() {
  asm volatile("fence.proxy.async.shared::cluster;" ::: "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T over both CTAs of the pair (M = 256), kind::tf32.
__device__ __forceinline__ void mma_tf32_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` (same offset) in every CTA of `cta_mask` once this thread's prior tcgen05 ops complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_addr(bar)),
      "h"(cta_mask)
      : "memory");
}

}  // namespace pq8
