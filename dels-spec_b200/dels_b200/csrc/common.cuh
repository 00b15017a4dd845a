// Shared device helpers for the DeLS draft-scoring kernels (sm_100a only).
//
// Everything here is hand-written inline PTX for the Blackwell async machinery the
// kernels use: mbarriers with bounded waits, TMA tile loads, and the tcgen05
// tensor-core / tensor-memory instructions.  Also the packed (score, index) key that
// turns "argmax with the lowest index on ties" into a single signed 64-bit max, which
// both the in-kernel atomics and the cross-rank NCCL all-reduce(MAX) use.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../../include/dels_b200.h"

namespace dels {

// A single mbarrier wait gives up after this long (the whole kernel normally runs in
// well under a millisecond per wave).  On expiry the kernel records
// DELS_ERR_DEVICE_TIMEOUT in the caller's status word, tells the other roles of the CTA
// to stop, and returns; the host reads the status after synchronising.
constexpr unsigned long long kWaitLimitNs = 2000ull * 1000ull * 1000ull;

// --------------------------------------------------------------------------------
// Packed argmax keys.
//
// key = (ordered_i32(score) << 32) | (0xFFFFFFFF - index)
//
// ordered_i32 maps IEEE floats to int32 so that signed integer order equals float
// order.  The low word is the complemented index, so among equal scores the lowest
// index has the largest key: max(key) is torch.argmax's "first occurrence" rule
// (reference: code/kernel/dels.py:134 strict '>' and torch.argmax in
// code/kernel/dels.py:456).  NaN maps above +inf, so a NaN score wins like it does in
// torch.argmax; -0.0 is folded onto +0.0 so that the two compare equal as in torch.
// --------------------------------------------------------------------------------
__host__ __device__ __forceinline__ int32_t ordered_i32(float f) {
  if (f != f) return 0x7FFFFFFF;
  if (f == 0.0f) f = 0.0f;
#ifdef __CUDA_ARCH__
  int32_t i = __float_as_int(f);
#else
  int32_t i;
  __builtin_memcpy(&i, &f, 4);
#endif
  return i < 0 ? (i ^ 0x7FFFFFFF) : i;
}

__host__ __device__ __forceinline__ float ordered_to_float(int32_t o) {
  int32_t i = o < 0 ? (o ^ 0x7FFFFFFF) : o;
#ifdef __CUDA_ARCH__
  return __int_as_float(i);
#else
  float f;
  __builtin_memcpy(&f, &i, 4);
  return f;
#endif
}

__host__ __device__ __forceinline__ long long pack_key(float score, uint32_t index) {
  return (long long)(((unsigned long long)(uint32_t)ordered_i32(score) << 32) |
                     (unsigned long long)(0xFFFFFFFFu - index));
}

__host__ __device__ __forceinline__ uint32_t key_index(long long key) {
  return 0xFFFFFFFFu - (uint32_t)((unsigned long long)key & 0xFFFFFFFFull);
}

__host__ __device__ __forceinline__ float key_score(long long key) {
  return ordered_to_float((int32_t)((unsigned long long)key >> 32));
}

constexpr long long kKeyEmpty = (long long)0x8000000000000000ull;

// ordered_i32 without branches, for the scoring epilogues: x + 0 turns -0 into +0 and
// leaves every other value (NaN included) as it is.
__device__ __forceinline__ int32_t ordered_i32_dev(float f) {
  const int32_t i = __float_as_int(__fadd_rn(f, 0.0f));
  const int32_t o = i ^ ((i >> 31) & 0x7FFFFFFF);
  return f != f ? 0x7FFFFFFF : o;
}

// max(a, b) / max(a, b, c) that return NaN when any input is NaN.
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}
__device__ __forceinline__ float fmax3_nan(float a, float b, float c) {
  float d;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// Score threshold of a running key for chunk_fold: -inf for the empty key, +inf once a
// NaN holds it (only a NaN at a lower index could still win, and NaN chunks always fold).
__device__ __forceinline__ float key_threshold(long long key) {
  if (key == kKeyEmpty) return -__int_as_float(0x7f800000);
  const float f = key_score(key);
  return f != f ? __int_as_float(0x7f800000) : f;
}

// Folds the chunk sc[0..valid) (global indices idx0 + j) into the running packed key
// best_key, i.e. best_key = max(best_key, max_j pack_key(sc[j], idx0 + j)): the largest
// score, NaN above everything, -0 equal to +0, the lowest index among equal scores.
//
// The NaN-propagating maximum m of the chunk comes from a tree of three-input maxima (entries past
// `valid` read as -inf).  A chunk with m below `thr` -- a score some column of the row
// already reached: this thread's best so far, or the row's global key read at the start
// of the tile -- cannot hold the argmax and is done.  Otherwise the lowest column whose
// score equals m (or is NaN when m is NaN) comes from a 32-bit match mask and ONE key is
// packed.  Packing and reducing a 64-bit key per column took ~11 instructions per column;
// issued on the SM sub-partitions that also run the MMA-issuing and TMA warps, that cost
// the paired scorer ~4 points of tensor-pipe utilisation (ncu).
__device__ __forceinline__ void chunk_fold(const float (&sc)[32], int valid, uint32_t idx0, long long& best_key,
                                           float& thr) {
  float x[32];
  if (valid >= 32) {
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = sc[j];
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) x[j] = j < valid ? sc[j] : -__int_as_float(0x7f800000);
  }
  // 32 -> 12 -> 4 -> 1 with three-input maxima
  float t[12];
#pragma unroll
  for (int j = 0; j < 10; ++j) t[j] = fmax3_nan(x[3 * j], x[3 * j + 1], x[3 * j + 2]);
  t[10] = x[30];
  t[11] = x[31];
  float u[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) u[j] = fmax3_nan(t[3 * j], t[3 * j + 1], t[3 * j + 2]);
  const float m = fmax_nan(fmax3_nan(u[0], u[1], u[2]), u[3]);
  if (m < thr) return;
  uint32_t mask = 0u;
  if (m == m) {
#pragma unroll
    for (int j = 0; j < 32; ++j) mask |= x[j] == m ? (1u << j) : 0u;
  } else {
#pragma unroll
    for (int j = 0; j < 32; ++j) mask |= x[j] != x[j] ? (1u << j) : 0u;
  }
  const uint32_t first = (uint32_t)(__ffs((int)mask) - 1);
  const long long key = (long long)(((unsigned long long)(uint32_t)ordered_i32_dev(m) << 32) |
                                    (unsigned long long)(0xFFFFFFFFu - (idx0 + first)));
  best_key = key > best_key ? key : best_key;
  thr = m == m ? m : __int_as_float(0x7f800000);
}

// Row position (the draft-block slot that selects alpha_p / beta_p).
__device__ __forceinline__ int row_position(const int* row_pos, int row, int n_pos) {
  return row_pos != nullptr ? row_pos[row] : (row % n_pos);
}

// --------------------------------------------------------------------------------
// Shared-memory addresses, timers
// --------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// --------------------------------------------------------------------------------
// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialisation may start while the previous kernel in the stream is still running; it
// calls pdl_wait() before it reads anything an earlier kernel wrote or writes anything
// an earlier kernel reads (the wait returns once the previous grid has completed and
// its memory is visible).  pdl_trigger() lets the next kernel launch now.  Both are
// no-ops in a normal launch.
// --------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// --------------------------------------------------------------------------------
// mbarrier
// --------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t"
      "}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false if the CTA's
// abort flag is raised or the wait runs past limit_ns (kWaitLimitNs unless given); in
// the latter case this thread raises the abort flag and records
// DELS_ERR_DEVICE_TIMEOUT in *status.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag,
                                          int* status, unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      *abort_flag = 1;
      if (status != nullptr) atomicCAS(status, 0, DELS_ERR_DEVICE_TIMEOUT);
      return false;
    }
  }
}

// --------------------------------------------------------------------------------
// TMA (tensor tile copies global -> shared, completion counted on an mbarrier)
// --------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int x,
                                            int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// --------------------------------------------------------------------------------
// Per-thread asynchronous 16-byte copies global -> shared (the epilogue's operand
// prefetch).  src_bytes < 16 zero-fills the rest of the 16 bytes without reading past
// src + src_bytes.
// --------------------------------------------------------------------------------
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

// --------------------------------------------------------------------------------
// tcgen05: tensor memory, MMA, commit, loads
// --------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Arrive (once) on an mbarrier when every tcgen05.mma issued so far by this thread
// has completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulator.
__device__ __forceinline__ void tc_mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B (both K-major),
// fp32 accumulator, shape M x N.
__host__ __device__ constexpr uint32_t make_idesc_bf16_f32(int M, int N) {
  return (1u << 4)                        // accumulator format: f32
         | (1u << 7)                      // A format: bf16
         | (1u << 10)                     // B format: bf16
         | ((uint32_t)(N >> 3) << 17)     // N / 8
         | ((uint32_t)(M >> 4) << 24);    // M / 16
}

// Shared-memory matrix descriptor for a K-major bf16 tile written by TMA with the
// 128-byte swizzle: rows of 64 elements (128 B), 8-row swizzle atoms 1024 B apart.
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr & 0x3FFFFu) >> 4);  // start address / 16
  d |= (uint64_t)1 << 16;                         // leading byte offset (unused with swizzle)
  d |= (uint64_t)(1024 >> 4) << 32;               // stride byte offset: 8 rows * 128 B
  d |= (uint64_t)1 << 46;                         // descriptor version for sm_100
  d |= (uint64_t)2 << 61;                         // layout: 128-byte swizzle
  return d;
}

// Load 32 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

// Wait for this thread's outstanding tcgen05.ld, then pin the loaded registers after
// the wait so that no consumer is scheduled ahead of it.
template <int N>
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&v)[N]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < N; ++i) asm volatile("" : "+r"(v[i]));
}

// 16 consecutive fp32 columns of this warp's 32 lanes (lane i of the warp <-> TMEM lane
// base + i).
__device__ __forceinline__ void tmem_ld_16cols(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}

// --------------------------------------------------------------------------------
// CTA pairs (2-CTA clusters): cluster rank, cross-CTA shared addresses, remote arrive,
// cluster barrier, and the cta_group::2 forms of the tensor-memory / MMA / TMA
// instructions.  In a pair, the MMA issued by rank 0 reads A and B from both CTAs'
// shared memory (same offsets) and writes each CTA's 128-row half of D into that CTA's
// tensor memory.
// --------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Shared::cluster address of the variable at local address `addr` in CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

// All threads of both CTAs of the cluster.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem of both CTAs] (+)= A[smem of both] * B[smem of both]^T, M = 256 across the pair.
__device__ __forceinline__ void tc_mma_pair_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                                 uint32_t accumulate) {
  asm volatile(
      "{\n\t"
      ".reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at local offset `bar` in BOTH CTAs of the pair when the
// issuing thread's prior tcgen05.mma operations have completed.
__device__ __forceinline__ void tc_commit_pair_both(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          bar),
      "h"((unsigned short)0x3)
      : "memory");
}

// TMA tile load into this CTA's shared memory whose completion is counted on the
// mbarrier at shared::cluster address `bar_cluster` (rank 0's barrier in a pair).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

// --------------------------------------------------------------------------------
// bf16 helpers
// --------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
// two floats rounded to bf16 (nearest-even), lo in the low half (the lower address)
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 p = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&p);
}

}  // namespace dels
